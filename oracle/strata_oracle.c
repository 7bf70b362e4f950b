/*
 * strata_oracle.c — CPU restatement of strata-rs's quantized-matmul path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product): see the header.
 * Build: oracle/Makefile (gcc -std=c11 -O2 -ffp-contract=off -fPIC -shared).
 *
 * Parity anchors (all paths relative to the strata-rs repository root):
 *   QuantType geometry ............ crates/strata-gguf/src/quant.rs:125-180
 *   f16 -> f32 (half 2.7.1) ....... crates/strata-gguf/src/dequant.rs:28-36
 *   dequantize_row ................ crates/strata-gguf/src/dequant.rs:45-61
 *   dequant_q8_0 .................. crates/strata-gguf/src/dequant.rs:123-128
 *   dequant_q6_k .................. crates/strata-gguf/src/dequant.rs:208-234
 *   get_scale_min_k4 .............. crates/strata-gguf/src/dequant.rs:237-245
 *   dequant_q4_k .................. crates/strata-gguf/src/dequant.rs:247-270
 *   dequant_q5_k .................. crates/strata-gguf/src/dequant.rs:272-302
 *   Q2_0, Q8_1, Q4_0/1, Q5_0/1 .... crates/strata-gguf/src/dequant.rs:87-180
 *   IQ4_NL, IQ4_XS ................ crates/strata-gguf/src/dequant.rs:182-206
 *   Q3_K, Q2_K .................... crates/strata-gguf/src/dequant.rs:304-380
 *   MXFP4, NVFP4 .................. crates/strata-gguf/src/dequant.rs:382-445
 *   ops::gemv ..................... crates/strata-core/src/ops.rs:14-28
 *   ops::expert_gemv .............. crates/strata-core/src/ops.rs:169-195
 *   ops::silu / sigmoid ........... crates/strata-core/src/ops.rs:84-92
 *   ops::rms_norm / l2_norm ....... crates/strata-core/src/ops.rs:45-56,71-81
 *   ops::softmax / rope_neox ...... crates/strata-core/src/ops.rs:107-140
 *   ops::add_into ................. crates/strata-core/src/ops.rs:164-168
 *   bf16_round (half 2.7.1) ....... crates/strata-core/src/hyper.rs:21-24
 *   MoeLayer::route / combine ..... crates/strata-core/src/moe.rs:48-144
 */
#define _GNU_SOURCE
#include "strata_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- geometry */

int64_t orc_block_size(uint32_t q) {
    switch (q) {
    case ORC_F32: case ORC_F16: case ORC_BF16: return 1;
    case ORC_Q4_0: case ORC_Q4_1: case ORC_Q5_0: case ORC_Q5_1: case ORC_Q8_0: case ORC_Q8_1:
    case ORC_IQ4_NL: case ORC_MXFP4: return 32;
    case ORC_NVFP4: case ORC_Q2_0: return 64;
    case ORC_Q2_K: case ORC_Q3_K: case ORC_Q4_K: case ORC_Q5_K: case ORC_Q6_K: case ORC_IQ4_XS: return 256;
    default: return 0;
    }
}

int64_t orc_type_size(uint32_t q) {
    switch (q) {
    case ORC_F32: return 4;
    case ORC_F16: case ORC_BF16: return 2;
    case ORC_Q4_0: case ORC_IQ4_NL: case ORC_Q2_0: return 18;
    case ORC_Q4_1: return 20;
    case ORC_Q5_0: return 22;
    case ORC_Q5_1: return 24;
    case ORC_Q8_0: return 34;
    case ORC_Q8_1: return 36;
    case ORC_Q2_K: return 84;
    case ORC_Q3_K: return 110;
    case ORC_Q4_K: return 144;
    case ORC_Q5_K: return 176;
    case ORC_Q6_K: return 210;
    case ORC_IQ4_XS: return 136;
    case ORC_MXFP4: return 17;
    case ORC_NVFP4: return 36;
    default: return 0;
    }
}

int64_t orc_byte_size(uint32_t q, int64_t n) {
    int64_t bs = orc_block_size(q);
    if (bs == 0) return 0;
    return ((n + bs - 1) / bs) * orc_type_size(q);
}

/* ------------------------------------------------------------ scalar codecs */

static float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* IEEE binary16 -> binary32, exact; NaNs keep their payload with the quiet bit
 * set, which is what half 2.7.1 returns (its software path and F16C agree). */
float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    if (exp == 0x1F) {
        if (man == 0) return bits_f32(sign | 0x7F800000u);
        return bits_f32(sign | 0x7FC00000u | (man << 13));
    }
    if (exp == 0) {
        if (man == 0) return bits_f32(sign);
        /* subnormal: man * 2^-24, normalised */
        int shift = 0;
        while ((man & 0x400u) == 0) { man <<= 1; ++shift; }
        man &= 0x3FFu;
        return bits_f32(sign | ((uint32_t)(127 - 15 + 1 - shift) << 23) | (man << 13));
    }
    return bits_f32(sign | ((exp + 112u) << 23) | (man << 13));
}

/* f32 -> bf16, round half to even; a NaN keeps its high bits and is quietened. */
uint16_t orc_f32_to_bf16_bits(float v) {
    uint32_t x = f32_bits(v);
    if ((x & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((x >> 16) | 0x0040u);
    uint32_t round_bit = 0x8000u;
    if ((x & round_bit) != 0 && (x & (3u * round_bit - 1u)) != 0) return (uint16_t)((x >> 16) + 1u);
    return (uint16_t)(x >> 16);
}

float orc_bf16_round(float v) { return bits_f32((uint32_t)orc_f32_to_bf16_bits(v) << 16); }

static uint16_t rd16(const uint8_t *b) { return (uint16_t)(b[0] | (b[1] << 8)); }

/* --------------------------------------------------------------- dequant */

/* dequant.rs:123-128 */
static void dequant_q8_0(const uint8_t *b, float *out) {
    float d = orc_f16_to_f32(rd16(b));
    for (int j = 0; j < 32; ++j) out[j] = (float)(int8_t)b[2 + j] * d;
}

/* dequant.rs:208-234; the 16 scales are read as u8 (not i8). */
static void dequant_q6_k(const uint8_t *b, float *out) {
    const uint8_t *ql = b, *qh = b + 128, *sc = b + 192;
    float d = orc_f16_to_f32(rd16(b + 208));
    int y = 0, ql_off = 0, qh_off = 0, sc_off = 0;
    for (int half = 0; half < 2; ++half) {
        for (int l = 0; l < 32; ++l) {
            int is = l / 16;
            int q1 = ((ql[ql_off + l] & 0x0F) | ((qh[qh_off + l] & 3) << 4)) - 32;
            int q2 = ((ql[ql_off + l + 32] & 0x0F) | (((qh[qh_off + l] >> 2) & 3) << 4)) - 32;
            int q3 = ((ql[ql_off + l] >> 4) | (((qh[qh_off + l] >> 4) & 3) << 4)) - 32;
            int q4 = ((ql[ql_off + l + 32] >> 4) | (((qh[qh_off + l] >> 6) & 3) << 4)) - 32;
            /* `d * sc as f32 * q as f32` evaluates left to right */
            out[y + l] = d * (float)sc[sc_off + is] * (float)q1;
            out[y + l + 32] = d * (float)sc[sc_off + is + 2] * (float)q2;
            out[y + l + 64] = d * (float)sc[sc_off + is + 4] * (float)q3;
            out[y + l + 96] = d * (float)sc[sc_off + is + 6] * (float)q4;
        }
        y += 128; ql_off += 64; qh_off += 32; sc_off += 8;
    }
}

/* dequant.rs:237-245 */
static void get_scale_min_k4(int j, const uint8_t *q, uint8_t *sc, uint8_t *m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (uint8_t)((q[j + 4] & 0x0F) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* dequant.rs:247-270 */
static void dequant_q4_k(const uint8_t *b, float *out) {
    float d = orc_f16_to_f32(rd16(b));
    float mn = orc_f16_to_f32(rd16(b + 2));
    const uint8_t *scales = b + 4, *q = b + 16;
    int y = 0, q_off = 0, is = 0;
    for (int c = 0; c < 4; ++c) {
        uint8_t s, m;
        get_scale_min_k4(is, scales, &s, &m);
        float d1 = d * (float)s, m1 = mn * (float)m;
        get_scale_min_k4(is + 1, scales, &s, &m);
        float d2 = d * (float)s, m2 = mn * (float)m;
        for (int l = 0; l < 32; ++l) {
            out[y + l] = d1 * (float)(q[q_off + l] & 0x0F) - m1;
            out[y + 32 + l] = d2 * (float)(q[q_off + l] >> 4) - m2;
        }
        y += 64; q_off += 32; is += 2;
    }
}

/* dequant.rs:272-302 */
static void dequant_q5_k(const uint8_t *b, float *out) {
    float d = orc_f16_to_f32(rd16(b));
    float mn = orc_f16_to_f32(rd16(b + 2));
    const uint8_t *sc = b + 4, *qh = b + 16, *ql = b + 48;
    int y = 0, ql_off = 0, is = 0;
    uint8_t u1 = 1, u2 = 2;
    for (int c = 0; c < 4; ++c) {
        uint8_t s, m;
        get_scale_min_k4(is, sc, &s, &m);
        float d1 = d * (float)s, m1 = mn * (float)m;
        get_scale_min_k4(is + 1, sc, &s, &m);
        float d2 = d * (float)s, m2 = mn * (float)m;
        for (int l = 0; l < 32; ++l) {
            out[y + l] = d1 * ((float)(ql[ql_off + l] & 0x0F) + ((qh[l] & u1) ? 16.0f : 0.0f)) - m1;
            out[y + 32 + l] = d2 * ((float)(ql[ql_off + l] >> 4) + ((qh[l] & u2) ? 16.0f : 0.0f)) - m2;
        }
        y += 64; ql_off += 32; is += 2;
        u1 = (uint8_t)(u1 << 2); u2 = (uint8_t)(u2 << 2);
    }
}

/* ---- the other block formats (dequant.rs:87-206, 304-445), each element in
 * the reference's operation order: f32 ops, one rounding each (no FMA). */

/* dequant.rs:87-96, Q2_0: 2-bit codes LSB first, v = (code - 1) * d. */
static void dequant_q2_0(const uint8_t *b, float *out) {
    float d = orc_f16_to_f32(rd16(b));
    for (int j = 0; j < 64; ++j) {
        int code = (b[2 + j / 4] >> ((j % 4) * 2)) & 3;
        out[j] = ((float)code - 1.0f) * d;
    }
}

/* dequant.rs:130-136, Q8_1: as Q8_0 with the quants after d and s. */
static void dequant_q8_1(const uint8_t *b, float *out) {
    float d = orc_f16_to_f32(rd16(b));
    for (int j = 0; j < 32; ++j) out[j] = (float)(int8_t)b[4 + j] * d;
}

/* dequant.rs:138-144, Q4_0: (nibble - 8) * d; low nibbles j, high j + 16. */
static void dequant_q4_0(const uint8_t *b, float *out) {
    float d = orc_f16_to_f32(rd16(b));
    for (int j = 0; j < 16; ++j) {
        out[j] = ((float)(b[2 + j] & 0x0F) - 8.0f) * d;
        out[j + 16] = ((float)(b[2 + j] >> 4) - 8.0f) * d;
    }
}

/* dequant.rs:146-153, Q4_1: nibble * d + m. */
static void dequant_q4_1(const uint8_t *b, float *out) {
    float d = orc_f16_to_f32(rd16(b)), m = orc_f16_to_f32(rd16(b + 2));
    for (int j = 0; j < 16; ++j) {
        out[j] = (float)(b[4 + j] & 0x0F) * d + m;
        out[j + 16] = (float)(b[4 + j] >> 4) * d + m;
    }
}

static uint32_t rd32(const uint8_t *b) {
    return (uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16) | ((uint32_t)b[3] << 24);
}

/* dequant.rs:155-166, Q5_0: 5th bit j (low) / j + 16 (high) of the 32-bit qh; (x - 16) * d. */
static void dequant_q5_0(const uint8_t *b, float *out) {
    float d = orc_f16_to_f32(rd16(b));
    uint32_t h = rd32(b + 2);
    const uint8_t *qs = b + 6;
    for (int j = 0; j < 16; ++j) {
        uint32_t x0 = (uint32_t)(qs[j] & 0x0F) | ((h >> j) & 1u) << 4;
        uint32_t x1 = (uint32_t)(qs[j] >> 4) | ((h >> (j + 16)) & 1u) << 4;
        out[j] = ((float)x0 - 16.0f) * d;
        out[j + 16] = ((float)x1 - 16.0f) * d;
    }
}

/* dequant.rs:168-180, Q5_1: x * d + m. */
static void dequant_q5_1(const uint8_t *b, float *out) {
    float d = orc_f16_to_f32(rd16(b)), m = orc_f16_to_f32(rd16(b + 2));
    uint32_t h = rd32(b + 4);
    const uint8_t *qs = b + 8;
    for (int j = 0; j < 16; ++j) {
        uint32_t x0 = (uint32_t)(qs[j] & 0x0F) | ((h >> j) & 1u) << 4;
        uint32_t x1 = (uint32_t)(qs[j] >> 4) | ((h >> (j + 16)) & 1u) << 4;
        out[j] = (float)x0 * d + m;
        out[j + 16] = (float)x1 * d + m;
    }
}

/* The IQ4_NL codebook: the 16 values a 4-bit index selects (IQ4_NL and
 * IQ4_XS; crates/strata-gguf/src/tables.rs KVALUES_IQ4NL). A format constant. */
static const int8_t kIq4nl[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

/* dequant.rs:182-189, IQ4_NL: d * codebook[nibble]. */
static void dequant_iq4_nl(const uint8_t *b, float *out) {
    float d = orc_f16_to_f32(rd16(b));
    for (int j = 0; j < 16; ++j) {
        out[j] = d * (float)kIq4nl[b[2 + j] & 0x0F];
        out[j + 16] = d * (float)kIq4nl[b[2 + j] >> 4];
    }
}

/* dequant.rs:191-206, IQ4_XS: 8 sub-blocks of 32 with 6-bit scales
 * (4 low bits in scales_l, 2 high in scales_h); dl = d * (ls - 32). As
 * strata-gguf writes it, every sub-block reads the same first 16 quant bytes
 * (its qs slice does not advance with the sub-block; ggml's does). */
static void dequant_iq4_xs(const uint8_t *b, float *out) {
    float d = orc_f16_to_f32(rd16(b));
    uint32_t scales_h = rd16(b + 2);
    const uint8_t *scales_l = b + 4, *qs = b + 8;
    for (int ib = 0; ib < 8; ++ib) {
        uint32_t ls = (uint32_t)((scales_l[ib / 2] >> (4 * (ib % 2))) & 0x0F) | ((scales_h >> (2 * ib)) & 3u) << 4;
        float dl = d * ((float)ls - 32.0f);
        for (int j = 0; j < 16; ++j) {
            out[32 * ib + j] = dl * (float)kIq4nl[qs[j] & 0x0F];
            out[32 * ib + j + 16] = dl * (float)kIq4nl[qs[j] >> 4];
        }
    }
}

/* dequant.rs:304-349, Q3_K: 2-bit quants, a high bit per element in hmask
 * (set: +0, clear: -4), 16 6-bit scales unpacked from 12 bytes, d at 108. */
static void dequant_q3_k(const uint8_t *b, float *out) {
    const uint8_t *hm = b, *q = b + 32;
    float d_all = orc_f16_to_f32(rd16(b + 108));
    const uint32_t kmask1 = 0x03030303u, kmask2 = 0x0f0f0f0fu;
    uint32_t aux[4];
    for (int i = 0; i < 3; ++i) aux[i] = rd32(b + 96 + 4 * i);
    uint32_t tmp = aux[2];
    aux[2] = ((aux[0] >> 4) & kmask2) | (((tmp >> 4) & kmask1) << 4);
    aux[3] = ((aux[1] >> 4) & kmask2) | (((tmp >> 6) & kmask1) << 4);
    aux[0] = (aux[0] & kmask2) | ((tmp & kmask1) << 4);
    aux[1] = (aux[1] & kmask2) | (((tmp >> 2) & kmask1) << 4);
    int8_t scales[16];
    for (int i = 0; i < 16; ++i) scales[i] = (int8_t)(uint8_t)(aux[i / 4] >> (8 * (i % 4)));
    int y = 0, is = 0, q_off = 0;
    uint8_t m = 1;
    for (int h = 0; h < 2; ++h) {
        int shift = 0;
        for (int g = 0; g < 4; ++g) {
            float dl = d_all * (float)(int8_t)(scales[is] - 32);
            ++is;
            for (int l = 0; l < 16; ++l)
                out[y + l] = dl * ((float)(int8_t)((q[q_off + l] >> shift) & 3) - ((hm[l] & m) ? 0.0f : 4.0f));
            dl = d_all * (float)(int8_t)(scales[is] - 32);
            ++is;
            for (int l = 0; l < 16; ++l)
                out[y + 16 + l] =
                    dl * ((float)(int8_t)((q[q_off + l + 16] >> shift) & 3) - ((hm[l + 16] & m) ? 0.0f : 4.0f));
            y += 32;
            shift += 2;
            m = (uint8_t)(m << 1);
        }
        q_off += 32;
    }
}

/* dequant.rs:351-380, Q2_K (strata-gguf's layout: d, dmin, scales[16],
 * qs[64]); (s, m) of sub-blocks is, is + 1 via get_scale_min_k4. */
static void dequant_q2_k(const uint8_t *b, float *out) {
    float d = orc_f16_to_f32(rd16(b)), mn = orc_f16_to_f32(rd16(b + 2));
    const uint8_t *sc = b + 4, *q = b + 20;
    int y = 0, q_off = 0, is = 0;
    for (int g = 0; g < 2; ++g) {
        uint8_t s, m;
        get_scale_min_k4(is, sc, &s, &m);
        float d1 = d * (float)s, m1 = mn * (float)m;
        get_scale_min_k4(is + 1, sc, &s, &m);
        float d2 = d * (float)s, m2 = mn * (float)m;
        for (int l = 0; l < 32; ++l) {
            out[y + l] = d1 * (float)(q[q_off + l] & 3) - m1;
            out[y + l + 32] = d2 * (float)((q[q_off + l] >> 2) & 3) - m2;
            out[y + l + 64] = d1 * (float)((q[q_off + l] >> 4) & 3) - m1;
            out[y + l + 96] = d2 * (float)((q[q_off + l] >> 6) & 3) - m2;
        }
        y += 128;
        q_off += 32;
        is += 2;
    }
}

/* E2M1 (FP4) codes in half units: magnitudes 0, 0.5, 1, 1.5, 2, 3, 4, 6 from
 * the format's 2-bit exponent and 1-bit mantissa, doubled; bit 3 the sign
 * (the values of strata-gguf's KVALUES_FP4, derived here from the format). */
static float fp4_half_units(uint32_t code) {
    uint32_t e = (code >> 1) & 3u, mbit = code & 1u;
    float mag = e == 0 ? (float)mbit : (float)((2u + mbit) << (e - 1));  /* x2: 0,1 | 2,3 | 4,6 | 8,12 */
    return (code & 8u) && mag != 0.0f ? -mag : mag;  /* code 8 is +0, as the table's 0 */
}

/* dequant.rs:386-395: E8M0 -> 2^(e-127); 0 is zero, 0xFF NaN. */
static float e8m0_to_f32(uint8_t e) {
    if (e == 0) return 0.0f;
    if (e == 0xFF) return bits_f32(0x7FC00000u);
    return bits_f32((uint32_t)e << 23);
}

/* dequant.rs:397-413: UE4M3 (no inf; 0x7F / 0xFF NaN). */
static float ue4m3_to_f32(uint8_t e) {
    int sign = (e & 0x80) != 0, ex = (e >> 3) & 0xF, man = e & 0x7;
    float v;
    if (ex == 0) v = (float)man / 8.0f * ldexpf(1.0f, -6);
    else if (ex == 15 && man == 7) v = bits_f32(0x7FC00000u);
    else v = ldexpf(1.0f, ex - 7) * (1.0f + (float)man / 8.0f);
    return sign ? -v : v;
}

/* dequant.rs:415-424, MXFP4: d * fp4 * 0.5; low nibble j, high j + 16. */
static void dequant_mxfp4(const uint8_t *b, float *out) {
    float d = e8m0_to_f32(b[0]);
    for (int j = 0; j < 16; ++j) {
        out[j] = d * fp4_half_units(b[1 + j] & 0x0F) * 0.5f;
        out[j + 16] = d * fp4_half_units(b[1 + j] >> 4) * 0.5f;
    }
}

/* dequant.rs:426-444, NVFP4: four sub-blocks of 16 with a UE4M3 scale each;
 * value j in the low nibble of qs[8s + j], j + 8 in the high one. */
static void dequant_nvfp4(const uint8_t *b, float *out) {
    for (int s = 0; s < 4; ++s) {
        float ds = ue4m3_to_f32(b[s]);
        for (int j = 0; j < 8; ++j) {
            out[16 * s + j] = ds * fp4_half_units(b[4 + 8 * s + j] & 0x0F) * 0.5f;
            out[16 * s + j + 8] = ds * fp4_half_units(b[4 + 8 * s + j] >> 4) * 0.5f;
        }
    }
}

static int dequant_block(uint32_t q, const uint8_t *b, float *out) {
    switch (q) {
    case ORC_F32: memcpy(out, b, 4); return ORC_OK;
    case ORC_F16: out[0] = orc_f16_to_f32(rd16(b)); return ORC_OK;
    case ORC_BF16: out[0] = bits_f32((uint32_t)rd16(b) << 16); return ORC_OK;
    case ORC_Q8_0: dequant_q8_0(b, out); return ORC_OK;
    case ORC_Q4_K: dequant_q4_k(b, out); return ORC_OK;
    case ORC_Q5_K: dequant_q5_k(b, out); return ORC_OK;
    case ORC_Q6_K: dequant_q6_k(b, out); return ORC_OK;
    case ORC_Q2_0: dequant_q2_0(b, out); return ORC_OK;
    case ORC_Q8_1: dequant_q8_1(b, out); return ORC_OK;
    case ORC_Q4_0: dequant_q4_0(b, out); return ORC_OK;
    case ORC_Q4_1: dequant_q4_1(b, out); return ORC_OK;
    case ORC_Q5_0: dequant_q5_0(b, out); return ORC_OK;
    case ORC_Q5_1: dequant_q5_1(b, out); return ORC_OK;
    case ORC_IQ4_NL: dequant_iq4_nl(b, out); return ORC_OK;
    case ORC_IQ4_XS: dequant_iq4_xs(b, out); return ORC_OK;
    case ORC_Q3_K: dequant_q3_k(b, out); return ORC_OK;
    case ORC_Q2_K: dequant_q2_k(b, out); return ORC_OK;
    case ORC_MXFP4: dequant_mxfp4(b, out); return ORC_OK;
    case ORC_NVFP4: dequant_nvfp4(b, out); return ORC_OK;
    default: return ORC_ERR_UNSUPPORTED;
    }
}

/* dequant.rs:45-61: Err(Truncated) when n is not a whole number of blocks or
 * the bytes are short. */
int orc_dequantize_row(uint32_t q, const uint8_t *block, size_t block_len, float *out, int64_t n) {
    int64_t bs = orc_block_size(q), ts = orc_type_size(q);
    if (bs == 0) return ORC_ERR_UNSUPPORTED;
    int64_t nb = (n + bs - 1) / bs;
    if (n % bs != 0 || (int64_t)block_len < nb * ts) return ORC_ERR_TRUNCATED;
    for (int64_t i = 0; i < nb; ++i) {
        int rc = dequant_block(q, block + i * ts, out + i * bs);
        if (rc) return rc;
    }
    return ORC_OK;
}

/* ------------------------------------------------------------------ gemv */

/* ops.rs:14-28 for rows [r0, r1): dequantize the row, f64 dot, round once. */
static int gemv_range(uint32_t q, const uint8_t *w, int64_t cols, const float *x, float *y,
                      int64_t r0, int64_t r1, float *scratch) {
    int64_t rb = orc_byte_size(q, cols);
    for (int64_t r = r0; r < r1; ++r) {
        int rc = orc_dequantize_row(q, w + r * rb, (size_t)rb, scratch, cols);
        if (rc) return rc;
        double acc = 0.0;
        for (int64_t c = 0; c < cols; ++c) acc += (double)scratch[c] * (double)x[c];
        y[r - r0] = (float)acc;
    }
    return ORC_OK;
}

static int check_dense(uint32_t q, size_t w_len, int64_t rows, int64_t cols) {
    if (orc_block_size(q) == 0) return ORC_ERR_UNSUPPORTED;
    if (rows < 0 || cols < 0) return ORC_ERR_INVALID;
    if ((int64_t)w_len < rows * orc_byte_size(q, cols)) return ORC_ERR_TRUNCATED;
    if (cols % orc_block_size(q) != 0) return ORC_ERR_TRUNCATED;
    return ORC_OK;
}

int orc_gemv(uint32_t q, const uint8_t *w, size_t w_len, int64_t rows, int64_t cols,
             const float *x, float *y) {
    int rc = check_dense(q, w_len, rows, cols);
    if (rc) return rc;
    float *scratch = (float *)malloc(sizeof(float) * (size_t)(cols > 0 ? cols : 1));
    if (!scratch) return ORC_ERR_INVALID;
    rc = gemv_range(q, w, cols, x, y, 0, rows, scratch);
    free(scratch);
    return rc;
}

typedef struct {
    uint32_t q; const uint8_t *w; int64_t cols; const float *x; float *y;
    int64_t r0, r1; int rc;
} gemv_job;

static void *gemv_worker(void *p) {
    gemv_job *j = (gemv_job *)p;
    float *scratch = (float *)malloc(sizeof(float) * (size_t)(j->cols > 0 ? j->cols : 1));
    j->rc = scratch ? gemv_range(j->q, j->w, j->cols, j->x, j->y, j->r0, j->r1, scratch) : ORC_ERR_INVALID;
    free(scratch);
    return NULL;
}

/* rows [row0, row_end) of one column, split over `threads` pthreads */
static int gemv_rows_par(uint32_t q, const uint8_t *w, int64_t cols, const float *x, float *y,
                         int64_t row0, int64_t row_end, int threads) {
    int64_t n = row_end - row0;
    if (threads < 1) threads = 1;
    if (threads > n) threads = n > 0 ? (int)n : 1;
    if (threads == 1) {
        gemv_job j = {q, w, cols, x, y, row0, row_end, 0};
        gemv_worker(&j);
        return j.rc;
    }
    gemv_job *jobs = (gemv_job *)calloc((size_t)threads, sizeof(gemv_job));
    pthread_t *tid = (pthread_t *)calloc((size_t)threads, sizeof(pthread_t));
    int rc = ORC_OK;
    for (int t = 0; t < threads; ++t) {
        int64_t a = row0 + n * t / threads, b = row0 + n * (t + 1) / threads;
        jobs[t] = (gemv_job){q, w, cols, x, y + (a - row0), a, b, 0};
        pthread_create(&tid[t], NULL, gemv_worker, &jobs[t]);
    }
    for (int t = 0; t < threads; ++t) {
        pthread_join(tid[t], NULL);
        if (jobs[t].rc) rc = jobs[t].rc;
    }
    free(jobs); free(tid);
    return rc;
}

int orc_gemv_batch(uint32_t q, const uint8_t *w, size_t w_len, int64_t rows, int64_t cols,
                   const float *x, float *y, int64_t batch, int threads) {
    int rc = check_dense(q, w_len, rows, cols);
    if (rc) return rc;
    for (int64_t b = 0; b < batch; ++b) {
        rc = gemv_rows_par(q, w, cols, x + b * cols, y + b * rows, 0, rows, threads);
        if (rc) return rc;
    }
    return ORC_OK;
}

int orc_gemv_rows(uint32_t q, const uint8_t *w, size_t w_len, int64_t rows, int64_t cols,
                  const float *x, float *y, int64_t row0, int64_t row_end, int threads) {
    int rc = check_dense(q, w_len, rows, cols);
    if (rc) return rc;
    if (row0 < 0 || row_end > rows || row0 > row_end) return ORC_ERR_INVALID;
    return gemv_rows_par(q, w, cols, x, y, row0, row_end, threads);
}

/* ops.rs:169-195: y[c] = sum_i x[i] * W_e[i][c], f64 accumulators, rows with
 * x[i] == 0 skipped (they never touch the sum). */
int orc_expert_gemv(uint32_t q, const uint8_t *w, size_t w_len, int64_t n_expert, int64_t rows,
                    int64_t cols, int64_t e, const float *x, float *y) {
    if (orc_block_size(q) == 0) return ORC_ERR_UNSUPPORTED;
    int64_t rb = orc_byte_size(q, cols);
    if (e < 0 || e >= n_expert) return ORC_ERR_INVALID;
    if ((int64_t)w_len < n_expert * rows * rb || cols % orc_block_size(q) != 0) return ORC_ERR_TRUNCATED;
    double *acc = (double *)calloc((size_t)(cols > 0 ? cols : 1), sizeof(double));
    float *row = (float *)malloc(sizeof(float) * (size_t)(cols > 0 ? cols : 1));
    int rc = ORC_OK;
    const uint8_t *base = w + e * rows * rb;
    for (int64_t i = 0; i < rows && rc == ORC_OK; ++i) {
        double xi = (double)x[i];
        if (xi == 0.0) continue;
        rc = orc_dequantize_row(q, base + i * rb, (size_t)rb, row, cols);
        for (int64_t c = 0; c < cols && rc == ORC_OK; ++c) acc[c] += xi * (double)row[c];
    }
    for (int64_t c = 0; c < cols && rc == ORC_OK; ++c) y[c] = (float)acc[c];
    free(acc); free(row);
    return rc;
}

/* ------------------------------------------------------------------- MoE */

float orc_silu(float x) { return x / (1.0f + expf(-x)); }
float orc_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

/* moe.rs:57-91 */
int orc_moe_route_logits(float *logits, int64_t n_expert, int64_t top_k, int64_t *ids,
                         float *weights) {
    if (n_expert <= 0 || top_k <= 0) return ORC_ERR_INVALID;
    float mx = -INFINITY;
    for (int64_t i = 0; i < n_expert; ++i) mx = fmaxf(mx, logits[i]);
    double sum = 0.0;
    for (int64_t i = 0; i < n_expert; ++i) {
        logits[i] = expf(logits[i] - mx);
        sum += (double)logits[i];
    }
    float inv = (float)(1.0 / sum);
    for (int64_t i = 0; i < n_expert; ++i) logits[i] *= inv;
    int64_t k = top_k < n_expert ? top_k : n_expert;
    /* The k first of the total order (prob desc, index asc); selection by
     * repeated scans keeps this obviously equal to select_nth_unstable_by. */
    unsigned char *taken = (unsigned char *)calloc((size_t)n_expert, 1);
    for (int64_t s = 0; s < k; ++s) {
        int64_t best = -1;
        for (int64_t i = 0; i < n_expert; ++i) {
            if (taken[i]) continue;
            if (best < 0 || logits[i] > logits[best]) best = i;
        }
        taken[best] = 1;
    }
    int64_t n = 0;
    for (int64_t i = 0; i < n_expert; ++i)
        if (taken[i]) ids[n++] = i; /* ascending id order */
    free(taken);
    double ws = 0.0;
    for (int64_t j = 0; j < k; ++j) {
        weights[j] = logits[ids[j]];
        ws += (double)weights[j];
    }
    double s = ws > ldexp(1.0, -14) ? ws : ldexp(1.0, -14);
    for (int64_t j = 0; j < k; ++j) weights[j] = (float)((double)weights[j] / s);
    for (int64_t j = k; j < top_k; ++j) { ids[j] = -1; weights[j] = 0.0f; }
    return ORC_OK;
}

int orc_moe_route(const orc_moe_weights *L, const float *x, int64_t *ids, float *weights) {
    float *xb = (float *)malloc(sizeof(float) * (size_t)L->n_embd);
    float *logits = (float *)malloc(sizeof(float) * (size_t)L->n_expert);
    for (int64_t i = 0; i < L->n_embd; ++i) xb[i] = orc_bf16_round(x[i]);
    int rc = orc_gemv(L->quant_router, L->router, L->router_len, L->n_expert, L->n_embd, xb, logits);
    if (rc == ORC_OK) rc = orc_moe_route_logits(logits, L->n_expert, L->top_k, ids, weights);
    free(xb); free(logits);
    return rc;
}

/* moe.rs:97-144 */
int orc_moe_combine(const orc_moe_weights *L, const float *x, const int64_t *ids,
                    const float *weights, float *out) {
    int64_t n = L->n_embd, ff = L->n_ff > L->n_ff_shexp ? L->n_ff : L->n_ff_shexp;
    float *h = (float *)malloc(sizeof(float) * (size_t)ff);
    float *part = (float *)malloc(sizeof(float) * (size_t)ff);
    float *down = (float *)malloc(sizeof(float) * (size_t)n);
    int rc = ORC_OK;
    for (int64_t i = 0; i < n; ++i) out[i] = 0.0f;
    int64_t k = L->top_k < L->n_expert ? L->top_k : L->n_expert;
    for (int64_t j = 0; j < k && rc == ORC_OK; ++j) {
        float w = weights[j];
        int64_t e = ids[j];
        if (w == 0.0f) continue;
        rc = orc_expert_gemv(L->quant_gate_exps, L->gate_exps, L->gate_exps_len, L->n_expert, n, L->n_ff, e, x, h);
        if (!rc) rc = orc_expert_gemv(L->quant_up_exps, L->up_exps, L->up_exps_len, L->n_expert, n, L->n_ff, e, x, part);
        if (rc) break;
        for (int64_t f = 0; f < L->n_ff; ++f) h[f] = orc_silu(h[f]) * part[f];
        rc = orc_expert_gemv(L->quant_down_exps, L->down_exps, L->down_exps_len, L->n_expert, L->n_ff, n, e, h, down);
        if (rc) break;
        for (int64_t i = 0; i < n; ++i) out[i] += w * down[i];
    }
    if (rc == ORC_OK && L->gate_shexp) {
        int64_t fs = L->n_ff_shexp;
        rc = orc_gemv(L->quant_gate_shexp, L->gate_shexp, L->gate_shexp_len, fs, n, x, h);
        if (!rc) rc = orc_gemv(L->quant_up_shexp, L->up_shexp, L->up_shexp_len, fs, n, x, part);
        if (!rc) {
            for (int64_t f = 0; f < fs; ++f) h[f] = orc_silu(h[f]) * part[f];
            rc = orc_gemv(L->quant_down_shexp, L->down_shexp, L->down_shexp_len, n, fs, h, down);
        }
        float sgate = 0.0f;
        if (!rc) rc = orc_gemv(L->quant_gate_inp_shexp, L->gate_inp_shexp, L->gate_inp_shexp_len, 1, n, x, &sgate);
        if (!rc) {
            float g = orc_sigmoid(sgate);
            for (int64_t i = 0; i < n; ++i) out[i] += g * down[i];
        }
    }
    free(h); free(part); free(down);
    return rc;
}

typedef struct {
    const orc_moe_weights *L; const float *x; const float *logits;
    float *out; int64_t *ids; float *weights; int64_t t0, t1; int rc;
} moe_job;

static void *moe_worker(void *p) {
    moe_job *j = (moe_job *)p;
    const orc_moe_weights *L = j->L;
    int64_t k = L->top_k;
    int64_t *ids = (int64_t *)malloc(sizeof(int64_t) * (size_t)k);
    float *w = (float *)malloc(sizeof(float) * (size_t)k);
    float *lg = (float *)malloc(sizeof(float) * (size_t)L->n_expert);
    j->rc = ORC_OK;
    for (int64_t t = j->t0; t < j->t1 && j->rc == ORC_OK; ++t) {
        const float *xt = j->x + t * L->n_embd;
        if (j->logits) {
            memcpy(lg, j->logits + t * L->n_expert, sizeof(float) * (size_t)L->n_expert);
            j->rc = orc_moe_route_logits(lg, L->n_expert, k, ids, w);
        } else {
            j->rc = orc_moe_route(L, xt, ids, w);
        }
        if (j->rc) break;
        if (j->ids) memcpy(j->ids + t * k, ids, sizeof(int64_t) * (size_t)k);
        if (j->weights) memcpy(j->weights + t * k, w, sizeof(float) * (size_t)k);
        j->rc = orc_moe_combine(L, xt, ids, w, j->out + t * L->n_embd);
    }
    free(ids); free(w); free(lg);
    return NULL;
}

int orc_moe_layer(const orc_moe_weights *L, const float *x, const float *logits, int64_t tokens,
                  float *out, int64_t *ids, float *weights, int threads) {
    if (tokens < 0 || !L) return ORC_ERR_INVALID;
    if (threads < 1) threads = 1;
    if (threads > tokens) threads = tokens > 0 ? (int)tokens : 1;
    moe_job *jobs = (moe_job *)calloc((size_t)threads, sizeof(moe_job));
    pthread_t *tid = (pthread_t *)calloc((size_t)threads, sizeof(pthread_t));
    int rc = ORC_OK;
    for (int t = 0; t < threads; ++t) {
        jobs[t] = (moe_job){L, x, logits, out, ids, weights, tokens * t / threads, tokens * (t + 1) / threads, 0};
        if (threads == 1) moe_worker(&jobs[t]);
        else pthread_create(&tid[t], NULL, moe_worker, &jobs[t]);
    }
    for (int t = 0; t < threads; ++t) {
        if (threads > 1) pthread_join(tid[t], NULL);
        if (jobs[t].rc) rc = jobs[t].rc;
    }
    free(jobs); free(tid);
    return rc;
}

/* ---------------------------------------------------------------- elementwise ops */

/* ops::rms_norm (ops.rs:45-56): sequential f64 sum of squares, divided by n;
 * scale = 1 / sqrt(ss + eps); x = f32((x * scale) * w) in f64. */
void orc_rms_norm(float *x, const float *w, int64_t n, double eps) {
    double ss = 0.0;
    for (int64_t i = 0; i < n; ++i) ss += (double)x[i] * (double)x[i];
    ss /= (double)n;
    const double scale = 1.0 / sqrt(ss + eps);
    for (int64_t i = 0; i < n; ++i) x[i] = (float)((double)x[i] * scale * (double)w[i]);
}

/* ops::l2_norm (ops.rs:71-81): inv = 1 / sqrt(sum x^2 + eps), x = f32(x * inv). */
void orc_l2_norm(float *head, int64_t n, double eps) {
    double ss = 0.0;
    for (int64_t i = 0; i < n; ++i) ss += (double)head[i] * (double)head[i];
    const double inv = 1.0 / sqrt(ss + eps);
    for (int64_t i = 0; i < n; ++i) head[i] = (float)((double)head[i] * inv);
}

/* ops::softmax (ops.rs:107-119): f32 max, v = expf(v - max) in f32, f64 sum,
 * v = f32(v * (1 / sum)). */
void orc_softmax(float *xs, int64_t n) {
    float mx = -INFINITY;
    for (int64_t i = 0; i < n; ++i) mx = xs[i] > mx ? xs[i] : mx;
    double sum = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        xs[i] = expf(xs[i] - mx);
        sum += (double)xs[i];
    }
    const double inv = 1.0 / sum;
    for (int64_t i = 0; i < n; ++i) xs[i] = (float)((double)xs[i] * inv);
}

/* ops::rope_neox (ops.rs:121-140): n_rot clamped to the head and made even;
 * pair (i, i + half) rotated by angle = base^(-2i/n_rot) * pos in f64. */
void orc_rope_neox(float *head, int64_t len, int64_t pos, int64_t n_rot, int64_t head_dim, double freq_base) {
    int64_t nr = n_rot < head_dim ? n_rot : head_dim;
    nr = nr < len ? nr : len;
    nr &= ~(int64_t)1;
    const int64_t half = nr / 2;
    for (int64_t i = 0; i < half; ++i) {
        const double theta = pow(freq_base, -2.0 * (double)i / (double)nr);
        const double angle = theta * (double)pos;
        const double s = sin(angle), c = cos(angle);
        const double a = head[i], b = head[i + half];
        head[i] = (float)(a * c - b * s);
        head[i + half] = (float)(a * s + b * c);
    }
}

/* ops::add_into (ops.rs:164-168): out += a in f32. */
void orc_add(float *out, const float *a, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] += a[i];
}

/* ---- test support (not a restatement): where the C library's expf, which
 * the reference's f32::exp is, is not correctly rounded. The correctly
 * rounded value is the x87 long double expl (64-bit significand) rounded to
 * f32. Inputs are scanned upward from lo to hi (both finite, lo <= hi, same
 * sign). */
static uint32_t orc_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float orc_float(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static float orc_expf_cr(float x) { return (float)expl((long double)x); }
static float orc_next_up(float x) {
    const uint32_t u = orc_bits(x);
    if (x == 0.0f) return orc_float(1u);
    return orc_float(x > 0.0f ? u + 1u : u - 1u);
}

/* Inputs x in [lo, hi] where expf(x) differs from the correctly rounded value;
 * at most cap of them into out. Returns the number written. */
int64_t orc_expf_misrounded(float lo, float hi, float *out, int64_t cap) {
    int64_t n = 0;
    for (float x = lo; x <= hi && n < cap; x = orc_next_up(x))
        if (orc_bits(expf(x)) != orc_bits(orc_expf_cr(x))) out[n++] = x;
    return n;
}

/* Pairs x1 < x2 in [lo, hi], at most 4 floats apart, where expf(x1) ==
 * expf(x2) but the correctly rounded values differ (so an ordering by the
 * correctly rounded exp separates what expf ties); at most cap pairs into
 * out[2 i], out[2 i + 1]. Returns the number of pairs written. */
int64_t orc_expf_tie_pairs(float lo, float hi, float *out, int64_t cap) {
    int64_t n = 0;
    for (float x = lo; x <= hi && n < cap; x = orc_next_up(x)) {
        if (orc_bits(expf(x)) == orc_bits(orc_expf_cr(x))) continue;  /* one of the pair is misrounded */
        /* neighbours on both sides */
        float y = x;
        for (int s = 1; s <= 4; ++s) {
            y = orc_next_up(y);
            if (orc_bits(expf(y)) == orc_bits(expf(x)) && orc_bits(orc_expf_cr(y)) != orc_bits(orc_expf_cr(x))) {
                out[2 * n] = x;
                out[2 * n + 1] = y;
                if (++n >= cap) return n;
                break;
            }
        }
        float w = x;
        for (int s = 1; s <= 4 && n < cap; ++s) {
            const uint32_t u = orc_bits(w);
            w = orc_float(x > 0.0f ? u - 1u : u + 1u);  /* next down */
            if (orc_bits(expf(w)) == orc_bits(expf(x)) && orc_bits(orc_expf_cr(w)) != orc_bits(orc_expf_cr(x))) {
                out[2 * n] = w;
                out[2 * n + 1] = x;
                ++n;
                break;
            }
        }
    }
    return n;
}
