// gemv_mma.cu — Q4_K / Q5_K decode GEMV (batch 1..8) on the tensor cores.
//
// Same product as ops::gemv (crates/strata-core/src/ops.rs:14-28), restated so
// that the tensor cores do every multiply-add:
//
//   sum_k W[n][k] x[k] = sum_blocks ( d * sum_k (sc_j q_k) x_k  -  dmin * sum_k m_j x_k )
//
// * A operand (fp16): sc_j * q_k is an integer <= 63*15 (Q4_K) or 63*31 (Q5_K),
//   so it is exact in fp16. It is built in registers straight from the packed
//   quants: a LOP3 drops two nibbles into the mantissas of 1024.0 (or 1024 +
//   16 q for a high nibble) and one HFMA2 with per-sub-block constants turns
//   that into sc*q, exactly (the fused multiply-add rounds once, and the
//   result is a small integer).
// * MMA rows 0..7 are 8 weight rows; rows 8..15 carry the same rows' 6-bit
//   mins m_j, so D[8+r] = sum_k m_j(k) x_k comes out of the same instruction.
// * B operand (fp16): each activation column is split into two fp16 limbs,
//   x*s = hi + lo * 2^-11 (22 significant bits), with a power-of-two scale s
//   per (column, block) chosen from the block's max |x|, so fp16 can neither
//   overflow nor lose the small entries. Columns are (batch, limb) pairs.
// * D (fp32) accumulates one 256-weight block (16 mma.sync m16n8k16), then is
//   folded into fp32 accumulators with d / dmin / s. The products are exact
//   and the sums are fp32, which is what the 1e-3 tolerance needs.
//
// Work split: a CTA owns 8*G rows; its warps split the K blocks; partial sums
// meet in shared memory. A prologue kernel writes the activation limbs in the
// order the B fragments are read (one 8-byte load per lane per mma).
#include <cuda_fp16.h>

#include "kernels.cuh"
#include "quant.cuh"

namespace strata {

namespace {

constexpr int kMmaWarps = 8;

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

__device__ __forceinline__ void mma16816(float d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------- prologue
//
// XF layout: [blk][s = sub-block 0..7][i = word 0..7][n = column 0..ncols)
// of uint2 {b0, b1}, where for e = 256 blk + 32 s + 4 i
//   b0 = half2(v[e], v[e+2]), b1 = half2(v[e+1], v[e+3]),
// v = limb (n & 1) of batch row (n >> 1) of x, scaled by XS^-1.
// XS layout: [batch][blk] float: the power of two that undoes the scaling.
__global__ void prep_x_limbs_kernel(const float* __restrict__ X, int64_t K, int batch, uint2* __restrict__ XF,
                                    float* __restrict__ XS) {
    const int nblk = (int)(K / 256);
    const int lane = threadIdx.x & 31;
    const int64_t wid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (wid >= (int64_t)nblk * batch) return;
    const int b = (int)(wid % batch);
    const int blk = (int)(wid / batch);
    // lane covers elements 8 lane .. 8 lane + 7 of the block: sub-block lane/4, words 2(lane%4), +1
    const float* xp = X + (int64_t)b * K + (int64_t)blk * 256 + 8 * lane;
    float4 v0 = __ldg(reinterpret_cast<const float4*>(xp));
    float4 v1 = __ldg(reinterpret_cast<const float4*>(xp) + 1);
    float mx = fmaxf(fmaxf(fmaxf(fabsf(v0.x), fabsf(v0.y)), fmaxf(fabsf(v0.z), fabsf(v0.w))),
                     fmaxf(fmaxf(fabsf(v1.x), fabsf(v1.y)), fmaxf(fabsf(v1.z), fabsf(v1.w))));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    // scale so that max |x| * s lies in [0.5, 1): s = 2^(126 - exp(max))
    int e = (int)((__float_as_uint(mx) >> 23) & 0xFF);
    if (e == 0 || e == 0xFF) e = 127;       // zero / denormal / non-finite: no scaling
    int se = 253 - e;                        // biased exponent of s
    se = se < 1 ? 1 : (se > 254 ? 254 : se);
    const float s = __uint_as_float((uint32_t)se << 23);
    const float inv = __uint_as_float((uint32_t)(254 - se) << 23);
    if (lane == 0) XS[(int64_t)b * nblk + blk] = inv;
    float v[8] = {v0.x * s, v0.y * s, v0.z * s, v0.w * s, v1.x * s, v1.y * s, v1.z * s, v1.w * s};
    __half hi[8], lo[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        hi[j] = __float2half_rn(v[j]);
        lo[j] = __float2half_rn((v[j] - __half2float(hi[j])) * 2048.0f);
    }
    const int ncols = 2 * batch;
    const int s_blk = lane >> 2;
#pragma unroll
    for (int w = 0; w < 2; ++w) {
        const int i = 2 * (lane & 3) + w;
        const int o = 4 * w;
        uint2 fh, fl;
        fh.x = h2u(__halves2half2(hi[o + 0], hi[o + 2]));
        fh.y = h2u(__halves2half2(hi[o + 1], hi[o + 3]));
        fl.x = h2u(__halves2half2(lo[o + 0], lo[o + 2]));
        fl.y = h2u(__halves2half2(lo[o + 1], lo[o + 3]));
        uint2* dst = XF + (((int64_t)blk * 8 + s_blk) * 8 + i) * ncols + 2 * b;
        dst[0] = fh;
        dst[1] = fl;
    }
}

// ---------------------------------------------------------------- main kernel

struct BlockRegs {
    uint4 hd;      // d, dmin, scales[12]
    uint4 qa, qb;  // this lane's 32 quant bytes (chunk t of the block)
    uint4 ha, hb;  // Q5_K: the block's 32 qh bytes
};

template <uint32_t Q>
__device__ __forceinline__ void load_block(const uint8_t* __restrict__ blk, int t, BlockRegs& r) {
    r.hd = __ldg(reinterpret_cast<const uint4*>(blk));
    if constexpr (Q == kQ4_K) {
        const uint4* q = reinterpret_cast<const uint4*>(blk + 16 + 32 * t);
        r.qa = __ldg(q);
        r.qb = __ldg(q + 1);
    } else {
        const uint4* q = reinterpret_cast<const uint4*>(blk + 48 + 32 * t);
        r.qa = __ldg(q);
        r.qb = __ldg(q + 1);
        const uint4* h = reinterpret_cast<const uint4*>(blk + 16);
        r.ha = __ldg(h);
        r.hb = __ldg(h + 1);
    }
}

__device__ __forceinline__ uint32_t word_of(const uint4& a, const uint4& b, int i) {
    switch (i) {
    case 0: return a.x; case 1: return a.y; case 2: return a.z; case 3: return a.w;
    case 4: return b.x; case 5: return b.y; case 6: return b.z; default: return b.w;
    }
}

template <uint32_t Q, int G, int NT>
__global__ void __launch_bounds__(kMmaWarps * 32)
gemv_kq_mma_kernel(const uint8_t* __restrict__ W, int64_t row_bytes, int64_t N, int nblk,
                   const uint2* __restrict__ XF, const float* __restrict__ XS, int batch,
                   float* __restrict__ Y) {
    constexpr int BB = block_bytes(Q);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int ncols = 2 * batch;
    const int64_t row0 = (int64_t)blockIdx.x * (8 * G);
    const int kb0 = warp * nblk / kMmaWarps, kb1 = (warp + 1) * nblk / kMmaWarps;

    const uint8_t* rowp[G];
#pragma unroll
    for (int gi = 0; gi < G; ++gi) {
        int64_t row = row0 + 8 * gi + g;
        row = row < N ? row : N - 1;
        rowp[gi] = W + row * row_bytes;
    }
    // per-lane constants: PRMT selector for bytes 2(t&1), 2(t&1)+1 under 0x64
    const uint32_t sel = (4u << 12) | ((uint32_t)(2 * (t & 1) + 1) << 8) | (4u << 4) | (uint32_t)(2 * (t & 1));
    const __half2 k1024 = __float2half2_rn(1024.0f);
    const __half2 kneg1024 = __float2half2_rn(-1024.0f);
    const __half2 k1_16 = __float2half2_rn(0.0625f);
    const __half2 kneg64 = __float2half2_rn(-64.0f);

    float acc[G][NT][2];
#pragma unroll
    for (int gi = 0; gi < G; ++gi)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) acc[gi][nt][0] = acc[gi][nt][1] = 0.0f;

    BlockRegs cur[G], nxt[G];
    if (kb0 < kb1) {
#pragma unroll
        for (int gi = 0; gi < G; ++gi) load_block<Q>(rowp[gi] + (int64_t)kb0 * BB, t, cur[gi]);
    }
    for (int kb = kb0; kb < kb1; ++kb) {
        if (kb + 1 < kb1) {
#pragma unroll
            for (int gi = 0; gi < G; ++gi) load_block<Q>(rowp[gi] + (int64_t)(kb + 1) * BB, t, nxt[gi]);
        }
        // activation fragments of this block: sub-blocks 2t (low) and 2t+1 (high), words 0..7
        const uint2* xf = XF + (int64_t)kb * 64 * ncols;
        float d_acc[G][NT][4];
#pragma unroll
        for (int gi = 0; gi < G; ++gi)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int c = 0; c < 4; ++c) d_acc[gi][nt][c] = 0.0f;

        // per-row, per-lane scale constants
        __half2 sAA[G], cA[G], sB16[G], cB[G], mAA[G], mBB[G];
        float dd[G], dm[G];
#pragma unroll
        for (int gi = 0; gi < G; ++gi) {
            const uint4 hd = cur[gi].hd;
            dd[gi] = f16_bits_to_f32(hd.x & 0xFFFFu);
            dm[gi] = f16_bits_to_f32(hd.x >> 16);
            uint32_t sl, sh, ml, mh;
            scales_k4_packed(hd.y, hd.z, hd.w, sl, sh, ml, mh);
            const uint32_t sw = t < 2 ? sl : sh, mw = t < 2 ? ml : mh;
            const __half2 sAB = __hsub2(u2h(__byte_perm(sw, 0x00006464u, sel)), k1024);
            const __half2 mAB = __hsub2(u2h(__byte_perm(mw, 0x00006464u, sel)), k1024);
            sAA[gi] = __low2half2(sAB);
            const __half2 sBB = __high2half2(sAB);
            cA[gi] = __hmul2(sAA[gi], kneg1024);
            sB16[gi] = __hmul2(sBB, k1_16);
            cB[gi] = __hmul2(sBB, kneg64);
            mAA[gi] = __low2half2(mAB);
            mBB[gi] = __high2half2(mAB);
        }

#pragma unroll
        for (int i = 0; i < 8; ++i) {
            uint2 blo[NT], bhi[NT];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int n = 8 * nt + g;
                if (n < ncols) {
                    blo[nt] = __ldg(xf + ((2 * t) * 8 + i) * ncols + n);
                    bhi[nt] = __ldg(xf + ((2 * t + 1) * 8 + i) * ncols + n);
                } else {
                    blo[nt] = make_uint2(0u, 0u);
                    bhi[nt] = make_uint2(0u, 0u);
                }
            }
#pragma unroll
            for (int gi = 0; gi < G; ++gi) {
                const uint32_t w = word_of(cur[gi].qa, cur[gi].qb, i);
                const uint32_t w8 = w >> 8;
                uint32_t lo0 = (w & 0x000F000Fu) | 0x64006400u;
                uint32_t lo1 = (w8 & 0x000F000Fu) | 0x64006400u;
                uint32_t hi0 = (w & 0x00F000F0u) | 0x64006400u;
                uint32_t hi1 = (w8 & 0x00F000F0u) | 0x64006400u;
                if constexpr (Q == kQ5_K) {
                    // qh byte l holds the 5th bit of element l of every sub-block:
                    // bit 2t for this lane's low sub-block, bit 2t+1 for the high one.
                    const uint32_t h = word_of(cur[gi].ha, cur[gi].hb, i) >> (2 * t);
                    lo0 |= (h << 4) & 0x00100010u;
                    lo1 |= (h >> 4) & 0x00100010u;
                    hi0 |= (h << 7) & 0x01000100u;
                    hi1 |= (h >> 1) & 0x01000100u;
                }
                const uint32_t a_lo0 = h2u(__hfma2(u2h(lo0), sAA[gi], cA[gi]));
                const uint32_t a_lo1 = h2u(__hfma2(u2h(lo1), sAA[gi], cA[gi]));
                const uint32_t a_hi0 = h2u(__hfma2(u2h(hi0), sB16[gi], cB[gi]));
                const uint32_t a_hi1 = h2u(__hfma2(u2h(hi1), sB16[gi], cB[gi]));
                const uint32_t mA = h2u(mAA[gi]), mB = h2u(mBB[gi]);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    mma16816(d_acc[gi][nt], a_lo0, mA, a_lo1, mA, blo[nt].x, blo[nt].y);
                    mma16816(d_acc[gi][nt], a_hi0, mB, a_hi1, mB, bhi[nt].x, bhi[nt].y);
                }
            }
        }
        // fold this block: columns 2t (limb 0) and 2t+1 (limb 1) of batch 4 nt + t
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int b = 4 * nt + t;
            const float xs = b < batch ? __ldg(XS + (int64_t)b * nblk + kb) : 0.0f;
#pragma unroll
            for (int gi = 0; gi < G; ++gi) {
                const float ds = dd[gi] * xs, ms = dm[gi] * xs;
                acc[gi][nt][0] = fmaf(ds, d_acc[gi][nt][0], fmaf(-ms, d_acc[gi][nt][2], acc[gi][nt][0]));
                acc[gi][nt][1] = fmaf(ds, d_acc[gi][nt][1], fmaf(-ms, d_acc[gi][nt][3], acc[gi][nt][1]));
            }
        }
#pragma unroll
        for (int gi = 0; gi < G; ++gi) cur[gi] = nxt[gi];
    }

    // combine the warps' partial sums
    __shared__ float red[kMmaWarps][G][NT][32];
#pragma unroll
    for (int gi = 0; gi < G; ++gi)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) red[warp][gi][nt][lane] = fmaf(acc[gi][nt][1], 1.0f / 2048.0f, acc[gi][nt][0]);
    __syncthreads();
    if (warp < G * NT) {
        const int gi = warp / NT, nt = warp % NT;
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < kMmaWarps; ++w) v += red[w][gi][nt][lane];
        const int b = 4 * nt + t;
        const int64_t row = row0 + 8 * gi + g;
        if (b < batch && row < N) Y[(int64_t)b * N + row] = v;
    }
}

template <uint32_t Q, int G, int NT>
void launch_mma(const GemvArgs& a, uint2* xf, float* xs, cudaStream_t s) {
    const int nblk = (int)(a.K / 256);
    const int64_t grid = (a.N + 8 * G - 1) / (8 * G);
    gemv_kq_mma_kernel<Q, G, NT><<<(unsigned)grid, kMmaWarps * 32, 0, s>>>(a.W, a.row_bytes, a.N, nblk, xf, xs,
                                                                          a.batch, a.Y);
}

}  // namespace

int64_t gemv_mma_work_bytes(int64_t K, int batch) {
    const int64_t nblk = K / 256;
    return nblk * 64 * 2 * batch * (int64_t)sizeof(uint2) + (int64_t)batch * nblk * 4 + 256;
}

bool gemv_mma_supported(uint32_t quant, const GemvArgs& a) {
    return (quant == kQ4_K || quant == kQ5_K) && a.K % 256 == 0 && a.batch >= 1 && a.batch <= 8 &&
           (a.row_bytes % 16) == 0 && ((uintptr_t)a.W % 16) == 0 && ((uintptr_t)a.X % 16) == 0;
}

// x limbs into `work` (gemv_mma_work_bytes), then the tensor-core GEMV.
int launch_gemv_mma(uint32_t quant, const GemvArgs& a, void* work, cudaStream_t s) {
    const int nblk = (int)(a.K / 256);
    uint2* xf = reinterpret_cast<uint2*>(work);
    float* xs = reinterpret_cast<float*>(reinterpret_cast<char*>(work) + (int64_t)nblk * 64 * 2 * a.batch * 8);
    const int64_t warps = (int64_t)nblk * a.batch;
    prep_x_limbs_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>(a.X, a.K, a.batch, xf, xs);
    const bool two = a.batch > 4;
    // rows per CTA: 16 when there are enough rows to fill the GPU twice over
    const bool wide = a.N >= (int64_t)a.sm_count * 16 * 2;
    if (quant == kQ4_K) {
        if (two) wide ? launch_mma<kQ4_K, 2, 2>(a, xf, xs, s) : launch_mma<kQ4_K, 1, 2>(a, xf, xs, s);
        else wide ? launch_mma<kQ4_K, 2, 1>(a, xf, xs, s) : launch_mma<kQ4_K, 1, 1>(a, xf, xs, s);
    } else {
        if (two) wide ? launch_mma<kQ5_K, 2, 2>(a, xf, xs, s) : launch_mma<kQ5_K, 1, 2>(a, xf, xs, s);
        else wide ? launch_mma<kQ5_K, 2, 1>(a, xf, xs, s) : launch_mma<kQ5_K, 1, 1>(a, xf, xs, s);
    }
    return 0;
}

}  // namespace strata
