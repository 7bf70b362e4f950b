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
// * An MMA covers 16 weight rows x 16 weights. The min term
//   sum_j m_j * (sum of x over sub-block j) is one more MMA per block whose 16
//   K slots are the block's 8 sub-blocks (and 8 zeros): A holds the rows'
//   6-bit mins, B the per-sub-block activation sums (as fp16 limbs).
// * B operand (fp16): each activation column is split into two fp16 limbs,
//   x*s = hi + lo * 2^-11 (22 significant bits), with a power-of-two scale s
//   per (column, block) chosen from the block's max |x|, so fp16 can neither
//   overflow nor lose the small entries. Columns are (batch, limb) pairs.
// * D (fp32) accumulates one 256-weight block (16 mma.sync m16n8k16, plus the
//   min MMA), then is folded into fp32 accumulators with d / dmin / s. The
//   products are exact and the sums are fp32, which is what the 1e-3
//   tolerance needs.
//
// Work split: row tiles of 16 rows; a producer warp streams each tile into
// shared memory with bulk copies while 4 (batch <= 4) or 8 consumer warps
// split its K blocks (see the kernel). Batch 1 keeps the scales out of the A
// operand (mma_blocks_diag). A prologue kernel writes the activation limbs in
// the order the B fragments are read (one 8-byte load per lane per mma); the
// GEMV is launched as its programmatic dependent, so it starts streaming
// weights while the prologue runs and waits only before reading the limbs.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <cstring>

#include "kernels.cuh"
#include "quant.cuh"

namespace strata {

namespace {

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

// d = (a & b) | c in one LOP3
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// d = A*B (accumulator input zero)
__device__ __forceinline__ void mma16816_z(float d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
    const float z = 0.0f;
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}

// ---------------------------------------------------------------- prologue
//
// XF layout: [blk][i = word 0..7][n = column 0..2*batch)][t = 0..3] of
// uint4 {b0(2t), b1(2t), b0(2t+1), b1(2t+1)}: the B fragments of the low- and
// high-nibble MMAs of word i for lane t, where for sub-block s and
// e = 256 blk + 32 s + 4 i
//   b0(s) = half2(v[e], v[e+2]), b1(s) = half2(v[e+1], v[e+3]),
// v = limb (n & 1) of batch row (n >> 1) of x, scaled by XS^-1. With t
// innermost, the 8 lanes of a quarter-warp (two columns x four t) read one
// contiguous 128-byte line per load.
// XS layout: [batch][blk] float: the power of two that undoes the scaling.
// XQ layout: [blk][t = 0..3][n][2] __half: the sums of v over sub-blocks 2t
// and 2t+1, limb (n & 1) of batch (n >> 1) -- the B operand of the min MMA.
__global__ void prep_x_limbs_kernel(const float* __restrict__ X, int64_t K, int batch, uint2* __restrict__ XF,
                                    float* __restrict__ XS, __half* __restrict__ XQ, int64_t chunk_bytes) {
    // XF is addressed here in uint2 halves of the uint4 entries.
    // Launched as a programmatic dependent of the previous kernel in the
    // stream: x may be that kernel's output, and the workspace written below
    // may still be read by it (a preceding GEMV), so wait for it first.
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // token chunk blockIdx.y: its own activation rows and workspace slice
    X += (int64_t)blockIdx.y * batch * K;
    XF = reinterpret_cast<uint2*>(reinterpret_cast<char*>(XF) + blockIdx.y * chunk_bytes);
    XS = reinterpret_cast<float*>(reinterpret_cast<char*>(XS) + blockIdx.y * chunk_bytes);
    XQ = reinterpret_cast<__half*>(reinterpret_cast<char*>(XQ) + blockIdx.y * chunk_bytes);
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
    if (e == 0 || e == 0xFF) e = 127;  // zero, denormal or non-finite maximum: s = 1/2
    int se = 253 - e;                  // biased exponent of s
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
    float sum = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
    sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
    sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 2);
    if ((lane & 3) == 0) {
        const __half shi = __float2half_rn(sum);
        const __half slo = __float2half_rn((sum - __half2float(shi)) * 2048.0f);
        __half* q = XQ + (((int64_t)blk * 4 + (s_blk >> 1)) * ncols + 2 * b) * 2 + (s_blk & 1);
        q[0] = shi;
        q[2] = slo;
    }
#pragma unroll
    for (int w = 0; w < 2; ++w) {
        const int i = 2 * (lane & 3) + w;
        const int o = 4 * w;
        uint2 fh, fl;
        fh.x = h2u(__halves2half2(hi[o + 0], hi[o + 2]));
        fh.y = h2u(__halves2half2(hi[o + 1], hi[o + 3]));
        fl.x = h2u(__halves2half2(lo[o + 0], lo[o + 2]));
        fl.y = h2u(__halves2half2(lo[o + 1], lo[o + 3]));
        // entry (blk, i, n, t = s/2) is 2 uint2; sub-block parity picks the half
        uint2* dst = XF + ((((int64_t)blk * 8 + i) * ncols + 2 * b) * 4 + (s_blk >> 1)) * 2 + (s_blk & 1);
        dst[0] = fh;   // column 2b   (limb 0)
        dst[8] = fl;   // column 2b+1 (limb 1): the next column, 4 uint4 = 8 uint2 on
    }
}

// ---------------------------------------------------------------- main kernel

// mbarrier / bulk-copy helpers (shared-memory addresses as 32-bit offsets)
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait on a phase parity: false (and *err set) if the phase has not
// completed within about a second (a stage's copies take microseconds).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err) {
    uint64_t t0 = 0;
    for (long long i = 0; i < kSpinLimit; ++i) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(bar), "r"(parity)
            : "memory");
        if (done) return true;
        if ((i & 255) == 0) {
            const uint64_t now = global_ns();
            if (i == 0) t0 = now;
            else if (now - t0 > 1000000000ull) break;
        }
    }
    if (err) atomicExch(err, 1);
    return false;
}
// 1-D bulk copy global -> this CTA's shared memory, completing on `bar` (this CTA only).
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

__device__ __forceinline__ uint32_t word_of(const uint4& a, const uint4& b, int i) {
    switch (i) {
    case 0: return a.x; case 1: return a.y; case 2: return a.z; case 3: return a.w;
    case 4: return b.x; case 5: return b.y; case 6: return b.z; default: return b.w;
    }
}

// 3-D tensor-map load into this CTA's shared memory, completing on `bar` (this CTA only).
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}

constexpr int kStages = 2;  // smem ring depth
constexpr int kChunk = 8;   // K blocks per stage (whole 128-byte lines for the tensor map)
// Consumer warps per CTA: four warps of two blocks per stage (three CTAs per
// SM) or eight warps of one block (two CTAs per SM). From batch 5 always eight
// (the registers of the larger accumulators); up to batch 4 eight when that
// takes no more rounds of tiles over the resident CTAs than four: a CTA then
// spends half the time on each stage, which is what bounds matrices of few
// tiles (their time does not change when the weights are L2-resident).
__host__ __device__ constexpr int min_ctas_for_consumers(int c) { return c == 8 ? 2 : 3; }
constexpr int kTileRows = 16;

// One (16-row tile, K block) work item of a consumer warp: rows g and g+8 of
// the tile, block kb (its bytes in shared memory at `blk0` / `blk1`), folded
// into acc. NB is the batch; its 2*NB (batch, limb) columns fill
// NT = ceil(2*NB / 8) n8 tiles. `xfl` / `xql` point at this lane's fragment
// column of block 0. The 16 sc*q MMAs alternate between two accumulator chains.
template <uint32_t Q, int NB, int U, bool SW>
__device__ __forceinline__ void mma_blocks(const uint8_t* stage, const uint32_t (&rowoff)[U][2], const int (&kbs)[U],
                                           const uint4* const (&xfl)[(2 * NB + 7) / 8],
                                           const uint32_t* const (&xql)[(2 * NB + 7) / 8],
                                           const float* __restrict__ XS, int nblk, int t, uint32_t sel,
                                           float (&acc)[(2 * NB + 7) / 8][4]) {
    constexpr int NC = 2 * NB, NT = (NC + 7) / 8;
    constexpr int QOFF = (Q == kQ4_K) ? 16 : 48;
    const __half2 k1024 = __float2half2_rn(1024.0f);
    const __half2 kneg1024 = __float2half2_rn(-1024.0f);
    const __half2 k1_16 = __float2half2_rn(0.0625f);
    const __half2 kneg64 = __float2half2_rn(-64.0f);
    // masks kept in registers so each nibble extraction is one LOP3
    const uint32_t kLoMask = 0x000F000Fu, kHiMask = 0x00F000F0u, kMagic = 0x64006400u;
    float d_acc[U][NT][2][4], d_min[U][NT][4];

    // per block u and row r (0: row g, 1: row g + 8): quant bytes, scale constants and mins
    uint4 qa[U][2], qb[U][2], ha[U][2], hb[U][2];
    __half2 sAB[U][2], cA[U][2], sB16[U][2], cB[U][2];
    uint32_t mAB[U][2];
    float dd[U][2], dm[U][2];
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            // a 16-byte unit at logical offset o of the stage; with the 128-byte
            // swizzle the unit index inside each 128-byte line is XORed with the
            // line index mod 8
            auto ld = [&](uint32_t o) {
                if constexpr (SW) o ^= (o >> 3) & 0x70u;
                return *reinterpret_cast<const uint4*>(stage + o);
            };
            const uint32_t o = rowoff[u][r];
            const uint4 hd = ld(o);
            qa[u][r] = ld(o + QOFF + 32 * t);
            qb[u][r] = ld(o + QOFF + 32 * t + 16);
            if constexpr (Q == kQ5_K) {
                ha[u][r] = ld(o + 16);
                hb[u][r] = ld(o + 32);
            }
            dd[u][r] = f16_bits_to_f32(hd.x & 0xFFFFu);
            dm[u][r] = f16_bits_to_f32(hd.x >> 16);
            uint32_t sl, sh, ml, mh;
            scales_k4_packed(hd.y, hd.z, hd.w, sl, sh, ml, mh);
            const uint32_t sw = t < 2 ? sl : sh, mw = t < 2 ? ml : mh;
            sAB[u][r] = __hsub2(u2h(__byte_perm(sw, 0x00006464u, sel)), k1024);
            mAB[u][r] = h2u(__hsub2(u2h(__byte_perm(mw, 0x00006464u, sel)), k1024));
            cA[u][r] = __hmul2(__low2half2(sAB[u][r]), kneg1024);
            sB16[u][r] = __hmul2(__high2half2(sAB[u][r]), k1_16);
            cB[u][r] = __hmul2(__high2half2(sAB[u][r]), kneg64);
        }
    // min MMA: K slots 2t, 2t+1 = sub-blocks 2t, 2t+1 (A: this lane's mins; B: sub-block sums)
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
            mma16816_z(d_min[u][nt], mAB[u][0], mAB[u][1], 0u, 0u, __ldg(xql[nt] + kbs[u] * (4 * NC)), 0u);

#pragma unroll
    for (int i = 0; i < 8; ++i) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            uint4 bf[NT];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) bf[nt] = __ldg(xfl[nt] + (kbs[u] * 8 + i) * NC * 4);
            uint32_t a_lo0[2], a_lo1[2], a_hi0[2], a_hi1[2];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const uint32_t w = word_of(qa[u][r], qb[u][r], i);
                const uint32_t w8 = w >> 8;
                uint32_t lo0 = and_or(w, kLoMask, kMagic);
                uint32_t lo1 = and_or(w8, kLoMask, kMagic);
                uint32_t hi0 = and_or(w, kHiMask, kMagic);
                uint32_t hi1 = and_or(w8, kHiMask, kMagic);
                if constexpr (Q == kQ5_K) {
                    // qh byte l holds the 5th bit of element l of every sub-block:
                    // bit 2t for this lane's low sub-block, bit 2t+1 for the high one.
                    const uint32_t h = word_of(ha[u][r], hb[u][r], i) >> (2 * t);
                    lo0 = and_or(h << 4, 0x00100010u, lo0);
                    lo1 = and_or(h >> 4, 0x00100010u, lo1);
                    hi0 = and_or(h << 7, 0x01000100u, hi0);
                    hi1 = and_or(h >> 1, 0x01000100u, hi1);
                }
                a_lo0[r] = h2u(__hfma2(u2h(lo0), __low2half2(sAB[u][r]), cA[u][r]));
                a_lo1[r] = h2u(__hfma2(u2h(lo1), __low2half2(sAB[u][r]), cA[u][r]));
                a_hi0[r] = h2u(__hfma2(u2h(hi0), sB16[u][r], cB[u][r]));
                a_hi1[r] = h2u(__hfma2(u2h(hi1), sB16[u][r], cB[u][r]));
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                if (i == 0) {  // each chain starts from zero
                    mma16816_z(d_acc[u][nt][0], a_lo0[0], a_lo0[1], a_lo1[0], a_lo1[1], bf[nt].x, bf[nt].y);
                    mma16816_z(d_acc[u][nt][1], a_hi0[0], a_hi0[1], a_hi1[0], a_hi1[1], bf[nt].z, bf[nt].w);
                } else {
                    mma16816(d_acc[u][nt][0], a_lo0[0], a_lo0[1], a_lo1[0], a_lo1[1], bf[nt].x, bf[nt].y);
                    mma16816(d_acc[u][nt][1], a_hi0[0], a_hi0[1], a_hi1[0], a_hi1[1], bf[nt].z, bf[nt].w);
                }
            }
        }
    }
    // fold: D columns 2t (limb 0) and 2t+1 (limb 1) of batch 4 nt + t; D rows
    // g (c = 0, 1) and g + 8 (c = 2, 3). Columns past the batch hold garbage
    // (their lanes loaded a clamped column) and are never stored.
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int b = min(4 * nt + t, NB - 1);
            const float xs = __ldg(XS + b * nblk + kbs[u]);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int r = c >> 1;
                const float v = d_acc[u][nt][0][c] + d_acc[u][nt][1][c];
                acc[nt][c] = fmaf(dd[u][r] * xs, v, fmaf(-dm[u][r] * xs, d_min[u][nt][c], acc[nt][c]));
            }
        }
}

// Batch 1: the same work item with the scales kept out of the A operand.
// A holds the raw quants as fp16 subnormals (a nibble ANDed into the low
// mantissa bits is q * 2^-24, or 16 q * 2^-24 for a high nibble; exact, no
// HFMA2), and B is block-diagonal in the sub-blocks: column (j, limb) of token
// b is nonzero only in the K slots of lane group t = j, so D column (t, limb)
// is lane t's own sub-block partial sum (2t for the low-nibble chain, 2t + 1
// for the high one) and the sub-block scales are applied in fp32 afterwards.
// Lane (g, t) loads a B fragment only when g / 2 == t (the other columns are
// zero); the fragment is the prologue's XF entry for column 2 b + (g & 1).
// acc2[b][r] collects lane t's sub-blocks of row g (r = 0) or g + 8 (r = 1),
// already scaled by XS; the four t lanes are summed when the tile ends.
template <uint32_t Q, int NB, int U, bool SW>
__device__ __forceinline__ void mma_blocks_diag(const uint8_t* stage, const uint32_t (&rowoff)[U][2],
                                                const int (&kbs)[U], const uint4* const (&xfd)[NB],
                                                const __half* __restrict__ XQ, const float* __restrict__ XS, int nblk,
                                                int t, bool active, uint32_t sel, float (&acc2)[NB][2]) {
    constexpr int NC = 2 * NB;
    constexpr int QOFF = (Q == kQ4_K) ? 16 : 48;
    const uint32_t kLoMask = 0x000F000Fu, kHiMask = 0x00F000F0u;
    uint4 qa[U][2], qb[U][2], ha[U][2], hb[U][2];
    float fs0[U][2], fs1[U][2], fm0[U][2], fm1[U][2];
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            auto ld = [&](uint32_t o) {
                if constexpr (SW) o ^= (o >> 3) & 0x70u;
                return *reinterpret_cast<const uint4*>(stage + o);
            };
            const uint32_t o = rowoff[u][r];
            const uint4 hd = ld(o);
            qa[u][r] = ld(o + QOFF + 32 * t);
            qb[u][r] = ld(o + QOFF + 32 * t + 16);
            if constexpr (Q == kQ5_K) {
                ha[u][r] = ld(o + 16);
                hb[u][r] = ld(o + 32);
            }
            const float d = f16_bits_to_f32(hd.x & 0xFFFFu), dmin = f16_bits_to_f32(hd.x >> 16);
            uint32_t sl, sh, ml, mh;
            scales_k4_packed(hd.y, hd.z, hd.w, sl, sh, ml, mh);
            const uint32_t sw = t < 2 ? sl : sh, mw = t < 2 ? ml : mh;
            // (sc, m) of sub-blocks 2t and 2t + 1 as exact fp16 integers, then fp32
            const float2 sc = __half22float2(__hsub2(u2h(__byte_perm(sw, 0x00006464u, sel)),
                                                     __float2half2_rn(1024.0f)));
            const float2 mn = __half22float2(__hsub2(u2h(__byte_perm(mw, 0x00006464u, sel)),
                                                     __float2half2_rn(1024.0f)));
            // undo the 2^-24 of the subnormal quants (and the 16 of a high nibble)
            fs0[u][r] = d * 16777216.0f * sc.x;
            fs1[u][r] = d * 1048576.0f * sc.y;
            fm0[u][r] = dmin * mn.x;
            fm1[u][r] = dmin * mn.y;
        }
#pragma unroll
    for (int u = 0; u < U; ++u) {
        float dlo[NB][4], dhi[NB][4];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            uint4 bf[NB];
#pragma unroll
            for (int b = 0; b < NB; ++b)
                bf[b] = active ? __ldg(xfd[b] + (kbs[u] * 8 + i) * NC * 4) : make_uint4(0u, 0u, 0u, 0u);
            uint32_t a_lo0[2], a_lo1[2], a_hi0[2], a_hi1[2];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const uint32_t w = word_of(qa[u][r], qb[u][r], i);
                const uint32_t w8 = w >> 8;
                uint32_t lo0 = w & kLoMask, lo1 = w8 & kLoMask, hi0 = w & kHiMask, hi1 = w8 & kHiMask;
                if constexpr (Q == kQ5_K) {
                    const uint32_t h = word_of(ha[u][r], hb[u][r], i) >> (2 * t);
                    lo0 = and_or(h << 4, 0x00100010u, lo0);
                    lo1 = and_or(h >> 4, 0x00100010u, lo1);
                    hi0 = and_or(h << 7, 0x01000100u, hi0);
                    hi1 = and_or(h >> 1, 0x01000100u, hi1);
                }
                a_lo0[r] = lo0;
                a_lo1[r] = lo1;
                a_hi0[r] = hi0;
                a_hi1[r] = hi1;
            }
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                if (i == 0) {
                    mma16816_z(dlo[b], a_lo0[0], a_lo0[1], a_lo1[0], a_lo1[1], bf[b].x, bf[b].y);
                    mma16816_z(dhi[b], a_hi0[0], a_hi0[1], a_hi1[0], a_hi1[1], bf[b].z, bf[b].w);
                } else {
                    mma16816(dlo[b], a_lo0[0], a_lo0[1], a_lo1[0], a_lo1[1], bf[b].x, bf[b].y);
                    mma16816(dhi[b], a_hi0[0], a_hi0[1], a_hi1[0], a_hi1[1], bf[b].z, bf[b].w);
                }
            }
        }
        // fold: D columns 2t (limb 0) and 2t + 1 (limb 1); rows g (c = 0, 1), g + 8 (c = 2, 3)
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            const float xs = __ldg(XS + b * nblk + kbs[u]);
            // sums of the scaled activations over sub-blocks 2t, 2t + 1: {hi0, hi1, lo0, lo1}
            const uint2 qs = __ldg(reinterpret_cast<const uint2*>(XQ + ((kbs[u] * 4 + t) * NC + 2 * b) * 2));
            const float2 shi = __half22float2(u2h(qs.x)), slo = __half22float2(u2h(qs.y));
            const float x0 = fmaf(slo.x, 1.0f / 2048.0f, shi.x), x1 = fmaf(slo.y, 1.0f / 2048.0f, shi.y);
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const float vlo = fmaf(dlo[b][2 * r + 1], 1.0f / 2048.0f, dlo[b][2 * r]);
                const float vhi = fmaf(dhi[b][2 * r + 1], 1.0f / 2048.0f, dhi[b][2 * r]);
                const float tr = fmaf(fs0[u][r], vlo, fmaf(fs1[u][r], vhi, -fmaf(fm0[u][r], x0, fm1[u][r] * x1)));
                acc2[b][r] = fmaf(xs, tr, acc2[b][r]);
            }
        }
    }
}

// Persistent, warp-specialised kernel. CTA c takes 16-row tiles c, c + grid,
// ...; each tile is cut into stages of kChunk K blocks. The last warp (the
// producer) copies every stage into a kStages-deep shared-memory ring with one
// bulk copy per row (a row's blocks are contiguous bytes), completing on the
// slot's `full` mbarrier; consumer warp w computes blocks kBpw*w .. kBpw*w +
// kBpw - 1 of each stage and releases the slot through its `empty` mbarrier. Consumers keep their
// partial sums across a tile's stages and combine them in shared memory when
// the tile ends. Every wait is bounded; a timeout sets *err and the CTA stops.
template <uint32_t Q, int NB, bool TM, int NCONS>
__global__ void __launch_bounds__((NCONS + 1) * 32, min_ctas_for_consumers(NCONS))
gemv_kq_tma_kernel(const uint8_t* __restrict__ W, int64_t row_bytes, int N, int nblk,
                   const uint2* __restrict__ XF, const float* __restrict__ XS, const __half* __restrict__ XQ,
                   float* __restrict__ Y, int* __restrict__ err, const __grid_constant__ CUtensorMap tmap,
                   int64_t chunk_bytes, int64_t ldy, const __grid_constant__ PeerOut po) {
    // The next kernel in the stream may launch now: its pre-wait part only
    // reads constant weights (a following GEMV's producer) or nothing at all,
    // so its CTAs can fill the SMs this grid's CTAs leave while it drains.
    asm volatile("griddepcontrol.launch_dependents;");
    // token chunk blockIdx.y (batches above 8): its limbs and its NB output rows
    XF = reinterpret_cast<const uint2*>(reinterpret_cast<const char*>(XF) + blockIdx.y * chunk_bytes);
    XS = reinterpret_cast<const float*>(reinterpret_cast<const char*>(XS) + blockIdx.y * chunk_bytes);
    XQ = reinterpret_cast<const __half*>(reinterpret_cast<const char*>(XQ) + blockIdx.y * chunk_bytes);
    Y += (int64_t)blockIdx.y * NB * ldy;
    constexpr int NC = 2 * NB, NT = (NC + 7) / 8;
    constexpr int BB = block_bytes(Q);
    constexpr int kConsumers = NCONS, kBpw = kChunk / kConsumers;
    static_assert(NCONS == 8 || (NCONS == 4 && NB <= 4), "four consumer warps serve batches up to 4");
    // Stage j's tile and chunk: running counters, or (batches from 5, whose
    // accumulators leave no registers to spare) recomputed from j each stage,
    // which measured faster there.
    constexpr bool kDivide = NB >= 5;
    // smem stride of one row of a stage. TM (one tensor-map copy per stage):
    // the rows are dense and 128-byte swizzled, which puts consecutive rows'
    // units on different banks. Otherwise (one bulk copy per row): each row is
    // padded by 16 bytes so that the 8 rows a 128-bit fragment read touches
    // start 4 banks apart (kChunk * BB is a multiple of 128 bytes).
    constexpr int ROWB = TM ? kChunk * BB : kChunk * BB + 16;
    constexpr int STAGE = kTileRows * ROWB;
    constexpr int LINES = kChunk * BB / 128;  // 128-byte lines per row of a stage (TM)
    extern __shared__ __align__(1024) uint8_t ring_raw[];  // kStages * STAGE (+ 1 KB for alignment)
    uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ring_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t full_bar[kStages], empty_bar[kStages];
    __shared__ float red[2][kConsumers][NT][2][32];
    __shared__ int abort_flag;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ntiles = (N + kTileRows - 1) / kTileRows;
    const int nchunks = (nblk + kChunk - 1) / kChunk;
    const int my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int nstages = my_tiles * nchunks;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(smem_u32(&full_bar[i]), 1);
            mbar_init(smem_u32(&empty_bar[i]), kConsumers);
        }
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == kConsumers) {
        // ---------------- producer: the weights do not depend on the prologue
        // (abort decisions are made warp-uniform: the loop has __syncwarp)
        int issued = 0;  // stages whose copies were issued
        int tile_c = blockIdx.x, c0_c = 0;  // tile and first K block of stage j (counters)
        for (int j = 0; j < nstages; ++j) {
            const int slot = j % kStages;
            const int tile = kDivide ? blockIdx.x + (j / nchunks) * gridDim.x : tile_c;
            const int c0 = kDivide ? (j % nchunks) * kChunk : c0_c;
            bool ok = true;
            if (j >= kStages) ok = mbar_wait(smem_u32(&empty_bar[slot]), ((j / kStages) - 1) & 1, err);
            ok = __all_sync(0xFFFFFFFFu, ok) && __shfl_sync(0xFFFFFFFFu, *(volatile int*)&abort_flag, 0) == 0;
            if (!ok) {
                abort_flag = 1;
                break;
            }
            const int nb = min(kChunk, nblk - c0);
            const uint32_t bytes = (uint32_t)(nb * BB);
            const uint32_t fb = smem_u32(&full_bar[slot]);
            if constexpr (TM) {
                // the whole 16-row x kChunk-block box (rows past N are zero-filled)
                if (lane == 0) {
                    mbar_expect_tx(fb, (uint32_t)STAGE);
                    tma_load_3d(smem_u32(ring + slot * STAGE), &tmap, 0, (c0 / kChunk) * LINES, tile * kTileRows, fb);
                }
                __syncwarp();
            } else {
                if (lane == 0) mbar_expect_tx(fb, bytes * kTileRows);
                __syncwarp();
                if (lane < kTileRows) {
                    int row = tile * kTileRows + lane;
                    row = row < N ? row : N - 1;
                    const uint8_t* src = W + (int64_t)row * row_bytes + (int64_t)c0 * BB;
                    bulk_g2s(smem_u32(ring + slot * STAGE + lane * ROWB), src, bytes, fb);
                }
            }
            issued = j + 1;
            if constexpr (!kDivide) {
                c0_c += kChunk;
                if (c0_c >= nblk) {
                    c0_c = 0;
                    tile_c += gridDim.x;
                }
            }
        }
        // drain: wait (bounded) for the copies of the last stages issued, which
        // may still be in flight (after an abort, stages never issued are not waited on)
        for (int j = max(0, issued - kStages); j < issued; ++j)
            mbar_wait(smem_u32(&full_bar[j % kStages]), (j / kStages) & 1, nullptr);
        return;
    }

    // ---------------- consumers
    constexpr bool kDiag = NB == 1;  // batch 1: mma_blocks_diag
    const int g = lane >> 2, t = lane & 3;
    const uint32_t sel = (4u << 12) | ((uint32_t)(2 * (t & 1) + 1) << 8) | (4u << 4) | (uint32_t)(2 * (t & 1));
    // diagonal B: lane (g, t) holds column (g / 2, g & 1), nonzero when g / 2 == t
    const bool active = (g >> 1) == t;
    const uint4* xfd[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) xfd[b] = reinterpret_cast<const uint4*>(XF) + (2 * b + (g & 1)) * 4 + t;
    float acc2[NB][2];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc2[b][0] = acc2[b][1] = 0.0f;
    // lane (g, t) feeds B column 8 nt + g; past the batch it reads the last
    // column instead (a valid address; those D columns are never stored)
    const uint4* xfl[NT];
    const uint32_t* xql[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int n = min(8 * nt + g, NC - 1);
        xfl[nt] = reinterpret_cast<const uint4*>(XF) + n * 4 + t;
        xql[nt] = reinterpret_cast<const uint32_t*>(XQ) + t * NC + n;
    }
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[nt][c] = 0.0f;

    // the activation limbs come from the preceding kernel in the stream
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // peer all-gather: where this call's outputs go in this rank's exchange buffer
    const unsigned half = po.G ? (*po.epoch & 1u) : 0u;
    const int64_t peer_off = (int64_t)half * po.half_floats + po.off + (int64_t)blockIdx.y * NB * ldy;

    // After an expired wait a consumer skips its waits and math but keeps
    // walking the same stages, so every consumer still reaches every
    // tile-end barrier (nothing can be left waiting there).
    bool live = true;
    int tile_c = blockIdx.x, chunk_c = 0, set_c = 0;  // stage j's tile, its chunk, the tile's scratch set
    for (int j = 0; j < nstages; ++j) {
        const int slot = j % kStages;
        if (live) {
            bool ok = mbar_wait(smem_u32(&full_bar[slot]), (j / kStages) & 1, err);
            live = __all_sync(0xFFFFFFFFu, ok) && __shfl_sync(0xFFFFFFFFu, *(volatile int*)&abort_flag, 0) == 0;
            if (!live) abort_flag = 1;
        }
        const int tile = kDivide ? blockIdx.x + (j / nchunks) * gridDim.x : tile_c;
        const int chunk = kDivide ? j % nchunks : chunk_c;
        const int kb0 = chunk * kChunk + warp * kBpw;
        if (live && kb0 + kBpw <= nblk) {
            // the warp's kBpw blocks, interleaved for instruction-level parallelism
            uint32_t rowoff[kBpw][2];
            int kbs[kBpw];
#pragma unroll
            for (int u = 0; u < kBpw; ++u) {
                const uint32_t ub = (uint32_t)((warp * kBpw + u) * BB);
                rowoff[u][0] = g * ROWB + ub;
                rowoff[u][1] = (g + 8) * ROWB + ub;
                kbs[u] = kb0 + u;
            }
            if constexpr (kDiag)
                mma_blocks_diag<Q, NB, kBpw, TM>(ring + slot * STAGE, rowoff, kbs, xfd, XQ, XS, nblk, t, active, sel,
                                                 acc2);
            else
                mma_blocks<Q, NB, kBpw, TM>(ring + slot * STAGE, rowoff, kbs, xfl, xql, XS, nblk, t, sel, acc);
        } else if (live) {
            // a ragged last chunk: the blocks that exist, one at a time
            for (int kb = kb0; kb < nblk && kb < kb0 + kBpw; ++kb) {
                const uint32_t ub = (uint32_t)((kb - chunk * kChunk) * BB);
                const uint32_t rowoff[1][2] = {{g * ROWB + ub, (g + 8) * ROWB + ub}};
                const int kbs[1] = {kb};
                if constexpr (kDiag)
                    mma_blocks_diag<Q, NB, 1, TM>(ring + slot * STAGE, rowoff, kbs, xfd, XQ, XS, nblk, t, active, sel,
                                                  acc2);
                else
                    mma_blocks<Q, NB, 1, TM>(ring + slot * STAGE, rowoff, kbs, xfl, xql, XS, nblk, t, sel, acc);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&empty_bar[slot]));
        if (chunk == nchunks - 1) {
            // tile done: lane (g, t) holds rows g, g + 8 x columns (2t, 2t+1) of
            // each n8 tile. The scratch alternates between two sets, so the
            // next tile's writes cannot race this tile's reads and one barrier
            // per tile suffices.
            const int set = kDivide ? (j / nchunks) & 1 : set_c;
            if constexpr (kDiag) {
                // sum the four t lanes of each row, then the warps: red[set][w] as [b][16 rows]
                float* rw = &red[set][warp][0][0][0];
#pragma unroll
                for (int b = 0; b < NB; ++b)
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        float v = acc2[b][r];
                        v += __shfl_xor_sync(0xFFFFFFFFu, v, 1);
                        v += __shfl_xor_sync(0xFFFFFFFFu, v, 2);
                        if (t == 0) rw[b * 16 + 8 * r + g] = v;
                        acc2[b][r] = 0.0f;
                    }
                asm volatile("bar.sync 1, %0;" ::"r"(kConsumers * 32) : "memory");
                if (warp == 0 && lane < NB * 16) {
                    const int b = lane >> 4, row = tile * kTileRows + (lane & 15);
                    float v = 0.0f;
#pragma unroll
                    for (int w = 0; w < kConsumers; ++w) v += (&red[set][w][0][0][0])[lane];
                    if (row < N) {
                        if (po.G) po.y[peer_off + b * ldy + row] = v;
                        else Y[b * ldy + row] = v;
                    }
                }
            } else {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    red[set][warp][nt][0][lane] = fmaf(acc[nt][1], 1.0f / 2048.0f, acc[nt][0]);
                    red[set][warp][nt][1][lane] = fmaf(acc[nt][3], 1.0f / 2048.0f, acc[nt][2]);
#pragma unroll
                    for (int c = 0; c < 4; ++c) acc[nt][c] = 0.0f;
                }
                asm volatile("bar.sync 1, %0;" ::"r"(kConsumers * 32) : "memory");
                if (warp < 2 * NT) {
                    const int nt = warp >> 1, r = warp & 1;
                    float v = 0.0f;
#pragma unroll
                    for (int w = 0; w < kConsumers; ++w) v += red[set][w][nt][r][lane];
                    const int b = 4 * nt + t;
                    const int row = tile * kTileRows + 8 * r + g;
                    if (b < NB && row < N) {
                        if (po.G) po.y[peer_off + b * ldy + row] = v;
                        else Y[b * ldy + row] = v;
                    }
                }
            }
        }
        if constexpr (!kDivide) {
            if (++chunk_c == nchunks) {
                chunk_c = 0;
                tile_c += gridDim.x;
                set_c ^= 1;
            }
        }
    }
}

template <uint32_t Q, int NB, bool TM>
constexpr int tma_smem_bytes() {
    return kStages * kTileRows * (kChunk * block_bytes(Q) + (TM ? 0 : 16)) + 1024;
}

// Resident CTAs per SM of one instantiation (computed once).
template <uint32_t Q, int NB, bool TM, int NCONS>
int tma_ctas_per_sm() {
    static int per_sm = 0;
    if (per_sm == 0) {
        constexpr int smem = tma_smem_bytes<Q, NB, TM>();
        cudaFuncSetAttribute(gemv_kq_tma_kernel<Q, NB, TM, NCONS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        int n = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemv_kq_tma_kernel<Q, NB, TM, NCONS>, (NCONS + 1) * 32,
                                                      smem);
        per_sm = n < 1 ? 1 : n;
    }
    return per_sm;
}

template <uint32_t Q, int NB, bool TM, int NCONS>
void launch_tma(const GemvArgs& a, const uint2* xf, const float* xs, const __half* xq, int* err, cudaStream_t s,
                unsigned chunks, int64_t chunk_bytes) {
    const int nblk = (int)(a.K / 256);
    const int64_t ntiles = (a.N + kTileRows - 1) / kTileRows;
    CUtensorMap map;
    if (TM) map = *reinterpret_cast<const CUtensorMap*>(a.tmap);
    else memset(&map, 0, sizeof(map));
    int64_t grid = (int64_t)a.sm_count * tma_ctas_per_sm<Q, NB, TM, NCONS>();
    if (grid > ntiles) grid = ntiles;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid, chunks);
    cfg.blockDim = dim3((NCONS + 1) * 32);
    cfg.dynamicSmemBytes = tma_smem_bytes<Q, NB, TM>();
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    PeerOut po{};
    if (a.peers) po = *a.peers;
    cudaLaunchKernelEx(&cfg, gemv_kq_tma_kernel<Q, NB, TM, NCONS>, a.W, a.row_bytes, (int)a.N, nblk, xf, xs, xq, a.Y,
                       err, map, chunk_bytes, ldy_of(a), po);
}

// Four or eight consumer warps (see min_ctas_for_consumers).
template <uint32_t Q, int NB, bool TM>
void launch_general(const GemvArgs& a, const uint2* xf, const float* xs, const __half* xq, int* err, cudaStream_t s,
                    unsigned chunks = 1, int64_t chunk_bytes = 0) {
    if constexpr (NB >= 5) {
        launch_tma<Q, NB, TM, 8>(a, xf, xs, xq, err, s, chunks, chunk_bytes);
    } else {
        const int64_t ntiles = (a.N + kTileRows - 1) / kTileRows;
        const int64_t cap4 = (int64_t)a.sm_count * tma_ctas_per_sm<Q, NB, TM, 4>();
        const int64_t cap8 = (int64_t)a.sm_count * tma_ctas_per_sm<Q, NB, TM, 8>();
        if ((ntiles + cap8 - 1) / cap8 <= (ntiles + cap4 - 1) / cap4)
            launch_tma<Q, NB, TM, 8>(a, xf, xs, xq, err, s, chunks, chunk_bytes);
        else
            launch_tma<Q, NB, TM, 4>(a, xf, xs, xq, err, s, chunks, chunk_bytes);
    }
}

template <uint32_t Q, bool TM>
void dispatch_mma(const GemvArgs& a, const uint2* xf, const float* xs, const __half* xq, int* err, cudaStream_t s,
                  unsigned chunks = 1, int64_t chunk_bytes = 0) {
    if (chunks > 1) return launch_general<Q, 8, TM>(a, xf, xs, xq, err, s, chunks, chunk_bytes);
    switch (a.batch) {
    case 1: return launch_general<Q, 1, TM>(a, xf, xs, xq, err, s);
    case 2: return launch_general<Q, 2, TM>(a, xf, xs, xq, err, s);
    case 3: return launch_general<Q, 3, TM>(a, xf, xs, xq, err, s);
    case 4: return launch_general<Q, 4, TM>(a, xf, xs, xq, err, s);
    case 5: return launch_general<Q, 5, TM>(a, xf, xs, xq, err, s);
    case 6: return launch_general<Q, 6, TM>(a, xf, xs, xq, err, s);
    case 7: return launch_general<Q, 7, TM>(a, xf, xs, xq, err, s);
    default: return launch_general<Q, 8, TM>(a, xf, xs, xq, err, s);
    }
}


// ============================================================ tall matrices, batch 1
//
// A second decode kernel for batch 1 on matrices with many rows (at least four
// 64-row items per SM, e.g. the 151936-row output projection): one CTA of 16
// consumer warps and a producer per SM streams 64-row x 8-block stages through
// a 3-deep ring (216 KB for Q4_K), each warp computing two m16 tiles of one
// block per stage, so the per-stage work outside the math is paid once per two
// tiles; the producer also adds the warps' partial sums, so no consumer ever
// waits for another. The general kernel above serves every other case.
namespace tall {

constexpr int kGroups = 2;               // row groups of 16 per 32-row half of a stage
constexpr int kWarps = 8 * kGroups;      // consumer warps: warp w computes block w % 8 of row group w / 8
constexpr int kThreads = (kWarps + 1) * 32;
constexpr int kHalfRows = 16 * kGroups;  // 32
constexpr int kT = 2;                    // m16 tiles per warp and stage
constexpr int kItemRows = kT * kHalfRows;  // 64 rows per stage
constexpr int kPitch = kItemRows + 8;    // floats per block row of a reduction slot
constexpr int kRedSlots = 4;
__host__ __device__ constexpr int stage_bytes(uint32_t q) { return kItemRows * kChunk * block_bytes(q); }
constexpr int kRedBytes = kRedSlots * 8 * kPitch * 4;
__host__ __device__ constexpr int stages_for(uint32_t q) {
    return (220 * 1024 - kRedBytes - 1024) / stage_bytes(q) > 4 ? 4 : (220 * 1024 - kRedBytes - 1024) / stage_bytes(q);
}
__host__ __device__ constexpr int smem_for(uint32_t q) { return stages_for(q) * stage_bytes(q) + kRedBytes + 1024; }

// Per-lane selectors for the 6-bit (scale, min) pairs of sub-blocks 2t and
// 2t + 1 (get_scale_min_k4, dequant.rs:237-245). With the 12 scale bytes as
// words y = bytes 0-3, z = 4-7, w = 8-11 and p = t & 1:
//   t < 2 : sc = y[2p..2p+1] & 63,                      m = z[2p..2p+1] & 63
//   t >= 2: sc = (w & 15) | (y >> 6) << 4 (same bytes),  m = (w >> 4) | (z >> 6) << 4
// Both pairs come out as two 16-bit integers (one per half), no branch.
struct LaneScale {
    uint32_t sel_lo;  // byte_perm selector: t < 2 bytes 2p, 2p+1 of the first word, else of w
    uint32_t sel_hi;  // byte_perm selector: t < 2 zero, else bytes 2p, 2p+1 of the first word
    uint32_t mlo;     // low-part mask: 6 bits (t < 2) or 4 bits
    uint32_t shm;     // shift of the min's low part: 0 (t < 2) or 4
};
__device__ __forceinline__ LaneScale lane_scale(int t) {
    const uint32_t p = 2u * (uint32_t)(t & 1);
    LaneScale s;
    if (t < 2) {
        s.sel_lo = p | (p << 4) | ((p + 1) << 8) | ((p + 1) << 12);
        s.sel_hi = 0x4444u;
        s.mlo = 0x003F003Fu;
        s.shm = 0;
    } else {
        s.sel_lo = (p + 4) | ((p + 4) << 4) | ((p + 5) << 8) | ((p + 5) << 12);
        s.sel_hi = p | (4u << 4) | ((p + 1) << 8) | (4u << 12);
        s.mlo = 0x000F000Fu;
        s.shm = 4;
    }
    return s;
}
// (sc, m) of this lane's two sub-blocks from a block header hd (hd.y/z/w =
// scale bytes 0-3 / 4-7 / 8-11).
__device__ __forceinline__ void sc_m_pair(const uint4& hd, const LaneScale& ls, uint32_t& SC, uint32_t& M) {
    const uint32_t p1 = __byte_perm(hd.y, hd.w, ls.sel_lo);
    const uint32_t p2 = __byte_perm(hd.y, 0u, ls.sel_hi);
    const uint32_t p3 = __byte_perm(hd.z, hd.w, ls.sel_lo);
    const uint32_t p4 = __byte_perm(hd.z, 0u, ls.sel_hi);
    SC = (p1 & ls.mlo) | ((p2 >> 2) & 0x00300030u);
    M = ((p3 >> ls.shm) & ls.mlo) | ((p4 >> 2) & 0x00300030u);
}
// the 16-bit integer in the low / high half of v as an exact float (2^23 + v - 2^23)
__device__ __forceinline__ float u16_lo_f(uint32_t v) {
    return __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7610)) - 8388608.0f;
}
__device__ __forceinline__ float u16_hi_f(uint32_t v) {
    return __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7632)) - 8388608.0f;
}
// two small integers (one per 16-bit half, < 1024) as an exact half2
__device__ __forceinline__ uint32_t u16x2_h2(uint32_t v) {
    return h2u(__hsub2(u2h(v | 0x64006400u), __float2half2_rn(1024.0f)));
}

// Shared-memory offsets of one lane's fields of one block in a stage: row r0
// of the stage, block position `w`. Row r0 + 8 follows at 8 * ROWB, a multiple
// of 1024 bytes (8 rows are 72 or 88 whole 128-byte lines), so the 128-byte
// swizzle of that row is the same and its offsets are a compile-time
// displacement from these.
struct LaneOff {
    uint32_t hd, qa, qb, ha, hb;
};
template <uint32_t Q, bool SW>
__device__ __forceinline__ LaneOff lane_offsets(int r0, int t, int w) {
    constexpr int BB = block_bytes(Q);
    constexpr int ROWB = SW ? kChunk * BB : kChunk * BB + 16;
    constexpr int QOFF = (Q == kQ4_K) ? 16 : 48;
    auto swz = [](uint32_t o) { return SW ? (o ^ ((o >> 3) & 0x70u)) : o; };
    const uint32_t base = (uint32_t)(r0 * ROWB + w * BB);
    LaneOff o;
    o.hd = swz(base);
    o.qa = swz(base + QOFF + 32 * t);
    o.qb = swz(base + QOFF + 32 * t + 16);
    o.ha = swz(base + 16);
    o.hb = swz(base + 32);
    return o;
}
__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

// Batch 1, one m16 tile (the lane's rows r0 and r0 + 8) of one block: A holds
// the raw quants as fp16 subnormals (a nibble ANDed into the low mantissa bits
// is q * 2^-24, a high nibble 16 q * 2^-24; exact) and B is block-diagonal in
// the sub-blocks, so D column (t, limb) is lane t's own sub-block partial sum
// and the scales are applied in fp32 once per block. The min term
// sum_j m_j * (sum of x over sub-block j) is one more MMA whose K slots are the
// 8 sub-blocks: A the rows' mins, B the per-sub-block activation sums (two fp16
// limbs; only columns 0 and 1 are non-zero).
// acc[r] collects lane t's share of row r0 (r = 0) or r0 + 8 (r = 1).
template <uint32_t Q, bool SW>
__device__ __forceinline__ void unit_diag(const uint8_t* st, const LaneOff& lo, const uint4 (&bf)[8], uint32_t bq,
                                          float xs24, float xs20, float xs, const LaneScale& ls, int t,
                                          float (&acc)[2]) {
    constexpr int BB = block_bytes(Q);
    constexpr int R8 = 8 * (SW ? kChunk * BB : kChunk * BB + 16);  // 8 rows of the stage
    (void)t;
    uint4 qa[2], qb[2], ha[2], hb[2];
    float fs0[2], fs1[2], fm[2];
    uint32_t ma[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const uint8_t* sr = st + r * R8;
        const uint4 hd = lds128(sr + lo.hd);
        qa[r] = lds128(sr + lo.qa);
        qb[r] = lds128(sr + lo.qb);
        if constexpr (Q == kQ5_K) {
            ha[r] = lds128(sr + lo.ha);
            hb[r] = lds128(sr + lo.hb);
        }
        uint32_t SC, M;
        sc_m_pair(hd, ls, SC, M);
        const float d = __low2float(u2h(hd.x)), dmin = __high2float(u2h(hd.x));
        fs0[r] = u16_lo_f(SC) * (d * xs24);
        fs1[r] = u16_hi_f(SC) * (d * xs20);
        fm[r] = dmin * xs;
        ma[r] = u16x2_h2(M);
    }
    float dm[4], dlo[4], dhi[4];
    mma16816_z(dm, ma[0], ma[1], 0u, 0u, bq, 0u);
    const uint32_t kLoMask = 0x000F000Fu, kHiMask = 0x00F000F0u;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        uint32_t a_lo0[2], a_lo1[2], a_hi0[2], a_hi1[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const uint32_t w = word_of(qa[r], qb[r], i);
            const uint32_t w8 = w >> 8;
            uint32_t lo0 = w & kLoMask, lo1 = w8 & kLoMask, hi0 = w & kHiMask, hi1 = w8 & kHiMask;
            if constexpr (Q == kQ5_K) {
                // qh byte l holds the 5th bit of element l of every sub-block:
                // bit 2t for this lane's low sub-block, bit 2t+1 for the high one.
                const uint32_t h = word_of(ha[r], hb[r], i) >> (2 * t);
                lo0 = and_or(h << 4, 0x00100010u, lo0);
                lo1 = and_or(h >> 4, 0x00100010u, lo1);
                hi0 = and_or(h << 7, 0x01000100u, hi0);
                hi1 = and_or(h >> 1, 0x01000100u, hi1);
            }
            a_lo0[r] = lo0;
            a_lo1[r] = lo1;
            a_hi0[r] = hi0;
            a_hi1[r] = hi1;
        }
        if (i == 0) {
            mma16816_z(dlo, a_lo0[0], a_lo0[1], a_lo1[0], a_lo1[1], bf[i].x, bf[i].y);
            mma16816_z(dhi, a_hi0[0], a_hi0[1], a_hi1[0], a_hi1[1], bf[i].z, bf[i].w);
        } else {
            mma16816(dlo, a_lo0[0], a_lo0[1], a_lo1[0], a_lo1[1], bf[i].x, bf[i].y);
            mma16816(dhi, a_hi0[0], a_hi0[1], a_hi1[0], a_hi1[1], bf[i].z, bf[i].w);
        }
    }
    // D columns 2t (limb 0) and 2t + 1 (limb 1); rows r0 (c = 0, 1), r0 + 8 (c = 2, 3)
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const float vlo = fmaf(dlo[2 * r + 1], 1.0f / 2048.0f, dlo[2 * r]);
        const float vhi = fmaf(dhi[2 * r + 1], 1.0f / 2048.0f, dhi[2 * r]);
        const float vm = fmaf(dm[2 * r + 1], 1.0f / 2048.0f, dm[2 * r]);
        acc[r] = fmaf(fs0[r], vlo, fmaf(fs1[r], vhi, fmaf(-fm[r], vm, acc[r])));
    }
}

// Bounded wait with a fast path: one try_wait (which itself may suspend the
// thread in hardware for a while), then, only if the phase is still open, a
// loop that sleeps between polls (suspend-time hint), gives up early once the
// CTA has aborted and records a timeout after about a second.
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}
__device__ __noinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity, int* err, const volatile int* abort) {
    const uint64_t t0 = global_ns();
    for (long long i = 0; i < kSpinLimit; ++i) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(bar), "r"(parity), "r"(1000000u)
            : "memory");
        if (done) return true;
        if (*abort) return false;
        if (global_ns() - t0 > 1000000000ull) break;
    }
    if (err) atomicExch(err, 1);
    return false;
}
__device__ __forceinline__ bool mbar_wait_ab(uint32_t bar, uint32_t parity, int* err, const volatile int* abort) {
    return mbar_try(bar, parity) || mbar_wait_slow(bar, parity, err, abort);
}

// Persistent, warp-specialised: CTA c takes 64-row items c, c + grid, ...; an
// item's K range is cut into stages of kChunk blocks. The producer (warp 16)
// copies each stage with four 16-row tensor-map boxes into the ring; consumer
// warp w computes block w % 8 of the stage for rows 16 (w / 8) + 32 u .. + 15,
// u = 0, 1, and releases the slot. At the end of an item every consumer writes
// its partial sums to a reduction slot; the producer, between copies, adds
// each row's eight blocks in order and stores the rows. Every wait is bounded;
// a timeout sets *err and the CTA stops.
template <uint32_t Q>
__global__ void __launch_bounds__(kThreads, 1)
gemv_b1_tall_kernel(int N, int nblk, const uint2* __restrict__ XF, const float* __restrict__ XS,
                    const __half* __restrict__ XQ, float* __restrict__ Y, int* __restrict__ err,
                    const __grid_constant__ CUtensorMap tmap, const __grid_constant__ PeerOut po) {
    // the next kernel in the stream may launch now (its pre-wait part reads only constant weights)
    asm volatile("griddepcontrol.launch_dependents;");
    constexpr int NC = 2;  // (limb 0, limb 1) of the one token
    constexpr int BB = block_bytes(Q);
    constexpr int ROWB = kChunk * BB;  // dense, 128-byte swizzled rows
    constexpr int HALF = kHalfRows * ROWB;
    constexpr int STAGE = kT * HALF;
    constexpr int kStages = stages_for(Q);
    static_assert(kStages >= 2, "the ring needs two stages");
    constexpr int LINES = kChunk * BB / 128;
    constexpr int RED = 8 * kPitch;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* red = reinterpret_cast<float*>(ring + kStages * STAGE);  // [kRedSlots][8 blocks][kPitch]
    __shared__ __align__(8) uint64_t full_bar[kStages], empty_bar[kStages], rfull_bar[kRedSlots],
        rempty_bar[kRedSlots];
    __shared__ int abort_flag;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nchunks = (nblk + kChunk - 1) / kChunk;
    const int nitems = (N + kItemRows - 1) / kItemRows;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(smem_u32(&full_bar[i]), 1);
            mbar_init(smem_u32(&empty_bar[i]), kWarps);
        }
        for (int i = 0; i < kRedSlots; ++i) {
            mbar_init(smem_u32(&rfull_bar[i]), kWarps);
            mbar_init(smem_u32(&rempty_bar[i]), 1);
        }
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const volatile int* abortp = &abort_flag;

    if (warp == kWarps) {
        // ---------------- producer: streams the stages and reduces finished items
        bool waited = false;  // griddepcontrol.wait done (before the first store)
        int64_t peer_off = 0;
        auto reduce = [&](int it, int q) -> bool {
            if (!waited) {
                asm volatile("griddepcontrol.wait;" ::: "memory");
                const unsigned half = po.G ? (*po.epoch & 1u) : 0u;
                peer_off = (int64_t)half * po.half_floats + po.off;
                waited = true;
            }
            const int rs = q & (kRedSlots - 1), use = q / kRedSlots;
            if (!__all_sync(0xFFFFFFFFu, mbar_wait_ab(smem_u32(&rfull_bar[rs]), use & 1, err, abortp)))
                return false;
            const float* rr = red + rs * RED;
            float v[kT];
#pragma unroll
            for (int u = 0; u < kT; ++u) {
                float sum = 0.0f;
#pragma unroll
                for (int w = 0; w < 8; ++w) sum += rr[w * kPitch + kHalfRows * u + lane];
                v[u] = sum;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&rempty_bar[rs]));
#pragma unroll
            for (int u = 0; u < kT; ++u) {
                const int row = it * kItemRows + kHalfRows * u + lane;
                if (row < N) {
                    if (po.G) po.y[peer_off + row] = v[u];
                    else Y[row] = v[u];
                }
            }
            return true;
        };
        int j = 0, slot = 0, par = 0;  // stages issued; ring slot and round parity of stage j
        int rit = blockIdx.x, rq = 0, rend = nchunks;  // next item to reduce, its ordinal, stage just past it
        bool ok = true;
        for (int it = blockIdx.x; it < nitems && ok; it += gridDim.x) {
            for (int c = 0; c < nchunks; ++c) {
                if (j >= kStages &&
                    !__all_sync(0xFFFFFFFFu, mbar_wait_ab(smem_u32(&empty_bar[slot]), par ^ 1, err, abortp))) {
                    abort_flag = 1;
                    ok = false;
                    break;
                }
                const uint32_t fb = smem_u32(&full_bar[slot]);
                if (lane == 0) {
                    // four 16-row boxes (rows past N are zero-filled)
                    mbar_expect_tx(fb, (uint32_t)STAGE);
#pragma unroll
                    for (int h = 0; h < kItemRows / 16; ++h)
                        tma_load_3d(smem_u32(ring + slot * STAGE + h * 16 * ROWB), &tmap, 0, c * LINES,
                                    it * kItemRows + 16 * h, fb);
                }
                __syncwarp();
                ++j;
                if (++slot == kStages) {
                    slot = 0;
                    par ^= 1;
                }
                // every consumer has released stage j - 1 - kStages: the items that
                // ended before it have their partials in place
                while (rit < nitems && rend <= j - 1 - kStages) {
                    if (!reduce(rit, rq)) {
                        abort_flag = 1;
                        ok = false;
                        break;
                    }
                    rit += gridDim.x;
                    ++rq;
                    rend += nchunks;
                }
                if (!ok) break;
            }
        }
        for (; ok && rit < nitems; rit += gridDim.x, ++rq)
            if (!reduce(rit, rq)) {
                abort_flag = 1;
                ok = false;
            }
        // drain after an abort: wait (bounded) for the copies issued that may still be in flight
        if (!ok)
            for (int i = max(0, j - kStages); i < j; ++i)
                mbar_wait(smem_u32(&full_bar[i % kStages]), (i / kStages) & 1, nullptr);
        return;
    }

    // ---------------- consumers
    const int g = lane >> 2, t = lane & 3;
    const int grp = warp >> 3, wb = warp & 7;  // row group, block position in the stage
    const LaneScale ls = lane_scale(t);
    const LaneOff lo = lane_offsets<Q, true>(g + 16 * grp, t, wb);
    // diagonal B: lane (g, t) holds column (g / 2, g & 1), nonzero when g / 2 == t
    const bool active = (g >> 1) == t;
    const uint4* xfd = reinterpret_cast<const uint4*>(XF) + (g & 1) * 4 + t;
    const uint32_t* xq32 = reinterpret_cast<const uint32_t*>(XQ);
    float acc[kT][2];
#pragma unroll
    for (int u = 0; u < kT; ++u) acc[u][0] = acc[u][1] = 0.0f;
    // the B fragments of the warp's current block (with one chunk per row they are loaded once)
    uint4 bf[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) bf[i] = make_uint4(0u, 0u, 0u, 0u);
    uint32_t bq = 0u;
    float xs = 0.0f;
    int cur_kb = -1;

    // the activation limbs come from the preceding kernel in the stream
    asm volatile("griddepcontrol.wait;" ::: "memory");

    int slot = 0, par = 0;
    int q = 0;
    bool live = true;
    for (int it = blockIdx.x; it < nitems && live; it += gridDim.x, ++q) {
        for (int c = 0; c < nchunks; ++c) {
            if (!__all_sync(0xFFFFFFFFu, mbar_wait_ab(smem_u32(&full_bar[slot]), par, err, abortp))) {
                abort_flag = 1;
                live = false;
                break;
            }
            const int kb = c * kChunk + wb;
            if (kb < nblk) {
                if (kb != cur_kb) {
                    cur_kb = kb;
                    if (active) {
#pragma unroll
                        for (int i = 0; i < 8; ++i) bf[i] = __ldg(xfd + (kb * 8 + i) * NC * 4);
                    }
                    bq = g < 2 ? __ldg(xq32 + (kb * 4 + t) * NC + g) : 0u;
                    xs = __ldg(XS + kb);
                }
                const uint8_t* st = ring + slot * STAGE;
#pragma unroll
                for (int u = 0; u < kT; ++u)
                    unit_diag<Q, true>(st + u * HALF, lo, bf, bq, xs * 16777216.0f, xs * 1048576.0f, xs, ls, t,
                                       acc[u]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&empty_bar[slot]));
            if (++slot == kStages) {
                slot = 0;
                par ^= 1;
            }
        }
        if (!live) break;
        // ---- item done: this warp's partial sums into reduction slot q % kRedSlots
        const int rs = q & (kRedSlots - 1), use = q / kRedSlots;
        if (use >= 1 &&
            !__all_sync(0xFFFFFFFFu, mbar_wait_ab(smem_u32(&rempty_bar[rs]), (use - 1) & 1, err, abortp))) {
            abort_flag = 1;
            break;
        }
        float* rw = red + rs * RED + wb * kPitch + 16 * grp;
        const bool hr = (t & 1) != 0;
#pragma unroll
        for (int u = 0; u < kT; ++u) {
            // sum over the four t lanes of each row: lanes t = 0, 1 end with rows g and g + 8
            float k = hr ? acc[u][1] : acc[u][0];
            k += __shfl_xor_sync(0xFFFFFFFFu, hr ? acc[u][0] : acc[u][1], 1);
            k += __shfl_xor_sync(0xFFFFFFFFu, k, 2);
            if (t < 2) rw[kHalfRows * u + 8 * t + g] = k;
            acc[u][0] = acc[u][1] = 0.0f;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&rfull_bar[rs]));
    }
}

// Whether the tall kernel takes this batch-1 GEMV: Q4_K / Q5_K with its
// tensor map and at least four 64-row items per SM.
inline bool takes(uint32_t quant, const GemvArgs& a) {
    return (quant == kQ4_K || quant == kQ5_K) && a.batch == 1 && a.tmap &&
           (a.N + kItemRows - 1) / kItemRows >= 4ll * a.sm_count;
}

template <uint32_t Q>
void launch(const GemvArgs& a, const uint2* xf, const float* xs, const __half* xq, int* err, cudaStream_t s) {
    constexpr int smem = smem_for(Q);
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(gemv_b1_tall_kernel<Q>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        attr_set = true;
    }
    const int64_t items = (a.N + kItemRows - 1) / kItemRows;
    const int64_t grid = items < a.sm_count ? items : a.sm_count;
    const CUtensorMap map = *reinterpret_cast<const CUtensorMap*>(a.tmap);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    PeerOut po{};
    if (a.peers) po = *a.peers;
    cudaLaunchKernelEx(&cfg, gemv_b1_tall_kernel<Q>, (int)a.N, (int)(a.K / 256), xf, xs, xq, a.Y, err, map, po);
}

}  // namespace tall

// ============================================================ Q8_0, batch 1-2
//
// Q8_0 rows are 34-byte blocks, so per-lane global loads of a block are 2-byte
// loads (17 per block). Here a producer warp copies each 16-row x 32-block
// stage into a 4-deep shared-memory ring with one bulk copy per row (1088
// bytes: a row's 32 blocks are contiguous and 16-byte aligned when K is a
// multiple of 1024), and each consumer warp owns kRpw rows of the tile:
// lane l takes block l of every row of the stage, reads its 34 bytes as 9
// aligned words from shared memory and funnel-shifts the quants into place.
// The arithmetic and its order are those of the CUDA-core Q8_0 kernel (per
// block: 32 FMAs in index order, then d * acc into the lane's sum; lanes
// summed by a butterfly at the end of the row), so the results are the same.
namespace q8 {

constexpr int kRows = 16;                  // rows per tile: 4 per consumer warp
constexpr int kBlocks = 32;                // blocks per row and stage: one per lane
constexpr int kRowBytes = kBlocks * 34;    // 1088
constexpr int kStages = 4;
constexpr int kConsumers = 4;
constexpr int kRpw = kRows / kConsumers;   // rows per consumer warp
constexpr int kThreads = (kConsumers + 1) * 32;
constexpr int kStage = kRows * kRowBytes;  // 17408 bytes
// + 16: lane 31's ninth word of the last row of the last slot lies past the ring
constexpr int kRing = kStages * kStage + 16;
// the activations follow the ring: NB x K floats, at most this many bytes
constexpr int kMaxXBytes = 48 * 1024;
inline int smem_bytes(int nb, int64_t K) { return kRing + nb * (int)K * 4; }

template <int NB>
__global__ void __launch_bounds__(kThreads, 3)
gemv_q8_0_bulk_kernel(const uint8_t* __restrict__ W, int64_t row_bytes, int N, int nblk,
                      const float* __restrict__ X, float* __restrict__ Y, int64_t ldy, int* __restrict__ err) {
    // the next kernel may launch now: it reads this grid's outputs only after its own wait
    asm volatile("griddepcontrol.launch_dependents;");
    extern __shared__ __align__(16) uint8_t q8_ring[];
    // activations, float4 (chunk, word i, lane) of token b at ((b * chunks + chunk) * 8 + i) * 32 + lane:
    // the 32 lanes of one (chunk, i) read 512 contiguous bytes
    float4* xs = reinterpret_cast<float4*>(q8_ring + kRing);
    __shared__ __align__(8) uint64_t full_bar[kStages], empty_bar[kStages];
    __shared__ int abort_flag;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ntiles = (N + kRows - 1) / kRows;
    const int nchunks = nblk / kBlocks;
    const int my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int nstages = my_tiles * nchunks;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(smem_u32(&full_bar[i]), 1);
            mbar_init(smem_u32(&empty_bar[i]), kConsumers);
        }
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == kConsumers) {
        // ---------------- producer (the weights do not depend on the previous kernel)
        int issued = 0, tile = blockIdx.x, chunk = 0;
        for (int j = 0; j < nstages; ++j) {
            const int slot = j % kStages;
            bool ok = true;
            if (j >= kStages) ok = mbar_wait(smem_u32(&empty_bar[slot]), ((j / kStages) - 1) & 1, err);
            ok = __all_sync(0xFFFFFFFFu, ok) && __shfl_sync(0xFFFFFFFFu, *(volatile int*)&abort_flag, 0) == 0;
            if (!ok) {
                abort_flag = 1;
                break;
            }
            const uint32_t fb = smem_u32(&full_bar[slot]);
            if (lane == 0) mbar_expect_tx(fb, (uint32_t)kStage);
            __syncwarp();
            if (lane < kRows) {
                int row = tile * kRows + lane;
                row = row < N ? row : N - 1;  // rows past N repeat the last (never stored)
                const uint8_t* src = W + (int64_t)row * row_bytes + (int64_t)chunk * kRowBytes;
                bulk_g2s(smem_u32(q8_ring + slot * kStage + lane * kRowBytes), src, (uint32_t)kRowBytes, fb);
            }
            issued = j + 1;
            if (++chunk == nchunks) {
                chunk = 0;
                tile += gridDim.x;
            }
        }
        // drain: the copies of the last stages issued may still be in flight
        for (int j = max(0, issued - kStages); j < issued; ++j)
            mbar_wait(smem_u32(&full_bar[j % kStages]), (j / kStages) & 1, nullptr);
        return;
    }

    // ---------------- consumers: x comes from the preceding kernel in the stream;
    // the CTA's 128 consumer threads stage all of it once (the weights of the
    // first stages are in flight meanwhile)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    {
        const int n4 = NB * nblk * 8;  // float4s of x
        const float4* x4 = reinterpret_cast<const float4*>(X);
        for (int g = threadIdx.x; g < n4; g += kConsumers * 32) {
            const int b = g / (nblk * 8), r = g - b * (nblk * 8);
            const int c = r >> 8, ln = (r >> 3) & 31, i = r & 7;  // global float4 (chunk c, lane ln, word i)
            xs[((b * nchunks + c) * 8 + i) * 32 + ln] = __ldg(x4 + g);
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kConsumers * 32) : "memory");
    }
    // the quants of block `lane` start at byte 34 lane + 2 of a row: the aligned
    // word below it and the shift that brings them into place (0 or 16 bits)
    const uint32_t qoff = 34u * (uint32_t)lane + 2u;
    const uint32_t qword = qoff & ~3u, qshift = (qoff & 3u) * 8u;
    float sum[kRpw][NB];
#pragma unroll
    for (int r = 0; r < kRpw; ++r)
#pragma unroll
        for (int b = 0; b < NB; ++b) sum[r][b] = 0.0f;
    bool live = true;
    int tile = blockIdx.x, chunk = 0;
    for (int j = 0; j < nstages; ++j) {
        const int slot = j % kStages;
        if (live) {
            const bool ok = mbar_wait(smem_u32(&full_bar[slot]), (j / kStages) & 1, err);
            live = __all_sync(0xFFFFFFFFu, ok) && __shfl_sync(0xFFFFFFFFu, *(volatile int*)&abort_flag, 0) == 0;
            if (!live) abort_flag = 1;
        }
        if (live) {
            const uint8_t* st = q8_ring + slot * kStage + (kRpw * warp) * kRowBytes;
            uint32_t q[kRpw][8];
            float d[kRpw];
#pragma unroll
            for (int r = 0; r < kRpw; ++r) {
                const uint8_t* row = st + r * kRowBytes;
                d[r] = f16_bits_to_f32(*reinterpret_cast<const unsigned short*>(row + 34 * lane));
                const uint32_t* wp = reinterpret_cast<const uint32_t*>(row + qword);
                uint32_t wv[9];
#pragma unroll
                for (int k = 0; k < 9; ++k) wv[k] = wp[k];
#pragma unroll
                for (int i = 0; i < 8; ++i) q[r][i] = __funnelshift_r(wv[i], wv[i + 1], qshift) ^ 0x80808080u;
            }
            float acc[kRpw][NB];
#pragma unroll
            for (int r = 0; r < kRpw; ++r)
#pragma unroll
                for (int b = 0; b < NB; ++b) acc[r][b] = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                float4 xv[NB];
#pragma unroll
                for (int b = 0; b < NB; ++b) xv[b] = xs[((b * nchunks + chunk) * 8 + i) * 32 + lane];
#pragma unroll
                for (int r = 0; r < kRpw; ++r) {
                    // 2^23 + (q + 128) - (2^23 + 128) = q, exactly
                    const float f0 = __uint_as_float(__byte_perm(q[r][i], 0x4B000000u, 0x7440u)) - 8388736.0f;
                    const float f1 = __uint_as_float(__byte_perm(q[r][i], 0x4B000000u, 0x7441u)) - 8388736.0f;
                    const float f2 = __uint_as_float(__byte_perm(q[r][i], 0x4B000000u, 0x7442u)) - 8388736.0f;
                    const float f3 = __uint_as_float(__byte_perm(q[r][i], 0x4B000000u, 0x7443u)) - 8388736.0f;
#pragma unroll
                    for (int b = 0; b < NB; ++b) {
                        acc[r][b] = fmaf(f0, xv[b].x, acc[r][b]);
                        acc[r][b] = fmaf(f1, xv[b].y, acc[r][b]);
                        acc[r][b] = fmaf(f2, xv[b].z, acc[r][b]);
                        acc[r][b] = fmaf(f3, xv[b].w, acc[r][b]);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < kRpw; ++r)
#pragma unroll
                for (int b = 0; b < NB; ++b) sum[r][b] = fmaf(d[r], acc[r][b], sum[r][b]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&empty_bar[slot]));
        if (++chunk == nchunks) {
            // the tile's rows are done: each warp sums its own rows over the lanes
#pragma unroll
            for (int r = 0; r < kRpw; ++r)
#pragma unroll
                for (int b = 0; b < NB; ++b) {
                    float v = sum[r][b];
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
                    const int row = tile * kRows + kRpw * warp + r;
                    if (live && lane == 0 && row < N) Y[b * ldy + row] = v;
                    sum[r][b] = 0.0f;
                }
            chunk = 0;
            tile += gridDim.x;
        }
    }
}

template <int NB>
void launch(const GemvArgs& a, int* err, cudaStream_t s) {
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(gemv_q8_0_bulk_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kRing + kMaxXBytes);
        configured = true;
    }
    const int smem = smem_bytes(NB, a.K);
    static int last_smem = -1, per_sm = 1;  // resident CTAs per SM at the last size asked
    if (smem != last_smem) {
        int n = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemv_q8_0_bulk_kernel<NB>, kThreads, smem);
        per_sm = n < 1 ? 1 : n;
        last_smem = smem;
    }
    const int64_t ntiles = (a.N + kRows - 1) / kRows;
    int64_t grid = (int64_t)a.sm_count * per_sm;
    if (grid > ntiles) grid = ntiles;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, gemv_q8_0_bulk_kernel<NB>, a.W, a.row_bytes, (int)a.N, (int)(a.K / 32), a.X, a.Y,
                       ldy_of(a), err);
}

}  // namespace q8

}  // namespace

bool gemv_q8_0_bulk_supported(const GemvArgs& a) {
    return a.batch >= 1 && a.batch <= 2 && a.K % 1024 == 0 && a.K > 0 && a.batch * a.K * 4 <= q8::kMaxXBytes && a.N > 0 &&
           a.N < (1ll << 31) && a.row_bytes == a.K / 32 * 34 && ((uintptr_t)a.W % 16) == 0 &&
           ((uintptr_t)a.X % 16) == 0 && !a.peers;
}

void launch_gemv_q8_0_bulk(const GemvArgs& a, int* err, cudaStream_t s) {
    if (a.batch == 1) q8::launch<1>(a, err, s);
    else q8::launch<2>(a, err, s);
}

// The 3-D view of a Q4_K / Q5_K matrix the tensor-core GEMV copies from:
// [8-byte units x 16][128-byte lines x row_bytes/128][rows], box
// [16][kChunk*BB/128][16] with 128-byte swizzle. Needs whole 8-block chunks
// per row (K a multiple of 2048). Returns false when not applicable.
bool encode_gemv_tmap(uint32_t quant, const void* base, int64_t rows, int64_t row_bytes, void* out128) {
    if (quant != kQ4_K && quant != kQ5_K) return false;
    const int bb = block_bytes(quant);
    if (rows <= 0 || row_bytes % ((int64_t)kChunk * bb) != 0 || ((uintptr_t)base % 16) != 0) return false;
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn)
            return false;
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    const cuuint64_t dims[3] = {16, (cuuint64_t)(row_bytes / 128), (cuuint64_t)rows};
    const cuuint64_t strides[2] = {128, (cuuint64_t)row_bytes};
    const cuuint32_t box[3] = {16, (cuuint32_t)(kChunk * bb / 128), (cuuint32_t)kTileRows};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = encode(reinterpret_cast<CUtensorMap*>(out128), CU_TENSOR_MAP_DATA_TYPE_UINT64, 3,
                        const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// workspace of one call of up to 8 tokens: XF (nblk*64*2B uint2), XS
// (B*nblk float), XQ (nblk*4*2B half2); larger batches take one such slice
// (256-byte aligned) per 8-token chunk plus one for the remainder.
static int64_t work_bytes_8(int64_t K, int batch) {
    const int64_t nblk = K / 256;
    const int64_t b = nblk * 64 * 2 * batch * 8 + (int64_t)batch * nblk * 4 + nblk * 4 * 2 * batch * 4 + 512;
    return (b + 255) / 256 * 256;
}

int64_t gemv_mma_work_bytes(int64_t K, int batch) {
    if (batch <= 8) return work_bytes_8(K, batch);
    return (batch / 8) * work_bytes_8(K, 8) + (batch % 8 ? work_bytes_8(K, batch % 8) : 0);
}

bool gemv_mma_supported(uint32_t quant, const GemvArgs& a) {
    return (quant == kQ4_K || quant == kQ5_K) && a.K % 256 == 0 && a.batch >= 1 && a.batch <= 4096 &&
           a.N < (1ll << 31) && a.N * a.batch < (1ll << 31) && a.K < (1ll << 26) &&
           (a.row_bytes % 16) == 0 && ((uintptr_t)a.W % 16) == 0 && ((uintptr_t)a.X % 16) == 0;
}

// x limbs into `work` (gemv_mma_work_bytes), then the tensor-core GEMV.
// With prep = false the limbs already in `work` are reused: they must come
// from a call on the same stream with the same x, K and batch.
int launch_gemv_mma(uint32_t quant, const GemvArgs& a, void* work, int* err, cudaStream_t s, bool prep) {
    const int nblk = (int)(a.K / 256);
    const int full = a.batch > 8 ? a.batch / 8 : 0;  // 8-token chunks on grid.y
    const int nb = full ? 8 : a.batch;
    const unsigned chunks = full ? (unsigned)full : 1u;
    const int64_t chunk_bytes = work_bytes_8(a.K, nb);
    char* base = reinterpret_cast<char*>(work);
    uint2* xf = reinterpret_cast<uint2*>(base);
    const int64_t xf_bytes = (int64_t)nblk * 64 * 2 * nb * 8;
    float* xs = reinterpret_cast<float*>(base + xf_bytes);
    const int64_t xs_bytes = ((int64_t)nb * nblk * 4 + 255) / 256 * 256;
    __half* xq = reinterpret_cast<__half*>(base + xf_bytes + xs_bytes);
    const int64_t warps = (int64_t)nblk * nb;
    if (prep) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)((warps + 7) / 8), chunks);
        cfg.blockDim = dim3(256);
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaLaunchKernelEx(&cfg, prep_x_limbs_kernel, a.X, a.K, nb, xf, xs, xq, chunk_bytes);
    }
    GemvArgs c = a;
    c.batch = nb;
    const bool tm = a.tmap != nullptr;
    if (!full && tall::takes(quant, c)) {
        if (quant == kQ4_K) tall::launch<kQ4_K>(c, xf, xs, xq, err, s);
        else tall::launch<kQ5_K>(c, xf, xs, xq, err, s);
        return 0;
    }
    if (quant == kQ4_K) tm ? dispatch_mma<kQ4_K, true>(c, xf, xs, xq, err, s, chunks, chunk_bytes)
                           : dispatch_mma<kQ4_K, false>(c, xf, xs, xq, err, s, chunks, chunk_bytes);
    else tm ? dispatch_mma<kQ5_K, true>(c, xf, xs, xq, err, s, chunks, chunk_bytes)
            : dispatch_mma<kQ5_K, false>(c, xf, xs, xq, err, s, chunks, chunk_bytes);
    if (full && a.batch % 8) {  // the remaining tokens, after the chunks' workspace
        GemvArgs r = a;
        r.X = a.X + (int64_t)full * 8 * a.K;
        r.Y = a.Y + (int64_t)full * 8 * ldy_of(a);
        r.batch = a.batch % 8;
        PeerOut pr{};
        if (a.peers) {
            pr = *a.peers;
            pr.off += (int64_t)full * 8 * ldy_of(a);
            r.peers = &pr;
        }
        return launch_gemv_mma(quant, r, base + (int64_t)full * chunk_bytes, err, s, prep);
    }
    return 0;
}

}  // namespace strata
