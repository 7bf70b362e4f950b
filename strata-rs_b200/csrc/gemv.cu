// gemv.cu — fused dequant-GEMV for decode (batch 1..8): y[b][n] = sum_k W[n][k] x[b][k].
//
// Replaces the per-row dequantize + f64 dot of ops::gemv
// (crates/strata-core/src/ops.rs:14-28) for Q4_K / Q5_K / Q6_K / Q8_0 weights.
//
// Shape of the work: one warp owns R consecutive output rows (a row tile);
// its 32 lanes stride over the row in "units" of 32 weights. A unit of a
// K-quant is 16 bytes of packed quants (one 128-bit load) plus the block's
// scales; each lane decodes its unit in registers for all R rows, reusing the
// activation values it loaded once for the R rows. Accumulation is fp32 and
// the lanes' partial sums are reduced with warp shuffles.
//
// Nibble -> float without an int->float conversion: a byte 1qqqq000 placed as
// bits 23..16 under 0x3F gives the float 1 + q/16, exactly. Summing
// (1 + q/16)·x over a run and subtracting the run's sum of x yields sum(q·x)/16.
// Q5_K uses 1 + q/32 and Q6_K 1 + u/64 the same way.
#include "dequant_elem.cuh"
#include "kernels.cuh"

namespace strata {

namespace {

__device__ __forceinline__ float as_f(uint32_t u) { return __uint_as_float(u); }

// byte k of t (k = 0..3) under 0x3F: the float 0x3F | t.byte_k | 00 | 00
template <int K>
__device__ __forceinline__ float mag(uint32_t t) {
    return as_f(__byte_perm(t, 0x3F000000u, 0x7044u | (K << 8)));
}

__device__ __forceinline__ float dot4_mag(uint32_t t, float4 x, float acc) {
    acc = fmaf(mag<0>(t), x.x, acc);
    acc = fmaf(mag<1>(t), x.y, acc);
    acc = fmaf(mag<2>(t), x.z, acc);
    acc = fmaf(mag<3>(t), x.w, acc);
    return acc;
}

__device__ __forceinline__ float hsum4(float4 v) { return (v.x + v.y) + (v.z + v.w); }

__device__ __forceinline__ uint4 ldg16(const uint8_t* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ float4 ldx4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// Per-type description of a 32-weight unit: 8 units per 256-element block
// for the K-quants. Each unit yields two runs of 16 weights (run A, run B)
// with one (scale, min) pair each; the element offsets of the runs within the
// block are baseA/baseB.
struct UnitGeom {
    int baseA, baseB;
};

template <uint32_t Q>
__device__ __forceinline__ UnitGeom unit_geom(int t) {
    if constexpr (Q == kQ4_K || Q == kQ5_K) {
        int c = t >> 1, h = t & 1;
        return {64 * c + 16 * h, 64 * c + 32 + 16 * h};
    } else {  // Q6_K
        int H = t >> 2, u = t & 3;
        int base = 128 * H + 32 * (u >> 1) + 16 * (u & 1);
        return {base, base + 64};
    }
}

// Loaded state of one unit of one row.
struct UnitData {
    uint4 q;     // 16 bytes of low-4-bit quants
    uint4 h;     // Q5_K: 16 bytes of qh; Q6_K: 16 bytes of qh
    float cA, kA, cB, kB;  // run A: sum = cA * acc - kA * sx ; same for run B
};

// Load the bytes of unit t of the block at `blk` and fold its scales into the
// run coefficients.
template <uint32_t Q>
__device__ __forceinline__ void load_unit(const uint8_t* __restrict__ blk, int t, UnitData& u) {
    if constexpr (Q == kQ4_K) {
        int c = t >> 1, h = t & 1;
        uint4 hd = ldg16(blk);  // d, dmin, scales[12]
        u.q = ldg16(blk + 16 + 32 * c + 16 * h);
        float d = f16_bits_to_f32(hd.x & 0xFFFFu), dm = f16_bits_to_f32(hd.x >> 16);
        uint32_t sl, sh, ml, mh;
        scales_k4_packed(hd.y, hd.z, hd.w, sl, sh, ml, mh);
        uint32_t sw = (c < 2) ? sl : sh, mw = (c < 2) ? ml : mh;
        int sft = 16 * (c & 1);
        float sA = (float)((sw >> sft) & 0xFFu), sB = (float)((sw >> (sft + 8)) & 0xFFu);
        float mA = (float)((mw >> sft) & 0xFFu), mB = (float)((mw >> (sft + 8)) & 0xFFu);
        // sum_l (d sA q_l - dm mA) x_l = 16 d sA * acc - (16 d sA + dm mA) * sx
        u.cA = 16.0f * d * sA; u.kA = u.cA + dm * mA;
        u.cB = 16.0f * d * sB; u.kB = u.cB + dm * mB;
    } else if constexpr (Q == kQ5_K) {
        int c = t >> 1, h = t & 1;
        uint4 hd = ldg16(blk);
        u.h = ldg16(blk + 16 + 16 * h);
        u.q = ldg16(blk + 48 + 32 * c + 16 * h);
        float d = f16_bits_to_f32(hd.x & 0xFFFFu), dm = f16_bits_to_f32(hd.x >> 16);
        uint32_t sl, sh, ml, mh;
        scales_k4_packed(hd.y, hd.z, hd.w, sl, sh, ml, mh);
        uint32_t sw = (c < 2) ? sl : sh, mw = (c < 2) ? ml : mh;
        int sft = 16 * (c & 1);
        float sA = (float)((sw >> sft) & 0xFFu), sB = (float)((sw >> (sft + 8)) & 0xFFu);
        float mA = (float)((mw >> sft) & 0xFFu), mB = (float)((mw >> (sft + 8)) & 0xFFu);
        u.cA = 32.0f * d * sA; u.kA = u.cA + dm * mA;
        u.cB = 32.0f * d * sB; u.kB = u.cB + dm * mB;
    } else {  // Q6_K: 210-byte blocks are only 2-byte aligned
        int H = t >> 2, uu = t & 3;
        const uint8_t* ql = blk + 64 * H + 16 * uu;
        const uint8_t* qh = blk + 128 + 32 * H + 16 * (uu & 1);
        const unsigned short* q16 = reinterpret_cast<const unsigned short*>(ql);
        const unsigned short* h16 = reinterpret_cast<const unsigned short*>(qh);
        uint32_t w[4], hw[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            w[i] = (uint32_t)__ldg(q16 + 2 * i) | ((uint32_t)__ldg(q16 + 2 * i + 1) << 16);
            hw[i] = (uint32_t)__ldg(h16 + 2 * i) | ((uint32_t)__ldg(h16 + 2 * i + 1) << 16);
        }
        u.q = make_uint4(w[0], w[1], w[2], w[3]);
        u.h = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        float d = f16_bits_to_f32(__ldg(reinterpret_cast<const unsigned short*>(blk + 208)));
        float sA = (float)__ldg(blk + 192 + 8 * H + uu);
        float sB = (float)__ldg(blk + 192 + 8 * H + uu + 4);
        // q = u - 32, u = 64 (mag - 1): sum q x = 64 acc - 96 sx
        u.cA = 64.0f * d * sA; u.kA = 96.0f * d * sA;
        u.cB = 64.0f * d * sB; u.kB = 96.0f * d * sB;
    }
}

// Magic bytes (1qqqq000-style) of word i of the unit: run A (lo) and run B (hi).
template <uint32_t Q>
__device__ __forceinline__ void unit_word(const UnitData& u, int t, int i, uint32_t& lo, uint32_t& hi) {
    uint32_t w = (i == 0) ? u.q.x : (i == 1) ? u.q.y : (i == 2) ? u.q.z : u.q.w;
    if constexpr (Q == kQ4_K) {
        lo = ((w << 3) & 0x78787878u) | 0x80808080u;
        hi = ((w >> 1) & 0x78787878u) | 0x80808080u;
    } else if constexpr (Q == kQ5_K) {
        uint32_t hw = (i == 0) ? u.h.x : (i == 1) ? u.h.y : (i == 2) ? u.h.z : u.h.w;
        int c = t >> 1;
        lo = ((w << 2) & 0x3C3C3C3Cu) | (((hw >> (2 * c)) & 0x01010101u) << 6) | 0x80808080u;
        hi = ((w >> 2) & 0x3C3C3C3Cu) | (((hw >> (2 * c + 1)) & 0x01010101u) << 6) | 0x80808080u;
    } else {  // Q6_K
        uint32_t hw = (i == 0) ? u.h.x : (i == 1) ? u.h.y : (i == 2) ? u.h.z : u.h.w;
        int s = 2 * ((t & 3) >> 1);
        lo = ((w << 1) & 0x1E1E1E1Eu) | (((hw >> s) & 0x03030303u) << 5) | 0x80808080u;
        hi = ((w >> 3) & 0x1E1E1E1Eu) | (((hw >> (s + 4)) & 0x03030303u) << 5) | 0x80808080u;
    }
}

// K-quant GEMV: each warp owns R rows; grid-stride over row tiles.
template <uint32_t Q, int NB, int R, int WARPS>
__global__ void __launch_bounds__(WARPS * 32)
gemv_kquant_kernel(const uint8_t* __restrict__ W, int64_t row_bytes, int64_t N, int64_t K,
                   const float* __restrict__ X, float* __restrict__ Y, int64_t ldy) {
    // token chunk blockIdx.y: rows [NB y, NB y + NB) of X and Y
    X += (int64_t)blockIdx.y * NB * K;
    Y += (int64_t)blockIdx.y * NB * ldy;
    constexpr int BB = block_bytes(Q);
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t units = (K / 256) * 8;
    const int64_t tiles = (N + R - 1) / R;
    for (int64_t tile = (int64_t)blockIdx.x * WARPS + warp; tile < tiles; tile += (int64_t)gridDim.x * WARPS) {
        const int64_t row0 = tile * R;
        float sum[R][NB];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int b = 0; b < NB; ++b) sum[r][b] = 0.0f;

        for (int64_t un = lane; un < units; un += 32) {
            const int64_t blk_i = un >> 3;
            const int t = (int)(un & 7);
            UnitData ud[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                int64_t row = row0 + r < N ? row0 + r : N - 1;
                load_unit<Q>(W + row * row_bytes + blk_i * BB, t, ud[r]);
            }
            const UnitGeom g = unit_geom<Q>(t);
            const int64_t kA = blk_i * 256 + g.baseA, kB = blk_i * 256 + g.baseB;
            float sxA[NB], sxB[NB], accA[R][NB], accB[R][NB];
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                sxA[b] = sxB[b] = 0.0f;
#pragma unroll
                for (int r = 0; r < R; ++r) accA[r][b] = accB[r][b] = 0.0f;
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float4 xa[NB], xb[NB];
#pragma unroll
                for (int b = 0; b < NB; ++b) {
                    xa[b] = ldx4(X + b * K + kA + 4 * i);
                    xb[b] = ldx4(X + b * K + kB + 4 * i);
                    sxA[b] += hsum4(xa[b]);
                    sxB[b] += hsum4(xb[b]);
                }
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    uint32_t lo, hi;
                    unit_word<Q>(ud[r], t, i, lo, hi);
#pragma unroll
                    for (int b = 0; b < NB; ++b) {
                        accA[r][b] = dot4_mag(lo, xa[b], accA[r][b]);
                        accB[r][b] = dot4_mag(hi, xb[b], accB[r][b]);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int b = 0; b < NB; ++b)
                    sum[r][b] += (ud[r].cA * accA[r][b] - ud[r].kA * sxA[b]) +
                                 (ud[r].cB * accB[r][b] - ud[r].kB * sxB[b]);
        }
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                float v = warp_sum(sum[r][b]);
                if (lane == 0 && row0 + r < N) Y[b * ldy + row0 + r] = v;
            }
    }
}

// Q8_0 GEMV: one lane per 34-byte block (32 weights), R rows per warp.
// Blocks are 2-byte aligned, so the 32 quants are gathered with 16-bit loads.
template <int NB, int R, int WARPS>
__global__ void __launch_bounds__(WARPS * 32)
gemv_q8_0_kernel(const uint8_t* __restrict__ W, int64_t row_bytes, int64_t N, int64_t K,
                 const float* __restrict__ X, float* __restrict__ Y, int64_t ldy) {
    X += (int64_t)blockIdx.y * NB * K;
    Y += (int64_t)blockIdx.y * NB * ldy;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t nblk = K / 32;
    const int64_t tiles = (N + R - 1) / R;
    for (int64_t tile = (int64_t)blockIdx.x * WARPS + warp; tile < tiles; tile += (int64_t)gridDim.x * WARPS) {
        const int64_t row0 = tile * R;
        float sum[R][NB];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int b = 0; b < NB; ++b) sum[r][b] = 0.0f;
        for (int64_t bi = lane; bi < nblk; bi += 32) {
            uint32_t q[R][8];
            float d[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                int64_t row = row0 + r < N ? row0 + r : N - 1;
                const unsigned short* p = reinterpret_cast<const unsigned short*>(W + row * row_bytes + bi * 34);
                d[r] = f16_bits_to_f32(__ldg(p));
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    q[r][i] = ((uint32_t)__ldg(p + 1 + 2 * i) | ((uint32_t)__ldg(p + 2 + 2 * i) << 16)) ^ 0x80808080u;
            }
            float acc[R][NB];
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int b = 0; b < NB; ++b) acc[r][b] = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                float4 xv[NB];
#pragma unroll
                for (int b = 0; b < NB; ++b) xv[b] = ldx4(X + b * K + bi * 32 + 4 * i);
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    // 2^23 + (q + 128) - (2^23 + 128) = q, exactly
                    float f0 = as_f(__byte_perm(q[r][i], 0x4B000000u, 0x7440u)) - 8388736.0f;
                    float f1 = as_f(__byte_perm(q[r][i], 0x4B000000u, 0x7441u)) - 8388736.0f;
                    float f2 = as_f(__byte_perm(q[r][i], 0x4B000000u, 0x7442u)) - 8388736.0f;
                    float f3 = as_f(__byte_perm(q[r][i], 0x4B000000u, 0x7443u)) - 8388736.0f;
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
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int b = 0; b < NB; ++b) sum[r][b] = fmaf(d[r], acc[r][b], sum[r][b]);
        }
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                float v = warp_sum(sum[r][b]);
                if (lane == 0 && row0 + r < N) Y[b * ldy + row0 + r] = v;
            }
    }
}

// Plain float weights (F32 / F16 / BF16): one warp per row, lanes stride over K.
template <uint32_t Q, int NB>
__global__ void gemv_float_kernel(const uint8_t* __restrict__ W, int64_t row_bytes, int64_t N, int64_t K,
                                  const float* __restrict__ X, float* __restrict__ Y, int64_t ldy) {
    X += (int64_t)blockIdx.y * NB * K;
    Y += (int64_t)blockIdx.y * NB * ldy;
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    for (int64_t row = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5); row < N; row += (int64_t)gridDim.x * warps) {
        const uint8_t* wr = W + row * row_bytes;
        float acc[NB];
#pragma unroll
        for (int b = 0; b < NB; ++b) acc[b] = 0.0f;
        for (int64_t k = lane; k < K; k += 32) {
            float w;
            if constexpr (Q == kF32) w = __ldg(reinterpret_cast<const float*>(wr) + k);
            else if constexpr (Q == kF16) w = f16_bits_to_f32(__ldg(reinterpret_cast<const unsigned short*>(wr) + k));
            else w = __uint_as_float((uint32_t)__ldg(reinterpret_cast<const unsigned short*>(wr) + k) << 16);
#pragma unroll
            for (int b = 0; b < NB; ++b) acc[b] = fmaf(w, __ldg(X + b * K + k), acc[b]);
        }
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            float v = warp_sum(acc[b]);
            if (lane == 0) Y[b * ldy + row] = v;
        }
    }
}

// The other block formats (Q4_0 .. NVFP4): one warp per row, lanes stride over
// K, each weight decoded by dequant_elem (the reference's exact values), fp32
// FMAs. Not a fused fast path: these formats are outside the benchmark.
template <uint32_t Q, int NB>
__global__ void gemv_elem_kernel(const uint8_t* __restrict__ W, int64_t row_bytes, int64_t N, int64_t K,
                                 const float* __restrict__ X, float* __restrict__ Y, int64_t ldy) {
    constexpr int BE = block_elems(Q), BB = block_bytes(Q);
    X += (int64_t)blockIdx.y * NB * K;
    Y += (int64_t)blockIdx.y * NB * ldy;
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    for (int64_t row = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5); row < N; row += (int64_t)gridDim.x * warps) {
        const uint8_t* wr = W + row * row_bytes;
        float acc[NB];
#pragma unroll
        for (int b = 0; b < NB; ++b) acc[b] = 0.0f;
        for (int64_t k = lane; k < K; k += 32) {
            const float w = dequant_elem<Q>(wr + (k / BE) * BB, (int)(k % BE));
#pragma unroll
            for (int b = 0; b < NB; ++b) acc[b] = fmaf(w, __ldg(X + b * K + k), acc[b]);
        }
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            float v = warp_sum(acc[b]);
            if (lane == 0) Y[b * ldy + row] = v;
        }
    }
}

template <uint32_t Q, int NB>
void launch_elem(const GemvArgs& a, cudaStream_t s, unsigned chunks = 1) {
    int64_t grid = (a.N + 7) / 8;
    int64_t cap = (int64_t)a.sm_count * 16;
    if (grid > cap) grid = cap;
    gemv_elem_kernel<Q, NB><<<dim3((unsigned)grid, chunks), 256, 0, s>>>(a.W, a.row_bytes, a.N, a.K, a.X, a.Y,
                                                                         ldy_of(a));
}

template <uint32_t Q>
int dispatch_elem(const GemvArgs& a, cudaStream_t s) {
    switch (a.batch) {
    case 1: launch_elem<Q, 1>(a, s); break;
    case 2: launch_elem<Q, 2>(a, s); break;
    case 3: launch_elem<Q, 3>(a, s); break;
    case 4: launch_elem<Q, 4>(a, s); break;
    case 5: launch_elem<Q, 5>(a, s); break;
    case 6: launch_elem<Q, 6>(a, s); break;
    case 7: launch_elem<Q, 7>(a, s); break;
    case 8: launch_elem<Q, 8>(a, s); break;
    default: return -1;
    }
    return 0;
}

#define STRATA_OTHER_FORMATS(X) \
    X(kQ4_0) X(kQ4_1) X(kQ5_0) X(kQ5_1) X(kQ8_1) X(kQ2_K) X(kQ3_K) X(kIQ4_NL) X(kIQ4_XS) X(kMXFP4) X(kNVFP4) X(kQ2_0)

template <uint32_t Q, int NB, int R>
void launch_kq(const GemvArgs& a, cudaStream_t s, unsigned chunks = 1) {
    constexpr int WARPS = 4;
    int64_t tiles = (a.N + R - 1) / R;
    int64_t grid = (tiles + WARPS - 1) / WARPS;
    int64_t cap = (int64_t)a.sm_count * 8;
    if (grid > cap) grid = cap;
    gemv_kquant_kernel<Q, NB, R, WARPS><<<dim3((unsigned)grid, chunks), WARPS * 32, 0, s>>>(a.W, a.row_bytes, a.N,
                                                                                       a.K, a.X, a.Y, ldy_of(a));
}

template <int NB, int R>
void launch_q8(const GemvArgs& a, cudaStream_t s, unsigned chunks = 1) {
    constexpr int WARPS = 4;
    int64_t tiles = (a.N + R - 1) / R;
    int64_t grid = (tiles + WARPS - 1) / WARPS;
    int64_t cap = (int64_t)a.sm_count * 8;
    if (grid > cap) grid = cap;
    gemv_q8_0_kernel<NB, R, WARPS><<<dim3((unsigned)grid, chunks), WARPS * 32, 0, s>>>(a.W, a.row_bytes, a.N, a.K,
                                                                                  a.X, a.Y, ldy_of(a));
}

template <uint32_t Q, int NB>
void launch_float(const GemvArgs& a, cudaStream_t s, unsigned chunks = 1) {
    int64_t grid = (a.N + 7) / 8;
    int64_t cap = (int64_t)a.sm_count * 16;
    if (grid > cap) grid = cap;
    gemv_float_kernel<Q, NB><<<dim3((unsigned)grid, chunks), 256, 0, s>>>(a.W, a.row_bytes, a.N, a.K, a.X, a.Y,
                                                                          ldy_of(a));
}

// Rows per warp by batch: more rows share each activation load when the batch
// is small; fewer when every row already carries NB accumulators.
template <uint32_t Q>
int dispatch_kq(const GemvArgs& a, cudaStream_t s) {
    switch (a.batch) {
    case 1: launch_kq<Q, 1, 4>(a, s); break;
    case 2: launch_kq<Q, 2, 2>(a, s); break;
    case 3: launch_kq<Q, 3, 2>(a, s); break;
    case 4: launch_kq<Q, 4, 2>(a, s); break;
    case 5: launch_kq<Q, 5, 1>(a, s); break;
    case 6: launch_kq<Q, 6, 1>(a, s); break;
    case 7: launch_kq<Q, 7, 1>(a, s); break;
    case 8: launch_kq<Q, 8, 1>(a, s); break;
    default: return -1;
    }
    return 0;
}

int dispatch_q8(const GemvArgs& a, cudaStream_t s) {
    switch (a.batch) {
    case 1: launch_q8<1, 4>(a, s); break;
    case 2: launch_q8<2, 2>(a, s); break;
    case 3: launch_q8<3, 2>(a, s); break;
    case 4: launch_q8<4, 2>(a, s); break;
    case 5: launch_q8<5, 1>(a, s); break;
    case 6: launch_q8<6, 1>(a, s); break;
    case 7: launch_q8<7, 1>(a, s); break;
    case 8: launch_q8<8, 1>(a, s); break;
    default: return -1;
    }
    return 0;
}

template <uint32_t Q>
int dispatch_float(const GemvArgs& a, cudaStream_t s) {
    switch (a.batch) {
    case 1: launch_float<Q, 1>(a, s); break;
    case 2: launch_float<Q, 2>(a, s); break;
    case 3: launch_float<Q, 3>(a, s); break;
    case 4: launch_float<Q, 4>(a, s); break;
    case 5: launch_float<Q, 5>(a, s); break;
    case 6: launch_float<Q, 6>(a, s); break;
    case 7: launch_float<Q, 7>(a, s); break;
    case 8: launch_float<Q, 8>(a, s); break;
    default: return -1;
    }
    return 0;
}

}  // namespace

// Batches above 8 run as full 8-token chunks (one launch, the chunk index on
// grid.y) plus one launch for the remainder.
static int launch_gemv_chunks(uint32_t quant, const GemvArgs& a, unsigned chunks, cudaStream_t s) {
    switch (quant) {
    case kQ4_K: launch_kq<kQ4_K, 8, 1>(a, s, chunks); return 0;
    case kQ5_K: launch_kq<kQ5_K, 8, 1>(a, s, chunks); return 0;
    case kQ6_K: launch_kq<kQ6_K, 8, 1>(a, s, chunks); return 0;
    case kQ8_0: launch_q8<8, 1>(a, s, chunks); return 0;
    case kF32: launch_float<kF32, 8>(a, s, chunks); return 0;
    case kF16: launch_float<kF16, 8>(a, s, chunks); return 0;
    case kBF16: launch_float<kBF16, 8>(a, s, chunks); return 0;
#define STRATA_CHUNK_CASE(QQ) \
    case QQ: launch_elem<QQ, 8>(a, s, chunks); return 0;
        STRATA_OTHER_FORMATS(STRATA_CHUNK_CASE)
#undef STRATA_CHUNK_CASE
    default: return -1;
    }
}

int launch_gemv(uint32_t quant, const GemvArgs& a, cudaStream_t s) {
    if (a.N <= 0 || a.batch <= 0) return 0;
    if (a.batch > 8) {
        const int full = a.batch / 8, rem = a.batch % 8;
        if (launch_gemv_chunks(quant, a, (unsigned)full, s)) return -1;
        if (rem == 0) return 0;
        GemvArgs r = a;
        r.X = a.X + (int64_t)full * 8 * a.K;
        r.Y = a.Y + (int64_t)full * 8 * ldy_of(a);
        r.batch = rem;
        return launch_gemv(quant, r, s);
    }
    switch (quant) {
    case kQ4_K: return dispatch_kq<kQ4_K>(a, s);
    case kQ5_K: return dispatch_kq<kQ5_K>(a, s);
    case kQ6_K: return dispatch_kq<kQ6_K>(a, s);
    case kQ8_0: return dispatch_q8(a, s);
    case kF32: return dispatch_float<kF32>(a, s);
    case kF16: return dispatch_float<kF16>(a, s);
    case kBF16: return dispatch_float<kBF16>(a, s);
#define STRATA_ELEM_CASE(QQ) \
    case QQ: return dispatch_elem<QQ>(a, s);
        STRATA_OTHER_FORMATS(STRATA_ELEM_CASE)
#undef STRATA_ELEM_CASE
    default: return -1;
    }
}

}  // namespace strata
