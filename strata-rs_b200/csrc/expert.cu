// expert.cu — expert GEMV on strata's 3-D expert layout.
//
// ops::expert_gemv (crates/strata-core/src/ops.rs:169-195) computes
//   y[c] = sum_i x[i] * W_e[i][c]
// over an expert tensor stored [n_expert][rows = IN][cols = OUT] with every
// IN row quantized along OUT (crates/strata-core/src/weights.rs:11-34). A
// thread therefore owns a fixed slice of OUT columns (16 of them: 8 bytes of
// packed quants for a K-quant) and walks IN rows, scaling each dequantized
// row slice by x[i]. Row ranges are split across CTAs; the per-range partial
// sums go to a workspace and a second kernel adds them in a fixed order, so
// results are deterministic run to run.
#include "dequant_elem.cuh"
#include "kernels.cuh"

namespace strata {

namespace {

constexpr int kEgThreads = 256;
constexpr int kEgTok = 4;  // tokens per pass

__device__ __forceinline__ uint32_t rd16g(const uint8_t* p) {
    return (uint32_t)__ldg(p) | ((uint32_t)__ldg(p + 1) << 8);
}

// Columns covered by unit t of a block: cols [colA, colA+8) and [colB, colB+8).
template <uint32_t Q>
__device__ __forceinline__ void unit16_cols(int t, int& colA, int& colB) {
    if constexpr (Q == kQ4_K || Q == kQ5_K) {
        int c = t >> 2, p = t & 3;
        colA = 64 * c + 8 * p; colB = colA + 32;
    } else if constexpr (Q == kQ6_K) {
        int H = t >> 3, u = t & 7;
        int l = 8 * (u & 3);
        colA = 128 * H + l + ((u >= 4) ? 32 : 0); colB = colA + 64;
    } else {  // Q8_0 and the other formats: unit t = 16 consecutive columns
        colA = 16 * t; colB = colA + 8;
    }
}

template <uint32_t Q>
__host__ __device__ constexpr int units16_per_block() {
    return (Q == kQ4_K || Q == kQ5_K || Q == kQ6_K) ? 16 : block_elems(Q) / 16;  // Q8_0: two halves
}
// elements covered by one block, for unit indexing
template <uint32_t Q>
__host__ __device__ constexpr int unit_block_elems() {
    return block_elems(Q);
}

// Dequantize the 16 weights of unit t of the block at blk (fp32; the fused
// paths only need the tolerance, so FMA contraction is allowed here).
template <uint32_t Q>
__device__ __forceinline__ void decode16(const uint8_t* __restrict__ blk, int t, float w[16]) {
    if constexpr (Q == kQ4_K || Q == kQ5_K) {
        int c = t >> 2, p = t & 3;
        float d = f16_bits_to_f32(rd16g(blk)), dm = f16_bits_to_f32(rd16g(blk + 2));
        uint32_t sA, mA, sB, mB;
        scale_min_k4(2 * c, blk + 4, sA, mA);
        scale_min_k4(2 * c + 1, blk + 4, sB, mB);
        float dA = d * (float)sA, nA = dm * (float)mA, dB = d * (float)sB, nB = dm * (float)mB;
        const uint8_t* q = blk + ((Q == kQ4_K) ? 16 : 48) + 32 * c + 8 * p;
        const uint8_t* qh = blk + 16 + 8 * p;
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            uint32_t b = __ldg(q + l);
            float lo = (float)(b & 0xFu), hi = (float)(b >> 4);
            if constexpr (Q == kQ5_K) {
                uint32_t h = __ldg(qh + l);
                lo += ((h >> (2 * c)) & 1u) ? 16.0f : 0.0f;
                hi += ((h >> (2 * c + 1)) & 1u) ? 16.0f : 0.0f;
            }
            w[l] = dA * lo - nA;
            w[8 + l] = dB * hi - nB;
        }
    } else if constexpr (Q == kQ6_K) {
        int H = t >> 3, u = t & 7;
        int l0 = 8 * (u & 3);
        int g = (u >= 4) ? 1 : 0;  // 0: ql[l] (+0 / +64); 1: ql[l+32] (+32 / +96)
        const uint8_t* ql = blk + 64 * H + 32 * g + l0;
        const uint8_t* qh = blk + 128 + 32 * H + l0;
        const uint8_t* sc = blk + 192 + 8 * H;
        float d = f16_bits_to_f32(rd16g(blk + 208));
        int is = l0 >> 4;
        float sA = d * (float)__ldg(sc + is + 2 * g);
        float sB = d * (float)__ldg(sc + is + 2 * g + 4);
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            uint32_t b = __ldg(ql + l), h = __ldg(qh + l);
            int qa = (int)((b & 0xFu) | (((h >> (2 * g)) & 3u) << 4)) - 32;
            int qb = (int)((b >> 4) | (((h >> (2 * g + 4)) & 3u) << 4)) - 32;
            w[l] = sA * (float)qa;
            w[8 + l] = sB * (float)qb;
        }
    } else if constexpr (Q == kQ8_0) {
        float d = f16_bits_to_f32(rd16g(blk));
#pragma unroll
        for (int l = 0; l < 16; ++l) w[l] = (float)(int8_t)__ldg(blk + 2 + 16 * t + l) * d;
    } else {
        // the other formats: columns 16 t .. 16 t + 15, the reference's exact values
#pragma unroll
        for (int l = 0; l < 16; ++l) w[l] = dequant_elem<Q>(blk, 16 * t + l);
    }
}

// Plain float experts: one thread per (token, column), rows walked in order.
template <uint32_t Q>
__global__ void expert_float_kernel(const uint8_t* __restrict__ W, int64_t row_bytes, int64_t IN, int64_t OUT,
                                    const float* __restrict__ X, int batch, float* __restrict__ Y) {
    int64_t n = (int64_t)batch * OUT;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < n;
         idx += (int64_t)gridDim.x * blockDim.x) {
        int64_t b = idx / OUT, c = idx - b * OUT;
        float acc = 0.0f;
        for (int64_t i = 0; i < IN; ++i) {
            const uint8_t* row = W + i * row_bytes;
            float w;
            if constexpr (Q == kF32) w = __ldg(reinterpret_cast<const float*>(row) + c);
            else if constexpr (Q == kF16) w = f16_bits_to_f32(rd16g(row + 2 * c));
            else w = __uint_as_float(rd16g(row + 2 * c) << 16);
            acc = fmaf(__ldg(X + b * IN + i), w, acc);
        }
        Y[idx] = acc;
    }
}

template <uint32_t Q>
int run_expert_float(const ExpertGemvArgs& a, cudaStream_t st) {
    int64_t n = (int64_t)a.batch * a.OUT;
    int64_t blocks = (n + 255) / 256;
    if (blocks > (int64_t)a.sm_count * 8) blocks = (int64_t)a.sm_count * 8;
    expert_float_kernel<Q><<<(unsigned)blocks, 256, 0, st>>>(a.W, a.row_bytes, a.IN, a.OUT, a.X, a.batch, a.Y);
    return 0;
}

// Pass 1: CTA (s, g) sums rows [s*rps, (s+1)*rps) for column units of group g
// and writes P[s][b][c] for its tokens [tok0, tok0 + nt).
template <uint32_t Q>
__global__ void __launch_bounds__(kEgThreads)
expert_partial_kernel(const uint8_t* __restrict__ W, int64_t row_bytes, int64_t IN, int64_t OUT,
                      const float* __restrict__ X, int tok0, int nt, int64_t rps, int ug,
                      float* __restrict__ P) {
    constexpr int UPB = units16_per_block<Q>();
    constexpr int BE = unit_block_elems<Q>();
    constexpr int BB = block_bytes(Q);
    __shared__ float red[kEgThreads][16 + 1];

    const int64_t units = (OUT / BE) * UPB;
    const int tid = threadIdx.x;
    const int lanes_u = ug;                     // threads along columns
    const int prow = kEgThreads / lanes_u;      // row lanes
    const int pu = tid % lanes_u, pr = tid / lanes_u;
    const int64_t u = (int64_t)blockIdx.y * lanes_u + pu;
    const bool active = (pr < prow) && (u < units);
    const int64_t blk_i = u / UPB;
    const int t = (int)(u % UPB);
    int colA = 0, colB = 0;
    unit16_cols<Q>(t, colA, colB);
    const int64_t r0 = (int64_t)blockIdx.x * rps;
    const int64_t r1 = (r0 + rps < IN) ? r0 + rps : IN;

    float acc[kEgTok][16];
#pragma unroll
    for (int b = 0; b < kEgTok; ++b)
#pragma unroll
        for (int l = 0; l < 16; ++l) acc[b][l] = 0.0f;

    if (active) {
        for (int64_t i = r0 + pr; i < r1; i += prow) {
            float w[16];
            decode16<Q>(W + i * row_bytes + blk_i * BB, t, w);
#pragma unroll
            for (int b = 0; b < kEgTok; ++b) {
                if (b < nt) {
                    float xi = __ldg(X + (int64_t)(tok0 + b) * IN + i);
#pragma unroll
                    for (int l = 0; l < 16; ++l) acc[b][l] = fmaf(xi, w[l], acc[b][l]);
                }
            }
        }
    }
    // reduce over the row lanes of this CTA, in a fixed order
    for (int b = 0; b < nt; ++b) {
#pragma unroll
        for (int l = 0; l < 16; ++l) red[tid][l] = acc[b][l];
        __syncthreads();
        if (pr == 0 && u < units) {
            float s[16];
#pragma unroll
            for (int l = 0; l < 16; ++l) s[l] = red[pu][l];
            for (int q = 1; q < prow; ++q)
#pragma unroll
                for (int l = 0; l < 16; ++l) s[l] += red[q * lanes_u + pu][l];
            float* dst = P + ((int64_t)blockIdx.x * nt + b) * OUT + blk_i * BE;
#pragma unroll
            for (int l = 0; l < 8; ++l) {
                dst[colA + l] = s[l];
                dst[colB + l] = s[8 + l];
            }
        }
        __syncthreads();
    }
}

// Pass 2: Y[tok0 + b][c] = sum_s P[s][b][c], s ascending.
__global__ void expert_reduce_kernel(const float* __restrict__ P, int64_t S, int nt, int64_t OUT,
                                     int tok0, float* __restrict__ Y) {
    int64_t n = (int64_t)nt * OUT;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < n;
         idx += (int64_t)gridDim.x * blockDim.x) {
        float s = 0.0f;
        for (int64_t k = 0; k < S; ++k) s += P[k * n + idx];
        Y[(int64_t)tok0 * OUT + idx] = s;
    }
}

template <uint32_t Q>
int run_expert(const ExpertGemvArgs& a, float* work, int64_t work_floats, cudaStream_t st) {
    constexpr int UPB = units16_per_block<Q>();
    constexpr int BE = unit_block_elems<Q>();
    if (a.OUT % BE != 0) return -1;
    const int64_t units = (a.OUT / BE) * UPB;
    int ug = 1;
    while (ug < units && ug < kEgThreads) ug <<= 1;
    const int64_t groups = (units + ug - 1) / ug;
    // row splits: enough CTAs to fill the GPU, at least 16 rows each
    int64_t want = ((int64_t)a.sm_count * 4 + groups - 1) / groups;
    int64_t S = a.IN / 16 > 0 ? a.IN / 16 : 1;
    if (S > want) S = want;
    if (S < 1) S = 1;
    int64_t rps = (a.IN + S - 1) / S;
    S = (a.IN + rps - 1) / rps;
    if (S < 1) S = 1;
    if (S * kEgTok * a.OUT > work_floats) return -2;
    for (int tok0 = 0; tok0 < a.batch; tok0 += kEgTok) {
        int nt = a.batch - tok0 < kEgTok ? a.batch - tok0 : kEgTok;
        dim3 grid((unsigned)S, (unsigned)groups);
        expert_partial_kernel<Q><<<grid, kEgThreads, 0, st>>>(a.W, a.row_bytes, a.IN, a.OUT, a.X, tok0, nt,
                                                               rps, ug, work);
        int64_t n = (int64_t)nt * a.OUT;
        int64_t rb = (n + 255) / 256;
        if (rb > (int64_t)a.sm_count * 8) rb = (int64_t)a.sm_count * 8;
        expert_reduce_kernel<<<(unsigned)rb, 256, 0, st>>>(work, S, nt, a.OUT, tok0, a.Y);
    }
    return 0;
}

}  // namespace

int64_t expert_gemv_work_floats(int64_t IN, int64_t OUT, int sm_count) {
    (void)IN;
    return (int64_t)sm_count * 4 * kEgTok * OUT + 1024;
}

int launch_expert_gemv_ws(uint32_t quant, const ExpertGemvArgs& a, float* work, int64_t work_floats,
                          cudaStream_t s) {
    if (a.OUT <= 0 || a.batch <= 0) return 0;
    switch (quant) {
    case kQ4_K: return run_expert<kQ4_K>(a, work, work_floats, s);
    case kQ5_K: return run_expert<kQ5_K>(a, work, work_floats, s);
    case kQ6_K: return run_expert<kQ6_K>(a, work, work_floats, s);
    case kQ8_0: return run_expert<kQ8_0>(a, work, work_floats, s);
    case kF32: return run_expert_float<kF32>(a, s);
    case kF16: return run_expert_float<kF16>(a, s);
    case kBF16: return run_expert_float<kBF16>(a, s);
    case kQ4_0: return run_expert<kQ4_0>(a, work, work_floats, s);
    case kQ4_1: return run_expert<kQ4_1>(a, work, work_floats, s);
    case kQ5_0: return run_expert<kQ5_0>(a, work, work_floats, s);
    case kQ5_1: return run_expert<kQ5_1>(a, work, work_floats, s);
    case kQ8_1: return run_expert<kQ8_1>(a, work, work_floats, s);
    case kQ2_K: return run_expert<kQ2_K>(a, work, work_floats, s);
    case kQ3_K: return run_expert<kQ3_K>(a, work, work_floats, s);
    case kIQ4_NL: return run_expert<kIQ4_NL>(a, work, work_floats, s);
    case kIQ4_XS: return run_expert<kIQ4_XS>(a, work, work_floats, s);
    case kMXFP4: return run_expert<kMXFP4>(a, work, work_floats, s);
    case kNVFP4: return run_expert<kNVFP4>(a, work, work_floats, s);
    case kQ2_0: return run_expert<kQ2_0>(a, work, work_floats, s);
    default: return -1;
    }
}

}  // namespace strata
