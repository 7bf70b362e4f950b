// moe.cu — the MoE FFN layer on the device: MoeLayer::route + MoeLayer::combine
// (crates/strata-core/src/moe.rs:48-144) for T tokens at once.
//
//   route      one CTA per token: softmax with the max shift, the f64 sum and
//              the f32 reciprocal of moe.rs:57-68, the k first experts in the
//              order (probability desc, id asc) of moe.rs:70-79, ids ascending,
//              weights renormalised with the 2^-14 floor of moe.rs:80-90;
//   assign     one CTA: per expert, the (token, slot) pairs routed to it in
//              token order, and the list of experts that received any;
//   gate/up    per active expert, column super-block and range of input rows:
//              partial sums of x W_gate and x W_up for that expert's tokens
//              (the expert layout [E][IN][OUT] is quantized along OUT, so a
//              thread owns 16 output columns and walks input rows);
//   swiglu     h = silu(sum gate) * (sum up), partials added in a fixed order;
//   down       the same grouped form over h and W_down;
//   combine    out[t] = sum over t's experts in ascending id of w * down
//              (moe.rs:111-127), then + sigmoid(x . gate_inp_shexp) *
//              shared(x) (moe.rs:129-142).
// The shared expert's dense projections use the CUDA-core GEMV. Every
// reduction has a fixed order, so the layer is deterministic run to run.
#include <cmath>

#include "kernels.cuh"
#include "moe.cuh"
#include "quant.cuh"

namespace strata {
namespace {

constexpr int kMoeThreads = 256;
constexpr int kUnits = 16;    // 16 units of 16 columns = one 256-column super-block
constexpr int kRowLanes = kMoeThreads / kUnits;
constexpr int kTokPass = 4;   // tokens per pass over the rows

// f32 exp rounded from a double exp (correctly rounded except within about
// 2^-29 ulp of a rounding boundary), standing in for Rust's f32::exp.
__device__ __forceinline__ float exp_f32(float x) { return (float)exp((double)x); }
__device__ __forceinline__ float silu_f32(float x) { return x / (1.0f + exp_f32(-x)); }      // ops.rs:85-87
__device__ __forceinline__ float sigmoid_f32(float x) { return 1.0f / (1.0f + exp_f32(-x)); }  // ops.rs:90-92

// ------------------------------------------------------------------ routing

__global__ void __launch_bounds__(256) moe_route_kernel(const float* __restrict__ logits, int E, int k,
                                                        int* __restrict__ ids, float* __restrict__ wts) {
    extern __shared__ float sp[];  // E probabilities
    __shared__ float red_f[256];
    __shared__ double red_d[256];
    __shared__ int sel[64];
    const int t = blockIdx.x, tid = threadIdx.x;
    const float* lg = logits + (int64_t)t * E;
    float mx = -INFINITY;
    for (int i = tid; i < E; i += blockDim.x) mx = fmaxf(mx, lg[i]);
    red_f[tid] = mx;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if (tid < s) red_f[tid] = fmaxf(red_f[tid], red_f[tid + s]);
        __syncthreads();
    }
    mx = red_f[0];
    double sum = 0.0;
    for (int i = tid; i < E; i += blockDim.x) {
        const float e = exp_f32(lg[i] - mx);
        sp[i] = e;
        sum += (double)e;
    }
    red_d[tid] = sum;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if (tid < s) red_d[tid] += red_d[tid + s];
        __syncthreads();
    }
    const float inv = (float)(1.0 / red_d[0]);
    for (int i = tid; i < E; i += blockDim.x) sp[i] = sp[i] * inv;
    __syncthreads();
    // expert i is chosen when fewer than k experts precede it in the order
    // (probability desc, index asc); its slot is the number of chosen ids below it
    const int kk = k < E ? k : E;
    int* chosen = reinterpret_cast<int*>(sp + E);  // E flags after the probabilities
    for (int i = tid; i < E; i += blockDim.x) {
        const float pi = sp[i];
        int rank = 0;
        for (int j = 0; j < E && rank < kk; ++j) {
            const float pj = sp[j];
            rank += (pj > pi || (pj == pi && j < i)) ? 1 : 0;
        }
        chosen[i] = rank < kk ? 1 : 0;
    }
    __syncthreads();
    for (int i = tid; i < E; i += blockDim.x) {
        if (!chosen[i]) continue;
        int slot = 0;
        for (int j = 0; j < i; ++j) slot += chosen[j];
        sel[slot] = i;
    }
    __syncthreads();
    if (tid == 0) {
        double ws = 0.0;
        for (int j = 0; j < kk; ++j) ws += (double)sp[sel[j]];
        const double s = ws > 0x1p-14 ? ws : 0x1p-14;
        for (int j = 0; j < kk; ++j) {
            ids[(int64_t)t * k + j] = sel[j];
            wts[(int64_t)t * k + j] = (float)((double)sp[sel[j]] / s);
        }
        for (int j = kk; j < k; ++j) {
            ids[(int64_t)t * k + j] = -1;
            wts[(int64_t)t * k + j] = 0.0f;
        }
    }
}

// ------------------------------------------------------------------ assignment

// One CTA of >= E threads; thread e handles expert e.
__global__ void moe_assign_kernel(const int* __restrict__ ids, int T, int k, int E, int e_begin, int e_end,
                                  MoeIndex ix) {
    __shared__ int scan[1024];
    const int e = threadIdx.x;
    const int64_t TK = (int64_t)T * k;
    for (int64_t i = threadIdx.x; i < TK; i += blockDim.x) ix.pos[i] = -1;
    const bool local = e < E && e >= e_begin && e < e_end;
    int c = 0;
    if (local)
        for (int64_t i = 0; i < TK; ++i) c += ids[i] == e ? 1 : 0;
    // exclusive scans (over e ascending) of the counts and of the active flags
    scan[e] = c;
    __syncthreads();
    for (int s = 1; s < (int)blockDim.x; s <<= 1) {
        const int v = e >= s ? scan[e - s] : 0;
        __syncthreads();
        scan[e] += v;
        __syncthreads();
    }
    const int off = scan[e] - c;
    const int total = scan[blockDim.x - 1];
    __syncthreads();
    scan[e] = c > 0 ? 1 : 0;
    __syncthreads();
    for (int s = 1; s < (int)blockDim.x; s <<= 1) {
        const int v = e >= s ? scan[e - s] : 0;
        __syncthreads();
        scan[e] += v;
        __syncthreads();
    }
    if (e < E) {
        ix.cnt[e] = c;
        ix.off[e] = off;
        if (c > 0) ix.active[scan[e] - 1] = e;
    }
    if (e == 0) {
        ix.n_active[0] = scan[blockDim.x - 1];
        ix.n_assign[0] = total;
    }
    if (c > 0) {
        int r = 0;
        for (int64_t i = 0; i < TK; ++i)
            if (ids[i] == e) {
                ix.tok[off + r] = (int)(i / k);
                ix.pos[i] = off + r;
                ++r;
            }
    }
}

// ------------------------------------------------------------------ grouped expert GEMV

__device__ __forceinline__ float h2f(uint32_t bits) { return f16_bits_to_f32(bits & 0xFFFFu); }

// The 16 weights of unit t (0..15) of one 256-column super-block: columns
// colA .. colA + 7 -> w[0..7] and colB .. colB + 7 -> w[8..15].
template <uint32_t Q>
__device__ __forceinline__ void unit_cols(int t, int& colA, int& colB) {
    if constexpr (Q == kQ4_K || Q == kQ5_K) {
        const int c = t >> 2, p = t & 3;
        colA = 64 * c + 8 * p;
        colB = colA + 32;
    } else if constexpr (Q == kQ6_K) {
        const int H = t >> 3, u = t & 7;
        colA = 128 * H + 8 * (u & 3) + ((u >= 4) ? 32 : 0);
        colB = colA + 64;
    } else {  // Q8_0: 8 blocks of 32; unit t = half t & 1 of block t >> 1
        colA = 16 * t;
        colB = colA + 8;
    }
}

template <uint32_t Q>
__device__ __forceinline__ void decode_unit(const uint8_t* __restrict__ blk, int t, float (&w)[16]) {
    if constexpr (Q == kQ4_K || Q == kQ5_K) {
        // 16-byte aligned: rows are whole 144 / 176-byte blocks from a 256-byte aligned base
        const int c = t >> 2, p = t & 3;
        const uint4 h = __ldg(reinterpret_cast<const uint4*>(blk));
        uint32_t sc_lo, sc_hi, m_lo, m_hi;
        scales_k4_packed(h.y, h.z, h.w, sc_lo, sc_hi, m_lo, m_hi);
        const float d = h2f(h.x), dm = h2f(h.x >> 16);
        const int jA = 2 * c, jB = 2 * c + 1;
        const float dA = d * (float)(((jA < 4 ? sc_lo : sc_hi) >> (8 * (jA & 3))) & 0xFFu);
        const float dB = d * (float)(((jB < 4 ? sc_lo : sc_hi) >> (8 * (jB & 3))) & 0xFFu);
        const float nA = dm * (float)(((jA < 4 ? m_lo : m_hi) >> (8 * (jA & 3))) & 0xFFu);
        const float nB = dm * (float)(((jB < 4 ? m_lo : m_hi) >> (8 * (jB & 3))) & 0xFFu);
        const uint2 q = __ldg(reinterpret_cast<const uint2*>(blk + ((Q == kQ4_K) ? 16 : 48) + 32 * c + 8 * p));
        uint2 qh = make_uint2(0, 0);
        if constexpr (Q == kQ5_K) qh = __ldg(reinterpret_cast<const uint2*>(blk + 16 + 8 * p));
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const uint32_t b = ((l < 4 ? q.x : q.y) >> (8 * (l & 3))) & 0xFFu;
            float lo = (float)(b & 0xFu), hi = (float)(b >> 4);
            if constexpr (Q == kQ5_K) {
                const uint32_t hb = ((l < 4 ? qh.x : qh.y) >> (8 * (l & 3))) & 0xFFu;
                lo += ((hb >> jA) & 1u) ? 16.0f : 0.0f;
                hi += ((hb >> jB) & 1u) ? 16.0f : 0.0f;
            }
            w[l] = fmaf(dA, lo, -nA);
            w[8 + l] = fmaf(dB, hi, -nB);
        }
    } else if constexpr (Q == kQ6_K) {
        const int H = t >> 3, u = t & 7;
        const int l0 = 8 * (u & 3), g = (u >= 4) ? 1 : 0;
        const uint8_t* ql = blk + 64 * H + 32 * g + l0;
        const uint8_t* qh = blk + 128 + 32 * H + l0;
        const uint8_t* sc = blk + 192 + 8 * H;
        const float d = f16_bits_to_f32((uint32_t)__ldg(blk + 208) | ((uint32_t)__ldg(blk + 209) << 8));
        const int is = l0 >> 4;
        // u8 scales, as the reference reads them (crates/strata-gguf/src/dequant.rs:208-234)
        const float sA = d * (float)__ldg(sc + is + 2 * g), sB = d * (float)__ldg(sc + is + 2 * g + 4);
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const uint32_t b = __ldg(ql + l), h = __ldg(qh + l);
            const int qa = (int)((b & 0xFu) | (((h >> (2 * g)) & 3u) << 4)) - 32;
            const int qb = (int)((b >> 4) | (((h >> (2 * g + 4)) & 3u) << 4)) - 32;
            w[l] = sA * (float)qa;
            w[8 + l] = sB * (float)qb;
        }
    } else {  // Q8_0
        const uint8_t* b = blk + 34 * (t >> 1);
        const float d = f16_bits_to_f32((uint32_t)__ldg(b) | ((uint32_t)__ldg(b + 1) << 8));
        const uint8_t* q = b + 2 + 16 * (t & 1);
#pragma unroll
        for (int l = 0; l < 16; ++l) w[l] = (float)(int8_t)__ldg(q + l) * d;
    }
}

template <uint32_t Q>
__host__ __device__ constexpr int sblock_bytes() {
    return Q == kQ8_0 ? 8 * 34 : block_bytes(Q);  // bytes of one 256-column group of a row
}

// Partial sums P[rc][m][a][OUT] (m < NMAT) of sum_i X[src(a)][i] W_m[e][i][c]
// over rows [IN rc / RC, IN (rc + 1) / RC) for the assignments a of the
// active expert in slot blockIdx.x / groups, columns of super-block
// blockIdx.x % groups. src(a) = tok[a] when by_token, else a itself.
template <uint32_t Q, int NMAT>
__global__ void __launch_bounds__(kMoeThreads)
moe_expert_partial_kernel(const uint8_t* __restrict__ W0, const uint8_t* __restrict__ W1, int64_t row_bytes,
                          int64_t expert_bytes, int IN, int OUT, const float* __restrict__ X, bool by_token,
                          MoeIndex ix, int e_begin, int A_cap, float* __restrict__ P) {
    __shared__ float red[kMoeThreads][17];
    const int groups = OUT / 256;
    const int slot = blockIdx.x / groups, cg = blockIdx.x % groups;
    if (slot >= ix.n_active[0]) return;
    const int e = ix.active[slot];
    const int a0 = ix.off[e], n = ix.cnt[e];
    const int RC = gridDim.y, rc = blockIdx.y;
    const int r0 = (int)((int64_t)IN * rc / RC), r1 = (int)((int64_t)IN * (rc + 1) / RC);
    const int tid = threadIdx.x, t = tid % kUnits, pr = tid / kUnits;
    int colA, colB;
    unit_cols<Q>(t, colA, colB);
    const int64_t ebase = (int64_t)(e - e_begin) * expert_bytes + (int64_t)cg * sblock_bytes<Q>();
    for (int p0 = 0; p0 < n; p0 += kTokPass) {
        const int np = n - p0 < kTokPass ? n - p0 : kTokPass;
        const float* xs[kTokPass];
#pragma unroll
        for (int b = 0; b < kTokPass; ++b) {
            const int a = a0 + p0 + (b < np ? b : 0);
            xs[b] = X + (int64_t)(by_token ? ix.tok[a] : a) * IN;
        }
        float acc[NMAT][kTokPass][16];
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (int b = 0; b < kTokPass; ++b)
#pragma unroll
                for (int l = 0; l < 16; ++l) acc[m][b][l] = 0.0f;
        for (int i = r0 + pr; i < r1; i += kRowLanes) {
            float xv[kTokPass];
#pragma unroll
            for (int b = 0; b < kTokPass; ++b) xv[b] = __ldg(xs[b] + i);
#pragma unroll
            for (int m = 0; m < NMAT; ++m) {
                float w[16];
                decode_unit<Q>((m == 0 ? W0 : W1) + ebase + (int64_t)i * row_bytes, t, w);
#pragma unroll
                for (int b = 0; b < kTokPass; ++b)
#pragma unroll
                    for (int l = 0; l < 16; ++l) acc[m][b][l] = fmaf(xv[b], w[l], acc[m][b][l]);
            }
        }
        // add the row lanes of each column unit in a fixed order
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
            for (int b = 0; b < np; ++b) {
#pragma unroll
                for (int l = 0; l < 16; ++l) red[tid][l] = acc[m][b][l];
                __syncthreads();
                if (pr == 0) {
                    float s[16];
#pragma unroll
                    for (int l = 0; l < 16; ++l) s[l] = red[t][l];
                    for (int q = 1; q < kRowLanes; ++q)
#pragma unroll
                        for (int l = 0; l < 16; ++l) s[l] += red[q * kUnits + t][l];
                    float* dst = P + (((int64_t)rc * NMAT + m) * A_cap + a0 + p0 + b) * OUT + cg * 256;
#pragma unroll
                    for (int l = 0; l < 8; ++l) {
                        dst[colA + l] = s[l];
                        dst[colB + l] = s[8 + l];
                    }
                }
                __syncthreads();
            }
        }
    }
}

// H[a][f] = silu(sum_rc P[rc][0][a][f]) * sum_rc P[rc][1][a][f]  (moe.rs:119-121)
__global__ void moe_swiglu_kernel(const float* __restrict__ P, int RC, int A_cap, int F, const int* __restrict__ n_assign,
                                  float* __restrict__ H) {
    const int64_t n = (int64_t)n_assign[0] * F;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float g = 0.0f, u = 0.0f;
        for (int rc = 0; rc < RC; ++rc) {
            g += P[((int64_t)rc * 2 + 0) * A_cap * F + i];
            u += P[((int64_t)rc * 2 + 1) * A_cap * F + i];
        }
        H[i] = silu_f32(g) * u;
    }
}

// Shared expert activation: Hs = silu(Gs) * Us, sg[t] = sigmoid(gi[t]) (moe.rs:129-140).
__global__ void moe_shared_act_kernel(const float* __restrict__ Gs, const float* __restrict__ Us,
                                      const float* __restrict__ gi, int T, int F, float* __restrict__ Hs,
                                      float* __restrict__ sg) {
    const int64_t n = (int64_t)T * F;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        Hs[i] = silu_f32(Gs[i]) * Us[i];
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < T; t += (int64_t)gridDim.x * blockDim.x)
        sg[t] = sigmoid_f32(gi[t]);
}

// out[t][c] = sum_j w[t][j] * down[pos(t,j)][c] over t's local experts in
// ascending id (skipping zero weights, moe.rs:111-113), + sg[t] * Ds[t][c].
__global__ void moe_combine_kernel(const float* __restrict__ Pd, int RC, int A_cap, int OUT, const int* __restrict__ pos,
                                   const float* __restrict__ wts, int T, int k, const float* __restrict__ Ds,
                                   const float* __restrict__ sg, float* __restrict__ out) {
    const int64_t n = (int64_t)T * OUT;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / OUT, c = i - t * OUT;
        float acc = 0.0f;
        for (int j = 0; j < k; ++j) {
            const int a = pos[t * k + j];
            const float w = wts[t * k + j];
            if (a < 0 || w == 0.0f) continue;
            float d = 0.0f;
            for (int rc = 0; rc < RC; ++rc) d += Pd[((int64_t)rc * A_cap + a) * OUT + c];
            acc += w * d;
        }
        if (Ds) acc += sg[t] * Ds[i];
        out[i] = acc;
    }
}

// bf16 rounding of the router input (hyper::bf16_round, crates/strata-core/src/hyper.rs:22-24)
__global__ void moe_bf16_round_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const uint32_t u = __float_as_uint(x[i]);
        uint32_t r;
        if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) r = (u | 0x00400000u) & 0xFFFF0000u;  // quiet NaN
        else r = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
        y[i] = __uint_as_float(r);
    }
}

unsigned grid_for(int64_t n, int sm_count, int per_sm = 8) {
    int64_t g = (n + 255) / 256;
    const int64_t cap = (int64_t)(sm_count > 0 ? sm_count : 148) * per_sm;
    if (g > cap) g = cap;
    return (unsigned)(g < 1 ? 1 : g);
}

template <int NMAT>
int launch_partial(uint32_t q, const uint8_t* W0, const uint8_t* W1, int64_t row_bytes, int64_t expert_bytes, int IN,
                   int OUT, const float* X, bool by_token, const MoeIndex& ix, int e_begin, int A_cap, float* P,
                   int slots, int RC, cudaStream_t s) {
    const dim3 grid((unsigned)(slots * (OUT / 256)), (unsigned)RC);
    switch (q) {
#define STRATA_MOE_Q(QQ)                                                                                     \
    case QQ:                                                                                                 \
        moe_expert_partial_kernel<QQ, NMAT><<<grid, kMoeThreads, 0, s>>>(W0, W1, row_bytes, expert_bytes, IN, \
                                                                         OUT, X, by_token, ix, e_begin,     \
                                                                         A_cap, P);                         \
        return 0;
        STRATA_MOE_Q(kQ4_K) STRATA_MOE_Q(kQ5_K) STRATA_MOE_Q(kQ6_K) STRATA_MOE_Q(kQ8_0)
#undef STRATA_MOE_Q
    default: return -1;
    }
}

}  // namespace

bool moe_expert_quant_supported(uint32_t q) { return q == kQ4_K || q == kQ5_K || q == kQ6_K || q == kQ8_0; }

// Row chunks for a grouped partial pass: enough CTAs for about two per SM, at
// least 64 rows per chunk.
int moe_row_chunks(int slots, int groups, int IN, int sm_count) {
    const int units = slots * groups;
    int rc = (2 * (sm_count > 0 ? sm_count : 148) + units - 1) / units;
    const int maxrc = IN / 64 > 0 ? IN / 64 : 1;
    if (rc > maxrc) rc = maxrc;
    return rc < 1 ? 1 : rc;
}

MoeWork moe_work_layout(const MoePlan& p) {
    MoeWork w{};
    int64_t o = 0;
    auto take = [&](int64_t bytes) {
        const int64_t at = o;
        o += (bytes + 255) & ~int64_t(255);
        return at;
    };
    const int64_t TK = (int64_t)p.T * p.k, A = TK;
    w.ids = take(TK * 4);
    w.wts = take(TK * 4);
    w.pos = take(TK * 4);
    w.tok = take(A * 4);
    w.cnt = take((int64_t)p.E * 4);
    w.off = take((int64_t)p.E * 4);
    w.active = take((int64_t)p.E * 4);
    w.counters = take(16);
    w.logits = p.need_router ? take((int64_t)p.T * p.E * 4) : -1;
    w.xb = p.need_router ? take((int64_t)p.T * p.n_embd * 4) : -1;
    w.pgu = take((int64_t)p.rc_gu * 2 * A * p.n_ff * 4);
    w.h = take(A * p.n_ff * 4);
    w.pd = take((int64_t)p.rc_d * A * p.n_embd * 4);
    if (p.shared) {
        w.gs = take((int64_t)p.T * p.n_ff_s * 4);
        w.us = take((int64_t)p.T * p.n_ff_s * 4);
        w.hs = take((int64_t)p.T * p.n_ff_s * 4);
        w.gi = take((int64_t)p.T * 4);
        w.sg = take((int64_t)p.T * 4);
        w.ds = take((int64_t)p.T * p.n_embd * 4);
    }
    w.bytes = o;
    return w;
}

int launch_moe_layer(const MoeLaunch& L, cudaStream_t s) {
    const MoePlan& p = L.plan;
    uint8_t* base = static_cast<uint8_t*>(L.work);
    auto F = [&](int64_t off) { return reinterpret_cast<float*>(base + off); };
    auto I = [&](int64_t off) { return reinterpret_cast<int*>(base + off); };
    const MoeWork& w = L.layout;
    MoeIndex ix{I(w.cnt), I(w.off), I(w.active), I(w.counters), I(w.counters) + 1, I(w.tok), I(w.pos)};
    const int A = p.T * p.k;

    // route
    const float* logits = L.logits;
    if (!logits) {
        const int64_t n = (int64_t)p.T * p.n_embd;
        moe_bf16_round_kernel<<<grid_for(n, p.sm_count), 256, 0, s>>>(L.x, F(w.xb), n);
        GemvArgs g{L.router.W, L.router.row_bytes, p.E, p.n_embd, F(w.xb), F(w.logits), p.T, p.sm_count, nullptr};
        if (launch_gemv(L.router.quant, g, s)) return -1;
        logits = F(w.logits);
    }
    moe_route_kernel<<<p.T, 256, (size_t)p.E * (sizeof(float) + sizeof(int)), s>>>(logits, p.E, p.k, I(w.ids), F(w.wts));
    int athreads = 32;
    while (athreads < p.E) athreads <<= 1;
    moe_assign_kernel<<<1, athreads, 0, s>>>(I(w.ids), p.T, p.k, p.E, p.e_begin, p.e_end, ix);

    // routed experts
    const int slots = p.slots;
    if (launch_partial<2>(L.gate.quant, L.gate.W, L.up.W, L.gate.row_bytes, L.gate.expert_bytes, p.n_embd, p.n_ff,
                          L.x, true, ix, p.e_begin, A, F(w.pgu), slots, p.rc_gu, s))
        return -2;
    moe_swiglu_kernel<<<grid_for((int64_t)A * p.n_ff, p.sm_count), 256, 0, s>>>(F(w.pgu), p.rc_gu, A, p.n_ff,
                                                                                 ix.n_assign, F(w.h));
    if (launch_partial<1>(L.down.quant, L.down.W, nullptr, L.down.row_bytes, L.down.expert_bytes, p.n_ff, p.n_embd,
                          F(w.h), false, ix, p.e_begin, A, F(w.pd), slots, p.rc_d, s))
        return -3;

    // shared expert (moe.rs:129-142)
    const float* Ds = nullptr;
    const float* sg = nullptr;
    if (p.shared) {
        GemvArgs gg{L.gate_s.W, L.gate_s.row_bytes, p.n_ff_s, p.n_embd, L.x, F(w.gs), p.T, p.sm_count, nullptr};
        GemvArgs gu{L.up_s.W, L.up_s.row_bytes, p.n_ff_s, p.n_embd, L.x, F(w.us), p.T, p.sm_count, nullptr};
        GemvArgs gi{L.gate_inp_s.W, L.gate_inp_s.row_bytes, 1, p.n_embd, L.x, F(w.gi), p.T, p.sm_count, nullptr};
        if (launch_gemv(L.gate_s.quant, gg, s) || launch_gemv(L.up_s.quant, gu, s) ||
            launch_gemv(L.gate_inp_s.quant, gi, s))
            return -4;
        moe_shared_act_kernel<<<grid_for((int64_t)p.T * p.n_ff_s, p.sm_count), 256, 0, s>>>(
            F(w.gs), F(w.us), F(w.gi), p.T, p.n_ff_s, F(w.hs), F(w.sg));
        GemvArgs gd{L.down_s.W, L.down_s.row_bytes, p.n_embd, p.n_ff_s, F(w.hs), F(w.ds), p.T, p.sm_count, nullptr};
        if (launch_gemv(L.down_s.quant, gd, s)) return -5;
        Ds = F(w.ds);
        sg = F(w.sg);
    }
    moe_combine_kernel<<<grid_for((int64_t)p.T * p.n_embd, p.sm_count), 256, 0, s>>>(
        F(w.pd), p.rc_d, A, p.n_embd, I(w.pos), F(w.wts), p.T, p.k, Ds, sg, L.out);
    if (L.ids_out) cudaMemcpyAsync(L.ids_out, I(w.ids), (size_t)A * 4, cudaMemcpyDeviceToDevice, s);
    if (L.wts_out) cudaMemcpyAsync(L.wts_out, F(w.wts), (size_t)A * 4, cudaMemcpyDeviceToDevice, s);
    return 0;
}

}  // namespace strata
