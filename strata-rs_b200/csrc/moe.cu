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
    // the k first experts of the order (probability desc, index asc): k rounds
    // of a block arg-max over the experts not yet taken
    const int kk = k < E ? k : E;
    int* taken = reinterpret_cast<int*>(sp + E);  // E flags after the probabilities
    for (int i = tid; i < E; i += blockDim.x) taken[i] = 0;
    __shared__ float wbest_p[32];
    __shared__ int wbest_i[32];
    __syncthreads();
    const int lane = tid & 31, wid = tid >> 5, nw = (blockDim.x + 31) >> 5;
    for (int r = 0; r < kk; ++r) {
        float bp = -1.0f;
        int bi = 0x7FFFFFFF;
        for (int i = tid; i < E; i += blockDim.x)
            if (!taken[i] && (sp[i] > bp || (sp[i] == bp && i < bi))) {
                bp = sp[i];
                bi = i;
            }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float op = __shfl_xor_sync(0xFFFFFFFFu, bp, o);
            const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
            if (op > bp || (op == bp && oi < bi)) {
                bp = op;
                bi = oi;
            }
        }
        if (lane == 0) {
            wbest_p[wid] = bp;
            wbest_i[wid] = bi;
        }
        __syncthreads();
        if (tid == 0) {
            float p = wbest_p[0];
            int i = wbest_i[0];
            for (int w = 1; w < nw; ++w)
                if (wbest_p[w] > p || (wbest_p[w] == p && wbest_i[w] < i)) {
                    p = wbest_p[w];
                    i = wbest_i[w];
                }
            sel[r] = i;
            taken[i] = 1;
        }
        __syncthreads();
    }
    if (tid == 0) {  // ids ascending
        for (int a = 1; a < kk; ++a) {
            const int v = sel[a];
            int b = a - 1;
            while (b >= 0 && sel[b] > v) {
                sel[b + 1] = sel[b];
                --b;
            }
            sel[b + 1] = v;
        }
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

// One CTA of >= E threads; thread e handles expert e. The routing ids are
// staged in shared memory when they fit (staged = true).
__global__ void moe_assign_kernel(const int* __restrict__ ids_g, int T, int k, int E, int e_begin, int e_end,
                                  bool staged, MoeIndex ix) {
    extern __shared__ int ids_s[];
    __shared__ int scan[1024];
    const int e = threadIdx.x;
    const int64_t TK = (int64_t)T * k;
    for (int64_t i = threadIdx.x; i < TK; i += blockDim.x) {
        ix.pos[i] = -1;
        if (staged) ids_s[i] = ids_g[i];
    }
    __syncthreads();
    const int* ids = staged ? ids_s : ids_g;
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
        for (int64_t i = 0; i < TK && r < c; ++i)
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
__device__ __forceinline__ void decode_unit(const uint8_t* blk, int t, float (&w)[16]) {
    if constexpr (Q == kQ4_K || Q == kQ5_K) {
        // 16-byte aligned: rows are whole 144 / 176-byte blocks from a 256-byte aligned base
        const int c = t >> 2, p = t & 3;
        const uint4 h = *reinterpret_cast<const uint4*>(blk);
        uint32_t sc_lo, sc_hi, m_lo, m_hi;
        scales_k4_packed(h.y, h.z, h.w, sc_lo, sc_hi, m_lo, m_hi);
        const float d = h2f(h.x), dm = h2f(h.x >> 16);
        const int jA = 2 * c, jB = 2 * c + 1;
        const float dA = d * (float)(((jA < 4 ? sc_lo : sc_hi) >> (8 * (jA & 3))) & 0xFFu);
        const float dB = d * (float)(((jB < 4 ? sc_lo : sc_hi) >> (8 * (jB & 3))) & 0xFFu);
        const float nA = dm * (float)(((jA < 4 ? m_lo : m_hi) >> (8 * (jA & 3))) & 0xFFu);
        const float nB = dm * (float)(((jB < 4 ? m_lo : m_hi) >> (8 * (jB & 3))) & 0xFFu);
        const uint2 q = *reinterpret_cast<const uint2*>(blk + ((Q == kQ4_K) ? 16 : 48) + 32 * c + 8 * p);
        uint2 qh = make_uint2(0, 0);
        if constexpr (Q == kQ5_K) qh = *reinterpret_cast<const uint2*>(blk + 16 + 8 * p);
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
        const float d = f16_bits_to_f32((uint32_t)blk[208] | ((uint32_t)blk[209] << 8));
        const int is = l0 >> 4;
        // u8 scales, as the reference reads them (crates/strata-gguf/src/dequant.rs:208-234)
        const float sA = d * (float)sc[is + 2 * g], sB = d * (float)sc[is + 2 * g + 4];
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const uint32_t b = ql[l], h = qh[l];
            const int qa = (int)((b & 0xFu) | (((h >> (2 * g)) & 3u) << 4)) - 32;
            const int qb = (int)((b >> 4) | (((h >> (2 * g + 4)) & 3u) << 4)) - 32;
            w[l] = sA * (float)qa;
            w[8 + l] = sB * (float)qb;
        }
    } else {  // Q8_0
        const uint8_t* b = blk + 34 * (t >> 1);
        const float d = f16_bits_to_f32((uint32_t)b[0] | ((uint32_t)b[1] << 8));
        const uint8_t* q = b + 2 + 16 * (t & 1);
#pragma unroll
        for (int l = 0; l < 16; ++l) w[l] = (float)(int8_t)q[l] * d;
    }
}

template <uint32_t Q>
__host__ __device__ constexpr int sblock_bytes() {
    return Q == kQ8_0 ? 8 * 34 : block_bytes(Q);  // bytes of one 256-column group of a row
}

// ---- streamed expert pass
//
// CTA (slot, m, rc): matrix m of the active expert in `slot`, input rows
// [IN rc / RC, IN (rc + 1) / RC). The rows of an expert are contiguous
// (row_bytes each, all output columns), so the CTA streams them through a
// kStages-deep shared-memory ring with cp.async (every thread copies 16 or 4
// bytes per request; several row tiles in flight), and thread (u, lane)
// decodes 16-column unit u of rows lane, lane + RL, ... of each tile from
// shared memory. Output: partial sums P[rc][m][a][OUT] of
// sum_i X[src(a)][i] W_m[e][i][c] for the expert's assignments a, TP tokens
// per pass over the rows; src(a) = tok[a] when by_token, else a.
constexpr int kStages = 4;
constexpr int kStageBytes = 16384;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
                 "l"(gmem)
                 : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
                 "l"(gmem)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Rows per tile: a multiple of the row lanes, about kStageBytes of weights.
__host__ __device__ inline int tile_rows(int64_t row_bytes, int RL) {
    int rs = (int)(kStageBytes / row_bytes);
    rs = rs < RL ? RL : rs;
    rs -= rs % RL;
    return rs > 64 ? 64 : rs;
}

template <uint32_t Q, int TP>
__global__ void __launch_bounds__(kMoeThreads, 2)
moe_stream_kernel(const uint8_t* __restrict__ W0, const uint8_t* __restrict__ W1, int64_t row_bytes,
                  int64_t expert_bytes, int IN, int OUT, const float* __restrict__ X, bool by_token, MoeIndex ix,
                  int e_begin, int A_cap, float* __restrict__ P) {
    extern __shared__ __align__(16) uint8_t dsm[];
    const int nmat = W1 ? 2 : 1;
    const int slot = blockIdx.x / nmat, m = blockIdx.x % nmat;
    if (slot >= ix.n_active[0]) return;
    const int e = ix.active[slot];
    const int a0 = ix.off[e], n = ix.cnt[e];
    const int RC = gridDim.y, rc = blockIdx.y;
    const int r0 = (int)((int64_t)IN * rc / RC), r1 = (int)((int64_t)IN * (rc + 1) / RC);
    const int U = OUT / 16, RL = kMoeThreads / U;
    const int tid = threadIdx.x, u = tid % U, lane = tid / U;
    const int RS = tile_rows(row_bytes, RL);
    const int64_t tile_bytes = (int64_t)RS * row_bytes;
    uint8_t* wring = dsm;                                                   // kStages x tile_bytes
    float* xring = reinterpret_cast<float*>(dsm + kStages * tile_bytes);    // kStages x TP x RS
    float* red = xring + kStages * TP * RS;                                 // kMoeThreads x 17
    const uint8_t* Wm = (m == 0 ? W0 : W1) + (int64_t)(e - e_begin) * expert_bytes;
    const bool vec16 = (row_bytes % 16) == 0;
    // unit u covers columns of 256-column group g = u / 16, unit t = u % 16 of that group
    const int g = u >> 4, t = u & 15;
    int colA, colB;
    unit_cols<Q>(t, colA, colB);
    const int ntiles = (r1 - r0 + RS - 1) / RS;

    for (int p0 = 0; p0 < n; p0 += TP) {
        const int np = n - p0 < TP ? n - p0 : TP;
        __shared__ int src[TP];  // activation row of each token of the pass
        if (tid < TP) {
            const int a = a0 + p0 + (tid < np ? tid : 0);
            src[tid] = by_token ? ix.tok[a] : a;
        }
        __syncthreads();
        auto issue = [&](int tile) {
            if (tile < ntiles) {
                const int i0 = r0 + tile * RS;
                const int rows = r1 - i0 < RS ? r1 - i0 : RS;
                uint8_t* dst = wring + (int64_t)(tile % kStages) * tile_bytes;
                const uint8_t* gsrc = Wm + (int64_t)i0 * row_bytes;
                const int64_t bytes = (int64_t)rows * row_bytes;
                if (vec16) {
                    for (int64_t c = tid; c < bytes / 16; c += kMoeThreads) cp_async16(dst + 16 * c, gsrc + 16 * c);
                } else {
                    for (int64_t c = tid; c < bytes / 4; c += kMoeThreads) cp_async4(dst + 4 * c, gsrc + 4 * c);
                }
                float* xd = xring + (tile % kStages) * TP * RS;
                for (int q = tid; q < TP * rows; q += kMoeThreads) {
                    const int b = q / rows, r = q % rows;
                    cp_async4(xd + b * RS + r, X + (int64_t)src[b] * IN + i0 + r);
                }
            }
            cp_async_commit();  // empty groups keep the count uniform
        };
        float acc[TP][16];
#pragma unroll
        for (int b = 0; b < TP; ++b)
#pragma unroll
            for (int l = 0; l < 16; ++l) acc[b][l] = 0.0f;
#pragma unroll
        for (int s = 0; s < kStages - 1; ++s) issue(s);
        for (int tile = 0; tile < ntiles; ++tile) {
            issue(tile + kStages - 1);
            cp_async_wait<kStages - 1>();
            __syncthreads();
            const int i0 = r0 + tile * RS;
            const int rows = r1 - i0 < RS ? r1 - i0 : RS;
            const uint8_t* wt = wring + (int64_t)(tile % kStages) * tile_bytes;
            const float* xt = xring + (tile % kStages) * TP * RS;
            for (int r = lane; r < rows; r += RL) {
                float w[16];
                decode_unit<Q>(wt + (int64_t)r * row_bytes + (int64_t)g * sblock_bytes<Q>(), t, w);
#pragma unroll
                for (int b = 0; b < TP; ++b) {
                    const float xv = xt[b * RS + r];
#pragma unroll
                    for (int l = 0; l < 16; ++l) acc[b][l] = fmaf(xv, w[l], acc[b][l]);
                }
            }
            __syncthreads();  // the stage is rewritten by the next issue
        }
        cp_async_wait<0>();
        // add the row lanes of each unit in a fixed order
        for (int b = 0; b < np; ++b) {
#pragma unroll
            for (int l = 0; l < 16; ++l) red[tid * 17 + l] = acc[b][l];
            __syncthreads();
            if (lane == 0) {
                float sum[16];
#pragma unroll
                for (int l = 0; l < 16; ++l) sum[l] = red[u * 17 + l];
                for (int q = 1; q < RL; ++q)
#pragma unroll
                    for (int l = 0; l < 16; ++l) sum[l] += red[(q * U + u) * 17 + l];
                float* dst = P + (((int64_t)rc * nmat + m) * A_cap + a0 + p0 + b) * OUT + (int64_t)g * 256;
#pragma unroll
                for (int l = 0; l < 8; ++l) {
                    dst[colA + l] = sum[l];
                    dst[colB + l] = sum[8 + l];
                }
            }
            __syncthreads();
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

size_t stream_smem(int64_t row_bytes, int OUT, int TP) {
    const int RL = kMoeThreads / (OUT / 16);
    const int RS = tile_rows(row_bytes, RL);
    return (size_t)kStages * RS * row_bytes + (size_t)kStages * TP * RS * 4 + (size_t)kMoeThreads * 17 * 4;
}

template <uint32_t Q, int TP>
int launch_stream_t(const uint8_t* W0, const uint8_t* W1, int64_t row_bytes, int64_t expert_bytes, int IN, int OUT,
                    const float* X, bool by_token, const MoeIndex& ix, int e_begin, int A_cap, float* P, int slots,
                    int RC, cudaStream_t s) {
    const size_t smem = stream_smem(row_bytes, OUT, TP);
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(moe_stream_kernel<Q, TP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
        return -1;
    const dim3 grid((unsigned)(slots * (W1 ? 2 : 1)), (unsigned)RC);
    moe_stream_kernel<Q, TP><<<grid, kMoeThreads, smem, s>>>(W0, W1, row_bytes, expert_bytes, IN, OUT, X, by_token,
                                                             ix, e_begin, A_cap, P);
    return 0;
}

template <uint32_t Q>
int launch_stream_q(int TP, const uint8_t* W0, const uint8_t* W1, int64_t row_bytes, int64_t expert_bytes, int IN,
                    int OUT, const float* X, bool by_token, const MoeIndex& ix, int e_begin, int A_cap, float* P,
                    int slots, int RC, cudaStream_t s) {
    if (TP == 1)
        return launch_stream_t<Q, 1>(W0, W1, row_bytes, expert_bytes, IN, OUT, X, by_token, ix, e_begin, A_cap, P,
                                     slots, RC, s);
    return launch_stream_t<Q, 4>(W0, W1, row_bytes, expert_bytes, IN, OUT, X, by_token, ix, e_begin, A_cap, P, slots,
                                 RC, s);
}

int launch_stream(uint32_t q, int TP, const uint8_t* W0, const uint8_t* W1, int64_t row_bytes, int64_t expert_bytes,
                  int IN, int OUT, const float* X, bool by_token, const MoeIndex& ix, int e_begin, int A_cap, float* P,
                  int slots, int RC, cudaStream_t s) {
    if (OUT % 256 != 0 || OUT / 16 > kMoeThreads) return -1;
    switch (q) {
    case kQ4_K: return launch_stream_q<kQ4_K>(TP, W0, W1, row_bytes, expert_bytes, IN, OUT, X, by_token, ix, e_begin,
                                              A_cap, P, slots, RC, s);
    case kQ5_K: return launch_stream_q<kQ5_K>(TP, W0, W1, row_bytes, expert_bytes, IN, OUT, X, by_token, ix, e_begin,
                                              A_cap, P, slots, RC, s);
    case kQ6_K: return launch_stream_q<kQ6_K>(TP, W0, W1, row_bytes, expert_bytes, IN, OUT, X, by_token, ix, e_begin,
                                              A_cap, P, slots, RC, s);
    case kQ8_0: return launch_stream_q<kQ8_0>(TP, W0, W1, row_bytes, expert_bytes, IN, OUT, X, by_token, ix, e_begin,
                                              A_cap, P, slots, RC, s);
    default: return -1;
    }
}

}  // namespace

bool moe_expert_quant_supported(uint32_t q) { return q == kQ4_K || q == kQ5_K || q == kQ6_K || q == kQ8_0; }

// Row chunks for a streamed pass over `mats` matrices: about four CTAs per SM
// in all, at least 32 rows per chunk.
int moe_row_chunks(int slots, int mats, int IN, int sm_count) {
    const int ctas = slots * mats;
    int rc = (4 * (sm_count > 0 ? sm_count : 148) + ctas - 1) / ctas;
    const int maxrc = IN / 32 > 0 ? IN / 32 : 1;
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
    const bool staged = (int64_t)p.T * p.k * 4 <= 40 * 1024;
    moe_assign_kernel<<<1, athreads, staged ? (size_t)p.T * p.k * 4 : 0, s>>>(I(w.ids), p.T, p.k, p.E, p.e_begin,
                                                                              p.e_end, staged, ix);

    // routed experts
    const int slots = p.slots;
    const int TP = p.T == 1 ? 1 : 4;
    if (launch_stream(L.gate.quant, TP, L.gate.W, L.up.W, L.gate.row_bytes, L.gate.expert_bytes, p.n_embd, p.n_ff,
                      L.x, true, ix, p.e_begin, A, F(w.pgu), slots, p.rc_gu, s))
        return -2;
    moe_swiglu_kernel<<<grid_for((int64_t)A * p.n_ff, p.sm_count), 256, 0, s>>>(F(w.pgu), p.rc_gu, A, p.n_ff,
                                                                                 ix.n_assign, F(w.h));
    if (launch_stream(L.down.quant, TP, L.down.W, nullptr, L.down.row_bytes, L.down.expert_bytes, p.n_ff, p.n_embd,
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
