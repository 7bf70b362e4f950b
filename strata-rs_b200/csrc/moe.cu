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
#include <cuda_fp16.h>

#include <cmath>

#include "expf_libm.cuh"
#include "kernels.cuh"
#include "moe.cuh"
#include "quant.cuh"

namespace strata {
namespace {

constexpr int kMoeThreads = 256;

// f32 exp rounded from a double exp (correctly rounded except within about
// 2^-29 ulp of a rounding boundary), standing in for Rust's f32::exp in silu
// and sigmoid (whose results the 1e-3 output bound covers); the router's
// softmax uses expf_libm, the C library's expf bit for bit.
__device__ __forceinline__ float exp_f32(float x) { return (float)exp((double)x); }
__device__ __forceinline__ float silu_f32(float x) { return x / (1.0f + exp_f32(-x)); }      // ops.rs:85-87
__device__ __forceinline__ float sigmoid_f32(float x) { return 1.0f / (1.0f + exp_f32(-x)); }  // ops.rs:90-92

// Programmatic dependent launch: every kernel of the layer's chain lets the
// next one launch at once (its CTAs start while this grid's last wave runs)
// and waits for the previous grid's completion and memory before reading it.
__device__ __forceinline__ void pdl_entry() {
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Launches `kern` as a programmatic dependent of the stream's previous kernel.
template <typename... KArgs, typename... Args>
void launch_dep(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// ------------------------------------------------------------------ routing

// Routing of one token by one warp (moe.rs:48-90): the E probabilities in
// `sp` (shared memory), ids ascending and renormalised weights to ids/wts
// (k each) and, when given, the ids to ids_s too.
__device__ void route_token(const float* __restrict__ lg, int E, int k, float* sp, int lane, int* __restrict__ ids,
                            float* __restrict__ wts, int* ids_s) {
    // the logits into sp (each lane its own entries i = lane mod 32) and their maximum
    float mx = -INFINITY;
    for (int i = lane; i < E; i += 32) {
        const float v = lg[i];
        sp[i] = v;
        mx = fmaxf(mx, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    // exp as the C library rounds it (expf_libm): the rounded double exp in a
    // loop without calls, the few inputs near a rounding midpoint (bit j of
    // `near`: entry lane + 32 j of the 1024-entry chunk) settled afterwards
    for (int i0 = 0; i0 < E; i0 += 1024) {
        uint32_t near = 0;
#pragma unroll 8
        for (int j = 0; j < 32; ++j) {
            const int i = i0 + 32 * j + lane;
            if (i < E) {
                bool exact;
                const float r = expf_libm_try(sp[i] - mx, exact);
                if (exact) sp[i] = r;
                else near |= 1u << j;
            }
        }
        while (near) {
            const int j = __ffs((int)near) - 1;
            near &= near - 1;
            const int i = i0 + 32 * j + lane;
            sp[i] = expf_libm_near(sp[i] - mx);
        }
    }
    double sum = 0.0;
    for (int i = lane; i < E; i += 32) sum += (double)sp[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
    const float inv = (float)(1.0 / sum);
    for (int i = lane; i < E; i += 32) sp[i] = sp[i] * inv;
    __syncwarp();
    // the k first experts of the order (probability desc, index asc): k rounds
    // of a warp arg-max over the experts not yet taken (lane-owned bit masks:
    // expert i belongs to lane i % 32, bit i / 32). `before` is the reference's
    // comparator (partial_cmp, unwrap_or(Equal), then the index): two values of
    // which one is NaN compare equal and fall back to the index. A NaN or +Inf
    // logit makes the f64 sum, and so every probability, NaN; the order is then
    // the index order and the ids are 0..k-1, as in the reference. The order is
    // total either way, so every round takes an expert that exists.
    auto before = [](float v, int i, float w, int j) {
        return (v != v || w != w) ? i < j : (v > w || (v == w && i < j));
    };
    const int kk = k < E ? k : E;
    uint32_t taken = 0;
    int sel = 0;  // lane j < kk ends holding the j-th chosen id
    for (int r = 0; r < kk; ++r) {
        float bp = -1.0f;
        int bi = 0x7FFFFFFF;
        for (int i = lane, m = 0; i < E; i += 32, ++m) {
            const float v = sp[i];
            if (!((taken >> m) & 1u) && before(v, i, bp, bi)) {
                bp = v;
                bi = i;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float op = __shfl_xor_sync(0xFFFFFFFFu, bp, o);
            const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
            if (before(op, oi, bp, bi)) {
                bp = op;
                bi = oi;
            }
        }
        bi = bi < E ? bi : E - 1;  // never taken: an untaken expert always exists (kk <= E)
        if (lane == r) sel = bi;
        if (lane == (bi & 31)) taken |= 1u << ((bi >> 5) & 31);
    }
    // ids ascending: lane q receives the chosen id of rank q
    const float psel = lane < kk ? sp[sel] : 0.0f;
    int rank = 0;
    for (int j = 0; j < kk; ++j) {
        const int oj = __shfl_sync(0xFFFFFFFFu, sel, j);
        rank += (lane < kk && oj < sel) ? 1 : 0;
    }
    int id_q = 0x7FFFFFFF;
    float p_q = 0.0f;
    for (int j = 0; j < kk; ++j) {
        const int rj = __shfl_sync(0xFFFFFFFFu, rank, j);
        const int sj = __shfl_sync(0xFFFFFFFFu, sel, j);
        const float pj = __shfl_sync(0xFFFFFFFFu, psel, j);
        if (lane == rj) {
            id_q = sj;
            p_q = pj;
        }
    }
    // weights: f64 sum in ascending id order, as moe.rs:80-90
    double ws = 0.0;
    for (int j = 0; j < kk; ++j) ws += (double)__shfl_sync(0xFFFFFFFFu, p_q, j);
    const double sden = ws > 0x1p-14 ? ws : 0x1p-14;
    if (lane < k) {
        const int id = lane < kk ? id_q : -1;
        ids[lane] = id;
        wts[lane] = lane < kk ? (float)((double)p_q / sden) : 0.0f;
        if (ids_s) ids_s[lane] = id;
    }
}

// One warp per token (kRouteWarps tokens per CTA); the token's E
// probabilities live in shared memory.
constexpr int kRouteWarps = 4;
__global__ void __launch_bounds__(kRouteWarps * 32) moe_route_kernel(const float* __restrict__ logits, int T, int E,
                                                                     int k, int* __restrict__ ids,
                                                                     float* __restrict__ wts) {
    pdl_entry();
    extern __shared__ float sp_all[];  // kRouteWarps x E
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * kRouteWarps + warp;
    if (t >= T) return;
    route_token(logits + (int64_t)t * E, E, k, sp_all + warp * E, lane, ids + (int64_t)t * k, wts + (int64_t)t * k,
                nullptr);
}

// ------------------------------------------------------------------ assignment

// One CTA (kAssignThreads threads, E <= 1024). Counts per expert come from
// shared-memory atomics (order-free); offsets and the active list from scans
// over the experts in ascending order; an entry's rank within its expert is
// the number of earlier entries (earlier tokens) routed to the same expert,
// so every list is in token order whatever the thread schedule.
constexpr int kAssignThreads = 1024;
__device__ void assign_block(const int* ids, int T, int k, int E, int e_begin, int e_end, MoeIndex ix) {
    __shared__ int cnt_s[1024], scan[1024], slot_s[1024];
    const int tid = threadIdx.x;
    const int64_t TK = (int64_t)T * k;
    if (TK <= 32) {
        // decode: one warp, entry i on lane i. Counts and offsets come from
        // comparisons with every other entry; only the active experts' cnt /
        // off are written (nothing reads the others).
        if (tid >= 32) return;
        const int lane = tid;
        const int e = lane < TK ? ids[lane] : -1;
        const bool held = lane < TK && e >= e_begin && e < e_end;
        int less = 0, same_before = 0, cnt = 0;
        bool first = true;
        for (int j = 0; j < (int)TK; ++j) {
            const int ej = __shfl_sync(0xFFFFFFFFu, e, j);
            const bool hj = ej >= e_begin && ej < e_end;
            if (held && hj) {
                less += ej < e ? 1 : 0;
                if (ej == e) {
                    ++cnt;
                    if (j < lane) {
                        ++same_before;
                        first = false;
                    }
                }
            }
        }
        const unsigned firsts = __ballot_sync(0xFFFFFFFFu, held && first);
        int distinct_less = 0;
        for (int j = 0; j < (int)TK; ++j) {
            const int ej = __shfl_sync(0xFFFFFFFFu, e, j);
            distinct_less += ((firsts >> j) & 1u) && ej < e ? 1 : 0;
        }
        const unsigned helds = __ballot_sync(0xFFFFFFFFu, held);
        if (held) {
            const int at = less + same_before;  // entries of smaller experts, then earlier tokens
            ix.tok[at] = lane / k;
            ix.pos[lane] = at;
            if (first) {
                ix.cnt[e] = cnt;
                ix.off[e] = less;
                ix.active[distinct_less] = e;
                if (distinct_less < ix.slots) ix.slot_info[distinct_less] = make_int4(e, less, cnt, lane / k);
            }
        } else if (lane < TK) {
            ix.pos[lane] = -1;
        }
        const int n_act = __popc(firsts);
        if (lane >= n_act && lane < ix.slots) ix.slot_info[lane] = make_int4(-1, 0, 0, 0);
        if (lane == 0) {
            ix.n_active[0] = n_act;
            ix.n_assign[0] = __popc(helds);
        }
        return;
    }
    for (int e = tid; e < 1024; e += blockDim.x) cnt_s[e] = 0;
    __syncthreads();
    for (int64_t i = tid; i < TK; i += blockDim.x) {
        const int e = ids[i];
        if (e >= e_begin && e < e_end) atomicAdd(&cnt_s[e], 1);
    }
    __syncthreads();
    // exclusive scans over e ascending: counts -> offsets, active flags -> slots
    const int c = tid < E ? cnt_s[tid] : 0;
    scan[tid] = c;
    __syncthreads();
    for (int sh = 1; sh < (int)blockDim.x; sh <<= 1) {
        const int v = tid >= sh ? scan[tid - sh] : 0;
        __syncthreads();
        scan[tid] += v;
        __syncthreads();
    }
    const int off = scan[tid] - c;
    const int total = scan[blockDim.x - 1];
    __syncthreads();
    scan[tid] = c > 0 ? 1 : 0;
    __syncthreads();
    for (int sh = 1; sh < (int)blockDim.x; sh <<= 1) {
        const int v = tid >= sh ? scan[tid - sh] : 0;
        __syncthreads();
        scan[tid] += v;
        __syncthreads();
    }
    if (tid < E) {
        ix.cnt[tid] = c;
        ix.off[tid] = off;
        if (c > 0) ix.active[scan[tid] - 1] = tid;
    }
    slot_s[tid] = c > 0 ? scan[tid] - 1 : -1;
    const int n_act = scan[blockDim.x - 1];
    if (tid == 0) {
        ix.n_active[0] = n_act;
        ix.n_assign[0] = total;
    }
    if (tid >= n_act && tid < ix.slots) ix.slot_info[tid] = make_int4(-1, 0, 0, 0);
    __syncthreads();
    scan[tid] = c;     // counts and
    cnt_s[tid] = off;  // offsets, for the placement below
    __syncthreads();
    for (int64_t i = tid; i < TK; i += blockDim.x) {
        const int e = ids[i];
        if (e < e_begin || e >= e_end) {
            ix.pos[i] = -1;
            continue;
        }
        int r = 0;
#pragma unroll 8
        for (int64_t q = 0; q < i; ++q) r += ids[q] == e ? 1 : 0;
        const int at = cnt_s[e] + r;
        ix.tok[at] = (int)(i / k);
        ix.pos[i] = at;
        if (r == 0 && slot_s[e] < ix.slots) ix.slot_info[slot_s[e]] = make_int4(e, cnt_s[e], scan[e], (int)(i / k));
    }
}

// The routing ids are staged in shared memory when they fit (staged = true).
__global__ void __launch_bounds__(kAssignThreads)
moe_assign_kernel(const int* __restrict__ ids_g, int T, int k, int E, int e_begin, int e_end, bool staged,
                  MoeIndex ix) {
    pdl_entry();
    extern __shared__ int ids_s[];
    if (staged) {
        for (int64_t i = threadIdx.x; i < (int64_t)T * k; i += blockDim.x) ids_s[i] = ids_g[i];
        __syncthreads();
    }
    assign_block(staged ? ids_s : ids_g, T, k, E, e_begin, e_end, ix);
}

// Up to 32 tokens: routing (a warp per token) and assignment in one CTA, the
// ids handed over in shared memory: one launch less on the decode path.
constexpr int kFusedRouteTokens = 32;
__global__ void __launch_bounds__(kAssignThreads)
moe_route_assign_kernel(const float* __restrict__ logits, int T, int E, int k, int* __restrict__ ids,
                        float* __restrict__ wts, int e_begin, int e_end, MoeIndex ix) {
    pdl_entry();
    extern __shared__ float dyn[];  // T x E probabilities, then T x k ids
    int* ids_s = reinterpret_cast<int*>(dyn + (int64_t)T * E);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp < T)
        route_token(logits + (int64_t)warp * E, E, k, dyn + (int64_t)warp * E, lane, ids + (int64_t)warp * k,
                    wts + (int64_t)warp * k, ids_s + warp * k);
    __syncthreads();
    assign_block(ids_s, T, k, E, e_begin, e_end, ix);
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

// Bytes b0 and b0 + 1 of v (each < 256) as exact floats: the byte lands in
// the mantissa of 2^23 and 2^23 is subtracted.
__device__ __forceinline__ float2 byte_pair_f(uint32_t v, int b0) {
    const float2 m = make_float2(__uint_as_float(__byte_perm(v, 0x4B000000u, 0x7540u | b0)),
                                 __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7540u | (b0 + 1))));
    return __fadd2_rn(m, make_float2(-8388608.0f, -8388608.0f));
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
    // a multiple of RL; even when rows are not 4-byte multiples (Q6_K), so
    // every tile starts on a 4-byte boundary
    const int step = (row_bytes % 4 != 0 && RL % 2 != 0) ? 2 * RL : RL;
    int rs = (int)(kStageBytes / row_bytes);
    rs = rs > 64 ? 64 : rs;
    rs -= rs % step;
    return rs < step ? step : rs;
}

// Pitches of the tensor-core pass's shared arrays: a staged row pitch whose
// 32-bit word count is 8 mod 32, and an x pitch of 4 mod 32 floats, so that
// the 4 consecutive rows a fragment load touches use different banks.
__host__ __device__ inline int64_t mma_row_pitch(int64_t row_bytes) {
    const int64_t words = row_bytes / 4;
    return row_bytes + 4 * ((8 - words % 32 + 32) % 32);
}
__host__ __device__ inline int mma_x_pitch(int rs) { return rs + (4 - rs % 32 + 32) % 32; }

// Rows per tile of the tensor-core pass: a multiple of 16 (one k-tile), about kStageBytes.
__host__ __device__ inline int mma_tile_rows(int64_t row_bytes) {
    int rs = (int)(kStageBytes / row_bytes);
    rs -= rs % 16;
    return rs < 16 ? 16 : (rs > 64 ? 64 : rs);
}

template <uint32_t Q, int TP>
__global__ void __launch_bounds__(kMoeThreads, 2)
moe_stream_kernel(const uint8_t* __restrict__ W0, const uint8_t* __restrict__ W1, int64_t row_bytes,
                  int64_t expert_bytes, int IN, int OUT, const float* __restrict__ X, bool by_token, MoeIndex ix,
                  int e_begin, int A_cap, float* __restrict__ P) {
    pdl_entry();
    extern __shared__ __align__(16) uint8_t dsm[];
    const int nmat = W1 ? 2 : 1;
    const int slot = blockIdx.x / nmat, m = blockIdx.x % nmat;
    if (slot >= ix.n_active[0]) return;
    const int e = ix.active[slot];
    const int a0 = ix.off[e], n = ix.cnt[e];
    // row chunk rc of RC on 16-row boundaries: a Q6_K row is 210 bytes per
    // block, so only an even first row keeps the 4-byte copies aligned
    const int RC = gridDim.y, rc = blockIdx.y, nk = IN / 16;
    const int r0 = 16 * (int)((int64_t)nk * rc / RC), r1 = 16 * (int)((int64_t)nk * (rc + 1) / RC);
    const int U = OUT / 16, RL = kMoeThreads / U;
    const int tid = threadIdx.x, u = tid % U, lane = tid / U;
    const int RS = tile_rows(row_bytes, RL);
    const int64_t tile_bytes = (int64_t)RS * row_bytes;
    uint8_t* wring = dsm;                                                   // kStages x tile_bytes
    float* xring = reinterpret_cast<float*>(dsm + kStages * tile_bytes);    // kStages x TP x RS
    float* red = xring + kStages * TP * RS;                                 // kMoeThreads x 17
    const int G = OUT / 256;
    float* tab = red + kMoeThreads * 17;                                    // RS x G x 16 scales
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
        float accm[TP][2];  // sum_i x dmin m of the unit's two sub-blocks (K-quants with mins)
#pragma unroll
        for (int b = 0; b < TP; ++b) {
            accm[b][0] = accm[b][1] = 0.0f;
#pragma unroll
            for (int l = 0; l < 16; ++l) acc[b][l] = 0.0f;
        }
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
            if constexpr (Q == kQ4_K || Q == kQ5_K) {
                // the tile's scales: d sc_j and dmin m_j of every (row, 256-column group)
                for (int q = tid; q < rows * G; q += kMoeThreads) {
                    const int rr = q / G, gg = q - rr * G;
                    const uint4 h = *reinterpret_cast<const uint4*>(wt + (int64_t)rr * row_bytes + gg * block_bytes(Q));
                    uint32_t sc_lo, sc_hi, m_lo, m_hi;
                    scales_k4_packed(h.y, h.z, h.w, sc_lo, sc_hi, m_lo, m_hi);
                    const float d = h2f(h.x), dm = h2f(h.x >> 16);
                    float* tb = tab + q * 16;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        tb[j] = d * (float)(((j < 4 ? sc_lo : sc_hi) >> (8 * (j & 3))) & 0xFFu);
                        tb[8 + j] = dm * (float)(((j < 4 ? m_lo : m_hi) >> (8 * (j & 3))) & 0xFFu);
                    }
                }
                __syncthreads();
                // y = sum_i q (x d sc) - sum_i x (dmin m): the scale rides on x
                const int cc = t >> 2, pp = t & 3, jA = 2 * cc;
                const int qoff = ((Q == kQ4_K) ? 16 : 48) + 32 * cc + 8 * pp;
                for (int r = lane; r < rows; r += RL) {
                    const uint8_t* blk = wt + (int64_t)r * row_bytes + (int64_t)g * block_bytes(Q);
                    const uint2 qv = *reinterpret_cast<const uint2*>(blk + qoff);
                    uint32_t lo0 = qv.x & 0x0F0F0F0Fu, lo1 = qv.y & 0x0F0F0F0Fu;
                    uint32_t hi0 = (qv.x >> 4) & 0x0F0F0F0Fu, hi1 = (qv.y >> 4) & 0x0F0F0F0Fu;
                    if constexpr (Q == kQ5_K) {
                        const uint2 hv = *reinterpret_cast<const uint2*>(blk + 16 + 8 * pp);
                        lo0 |= ((hv.x >> jA) & 0x01010101u) << 4;
                        lo1 |= ((hv.y >> jA) & 0x01010101u) << 4;
                        hi0 |= ((hv.x >> (jA + 1)) & 0x01010101u) << 4;
                        hi1 |= ((hv.y >> (jA + 1)) & 0x01010101u) << 4;
                    }
                    float2 qf[8];  // columns colA..colA+7 (pairs), then colB..colB+7
                    qf[0] = byte_pair_f(lo0, 0);
                    qf[1] = byte_pair_f(lo0, 2);
                    qf[2] = byte_pair_f(lo1, 0);
                    qf[3] = byte_pair_f(lo1, 2);
                    qf[4] = byte_pair_f(hi0, 0);
                    qf[5] = byte_pair_f(hi0, 2);
                    qf[6] = byte_pair_f(hi1, 0);
                    qf[7] = byte_pair_f(hi1, 2);
                    const float* tb = tab + (r * G + g) * 16;
                    const float2 dsc = *reinterpret_cast<const float2*>(tb + jA);
                    const float2 dmm = *reinterpret_cast<const float2*>(tb + 8 + jA);
#pragma unroll
                    for (int b = 0; b < TP; ++b) {
                        if (b < np) {
                            const float xv = xt[b * RS + r];
                            const float2 xa = make_float2(xv * dsc.x, xv * dsc.x);
                            const float2 xb = make_float2(xv * dsc.y, xv * dsc.y);
                            accm[b][0] = fmaf(xv, dmm.x, accm[b][0]);
                            accm[b][1] = fmaf(xv, dmm.y, accm[b][1]);
                            float2* a2 = reinterpret_cast<float2*>(acc[b]);
#pragma unroll
                            for (int k2 = 0; k2 < 4; ++k2) a2[k2] = __ffma2_rn(qf[k2], xa, a2[k2]);
#pragma unroll
                            for (int k2 = 4; k2 < 8; ++k2) a2[k2] = __ffma2_rn(qf[k2], xb, a2[k2]);
                        }
                    }
                }
            } else {
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
            }
            __syncthreads();  // the stage is rewritten by the next issue
        }
        cp_async_wait<0>();
        if constexpr (Q == kQ4_K || Q == kQ5_K) {
#pragma unroll
            for (int b = 0; b < TP; ++b)
#pragma unroll
                for (int l = 0; l < 8; ++l) {
                    acc[b][l] -= accm[b][0];
                    acc[b][8 + l] -= accm[b][1];
                }
        }
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
    pdl_entry();
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

// out[t][c] = sum_j w[t][j] * down[pos(t,j)][c] over t's local experts
// (skipping zero weights, moe.rs:111-113), + sg[t] * Ds[t][c]. A group of
// L >= k lanes serves one output: lane j adds expert j's row-chunk partials,
// the group sums its lanes with a fixed shuffle tree.
__global__ void moe_combine_kernel(const float* __restrict__ Pd, int RC, int A_cap, int OUT, const int* __restrict__ pos,
                                   const float* __restrict__ wts, int T, int k, int L, const float* __restrict__ Ds,
                                   const float* __restrict__ sg, float* __restrict__ out) {
    pdl_entry();
    const int64_t n = (int64_t)T * OUT;
    const int j = threadIdx.x % L;
    const int64_t per_block = blockDim.x / L;
    for (int64_t base = blockIdx.x * per_block; base < n; base += (int64_t)gridDim.x * per_block) {
        const int64_t i = base + threadIdx.x / L;
        const bool live = i < n;
        const int64_t t = live ? i / OUT : 0, c = live ? i - t * OUT : 0;
        float v = 0.0f;
        if (live && j < k) {
            const int a = pos[t * k + j];
            const float w = wts[t * k + j];
            if (a >= 0 && w != 0.0f) {
                float d = 0.0f;
                for (int rc = 0; rc < RC; ++rc) d += Pd[((int64_t)rc * A_cap + a) * OUT + c];
                v = w * d;
            }
        }
        for (int o = L / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
        if (live && j == 0) {
            if (Ds) v += sg[t] * Ds[i];
            out[i] = v;
        }
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

// ---- tensor-core form of the streamed pass (Q4_K / Q5_K)
//
// Same CTA shape, ring and scale table as moe_stream_kernel; the products
// run on mma.sync m16n8k16 (f16 in, f32 out, one k-tile per MMA, summed over
// k-tiles with fp32 adds). With m = 16 output
// columns of one sub-block j and k = 16 input rows:
//   A[c][i] = q[i][c]                       exact small integers in fp16
//   B[i][n] = x_t[i] S_t d_i sc_ij          n = (token t, limb): two fp16
//                                           limbs, hi + lo 2^-11 (22 bits)
//   D[c][n] = sum_i A B                     f32
// so that y[t][c] = (D[c][t,hi] + D[c][t,lo] 2^-11) / S_t
//                   - sum_i x_t[i] dmin_i m_ij   (min term, CUDA cores).
// S_t is a power of two chosen per CTA pass from max|x_t| and max d over the
// CTA's rows so that |B| < 2^14 (no fp16 overflow; the limbs keep ~22 bits).
// Warp w owns m-tiles MPW w .. MPW w + MPW - 1 (MPW = OUT / 128). Within a
// sub-block's two m-tiles, fragment row g of m-tile mt holds column 4g + 2mt
// and row g + 8 column 4g + 2mt + 1, so a lane's four columns are one 32-bit
// word of every quant row.
// d = A B (zero accumulator input): one k-tile's products, added to the running
// sums by the caller with fp32 adds (the tensor cores' own accumulation of
// long chains loses low bits; one 16-product sum does not)
__device__ __forceinline__ void mma16816z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    const float z = 0.0f;
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));  // (a & b) | c
    return d;
}
// f16x2 arithmetic on bit patterns (constants as immediate bit patterns:
// 0x6400 = 1024, 0x2C00 = 1/16, 0xD400 = -64)
__device__ __forceinline__ uint32_t hsub2_bits(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t hfma2_bits(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t f16x2_bits(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

template <uint32_t Q, int MPW>
__global__ void __launch_bounds__(kMoeThreads, 2)
moe_mma_kernel(const uint8_t* __restrict__ W0, const uint8_t* __restrict__ W1, int64_t row_bytes,
               int64_t expert_bytes, int IN, int OUT, const float* __restrict__ X, bool by_token, MoeIndex ix,
               int e_begin, int A_cap, float* __restrict__ P) {
    pdl_entry();
    constexpr int TP = 4;  // tokens per pass: n = 8 = 4 tokens x 2 limbs
    constexpr int SPW = MPW / 2;  // sub-blocks per warp
    extern __shared__ __align__(16) uint8_t dsm[];
    const int nmat = W1 ? 2 : 1;
    const int slot = blockIdx.x / nmat, m = blockIdx.x % nmat;
    if (slot >= ix.n_active[0]) return;
    const int e = ix.active[slot];
    const int a0 = ix.off[e], n = ix.cnt[e];
    // row chunk rc of RC, on 16-row (k-tile) boundaries
    const int RC = gridDim.y, rc = blockIdx.y, nk = IN / 16;
    const int r0 = 16 * (int)((int64_t)nk * rc / RC), r1 = 16 * (int)((int64_t)nk * (rc + 1) / RC);
    const int G = OUT / 256;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
    // shared-memory pitches chosen so that the 4 rows a fragment load touches
    // (t4 = 0..3, consecutive rows) fall on different banks
    const int RS = mma_tile_rows(row_bytes);
    const int64_t RB = mma_row_pitch(row_bytes);  // staged row pitch (bytes)
    const int RSX = mma_x_pitch(RS);              // x ring pitch per token (floats)
    const int TPITCH = G * 16 + 8;                // scale table pitch per row (floats)
    const int64_t tile_bytes = (int64_t)RS * RB;
    uint8_t* wring = dsm;
    float* xring = reinterpret_cast<float*>(dsm + kStages * tile_bytes);  // kStages x TP x RSX
    float* tab = xring + kStages * TP * RSX;                              // RS x TPITCH
    __shared__ float red_max[2][kMoeThreads / 32];
    __shared__ int src[TP];
    __shared__ float sinv[TP], sval[TP];
    const uint8_t* Wm = (m == 0 ? W0 : W1) + (int64_t)(e - e_begin) * expert_bytes;
    // this warp's sub-blocks: global sub-block index sb = SPW warp + s (8 per group)
    const int sb0 = SPW * warp;
    const int ntiles = (r1 - r0 + RS - 1) / RS;

    // max d over the CTA's rows (once per CTA)
    float dmax = 0.0f;
    for (int q = tid; q < (r1 - r0) * G; q += kMoeThreads) {
        const int rr = q / G, gg = q - rr * G;
        const uint8_t* hb = Wm + (int64_t)(r0 + rr) * row_bytes + gg * block_bytes(Q);
        dmax = fmaxf(dmax, fabsf(h2f((uint32_t)hb[0] | ((uint32_t)hb[1] << 8))));
    }
    for (int o = 16; o > 0; o >>= 1) dmax = fmaxf(dmax, __shfl_xor_sync(0xFFFFFFFFu, dmax, o));
    if (lane == 0) red_max[0][warp] = dmax;
    __syncthreads();
    if (tid == 0) {
        float v = 0.0f;
        for (int w = 0; w < kMoeThreads / 32; ++w) v = fmaxf(v, red_max[0][w]);
        red_max[1][0] = v;
    }
    __syncthreads();
    dmax = red_max[1][0];

    for (int p0 = 0; p0 < n; p0 += TP) {
        const int np = n - p0 < TP ? n - p0 : TP;
        if (tid < TP) {
            const int a = a0 + p0 + (tid < np ? tid : 0);
            src[tid] = by_token ? ix.tok[a] : a;
        }
        __syncthreads();
        // per-token scale S = 2^e with max |x| d 63 S <= 2^14 (|sc| <= 63)
        if (warp < TP) {
            float xm = 0.0f;
            const float* xr = X + (int64_t)src[warp] * IN;
            for (int i = r0 + lane; i < r1; i += 32) xm = fmaxf(xm, fabsf(xr[i]));
            for (int o = 16; o > 0; o >>= 1) xm = fmaxf(xm, __shfl_xor_sync(0xFFFFFFFFu, xm, o));
            if (lane == 0) {
                const float bound = xm * dmax * 63.0f;
                int ex = 0;
                if (bound > 0.0f && bound < INFINITY) {
                    frexpf(bound, &ex);        // bound < 2^ex
                    ex = 14 - ex;              // bound * 2^ex < 2^14
                    ex = ex > 100 ? 100 : (ex < -100 ? -100 : ex);
                }
                sval[warp] = ldexpf(1.0f, ex);
                sinv[warp] = ldexpf(1.0f, -ex);
            }
        }
        __syncthreads();
        auto issue = [&](int tile) {
            if (tile < ntiles) {
                const int i0 = r0 + tile * RS;
                const int rows = r1 - i0 < RS ? r1 - i0 : RS;
                uint8_t* dst = wring + (int64_t)(tile % kStages) * tile_bytes;
                const uint8_t* gsrc = Wm + (int64_t)i0 * row_bytes;
                const int cpr = (int)(row_bytes / 16);  // 16-byte chunks per row
                for (int c = tid; c < rows * cpr; c += kMoeThreads) {
                    const int rr = c / cpr, cc = c - rr * cpr;
                    cp_async16(dst + rr * RB + 16 * cc, gsrc + (int64_t)rr * row_bytes + 16 * cc);
                }
                float* xd = xring + (tile % kStages) * TP * RSX;
                for (int q = tid; q < TP * rows; q += kMoeThreads) {
                    const int b = q / rows, r = q % rows;
                    cp_async4(xd + b * RSX + r, X + (int64_t)src[b] * IN + i0 + r);
                }
            }
            cp_async_commit();
        };
        float acc[MPW][4];
        float accm[SPW];  // min term of this thread's token (g >> 1) and rows, per sub-block
#pragma unroll
        for (int mt = 0; mt < MPW; ++mt)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[mt][c] = 0.0f;
#pragma unroll
        for (int s2 = 0; s2 < SPW; ++s2) accm[s2] = 0.0f;
        const int tok = g >> 1, limb = g & 1;
        const float S = sval[tok];
#pragma unroll
        for (int s = 0; s < kStages - 1; ++s) issue(s);
        for (int tile = 0; tile < ntiles; ++tile) {
            // one barrier per tile: after it this tile's copies (every thread's
            // part) are visible, and every warp is done with the previous tile,
            // whose stage the issue below rewrites
            cp_async_wait<kStages - 2>();
            __syncthreads();
            issue(tile + kStages - 1);
            const int i0 = r0 + tile * RS;
            const int rows = r1 - i0 < RS ? r1 - i0 : RS;
            const uint8_t* wt = wring + (int64_t)(tile % kStages) * tile_bytes;
            const float* xt = xring + (tile % kStages) * TP * RSX;
            // the scale table entries of this warp's own sub-blocks (d sc and dmin m
            // per row): no other warp reads them, so a warp needs no barrier to use them
            for (int rr = lane; rr < rows; rr += 32) {
                int gcur = -1;
                uint32_t sc_lo = 0, sc_hi = 0, m_lo = 0, m_hi = 0;
                float d = 0.0f, dm = 0.0f;
#pragma unroll
                for (int s2 = 0; s2 < SPW; ++s2) {
                    const int sbg = sb0 + s2, gg = sbg >> 3, j = sbg & 7;
                    if (gg >= G) break;
                    if (gg != gcur) {
                        const uint4 h = *reinterpret_cast<const uint4*>(wt + (int64_t)rr * RB + gg * block_bytes(Q));
                        scales_k4_packed(h.y, h.z, h.w, sc_lo, sc_hi, m_lo, m_hi);
                        d = h2f(h.x);
                        dm = h2f(h.x >> 16);
                        gcur = gg;
                    }
                    float* tb = tab + rr * TPITCH + gg * 16;
                    tb[j] = d * (float)(((j < 4 ? sc_lo : sc_hi) >> (8 * (j & 3))) & 0xFFu);
                    tb[8 + j] = dm * (float)(((j < 4 ? m_lo : m_hi) >> (8 * (j & 3))) & 0xFFu);
                }
            }
            __syncwarp();
            for (int k0 = 0; k0 + 16 <= rows; k0 += 16) {
                // the k index of the MMA maps to rows of the tile as k = 2t4 -> t4,
                // 2t4 + 1 -> t4 + 4, 2t4 + 8 -> t4 + 8, 2t4 + 9 -> t4 + 12 (A and B
                // agree, so the sum over k is the sum over the 16 rows); the 4 lanes
                // t4 of a load then read 4 consecutive rows. B column: token `tok`, limb `limb`.
                const int ra = k0 + t4, rb = ra + 8;
                const float xa0 = xt[tok * RSX + ra], xa1 = xt[tok * RSX + ra + 4];
                const float xb0 = xt[tok * RSX + rb], xb1 = xt[tok * RSX + rb + 4];
                const float sa0 = xa0 * S, sa1 = xa1 * S, sb0v = xb0 * S, sb1v = xb1 * S;
                // Q5_K: the fifth bits of this lane's 4 columns, rows ra .. rb + 1
                uint32_t qh_a0 = 0, qh_a1 = 0, qh_b0 = 0, qh_b1 = 0;
                int grp_loaded = -1;
                uint32_t wa0 = 0, wa1 = 0, wb0 = 0, wb1 = 0;
#pragma unroll
                for (int s2 = 0; s2 < SPW; ++s2) {
                    const int sbg = sb0 + s2;            // sub-block over the whole row
                    const int grp = sbg >> 3, j = sbg & 7;
                    const int cc = j >> 1, h = j & 1;
                    const uint8_t* rowa = wt + (int64_t)ra * RB + grp * block_bytes(Q);
                    const uint8_t* rowb = wt + (int64_t)rb * RB + grp * block_bytes(Q);
                    constexpr int R4 = 4;  // the second row of each pair is 4 rows on
                    // the 4 quant bytes of columns 4g .. 4g + 3 of sub-blocks 2cc, 2cc + 1,
                    // loaded once for both nibbles (h = 0 then h = 1 on the next s2)
                    if (h == 0 || s2 == 0) {
                        const int qo = ((Q == kQ4_K) ? 16 : 48) + 32 * cc + 4 * g;
                        wa0 = *reinterpret_cast<const uint32_t*>(rowa + qo);
                        wa1 = *reinterpret_cast<const uint32_t*>(rowa + R4 * RB + qo);
                        wb0 = *reinterpret_cast<const uint32_t*>(rowb + qo);
                        wb1 = *reinterpret_cast<const uint32_t*>(rowb + R4 * RB + qo);
                    }
                    if constexpr (Q == kQ5_K) {
                        if (grp != grp_loaded) {
                            qh_a0 = *reinterpret_cast<const uint32_t*>(rowa + 16 + 4 * g);
                            qh_a1 = *reinterpret_cast<const uint32_t*>(rowa + R4 * RB + 16 + 4 * g);
                            qh_b0 = *reinterpret_cast<const uint32_t*>(rowb + 16 + 4 * g);
                            qh_b1 = *reinterpret_cast<const uint32_t*>(rowb + R4 * RB + 16 + 4 * g);
                            grp_loaded = grp;
                        }
                    }
                    // B fragment: both limbs computed, the lane's one selected (no divergence)
                    const float* ta = tab + ra * TPITCH + grp * 16;
                    const float* tbp = tab + rb * TPITCH + grp * 16;
                    const float va0 = sa0 * ta[j], va1 = sa1 * ta[R4 * TPITCH + j];
                    const float vb0 = sb0v * tbp[j], vb1 = sb1v * tbp[R4 * TPITCH + j];
                    const uint32_t ha = f16x2_bits(va0, va1), hbw = f16x2_bits(vb0, vb1);
                    const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&ha));
                    const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&hbw));
                    const uint32_t la = f16x2_bits((va0 - fa.x) * 2048.0f, (va1 - fa.y) * 2048.0f);
                    const uint32_t lb = f16x2_bits((vb0 - fb.x) * 2048.0f, (vb1 - fb.y) * 2048.0f);
                    const uint32_t b0 = limb ? la : ha, b1 = limb ? lb : hbw;
                    accm[s2] = fmaf(xa0, ta[8 + j], accm[s2]);
                    accm[s2] = fmaf(xa1, ta[R4 * TPITCH + 8 + j], accm[s2]);
                    accm[s2] = fmaf(xb0, tbp[8 + j], accm[s2]);
                    accm[s2] = fmaf(xb1, tbp[R4 * TPITCH + 8 + j], accm[s2]);
                    // A fragments. Column permutation: m-tile mt, fragment row g -> column
                    // 4g + 2mt, row g + 8 -> column 4g + 2mt + 1 (all 4 in one word per row).
#pragma unroll
                    for (int mt = 0; mt < 2; ++mt) {
                        uint32_t a[4];
#pragma unroll
                        for (int q = 0; q < 4; ++q) {  // a0 (ra, m=g), a1 (ra, g+8), a2 (rb, g), a3 (rb, g+8)
                            const int bsel = 2 * mt + (q & 1);
                            const uint32_t sel = (uint32_t)(bsel | (bsel << 4) | ((4 + bsel) << 8) | ((4 + bsel) << 12));
                            const uint32_t pr = (q < 2) ? __byte_perm(wa0, wa1, sel) : __byte_perm(wb0, wb1, sel);
                            uint32_t hb5 = 0;
                            if constexpr (Q == kQ5_K) {
                                const uint32_t ph = (q < 2) ? __byte_perm(qh_a0, qh_a1, sel) : __byte_perm(qh_b0, qh_b1, sel);
                                hb5 = ((ph >> j) & 0x00010001u) << (h ? 8 : 4);
                            }
                            if (h == 0) {  // 1024 + q -> q
                                a[q] = hsub2_bits(lop3_and_or(pr, 0x000F000Fu, 0x64006400u | hb5), 0x64006400u);
                            } else {       // 1024 + 16 q -> q (exact: 1/16 and 64 are powers of two)
                                a[q] = hfma2_bits(lop3_and_or(pr, 0x00F000F0u, 0x64006400u | hb5), 0x2C002C00u,
                                                  0xD400D400u);
                            }
                        }
                        float dk[4];
                        mma16816z(dk, a[0], a[1], a[2], a[3], b0, b1);
#pragma unroll
                        for (int c = 0; c < 4; ++c) acc[2 * s2 + mt][c] += dk[c];
                    }
                }
            }
        }
        cp_async_wait<0>();
        // min term of (sub-block, token): sum over the 4 lanes t4 (every lane of a
        // token holds the same sums)
#pragma unroll
        for (int s2 = 0; s2 < SPW; ++s2) {
            accm[s2] += __shfl_xor_sync(0xFFFFFFFFu, accm[s2], 1);
            accm[s2] += __shfl_xor_sync(0xFFFFFFFFu, accm[s2], 2);
        }
        // outputs: lane (g, t4) holds columns g and g + 8 of each m-tile for token t4
        // (D columns 2 t4 and 2 t4 + 1 are its hi and lo limbs). The min term of token
        // t4 lives on lanes with g = 2 t4 (lane 8 t4 + t4').
        const float invS = sinv[t4 < TP ? t4 : 0];
#pragma unroll
        for (int s2 = 0; s2 < SPW; ++s2) {
            const float mn = __shfl_sync(0xFFFFFFFFu, accm[s2], 8 * t4);
            const int sbg = sb0 + s2, grp = sbg >> 3, j = sbg & 7;
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
                const float* dd = acc[2 * s2 + mt];
                const float y0 = fmaf(dd[1], 1.0f / 2048.0f, dd[0]) * invS - mn;
                const float y1 = fmaf(dd[3], 1.0f / 2048.0f, dd[2]) * invS - mn;
                if (t4 < np) {  // columns 4g + 2mt and 4g + 2mt + 1 of the sub-block
                    float* dst = P + (((int64_t)rc * nmat + m) * A_cap + a0 + p0 + t4) * OUT + grp * 256 + 32 * j +
                                 4 * g + 2 * mt;
                    dst[0] = y0;
                    dst[1] = y1;
                }
            }
        }
        __syncthreads();
    }
}

size_t stream_smem(int64_t row_bytes, int OUT, int TP) {
    const int RL = kMoeThreads / (OUT / 16);
    const int RS = tile_rows(row_bytes, RL);
    return (size_t)kStages * RS * row_bytes + (size_t)kStages * TP * RS * 4 + (size_t)kMoeThreads * 17 * 4 +
           (size_t)RS * (OUT / 256) * 16 * 4;
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
    launch_dep(moe_stream_kernel<Q, TP>, grid, dim3(kMoeThreads), smem, s, W0, W1, row_bytes, expert_bytes, IN, OUT, X,
               by_token, ix, e_begin, A_cap, P);
    return 0;
}

// ------------------------------------------------------------------ few-token pass (CUDA cores)
//
// One or two tokens per expert (decode): the tensor-core pass spends the same
// instructions per weight whatever the token count, so with one token its
// MMAs are mostly empty. Here every thread owns 16 output columns of a row --
// bytes [8 u, 8 u + 8) of quant group `grp` of a block, i.e. columns
// 64 grp + 8 u .. + 7 (low nibbles, sub-block 2 grp) and the same + 32 (high
// nibbles, sub-block 2 grp + 1), so one row's scales serve all 16 -- and walks
// its rows with fp32 FMAs: a nibble q becomes the float 1 + q/16 (one shift
// and one LOP3; 1 + q/32 for a 5-bit Q5_K value), and
//   sum_i x_i (d_i sc_i q_i - dmin_i m_i)
//     = sum_i A_i f_i - sum_i (A_i + x_i dmin_i m_i),  A_i = 16 x_i d_i sc_i
// (32 for Q5_K). Row groups of the CTA are summed in shared memory and the
// row chunk's partials go to P like the other passes'.
constexpr int kLaneUnroll = 8;  // rows in flight per thread

template <uint32_t Q, int TPL>
__global__ void __launch_bounds__(kMoeThreads, 2)
moe_lane_kernel(const uint8_t* __restrict__ W0, const uint8_t* __restrict__ W1, int64_t row_bytes,
                int64_t expert_bytes, int IN, int OUT, const float* __restrict__ X, bool by_token, MoeIndex ix,
                int e_begin, int A_cap, float* __restrict__ P, const float* __restrict__ PG, int RCG) {
    pdl_entry();
    constexpr int BB = block_bytes(Q);
    constexpr int QOFF = (Q == kQ4_K) ? 16 : 48;
    constexpr float kUnit = (Q == kQ4_K) ? 16.0f : 32.0f;  // f = 1 + q / kUnit
    extern __shared__ float red[];  // [RG][TPL][OUT], then (PG) the activations [TPL][rows]
    const int nmat = W1 ? 2 : 1;
    const int slot = blockIdx.x / nmat, m = blockIdx.x % nmat;
    const int4 si = ix.slot_info[slot];  // {expert, first position, count, first token}
    if (si.x < 0) return;
    const int e = si.x, a0 = si.y, n = si.z;
    const int RC = gridDim.y, rc = blockIdx.y, nk = IN / 16;  // 16-row chunk boundaries, as the other passes
    const int r0 = 16 * (int)((int64_t)nk * rc / RC), r1 = 16 * (int)((int64_t)nk * (rc + 1) / RC);
    const int TPR = OUT / 16, RG = kMoeThreads / TPR;
    const int tid = threadIdx.x, c16 = tid % TPR, rg = tid / TPR;
    const int blk = c16 >> 4, grp = (c16 >> 2) & 3, u = c16 & 3;
    const int col = blk * 256 + 64 * grp + 8 * u;  // low columns col..col+7, high col+32..col+39
    const uint8_t* Wm = (m == 0 ? W0 : W1) + (int64_t)(e - e_begin) * expert_bytes + (int64_t)blk * BB;
    const int sh = 16 * (grp & 1);
    __shared__ int src[TPL];

    for (int p0 = 0; p0 < n; p0 += TPL) {
        const int np = n - p0 < TPL ? n - p0 : TPL;
        __syncthreads();  // the previous pass's reads of src and red are done
        if (tid < TPL) {
            const int a = a0 + p0 + (tid < np ? tid : 0);
            src[tid] = by_token ? (a == a0 ? si.w : ix.tok[a]) : a;
        }
        __syncthreads();
        const float* xr[TPL];
#pragma unroll
        for (int p = 0; p < TPL; ++p) xr[p] = X + (int64_t)src[p] * IN;
        // down pass fused with the SwiGLU: this chunk's activations
        // silu(sum gate partials) * (sum up partials), summed in chunk order
        const int rows = r1 - r0;
        float* xs = red + (int64_t)RG * TPL * OUT;
        if (PG) {
            // every partial loaded at once into shared memory (one round of
            // independent loads), then each activation sums its chunks in order
            float* pb = xs + TPL * rows;  // [TPL][2][RCG][rows]
            for (int q = tid; q < np * 2 * RCG * rows; q += kMoeThreads) {
                const int ii = q % rows, c = (q / rows) % RCG, mm = (q / (rows * RCG)) & 1, p = q / (2 * rows * RCG);
                pb[q] = PG[(((int64_t)c * 2 + mm) * A_cap + src[p]) * IN + r0 + ii];
            }
            __syncthreads();
            for (int q = tid; q < TPL * rows; q += kMoeThreads) {
                const int p = q / rows, ii = q - p * rows;
                float v = 0.0f;
                if (p < np) {
                    float g = 0.0f, uu = 0.0f;
                    const float* pg = pb + (int64_t)p * 2 * RCG * rows + ii;
                    for (int c = 0; c < RCG; ++c) {
                        g += pg[c * rows];
                        uu += pg[(RCG + c) * rows];
                    }
                    v = silu_f32(g) * uu;
                }
                xs[q] = v;
            }
            __syncthreads();
        }
        float acc[TPL][16], bias[TPL][2];
#pragma unroll
        for (int p = 0; p < TPL; ++p) {
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[p][j] = 0.0f;
            bias[p][0] = bias[p][1] = 0.0f;
        }
        for (int i0 = r0 + rg; i0 < r1; i0 += RG * kLaneUnroll) {
            uint4 hd[kLaneUnroll];
            uint2 qw[kLaneUnroll], hw[kLaneUnroll];
            float xv[kLaneUnroll][TPL];
#pragma unroll
            for (int r = 0; r < kLaneUnroll; ++r) {
                const int i = i0 + r * RG;
                if (i < r1) {
                    const uint8_t* row = Wm + (int64_t)i * row_bytes;
                    hd[r] = __ldg(reinterpret_cast<const uint4*>(row));
                    qw[r] = __ldg(reinterpret_cast<const uint2*>(row + QOFF + 32 * grp + 8 * u));
                    if constexpr (Q == kQ5_K) hw[r] = __ldg(reinterpret_cast<const uint2*>(row + 16 + 8 * u));
#pragma unroll
                    for (int p = 0; p < TPL; ++p) xv[r][p] = PG ? xs[p * rows + (i - r0)] : __ldg(xr[p] + i);
                } else {
                    hd[r] = make_uint4(0u, 0u, 0u, 0u);  // d = dmin = 0: contributes nothing
                    qw[r] = make_uint2(0u, 0u);
                    hw[r] = make_uint2(0u, 0u);
#pragma unroll
                    for (int p = 0; p < TPL; ++p) xv[r][p] = 0.0f;
                }
            }
#pragma unroll
            for (int r = 0; r < kLaneUnroll; ++r) {
                const float d = h2f(hd[r].x), dmin = h2f(hd[r].x >> 16);
                uint32_t sl, shi, ml, mh;
                scales_k4_packed(hd[r].y, hd[r].z, hd[r].w, sl, shi, ml, mh);
                const uint32_t sw = (grp < 2 ? sl : shi) >> sh, mw = (grp < 2 ? ml : mh) >> sh;
                const float ds0 = d * kUnit * (float)(sw & 63u), ds1 = d * kUnit * (float)((sw >> 8) & 63u);
                const float dm0 = dmin * (float)(mw & 63u), dm1 = dmin * (float)((mw >> 8) & 63u);
                float f[16];
#pragma unroll
                for (int w = 0; w < 2; ++w) {
                    const uint32_t q = w ? qw[r].y : qw[r].x;
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        uint32_t lo, hi;
                        if constexpr (Q == kQ4_K) {
                            // nibble to bits 19..22 under the exponent of 1.0
                            lo = (19 - 8 * b) >= 0 ? q << (19 - 8 * b) : q >> (8 * b - 19);
                            hi = (15 - 8 * b) >= 0 ? q << (15 - 8 * b) : q >> (8 * b - 15);
                            lo = (lo & 0x00780000u) | 0x3F800000u;
                            hi = (hi & 0x00780000u) | 0x3F800000u;
                        } else {
                            // nibble to bits 18..21, its high bit (qh bit 2 grp / 2 grp + 1 of byte 4w + b) to 22
                            const uint32_t h = w ? hw[r].y : hw[r].x;
                            const int hb = 8 * b + 2 * grp;
                            lo = (18 - 8 * b) >= 0 ? q << (18 - 8 * b) : q >> (8 * b - 18);
                            hi = (14 - 8 * b) >= 0 ? q << (14 - 8 * b) : q >> (8 * b - 14);
                            const uint32_t hl = (22 - hb) >= 0 ? h << (22 - hb) : h >> (hb - 22);
                            const uint32_t hh = (21 - hb) >= 0 ? h << (21 - hb) : h >> (hb - 21);
                            lo = (lo & 0x003C0000u) | (hl & 0x00400000u) | 0x3F800000u;
                            hi = (hi & 0x003C0000u) | (hh & 0x00400000u) | 0x3F800000u;
                        }
                        f[4 * w + b] = __uint_as_float(lo);
                        f[8 + 4 * w + b] = __uint_as_float(hi);
                    }
                }
#pragma unroll
                for (int p = 0; p < TPL; ++p) {
                    const float A0 = xv[r][p] * ds0, A1 = xv[r][p] * ds1;
                    bias[p][0] += fmaf(xv[r][p], dm0, A0);
                    bias[p][1] += fmaf(xv[r][p], dm1, A1);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        acc[p][j] = fmaf(A0, f[j], acc[p][j]);
                        acc[p][8 + j] = fmaf(A1, f[8 + j], acc[p][8 + j]);
                    }
                }
            }
        }
        // this thread's 16 columns, then the row groups summed in a fixed order
#pragma unroll
        for (int p = 0; p < TPL; ++p) {
            float* rr = red + ((int64_t)rg * TPL + p) * OUT;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                rr[col + j] = acc[p][j] - bias[p][0];
                rr[col + 32 + j] = acc[p][8 + j] - bias[p][1];
            }
        }
        __syncthreads();
        for (int q = tid; q < np * OUT; q += kMoeThreads) {
            const int p = q / OUT, c = q - p * OUT;
            float v = 0.0f;
            for (int g = 0; g < RG; ++g) v += red[((int64_t)g * TPL + p) * OUT + c];
            P[(((int64_t)rc * nmat + m) * A_cap + a0 + p0 + p) * OUT + c] = v;
        }
    }
}

// Dynamic shared memory of the few-token pass: the row groups' sums and,
// with the fused SwiGLU, the chunk's activations and their partials.
size_t lane_smem(int TPL, int IN, int OUT, int RC, bool fused, int RCG) {
    const int RG = kMoeThreads / (OUT / 16);
    const int max_rows = 16 * ((IN / 16 + RC - 1) / RC);
    return ((size_t)RG * TPL * OUT + (fused ? (size_t)TPL * max_rows * (1 + 2 * (size_t)RCG) : 0)) * sizeof(float);
}
constexpr size_t kLaneSmemMax = 200 * 1024;

template <uint32_t Q>
int launch_lane_q(int TPL, const uint8_t* W0, const uint8_t* W1, int64_t row_bytes, int64_t expert_bytes, int IN,
                  int OUT, const float* X, bool by_token, const MoeIndex& ix, int e_begin, int A_cap, float* P,
                  int slots, int RC, cudaStream_t s, const float* PG, int RCG) {
    const size_t smem = lane_smem(TPL, IN, OUT, RC, PG != nullptr, RCG);  // rows per chunk <= 16 ceil(IN / 16 / RC)
    if (smem > kLaneSmemMax) return -1;
    const dim3 grid((unsigned)(slots * (W1 ? 2 : 1)), (unsigned)RC);
    if (TPL == 1) {
        if (cudaFuncSetAttribute(moe_lane_kernel<Q, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
            return -1;
        launch_dep(moe_lane_kernel<Q, 1>, grid, dim3(kMoeThreads), smem, s, W0, W1, row_bytes, expert_bytes, IN, OUT,
                   X, by_token, ix, e_begin, A_cap, P, PG, RCG);
    } else {
        if (cudaFuncSetAttribute(moe_lane_kernel<Q, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
            return -1;
        launch_dep(moe_lane_kernel<Q, 2>, grid, dim3(kMoeThreads), smem, s, W0, W1, row_bytes, expert_bytes, IN, OUT,
                   X, by_token, ix, e_begin, A_cap, P, PG, RCG);
    }
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

size_t mma_smem(int64_t row_bytes, int OUT) {
    const int RS = mma_tile_rows(row_bytes);
    return (size_t)kStages * RS * mma_row_pitch(row_bytes) + (size_t)kStages * 4 * mma_x_pitch(RS) * 4 +
           (size_t)RS * ((OUT / 256) * 16 + 8) * 4;
}

template <uint32_t Q, int MPW>
int launch_mma_t(const uint8_t* W0, const uint8_t* W1, int64_t row_bytes, int64_t expert_bytes, int IN, int OUT,
                 const float* X, bool by_token, const MoeIndex& ix, int e_begin, int A_cap, float* P, int slots,
                 int RC, cudaStream_t s) {
    const size_t smem = mma_smem(row_bytes, OUT);
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(moe_mma_kernel<Q, MPW>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
        return -1;
    const dim3 grid((unsigned)(slots * (W1 ? 2 : 1)), (unsigned)RC);
    launch_dep(moe_mma_kernel<Q, MPW>, grid, dim3(kMoeThreads), smem, s, W0, W1, row_bytes, expert_bytes, IN, OUT, X,
               by_token, ix, e_begin, A_cap, P);
    return 0;
}

template <uint32_t Q>
int launch_mma_q(const uint8_t* W0, const uint8_t* W1, int64_t row_bytes, int64_t expert_bytes, int IN, int OUT,
                 const float* X, bool by_token, const MoeIndex& ix, int e_begin, int A_cap, float* P, int slots,
                 int RC, cudaStream_t s) {
    switch (OUT / 128) {
    case 2: return launch_mma_t<Q, 2>(W0, W1, row_bytes, expert_bytes, IN, OUT, X, by_token, ix, e_begin, A_cap, P,
                                      slots, RC, s);
    case 4: return launch_mma_t<Q, 4>(W0, W1, row_bytes, expert_bytes, IN, OUT, X, by_token, ix, e_begin, A_cap, P,
                                      slots, RC, s);
    case 8: return launch_mma_t<Q, 8>(W0, W1, row_bytes, expert_bytes, IN, OUT, X, by_token, ix, e_begin, A_cap, P,
                                      slots, RC, s);
    case 16: return launch_mma_t<Q, 16>(W0, W1, row_bytes, expert_bytes, IN, OUT, X, by_token, ix, e_begin, A_cap,
                                        P, slots, RC, s);
    default: return -1;
    }
}

// Whether a pass takes the few-token form: one or two tokens per pass, Q4_K /
// Q5_K, OUT / 16 threads per row dividing the CTA.
bool lane_pass(uint32_t q, int TP, int OUT, int64_t row_bytes) {
    return TP <= 2 && (q == kQ4_K || q == kQ5_K) && row_bytes % 16 == 0 && OUT % 256 == 0 &&
           OUT / 16 <= kMoeThreads && kMoeThreads % (OUT / 16) == 0;
}

// PG (few-token form only): the down pass computes its activations from the
// gate/up partials (RCG chunks) instead of reading X.
int launch_stream(uint32_t q, int TP, const uint8_t* W0, const uint8_t* W1, int64_t row_bytes, int64_t expert_bytes,
                  int IN, int OUT, const float* X, bool by_token, const MoeIndex& ix, int e_begin, int A_cap, float* P,
                  int slots, int RC, cudaStream_t s, const float* PG = nullptr, int RCG = 0) {
    if (OUT % 256 != 0 || OUT / 16 > kMoeThreads) return -1;
    if (lane_pass(q, TP, OUT, row_bytes)) {
        if (q == kQ4_K)
            return launch_lane_q<kQ4_K>(TP, W0, W1, row_bytes, expert_bytes, IN, OUT, X, by_token, ix, e_begin, A_cap,
                                        P, slots, RC, s, PG, RCG);
        return launch_lane_q<kQ5_K>(TP, W0, W1, row_bytes, expert_bytes, IN, OUT, X, by_token, ix, e_begin, A_cap, P,
                                    slots, RC, s, PG, RCG);
    }
    if (PG) return -1;
    // Q4_K / Q5_K with up to 2048 output columns: the tensor-core form
    const int mpw = OUT / 128;
    if ((q == kQ4_K || q == kQ5_K) && IN % 16 == 0 && row_bytes % 16 == 0 &&
        (mpw == 2 || mpw == 4 || mpw == 8 || mpw == 16)) {
        if (q == kQ4_K)
            return launch_mma_q<kQ4_K>(W0, W1, row_bytes, expert_bytes, IN, OUT, X, by_token, ix, e_begin, A_cap, P,
                                       slots, RC, s);
        return launch_mma_q<kQ5_K>(W0, W1, row_bytes, expert_bytes, IN, OUT, X, by_token, ix, e_begin, A_cap, P,
                                   slots, RC, s);
    }
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
// in all. Up to 8 tokens every chunk adds one partial per output to the
// reductions, which then dominate the tensor-core pass: at most 8 chunks (at
// least 32 rows each). The few-token pass (1 or 2 tokens) runs one wave of
// two CTAs per SM (up to 64 chunks of at least 16 rows).
int moe_row_chunks(int slots, int mats, int IN, int sm_count, int T) {
    const int ctas = slots * mats;
    int rc = (4 * (sm_count > 0 ? sm_count : 148) + ctas - 1) / ctas;
    int maxrc = IN / 32 > 0 ? IN / 32 : 1;
    if (T <= 2) {
        // one wave at two CTAs per SM: each CTA pays its index and first
        // load latencies once
        rc = (2 * (sm_count > 0 ? sm_count : 148)) / ctas;
        maxrc = IN / 16 > 0 ? IN / 16 : 1;
        if (maxrc > 64) maxrc = 64;
    } else if (T <= 8 && maxrc > 8) {
        maxrc = 8;
    }
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
    w.slot_info = take((int64_t)(p.slots > 0 ? p.slots : 1) * 16);
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
    const int64_t kmax = p.n_embd > p.n_ff_s ? p.n_embd : p.n_ff_s;
    w.xfrag = take(gemv_mma_work_bytes(kmax, p.T));
    w.xfrag_s = p.shared ? take(gemv_mma_work_bytes(kmax, p.T)) : -1;  // the shared expert's, on its own stream
    w.bytes = o;
    return w;
}

int launch_moe_layer(const MoeLaunch& L, cudaStream_t s) {
    const MoePlan& p = L.plan;
    uint8_t* base = static_cast<uint8_t*>(L.work);
    auto F = [&](int64_t off) { return reinterpret_cast<float*>(base + off); };
    auto I = [&](int64_t off) { return reinterpret_cast<int*>(base + off); };
    const MoeWork& w = L.layout;
    MoeIndex ix{I(w.cnt), I(w.off), I(w.active), I(w.counters), I(w.counters) + 1, I(w.tok), I(w.pos),
                reinterpret_cast<int4*>(base + w.slot_info), p.slots};
    const int A = p.T * p.k;

    // dense projections (router, shared expert): tensor-core GEMV where it applies
    // `prepped`: the limbs of X already sit in this workspace (the previous
    // tensor-core projection on this stream read the same X)
    auto dense_on = [&](cudaStream_t st, int64_t xf, const MoeTensor& Wt, int64_t rows, int64_t cols, const float* X,
                        float* Y, bool* prepped = nullptr) -> int {
        GemvArgs g{Wt.W, Wt.row_bytes, rows, cols, X, Y, p.T, p.sm_count, Wt.tmap};
        if (gemv_mma_supported(Wt.quant, g)) {
            const bool reuse = prepped && *prepped;
            if (prepped) *prepped = true;
            return launch_gemv_mma(Wt.quant, g, base + xf, L.err, st, !reuse);
        }
        return launch_gemv(Wt.quant, g, st);
    };
    auto dense = [&](const MoeTensor& Wt, int64_t rows, int64_t cols, const float* X, float* Y) -> int {
        return dense_on(s, w.xfrag, Wt, rows, cols, X, Y);
    };

    // shared expert (moe.rs:129-142): independent of the routing until the
    // combine, so it runs on the auxiliary stream beside the routed path
    const float* Ds = nullptr;
    const float* sg = nullptr;
    const bool fork = p.shared && L.aux && L.fork && L.join;
    if (p.shared) {
        cudaStream_t ss = s;
        if (fork) {
            cudaEventRecord(L.fork, s);
            cudaStreamWaitEvent(L.aux, L.fork, 0);
            ss = L.aux;
        }
        // gate, up and gate-input projections read the same x: one set of limbs
        bool prepped = false;
        if (dense_on(ss, w.xfrag_s, L.gate_s, p.n_ff_s, p.n_embd, L.x, F(w.gs), &prepped) ||
            dense_on(ss, w.xfrag_s, L.up_s, p.n_ff_s, p.n_embd, L.x, F(w.us), &prepped) ||
            dense_on(ss, w.xfrag_s, L.gate_inp_s, 1, p.n_embd, L.x, F(w.gi), &prepped))
            return -4;
        moe_shared_act_kernel<<<grid_for((int64_t)p.T * p.n_ff_s, p.sm_count), 256, 0, ss>>>(
            F(w.gs), F(w.us), F(w.gi), p.T, p.n_ff_s, F(w.hs), F(w.sg));
        if (dense_on(ss, w.xfrag_s, L.down_s, p.n_embd, p.n_ff_s, F(w.hs), F(w.ds))) return -5;
        if (fork) cudaEventRecord(L.join, L.aux);
        Ds = F(w.ds);
        sg = F(w.sg);
    }

    // route
    const float* logits = L.logits;
    if (!logits) {
        const int64_t n = (int64_t)p.T * p.n_embd;
        moe_bf16_round_kernel<<<grid_for(n, p.sm_count), 256, 0, s>>>(L.x, F(w.xb), n);
        if (dense(L.router, p.E, p.n_embd, F(w.xb), F(w.logits))) return -1;
        logits = F(w.logits);
    }
    const size_t fused_smem = ((size_t)p.T * p.E + (size_t)p.T * p.k) * 4;
    if (p.T <= kFusedRouteTokens && fused_smem <= 48 * 1024) {
        launch_dep(moe_route_assign_kernel, dim3(1), dim3(kAssignThreads), fused_smem, s, logits, p.T, p.E, p.k,
                   I(w.ids), F(w.wts), p.e_begin, p.e_end, ix);
    } else {
        launch_dep(moe_route_kernel, dim3((p.T + kRouteWarps - 1) / kRouteWarps), dim3(kRouteWarps * 32),
                   (size_t)kRouteWarps * p.E * sizeof(float), s, logits, p.T, p.E, p.k, I(w.ids), F(w.wts));
        const bool staged = (int64_t)p.T * p.k * 4 <= 32 * 1024;
        launch_dep(moe_assign_kernel, dim3(1), dim3(kAssignThreads), staged ? (size_t)p.T * p.k * 4 : 0, s, I(w.ids),
                   p.T, p.k, p.E, p.e_begin, p.e_end, staged, ix);
    }

    // routed experts
    const int slots = p.slots;
    const int TP = p.T <= 2 ? p.T : 4;  // tokens per pass: 1 or 2 take the few-token form
    if (launch_stream(L.gate.quant, TP, L.gate.W, L.up.W, L.gate.row_bytes, L.gate.expert_bytes, p.n_embd, p.n_ff,
                      L.x, true, ix, p.e_begin, A, F(w.pgu), slots, p.rc_gu, s))
        return -2;
    // the few-token down pass computes the SwiGLU itself from the gate/up partials
    const bool fuse_act = lane_pass(L.down.quant, TP, p.n_embd, L.down.row_bytes) &&
                          lane_smem(TP, p.n_ff, p.n_embd, p.rc_d, true, p.rc_gu) <= kLaneSmemMax;
    if (!fuse_act)
        launch_dep(moe_swiglu_kernel, dim3(grid_for((int64_t)A * p.n_ff, p.sm_count)), dim3(256), 0, s, F(w.pgu),
                   p.rc_gu, A, p.n_ff, ix.n_assign, F(w.h));
    if (launch_stream(L.down.quant, TP, L.down.W, nullptr, L.down.row_bytes, L.down.expert_bytes, p.n_ff, p.n_embd,
                      F(w.h), false, ix, p.e_begin, A, F(w.pd), slots, p.rc_d, s, fuse_act ? F(w.pgu) : nullptr,
                      p.rc_gu))
        return -3;

    if (fork) cudaStreamWaitEvent(s, L.join, 0);
    int lanes = 1;
    while (lanes < p.k) lanes <<= 1;
    const unsigned cgrid = (unsigned)grid_for((int64_t)p.T * p.n_embd * lanes, p.sm_count);
    if (fork)  // after the join: a full dependency on both streams
        moe_combine_kernel<<<cgrid, 256, 0, s>>>(F(w.pd), p.rc_d, A, p.n_embd, I(w.pos), F(w.wts), p.T, p.k, lanes, Ds,
                                                 sg, L.out);
    else
        launch_dep(moe_combine_kernel, dim3(cgrid), dim3(256), 0, s, F(w.pd), p.rc_d, A, p.n_embd, I(w.pos), F(w.wts),
                   p.T, p.k, lanes, Ds, sg, L.out);
    if (L.ids_out) cudaMemcpyAsync(L.ids_out, I(w.ids), (size_t)A * 4, cudaMemcpyDeviceToDevice, s);
    if (L.wts_out) cudaMemcpyAsync(L.wts_out, F(w.wts), (size_t)A * 4, cudaMemcpyDeviceToDevice, s);
    return 0;
}

}  // namespace strata
