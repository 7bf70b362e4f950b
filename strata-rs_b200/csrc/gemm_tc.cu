// gemm_tc.cu — prefill GEMM on the 5th-generation tensor cores (tcgen05 / TMEM).
//
// Y[m][n] = sum_k X[m][k] * W[n][k] for M >= 64 tokens: the batched form of
// ops::gemv (crates/strata-core/src/ops.rs:14-28), which the reference runs
// once per prompt token (crates/strata-core/src/generate.rs:116-118). X is
// bf16 (row-major, K contiguous), W a Q4_K / Q5_K / Q6_K matrix in
// strata-gguf's byte layout (crates/strata-gguf/src/dequant.rs), Y f32.
//
// One CTA computes a 128-weight-row x TN-token tile over a range of K:
//   warp 0      producer: per 256-weight super-block one TMA box of raw quant
//               bytes [BW bytes x 128 rows]; per 64-wide K step one TMA box of
//               X [64 x TN] bf16 with the 128-byte swizzle (UMMA's K-major
//               SW128 layout);
//   warp 1      MMA issuer: one thread issues tcgen05.mma kind::f16
//               (A = dequantized weights, B = X, D in TMEM) and commits each
//               stage's release to an mbarrier;
//   warps 2..9  two threads per weight row, each dequantizing half of every K
//               step into bf16 in the same SW128 layout (two such warps per
//               scheduler hide each other's latency), then read the
//               accumulators back with tcgen05.ld and store Y.
// X and W have separate rings (up to 4 and 3 stages as shared memory allows):
// the X copy of a step is issued several MMA steps ahead of its use.
// Precision: a single bf16 copy of a K-quant weight keeps 8 of its up to 17
// significant bits, which misses the 1e-2 bound of the parity metric
// (max |y - ref| / max(|ref|, 1e-3 |ref|inf)) by two orders of magnitude.
// TERMS = 2 stages the weight as hi = bf16(w) plus lo = bf16(w - hi) (w to
// ~2^-17 relative; x is bf16 already, so every product is exact) and
// accumulates the two products in separate TMEM accumulators, added in fp32 by
// the epilogue: the tensor core's accumulation error grows with the number of
// additions into a large running sum, and the lo products then add none.
// Every mbarrier wait is bounded (about a second); a timeout sets *err and the
// CTA drains its copies in flight and finishes.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <cstring>

#include "kernels.cuh"
#include "quant.cuh"

namespace strata {
namespace {

constexpr int kRowsTile = 128;  // UMMA M
constexpr int kKStep = 64;      // bf16 elements per 128-byte swizzled row
constexpr int kRawSlots = 2;    // raw super-block ring depth
constexpr int kDequantWarps = 8;
constexpr int kThreadsG = (2 + kDequantWarps) * 32;

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void bar_init(uint32_t b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(b), "r"(n) : "memory");
}
__device__ __forceinline__ void bar_expect_tx(uint32_t b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(b), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint32_t b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(b) : "memory");
}
// Bounded wait for the completion of the phase with parity `par`; returns
// false (and sets *err) after about a second.
__device__ __forceinline__ bool bar_wait(uint32_t b, uint32_t par, int* err) {
    uint64_t t0 = 0;
    for (long long i = 0; i < kSpinLimit; ++i) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(b), "r"(par)
            : "memory");
        if (ok) return true;
        if ((i & 255) == 0) {
            const uint64_t t = now_ns();
            if (i == 0) t0 = t;
            else if (t - t0 > 1000000000ull) break;
        }
    }
    if (err) atomicExch(err, 1);
    return false;
}
__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// K-major, 128-byte-swizzled UMMA shared-memory descriptor: rows 128 B apart,
// 8-row atoms 1024 B apart (stride byte offset), descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// kind::f16 instruction descriptor: D f32, A and B bf16, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// Byte offset of the 16-byte unit u (elements 8u..8u+7) of row r in a
// [rows][64] bf16 tile laid out with the 128-byte swizzle.
__device__ __forceinline__ uint32_t sw128_unit(int r, int u) {
    return (uint32_t)(r * 128 + (((u ^ (r & 7)) & 7) << 4));
}

// Raw bytes per row per super-block in the staged box. Q6_K blocks (210 B)
// start on 2-byte boundaries; the box is the 16-byte-aligned 240-byte window
// that contains the block.
template <uint32_t Q>
constexpr int raw_box_bytes() {
    return Q == kQ6_K ? 240 : block_bytes(Q);
}

// Bytes b0 and b0+1 of v (each < 256) as exact floats.
__device__ __forceinline__ float2 byte_pair_f(uint32_t v, int b0) {
    const float2 m = make_float2(__uint_as_float(__byte_perm(v, 0x4B000000u, 0x7540u | b0)),
                                 __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7540u | (b0 + 1))));
    return __fadd2_rn(m, make_float2(-8388608.0f, -8388608.0f));
}

// Two weights -> bf16x2 hi word (and lo word for TERMS == 2).
template <int TERMS>
__device__ __forceinline__ void split_pair(float2 w, uint32_t& hi, uint32_t& lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(w.x, w.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    if constexpr (TERMS == 2) {
        const float2 hf = make_float2(__uint_as_float(hi << 16), __uint_as_float(hi & 0xFFFF0000u));
        const float2 r = __fadd2_rn(w, make_float2(-hf.x, -hf.y));
        const __nv_bfloat162 l = __floats2bfloat162_rn(r.x, r.y);
        lo = *reinterpret_cast<const uint32_t*>(&l);
    } else {
        lo = 0;
    }
}

template <int TERMS>
__device__ __forceinline__ void store_unit(uint8_t* tile, uint32_t off, const uint32_t (&hi)[4],
                                           const uint32_t (&lo)[4]) {
    *reinterpret_cast<uint4*>(tile + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    if constexpr (TERMS == 2)
        *reinterpret_cast<uint4*>(tile + kRowsTile * 128 + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
}

// 32-bit words of a 2-byte-aligned shared-memory byte run.
template <int NW>
__device__ __forceinline__ void ld_words(const uint8_t* p, uint32_t (&o)[NW]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
    const uint32_t sh = (uint32_t)(a & 3u) * 8u;
    uint32_t prev = w[0];
#pragma unroll
    for (int i = 0; i < NW; ++i) {
        const uint32_t next = w[i + 1];
        o[i] = __funnelshift_r(prev, next, sh);
        prev = next;
    }
}

// Per-super-block state of one weight row (loaded once, used by 4 K steps).
template <uint32_t Q>
struct SbState;

template <>
struct SbState<kQ4_K> {
    float d, dmin;
    uint32_t sc_lo, sc_hi, m_lo, m_hi;
};
template <>
struct SbState<kQ5_K> {
    float d, dmin;
    uint32_t sc_lo, sc_hi, m_lo, m_hi;
    uint32_t qh[8];
};
template <>
struct SbState<kQ6_K> {
    float d;
    uint32_t sc[4];
};

template <uint32_t Q>
__device__ __forceinline__ void load_sb(const uint8_t* b, SbState<Q>& s) {
    if constexpr (Q == kQ4_K || Q == kQ5_K) {
        const uint4 h = *reinterpret_cast<const uint4*>(b);
        s.d = __half2float(__ushort_as_half((unsigned short)(h.x & 0xFFFFu)));
        s.dmin = __half2float(__ushort_as_half((unsigned short)(h.x >> 16)));
        scales_k4_packed(h.y, h.z, h.w, s.sc_lo, s.sc_hi, s.m_lo, s.m_hi);
        if constexpr (Q == kQ5_K) {
            const uint4 a = *reinterpret_cast<const uint4*>(b + 16);
            const uint4 c = *reinterpret_cast<const uint4*>(b + 32);
            s.qh[0] = a.x; s.qh[1] = a.y; s.qh[2] = a.z; s.qh[3] = a.w;
            s.qh[4] = c.x; s.qh[5] = c.y; s.qh[6] = c.z; s.qh[7] = c.w;
        }
    } else {
        uint32_t w[5];
        ld_words<5>(b + 192, w);
        s.sc[0] = w[0]; s.sc[1] = w[1]; s.sc[2] = w[2]; s.sc[3] = w[3];
        s.d = __half2float(__ushort_as_half((unsigned short)(w[4] & 0xFFFFu)));
    }
}

// Dequantize half h of K step kk -- elements 64 kk + 32 h .. + 31, the 16-byte
// units 4h .. 4h + 3 -- of this thread's super-block into row r of the
// stage's A tile(s). h is warp-uniform.
template <uint32_t Q, int TERMS>
__device__ __forceinline__ void dequant_half(const uint8_t* b, const SbState<Q>& s, int kk, int h, int r,
                                             uint8_t* tile) {
    if constexpr (Q == kQ4_K || Q == kQ5_K) {
        // sub-block j = 2kk + h: low nibbles of qs[32kk..] for h = 0, high nibbles for h = 1
        const int j = 2 * kk + h;
        const uint32_t scb = ((j < 4 ? s.sc_lo : s.sc_hi) >> (8 * (j & 3))) & 0xFFu;
        const uint32_t mnb = ((j < 4 ? s.m_lo : s.m_hi) >> (8 * (j & 3))) & 0xFFu;
        const float dA = s.d * (float)scb, nA = -(s.dmin * (float)mnb);
        const float2 sc2 = make_float2(dA, dA), mn2 = make_float2(nA, nA);
        const uint8_t* qs = b + ((Q == kQ4_K) ? 16 : 48) + 32 * kk;
        const uint4 qa = *reinterpret_cast<const uint4*>(qs);
        const uint4 qb = *reinterpret_cast<const uint4*>(qs + 16);
        const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        const int nsh = 4 * h;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int wi = 0; wi < 2; ++wi) {
                const int i = 2 * u + wi;
                uint32_t v = (qw[i] >> nsh) & 0x0F0F0F0Fu;
                if constexpr (Q == kQ5_K) v |= ((s.qh[i] >> j) & 0x01010101u) << 4;
#pragma unroll
                for (int p = 0; p < 2; ++p) {
                    const float2 w = __ffma2_rn(sc2, byte_pair_f(v, 2 * p), mn2);
                    split_pair<TERMS>(w, hi[2 * wi + p], lo[2 * wi + p]);
                }
            }
            store_unit<TERMS>(tile, sw128_unit(r, 4 * h + u), hi, lo);
        }
    } else {
        // Q6_K: half H = kk / 2 of the block; quarter g = 2 (kk & 1) + h of that half:
        // ql bytes 64H + 32 (g & 1) + l (low nibble for g < 2, high for g >= 2),
        // qh bytes 128 + 32H + l (bits 2g, 2g + 1), u8 scale 8H + 2g + l / 16
        const int H = kk >> 1, g = 2 * (kk & 1) + h;
        uint32_t ql[8], qh[8];
        ld_words<8>(b + 64 * H + 32 * (g & 1), ql);
        ld_words<8>(b + 128 + 32 * H, qh);
        const uint64_t sc64 = H ? (((uint64_t)s.sc[3] << 32) | s.sc[2]) : (((uint64_t)s.sc[1] << 32) | s.sc[0]);
        const int nsh = 4 * (g >> 1), hsh = 2 * g;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            // the reference reads Q6_K scales as u8 (crates/strata-gguf/src/dequant.rs:208-234)
            const uint32_t scv = (uint32_t)(sc64 >> (8 * (2 * g + (u >> 1)))) & 0xFFu;
            const float ds = s.d * (float)scv;
            const float2 ds2 = make_float2(ds, ds);
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int wi = 0; wi < 2; ++wi) {
                const int i = 2 * u + wi;
                uint32_t v = (ql[i] >> nsh) & 0x0F0F0F0Fu;
                v |= ((qh[i] >> hsh) & 0x03030303u) << 4;
#pragma unroll
                for (int p = 0; p < 2; ++p) {
                    const float2 q = __fadd2_rn(byte_pair_f(v, 2 * p), make_float2(-32.0f, -32.0f));
                    const float2 w = __fmul2_rn(ds2, q);
                    split_pair<TERMS>(w, hi[2 * wi + p], lo[2 * wi + p]);
                }
            }
            store_unit<TERMS>(tile, sw128_unit(r, 4 * h + u), hi, lo);
        }
    }
}

// 16 consecutive f32 columns of this warp's 32 TMEM lanes (one lane per thread).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}

// Ring depths: X (activation) stages, W (dequantized weight) stages. Deeper
// rings where shared memory allows; TN = 256 with two terms takes 2 W + 3 X.
template <uint32_t Q, int TN, int TERMS>
struct GemmCfg {
    static constexpr int kBW = raw_box_bytes<Q>();
    static constexpr int kRawSlot = kRowsTile * kBW;
    static constexpr int kWTile = kRowsTile * 128;
    static constexpr int kWStage = TERMS * kWTile;
    static constexpr int kXStage = TN * 128;
    static constexpr int bytes(int ws, int xs) { return ws * kWStage + xs * kXStage + kRawSlots * kRawSlot + 1024; }
    static constexpr int kBudget = 227 * 1024 - 256;  // opt-in maximum less the static barriers
    static constexpr int kWS = bytes(3, 4) <= kBudget ? 3 : 2;
    static constexpr int kXS = bytes(kWS, 4) <= kBudget ? 4 : bytes(kWS, 3) <= kBudget ? 3 : 2;
    static constexpr int kSmem = bytes(kWS, kXS);
    static_assert(kSmem <= kBudget, "GEMM tile does not fit shared memory");
    static_assert(kRawSlot % 1024 == 0 && kWStage % 1024 == 0 && kXStage % 1024 == 0,
                  "tiles must stay 1024-byte aligned");
};

template <uint32_t Q, int TN, int TERMS>
__global__ void __launch_bounds__(kThreadsG, 1)
gemm_kq_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap, int M,
                  int N, int nblk, float* __restrict__ Y, int64_t split_stride, int* __restrict__ err) {
    using C = GemmCfg<Q, TN, TERMS>;
    constexpr int BW = C::kBW, RAW_SLOT = C::kRawSlot, WTILE = C::kWTile;
    constexpr int WS = C::kWS, XS = C::kXS;
    // one TN-column f32 accumulator per weight term: the small lo products get
    // their own, so only the hi products round against the large running sums
    constexpr int TMEM_COLS = TN * TERMS <= 32 ? 32 : TN * TERMS <= 64 ? 64 : TN * TERMS <= 128 ? 128
                            : TN * TERMS <= 256 ? 256 : 512;
    static_assert(TN * TERMS <= 512, "accumulators exceed TMEM");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* wst = sm;                             // WS x [TERMS][128][64] bf16
    uint8_t* xst = wst + WS * C::kWStage;          // XS x [TN][64] bf16
    uint8_t* raw = xst + XS * C::kXStage;          // kRawSlots x [128][BW] bytes
    __shared__ __align__(8) uint64_t raw_full[kRawSlots], raw_empty[kRawSlots];
    __shared__ __align__(8) uint64_t x_full[XS], x_empty[XS], w_full[WS], w_empty[WS], acc_full;
    __shared__ uint32_t tmem_base;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * kRowsTile;
    const int tok0 = blockIdx.y * TN;
    // this CTA's super-blocks: [sb0, sb1) of the split-K range blockIdx.z
    const int sb0 = (int)((int64_t)nblk * blockIdx.z / gridDim.z);
    const int sb1 = (int)((int64_t)nblk * (blockIdx.z + 1) / gridDim.z);
    const int nsb = sb1 - sb0;
    const int nsteps = nsb * 4;
    float* Yz = Y + (int64_t)blockIdx.z * split_stride;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kRawSlots; ++i) {
            bar_init(smem_addr(&raw_full[i]), 1);
            bar_init(smem_addr(&raw_empty[i]), kDequantWarps);
        }
        for (int i = 0; i < XS; ++i) {
            bar_init(smem_addr(&x_full[i]), 1);
            bar_init(smem_addr(&x_empty[i]), 1);
        }
        for (int i = 0; i < WS; ++i) {
            bar_init(smem_addr(&w_full[i]), kDequantWarps);
            bar_init(smem_addr(&w_empty[i]), 1);
        }
        bar_init(smem_addr(&acc_full), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {  // TMEM accumulators: 128 lanes x TMEM_COLS f32 columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem_d = tmem_base;

    if (warp == 0) {
        // ---------------- producer; every wait is warp-uniform, lane 0 issues.
        // Raw super-blocks run ahead of the X steps by up to kRawSlots blocks.
        int j = 0, n_raw = 0;
        bool live = true;
        for (int t = 0; t < nsb && live; ++t) {
            const int rs = t % kRawSlots;
            if (t >= kRawSlots)
                live = __all_sync(0xFFFFFFFFu, bar_wait(smem_addr(&raw_empty[rs]), ((t / kRawSlots) - 1) & 1, err));
            if (!live) break;
            const int sb = sb0 + t;
            if (lane == 0) {
                const uint32_t fb = smem_addr(&raw_full[rs]);
                bar_expect_tx(fb, RAW_SLOT);
                const int x = (Q == kQ6_K) ? ((sb * 210) & ~15) : sb * block_bytes(Q);
                tma_2d(smem_addr(raw + rs * RAW_SLOT), &wmap, x, row0, fb);
            }
            ++n_raw;
            for (int kk = 0; kk < 4; ++kk) {
                const int s = j % XS;
                if (j >= XS)
                    live = __all_sync(0xFFFFFFFFu, bar_wait(smem_addr(&x_empty[s]), ((j / XS) - 1) & 1, err));
                if (!live) break;
                if (lane == 0) {
                    const uint32_t fb = smem_addr(&x_full[s]);
                    bar_expect_tx(fb, C::kXStage);
                    tma_2d(smem_addr(xst + s * C::kXStage), &xmap, (sb * 4 + kk) * kKStep, tok0, fb);
                }
                ++j;
            }
        }
        // drain: the last phase of every barrier a copy was issued on has
        // completed (immediate when the consumers already waited on it)
        for (int s = 0; s < XS; ++s) {
            const int uses = j > s ? (j - s + XS - 1) / XS : 0;
            if (uses) bar_wait(smem_addr(&x_full[s]), (uses - 1) & 1, err);
        }
        for (int rs = 0; rs < kRawSlots; ++rs) {
            const int uses = n_raw > rs ? (n_raw - rs + kRawSlots - 1) / kRawSlots : 0;
            if (uses) bar_wait(smem_addr(&raw_full[rs]), (uses - 1) & 1, err);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        constexpr uint32_t idesc = idesc_bf16(kRowsTile, TN);
        for (int j = 0; j < nsteps; ++j) {
            const int xs = j % XS, ws = j % WS;
            const bool ok = bar_wait(smem_addr(&x_full[xs]), (j / XS) & 1, err) &&
                            bar_wait(smem_addr(&w_full[ws]), (j / WS) & 1, err);
            if (!__all_sync(0xFFFFFFFFu, ok)) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            if (lane == 0) {
                const uint32_t wa = smem_addr(wst + ws * C::kWStage);
                const uint32_t xa = smem_addr(xst + xs * C::kXStage);
#pragma unroll
                for (int k16 = 0; k16 < kKStep / 16; ++k16) {
#pragma unroll
                    for (int term = 0; term < TERMS; ++term) {
                        const uint64_t da = sw128_desc(wa + term * WTILE + 32 * k16);
                        const uint64_t db = sw128_desc(xa + 32 * k16);
                        const uint32_t acc = (j > 0 || k16 > 0) ? 1u : 0u;
                        asm volatile(
                            "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                            " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
                                tmem_d + (uint32_t)(term * TN)),
                            "l"(da), "l"(db), "r"(idesc), "r"(acc)
                            : "memory");
                    }
                }
                // both stages are free once these MMAs have read them
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 smem_addr(&x_empty[xs]))
                             : "memory");
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 smem_addr(&w_empty[ws]))
                             : "memory");
            }
            __syncwarp();
        }
        // fires when every MMA issued above has completed (at once when none was)
        if (lane == 0)
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_addr(&acc_full))
                         : "memory");
        __syncwarp();
    } else {
        // ---------------- dequantizers: thread (h, r) converts half h of each K
        // step of weight row r (warps 2-5: h = 0, warps 6-9: h = 1, so every
        // scheduler runs two of them); then the epilogue
        const int idx = threadIdx.x - 64;
        const int r = idx & (kRowsTile - 1), h = idx >> 7;
        int j = 0;
        bool live = true;
        for (int t = 0; t < nsb && live; ++t) {
            const int rs = t % kRawSlots;
            live = __all_sync(0xFFFFFFFFu, bar_wait(smem_addr(&raw_full[rs]), (t / kRawSlots) & 1, err));
            if (!live) break;
            const int sb = sb0 + t;
            const uint8_t* blk = raw + rs * RAW_SLOT + r * BW + ((Q == kQ6_K) ? ((sb * 210) & 15) : 0);
            SbState<Q> st;
            load_sb<Q>(blk, st);
#pragma unroll 1
            for (int kk = 0; kk < 4; ++kk, ++j) {
                const int s = j % WS;
                if (j >= WS) {
                    live = __all_sync(0xFFFFFFFFu, bar_wait(smem_addr(&w_empty[s]), ((j / WS) - 1) & 1, err));
                    if (!live) break;
                }
                dequant_half<Q, TERMS>(blk, st, kk, h, r, wst + s * C::kWStage);
                // make the generic-proxy stores visible to the tensor core, then publish
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) bar_arrive(smem_addr(&w_full[s]));
            }
            __syncwarp();
            if (live && lane == 0) bar_arrive(smem_addr(&raw_empty[rs]));
        }
        // epilogue: TMEM lane 32 (warp % 4) + lane holds weight row row0 + that
        // lane; half h stores token columns [h TN / 2, (h + 1) TN / 2)
        const bool ready = bar_wait(smem_addr(&acc_full), 0, err);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int lane_base = 32 * (warp & 3);
        const int row = row0 + lane_base + lane;
#pragma unroll 1
        for (int c = h * (TN / 2); c < (h + 1) * (TN / 2); c += 16) {
            uint32_t v[16], vl[16];
            const uint32_t taddr = tmem_d + ((uint32_t)lane_base << 16) + (uint32_t)c;
            tmem_ld16(taddr, v);
            if constexpr (TERMS == 2) tmem_ld16(taddr + TN, vl);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (ready && live && row < N) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int t = tok0 + c + i;
                    float y = __uint_as_float(v[i]);
                    if constexpr (TERMS == 2) y += __uint_as_float(vl[i]);
                    if (t < M) Yz[(int64_t)t * N + row] = y;
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(TMEM_COLS));
    }
}

// Split-K partial slabs are `split_stride` floats apart: M * N rounded up to a
// multiple of 4, so every slab starts 16-byte aligned.
__host__ __device__ constexpr int64_t split_stride_of(int64_t n) { return (n + 3) & ~int64_t(3); }

// Y[i] = sum over splits z of P[z][i], in split order (deterministic).
__global__ void splitk_reduce_kernel(const float* __restrict__ P, float* __restrict__ Y, int64_t n, int S) {
    const int64_t n4 = n / 4;
    const int64_t stride = split_stride_of(n);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        float4 acc = reinterpret_cast<const float4*>(P)[i];
        for (int z = 1; z < S; ++z) {
            const float4 v = reinterpret_cast<const float4*>(P + (int64_t)z * stride)[i];
            acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
        }
        reinterpret_cast<float4*>(Y)[i] = acc;
    }
    for (int64_t i = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        float acc = P[i];
        for (int z = 1; z < S; ++z) acc += P[(int64_t)z * stride + i];
        Y[i] = acc;
    }
}

// bf16 bits of f32 values, round to nearest even (NaN stays NaN).
__global__ void f32_to_bf16_kernel(const float* __restrict__ x, uint16_t* __restrict__ y, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = __bfloat16_as_ushort(__float2bfloat16_rn(x[i]));
}

PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

int pick_tn(int64_t M) { return M <= 64 ? 64 : M <= 128 ? 128 : 256; }

template <uint32_t Q, int TN, int TERMS>
int launch_gemm_t(const GemmArgs& a, int splits, cudaStream_t s) {
    constexpr int BW = raw_box_bytes<Q>();
    auto enc = tmap_encoder();
    if (!enc) return -3;
    CUtensorMap wmap, xmap;
    {   // raw weight bytes: [row_bytes] x [N], box [BW] x [128]
        const cuuint64_t dims[2] = {(cuuint64_t)a.row_bytes, (cuuint64_t)a.N};
        const cuuint64_t strides[1] = {(cuuint64_t)a.row_bytes};
        const cuuint32_t box[2] = {(cuuint32_t)BW, (cuuint32_t)kRowsTile};
        const cuuint32_t es[2] = {1, 1};
        if (enc(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(a.W), dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return -4;
    }
    {   // activations: bf16 [K] x [M], box [64] x [TN], 128-byte swizzle
        const cuuint64_t dims[2] = {(cuuint64_t)a.K, (cuuint64_t)a.M};
        const cuuint64_t strides[1] = {(cuuint64_t)a.K * 2};
        const cuuint32_t box[2] = {(cuuint32_t)kKStep, (cuuint32_t)TN};
        const cuuint32_t es[2] = {1, 1};
        if (enc(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(a.X), dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return -5;
    }
    constexpr int smem = GemmCfg<Q, TN, TERMS>::kSmem;
    static bool configured[64] = {};  // the attribute is per device
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -6;
    if (!configured[dev]) {
        if (cudaFuncSetAttribute(gemm_kq_tc_kernel<Q, TN, TERMS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 smem) != cudaSuccess)
            return -6;
        configured[dev] = true;
    }
    const dim3 grid((unsigned)((a.N + kRowsTile - 1) / kRowsTile), (unsigned)((a.M + TN - 1) / TN),
                    (unsigned)splits);
    float* out = splits > 1 ? a.work : a.Y;
    gemm_kq_tc_kernel<Q, TN, TERMS><<<grid, kThreadsG, smem, s>>>(
        wmap, xmap, (int)a.M, (int)a.N, (int)(a.K / 256), out, split_stride_of(a.M * a.N), a.err);
    if (splits > 1) {
        const int64_t n = a.M * a.N;
        const int threads = 256;
        const int64_t want = (n / 4 + threads - 1) / threads;
        const int blocks = (int)(want < 4 * (int64_t)a.sm_count ? (want > 0 ? want : 1) : 4 * (int64_t)a.sm_count);
        splitk_reduce_kernel<<<blocks, threads, 0, s>>>(a.work, a.Y, n, splits);
    }
    return 0;
}

template <uint32_t Q, int TERMS>
int dispatch_tn(const GemmArgs& a, int splits, cudaStream_t s) {
    switch (pick_tn(a.M)) {
    case 64: return launch_gemm_t<Q, 64, TERMS>(a, splits, s);
    case 128: return launch_gemm_t<Q, 128, TERMS>(a, splits, s);
    default: return launch_gemm_t<Q, 256, TERMS>(a, splits, s);
    }
}

}  // namespace

int gemm_tc_splits(const GemmArgs& a) {
    const int64_t tiles = ((a.N + kRowsTile - 1) / kRowsTile) * ((a.M + pick_tn(a.M) - 1) / pick_tn(a.M));
    const int64_t sms = a.sm_count > 0 ? a.sm_count : 148;
    const int64_t nblk = a.K / 256;
    if (tiles >= 2 * sms) return 1;
    // one CTA per SM: time ~ waves x super-blocks per CTA, plus a few percent
    // per split for the partial-sum traffic and the reduction
    int best = 1;
    double best_cost = 1e300;
    for (int S = 1; S <= 8; ++S) {
        if (nblk / S < 2) break;
        const int64_t waves = (tiles * S + sms - 1) / sms;
        const double cost = (double)waves * (double)((nblk + S - 1) / S) * (1.0 + 0.02 * (S - 1));
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = S;
        }
    }
    return best;
}

int64_t gemm_tc_work_floats(const GemmArgs& a) {
    const int S = gemm_tc_splits(a);
    return S > 1 ? (int64_t)S * split_stride_of(a.M * a.N) : 0;
}

bool gemm_tc_supported(uint32_t quant, const GemmArgs& a) {
    if (quant != kQ4_K && quant != kQ5_K && quant != kQ6_K) return false;
    if (a.K % 256 != 0 || a.K <= 0 || a.M < 1 || a.N < 1 || a.M >= (1ll << 31) || a.N >= (1ll << 31)) return false;
    if (a.row_bytes >= (1ll << 31) - 256) return false;  // TMA x coordinates stay in int range
    if (a.row_bytes % 16 != 0 || ((uintptr_t)a.W % 16) != 0 || ((uintptr_t)a.X % 16) != 0) return false;
    if ((a.K * 2) % 16 != 0) return false;  // X row stride: a multiple of 16 bytes
    return true;
}

void launch_f32_to_bf16(const float* x, uint16_t* y, int64_t n, int sm_count, cudaStream_t s) {
    const int64_t want = (n + 255) / 256;
    const int64_t cap = 8 * (int64_t)(sm_count > 0 ? sm_count : 148);
    f32_to_bf16_kernel<<<(unsigned)(want < 1 ? 1 : want < cap ? want : cap), 256, 0, s>>>(x, y, n);
}

int launch_gemm_tc(uint32_t quant, const GemmArgs& a, cudaStream_t s) {
    const int splits = gemm_tc_splits(a);
    if (splits > 1 && !a.work) return -2;
    const bool two = a.terms >= 2;
    switch (quant) {
    case kQ4_K: return two ? dispatch_tn<kQ4_K, 2>(a, splits, s) : dispatch_tn<kQ4_K, 1>(a, splits, s);
    case kQ5_K: return two ? dispatch_tn<kQ5_K, 2>(a, splits, s) : dispatch_tn<kQ5_K, 1>(a, splits, s);
    case kQ6_K: return two ? dispatch_tn<kQ6_K, 2>(a, splits, s) : dispatch_tn<kQ6_K, 1>(a, splits, s);
    default: return -1;
    }
}

}  // namespace strata
