// elementwise.cu — the elementwise trait methods of ComputeBackend
// (crates/strata-core/src/backend.rs:37-50) on the device, so a layer's
// activations can stay in HBM between the projections.
//
// Same arithmetic as CpuBackend (crates/strata-backend-cpu/src/lib.rs:44-67):
//   rms_norm   ops.rs:45-56    f64 sum of squares / n; x = f32((x * scale) * w)
//   l2_norm    ops.rs:71-81    f64 sum of squares;     x = f32(x * inv)
//   softmax    ops.rs:107-119  f32 max shift, f32 exp, f64 sum; x = f32(e * inv)
//   rope_neox  ops.rs:121-140  NEOX pairs (i, i + n_rot/2), f64 angles and products
//   add        ops.rs:164-168  a += b in f32
// The f64 sums are reduced across a CTA instead of left to right (both
// exact to about 1e-16 relative, far inside an f32 ulp); products that the
// reference forms separately are kept unfused (__dmul_rn / __dadd_rn); the
// f32 exp is the f64 exp rounded to f32 (the correctly rounded value in all
// but double-rounding ties). One CTA per vector for the reductions.
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>

#include "expf_libm.cuh"
#include "runtime.cuh"

namespace strata {
namespace {

constexpr int kEwThreads = 256;

// CTA-wide sum / max; every thread gets the result (sh: 32 entries).
__device__ double block_sum(double v, double* sh) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();  // sh may still be read from a previous reduction
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    v = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) v += sh[w];
    return v;
}
__device__ float block_max(float v, float* sh) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    v = -INFINITY;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) v = fmaxf(v, sh[w]);
    return v;
}

// rows x n, row r normalised with w (n): ops::rms_norm per row.
__global__ void __launch_bounds__(kEwThreads) rms_norm_kernel(float* __restrict__ x, const float* __restrict__ w,
                                                              int64_t n, double eps) {
    __shared__ double sh[32];
    float* row = x + (int64_t)blockIdx.x * n;
    double ss = 0.0;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) ss += __dmul_rn((double)row[i], (double)row[i]);
    ss = block_sum(ss, sh) / (double)n;
    const double scale = 1.0 / sqrt(ss + eps);
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x)
        row[i] = (float)__dmul_rn(__dmul_rn((double)row[i], scale), (double)w[i]);
}

// heads x head_dim: ops::l2_norm per head.
__global__ void __launch_bounds__(kEwThreads) l2_norm_kernel(float* __restrict__ x, int64_t n, double eps) {
    __shared__ double sh[32];
    float* row = x + (int64_t)blockIdx.x * n;
    double ss = 0.0;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) ss += __dmul_rn((double)row[i], (double)row[i]);
    ss = block_sum(ss, sh);
    const double inv = 1.0 / sqrt(ss + eps);
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) row[i] = (float)__dmul_rn((double)row[i], inv);
}

// rows x n: ops::softmax per row.
__global__ void __launch_bounds__(kEwThreads) softmax_kernel(float* __restrict__ x, int64_t n) {
    __shared__ double sh[32];
    __shared__ float shf[32];
    float* row = x + (int64_t)blockIdx.x * n;
    float mx = -INFINITY;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) mx = fmaxf(mx, row[i]);
    mx = block_max(mx, shf);
    double sum = 0.0;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float e = expf_libm(row[i] - mx);  // f32::exp, as the C library rounds it
        row[i] = e;
        sum += (double)e;
    }
    sum = block_sum(sum, sh);
    const double inv = 1.0 / sum;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) row[i] = (float)__dmul_rn((double)row[i], inv);
}

// heads of `stride` floats: ops::rope_neox on the first nr (even) dims of each.
__global__ void __launch_bounds__(kEwThreads) rope_neox_kernel(float* __restrict__ x, int64_t stride, int64_t nr,
                                                               int64_t pos, double base) {
    float* head = x + (int64_t)blockIdx.x * stride;
    const int64_t half = nr / 2;
    for (int64_t i = threadIdx.x; i < half; i += blockDim.x) {
        const double theta = pow(base, -2.0 * (double)i / (double)nr);
        const double angle = __dmul_rn(theta, (double)pos);
        double s, c;
        sincos(angle, &s, &c);
        const double a = head[i], b = head[i + half];
        head[i] = (float)__dsub_rn(__dmul_rn(a, c), __dmul_rn(b, s));
        head[i + half] = (float)__dadd_rn(__dmul_rn(a, s), __dmul_rn(b, c));
    }
}

__global__ void add_kernel(float* __restrict__ a, const float* __restrict__ b, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        a[i] += b[i];
}

constexpr int64_t kMaxRows = int64_t(1) << 31;  // grid.x limit

int ew_checked(strata_ctx* ctx, int64_t n, int64_t rows) {
    if (n < 1 || rows < 1 || rows >= kMaxRows) return fail(ctx, STRATA_ERR_INVALID, "bad shape %lld x %lld",
                                                          (long long)rows, (long long)n);
    return STRATA_OK;
}

// Host-buffer form of one op on `n` floats (plus an optional read-only
// second operand of n2 floats): stage, run `launch` on ctx->stream, copy back.
template <typename F>
int ew_host(strata_ctx* ctx, float* x, int64_t n, const float* b, int64_t n2, F launch) {
    const size_t xb = (size_t)n * 4, bb = b ? (size_t)n2 * 4 : 0;
    int rc;
    if ((rc = ensure_device(ctx, ctx->x_dev, xb + bb, "cudaMalloc(x)"))) return rc;
    if ((rc = ensure_pinned(ctx, ctx->x_host, xb + bb, "cudaMallocHost(x)"))) return rc;
    char* hp = static_cast<char*>(ctx->x_host.ptr);
    memcpy(hp, x, xb);
    if (b) memcpy(hp + xb, b, bb);
    cudaError_t e = cudaMemcpyAsync(ctx->x_dev.ptr, hp, xb + bb, cudaMemcpyHostToDevice, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMemcpyAsync(H2D)");
    float* xd = static_cast<float*>(ctx->x_dev.ptr);
    launch(xd, b ? xd + n : nullptr, ctx->stream);
    if ((rc = check_launch(ctx, "elementwise kernel"))) return rc;
    e = cudaMemcpyAsync(hp, xd, xb, cudaMemcpyDeviceToHost, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMemcpyAsync(D2H)");
    if ((rc = wait_stream(ctx, ctx->stream))) return rc;
    memcpy(x, hp, xb);
    return STRATA_OK;
}

int64_t rope_pairs(int64_t n_rot, int64_t head_dim, int64_t len) {
    int64_t nr = n_rot < head_dim ? n_rot : head_dim;
    nr = nr < len ? nr : len;
    return nr < 0 ? 0 : (nr & ~int64_t(1));
}

unsigned add_grid(int64_t n, int sm) {
    int64_t g = (n + kEwThreads - 1) / kEwThreads;
    const int64_t cap = 8 * (int64_t)(sm > 0 ? sm : 148);
    return (unsigned)(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace
}  // namespace strata

using namespace strata;

extern "C" {

int strata_cuda_rms_norm_dev(strata_ctx* ctx, float* x_dev, const float* w_dev, int64_t n, int64_t rows, double eps,
                             void* stream) {
    if (!ctx || !x_dev || !w_dev) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = ew_checked(ctx, n, rows);
    if (rc) return rc;
    cudaSetDevice(ctx->device);
    rms_norm_kernel<<<(unsigned)rows, kEwThreads, 0, pick_stream(ctx, stream)>>>(x_dev, w_dev, n, eps);
    return check_launch(ctx, "rms_norm kernel");
}

int strata_cuda_l2_norm_dev(strata_ctx* ctx, float* x_dev, int64_t head_dim, int64_t heads, double eps,
                            void* stream) {
    if (!ctx || !x_dev) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = ew_checked(ctx, head_dim, heads);
    if (rc) return rc;
    cudaSetDevice(ctx->device);
    l2_norm_kernel<<<(unsigned)heads, kEwThreads, 0, pick_stream(ctx, stream)>>>(x_dev, head_dim, eps);
    return check_launch(ctx, "l2_norm kernel");
}

int strata_cuda_softmax_dev(strata_ctx* ctx, float* x_dev, int64_t n, int64_t rows, void* stream) {
    if (!ctx || !x_dev) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = ew_checked(ctx, n, rows);
    if (rc) return rc;
    cudaSetDevice(ctx->device);
    softmax_kernel<<<(unsigned)rows, kEwThreads, 0, pick_stream(ctx, stream)>>>(x_dev, n);
    return check_launch(ctx, "softmax kernel");
}

int strata_cuda_rope_neox_dev(strata_ctx* ctx, float* x_dev, int64_t head_dim, int64_t heads, int64_t n_rot,
                              int64_t pos, double freq_base, void* stream) {
    if (!ctx || !x_dev || pos < 0 || n_rot < 0) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = ew_checked(ctx, head_dim, heads);
    if (rc) return rc;
    const int64_t nr = rope_pairs(n_rot, head_dim, head_dim);
    if (nr == 0) return STRATA_OK;
    cudaSetDevice(ctx->device);
    rope_neox_kernel<<<(unsigned)heads, kEwThreads, 0, pick_stream(ctx, stream)>>>(x_dev, head_dim, nr, pos,
                                                                                   freq_base);
    return check_launch(ctx, "rope_neox kernel");
}

int strata_cuda_add_dev(strata_ctx* ctx, float* a_dev, const float* b_dev, int64_t n, void* stream) {
    if (!ctx || !a_dev || !b_dev) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = ew_checked(ctx, n, 1);
    if (rc) return rc;
    cudaSetDevice(ctx->device);
    add_kernel<<<add_grid(n, ctx->sm_count), kEwThreads, 0, pick_stream(ctx, stream)>>>(a_dev, b_dev, n);
    return check_launch(ctx, "add kernel");
}

// ---- the trait methods on host slices (one vector per call, as CpuBackend)

int strata_cuda_rms_norm(strata_ctx* ctx, float* x, const float* w, int64_t n, double eps) {
    if (!ctx || !x || !w) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = ew_checked(ctx, n, 1);
    if (rc) return rc;
    cudaSetDevice(ctx->device);
    return ew_host(ctx, x, n, w, n, [&](float* xd, float* wd, cudaStream_t s) {
        rms_norm_kernel<<<1, kEwThreads, 0, s>>>(xd, wd, n, eps);
    });
}

int strata_cuda_l2_norm(strata_ctx* ctx, float* head, int64_t n, double eps) {
    if (!ctx || !head) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = ew_checked(ctx, n, 1);
    if (rc) return rc;
    cudaSetDevice(ctx->device);
    return ew_host(ctx, head, n, nullptr, 0, [&](float* xd, float*, cudaStream_t s) {
        l2_norm_kernel<<<1, kEwThreads, 0, s>>>(xd, n, eps);
    });
}

int strata_cuda_softmax(strata_ctx* ctx, float* xs, int64_t n) {
    if (!ctx || !xs) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = ew_checked(ctx, n, 1);
    if (rc) return rc;
    cudaSetDevice(ctx->device);
    return ew_host(ctx, xs, n, nullptr, 0, [&](float* xd, float*, cudaStream_t s) {
        softmax_kernel<<<1, kEwThreads, 0, s>>>(xd, n);
    });
}

int strata_cuda_rope_neox(strata_ctx* ctx, float* head, int64_t len, int64_t pos, int64_t n_rot, int64_t head_dim,
                          double freq_base) {
    if (!ctx || !head || pos < 0 || n_rot < 0) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = ew_checked(ctx, len, 1);
    if (rc) return rc;
    const int64_t nr = rope_pairs(n_rot, head_dim, len);
    if (nr == 0) return STRATA_OK;
    cudaSetDevice(ctx->device);
    return ew_host(ctx, head, len, nullptr, 0, [&](float* xd, float*, cudaStream_t s) {
        rope_neox_kernel<<<1, kEwThreads, 0, s>>>(xd, len, nr, pos, freq_base);
    });
}

int strata_cuda_add(strata_ctx* ctx, float* a, const float* b, int64_t n) {
    if (!ctx || !a || !b) return STRATA_ERR_INVALID;
    STRATA_CALL_RANGE();
    std::lock_guard<std::mutex> g(ctx->mu);
    int rc = ew_checked(ctx, n, 1);
    if (rc) return rc;
    cudaSetDevice(ctx->device);
    return ew_host(ctx, a, n, b, n, [&](float* ad, float* bd, cudaStream_t s) {
        add_kernel<<<add_grid(n, ctx->sm_count), kEwThreads, 0, s>>>(ad, bd, n);
    });
}

}  // extern "C"
