// expf_libm.cuh — the host C library's expf on the device, bit for bit, on the
// max-shifted softmax domain x in [-104, 0] (strata-core's softmax and router
// call Rust's f32::exp there: crates/strata-core/src/ops.rs:105-116,
// crates/strata-core/src/moe.rs:57-68).
//
// y = exp((double)x) rounded to f32 is the correctly rounded exp unless y lies
// within a few double ulps of a rounding midpoint, and the C library's expf
// (error below 0.502 ulp) is correctly rounded except within 2^-9.25 ulp of
// one. So: when y is at least 2^-9 ulp from the midpoint on its side (all but
// 0.1% of the domain) the rounded y is the answer; otherwise x is looked up in
// the table gen_expf_fix.c builds from the host's expf (every input where expf
// is not correctly rounded, and every input within 16 double ulps of a
// midpoint), and the rounded y stands when x is not there. gen_expf_fix.c
// replays this rule on every float of the domain and the build fails unless
// all results equal expf's. Outside the domain: the rounded y.
#pragma once
#include <cstdint>

#include "expf_fix.inc"  // kExpfFix, kExpfFixBits, kExpfFixMaxProbe: generated into the build directory

namespace strata {

// The table entry for x, or r when x has none: open addressing over
// kExpfFix ({|x|'s bits, expf's bits}; Fibonacci hashing, linear probing, an
// empty slot has key 0xFFFFFFFF), at most kExpfFixMaxProbe slots.
static __device__ __noinline__ float expf_fix_lookup(float x, float r) {
    const uint32_t v = __float_as_uint(x) & 0x7FFFFFFFu;
    uint32_t h = (v * 0x9E3779B1u) >> (32 - kExpfFixBits);
    for (uint32_t p = 0; p < kExpfFixMaxProbe; ++p) {
        const uint2 s = kExpfFix[h];
        if (s.x == v) return __uint_as_float(s.y);
        if (s.x == 0xFFFFFFFFu) break;
        h = (h + 1) & ((1u << kExpfFixBits) - 1);
    }
    return r;
}

// The rounded double exp, and in `exact` whether it is also the C library's
// value (false only near a rounding midpoint: expf_libm_near gives it then).
// No loads and no calls, so loops over many inputs stay pipelined.
static __device__ __forceinline__ float expf_libm_try(float x, bool& exact) {
    const double y = exp((double)x);
    const float r = __double2float_rn(y);
    exact = true;
    if (!(x <= 0.0f && x >= -104.0f)) return r;  // also NaN
    const uint32_t ur = __float_as_uint(r);
    const double e = y - (double)r;  // exact: y and r are within a factor of two
    // the neighbour of r on y's side (r >= 0 here; r = 0 only with e >= 0)
    const float nb = __uint_as_float(e >= 0.0 ? ur + 1u : ur - 1u);
    const double half = 0.5 * fabs((double)nb - (double)r);  // r to the midpoint
    exact = fabs(fabs(e) - half) >= half * (1.0 / 256.0);  // at least 2^-9 ulp from the midpoint
    return r;
}

// The C library's expf for an input expf_libm_try did not settle.
static __device__ __noinline__ float expf_libm_near(float x) {
    return expf_fix_lookup(x, __double2float_rn(exp((double)x)));
}

static __device__ __forceinline__ float expf_libm(float x) {
    bool exact;
    const float r = expf_libm_try(x, exact);
    return exact ? r : expf_libm_near(x);
}

}  // namespace strata
