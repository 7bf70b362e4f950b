// expf_libm.cuh — the host C library's expf on the device, bit for bit, on the
// max-shifted softmax domain x in [-104, 0] (strata-core's softmax and router
// call Rust's f32::exp there: crates/strata-core/src/ops.rs:105-116,
// crates/strata-core/src/moe.rs:57-68).
//
// y = exp((double)x) rounded to f32 is the correctly rounded exp unless y lies
// within a few double ulps of a rounding midpoint, and the C library's expf
// (error below 0.502 ulp) is correctly rounded except within 1/256 ulp of one.
// So: when y is at least 2^-7 ulp from the midpoint on its side (all but about
// 0.2% of the domain) the rounded y is the answer; otherwise x is looked up in
// the table gen_expf_fix.c builds from the host's expf (every input where expf
// is not correctly rounded, and every input within 16 double ulps of a
// midpoint), and the rounded y stands when x is not there. gen_expf_fix.c
// replays this rule on every float of the domain and the build fails unless
// all results equal expf's. Outside the domain: the rounded y.
#pragma once
#include <cstdint>

#include "expf_fix.inc"  // kExpfFixIdx / kExpfFixKey / kExpfFixVal, generated into the build directory

namespace strata {

// The table entry for x (v = |x|'s bits), or r when x has none. Buckets are the
// high 16 bits of v; keys are the low 16, ascending within a bucket.
static __device__ __noinline__ float expf_fix_lookup(float x, float r) {
    const uint32_t v = __float_as_uint(x) & 0x7FFFFFFFu;
    const uint32_t b = v >> 16, key = v & 0xFFFFu;
    const uint32_t end = kExpfFixIdx[b + 1];
    for (uint32_t i = kExpfFixIdx[b]; i < end; ++i) {
        const uint32_t k = kExpfFixKey[i];
        if (k == key) return __uint_as_float(kExpfFixVal[i]);
        if (k > key) break;
    }
    return r;
}

static __device__ __forceinline__ float expf_libm(float x) {
    const double y = exp((double)x);
    const float r = __double2float_rn(y);
    if (!(x <= 0.0f && x >= -104.0f)) return r;  // also NaN
    const uint32_t ur = __float_as_uint(r);
    const double e = y - (double)r;  // exact: y and r are within a factor of two
    // the neighbour of r on y's side (r >= 0 here; r = 0 only with e >= 0)
    const float nb = __uint_as_float(e >= 0.0 ? ur + 1u : ur - 1u);
    const double half = 0.5 * fabs((double)nb - (double)r);  // r to the midpoint
    if (fabs(fabs(e) - half) >= half * (1.0 / 64.0)) return r;
    return expf_fix_lookup(x, r);
}

}  // namespace strata
