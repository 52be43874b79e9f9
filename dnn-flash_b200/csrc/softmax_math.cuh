// softmax_math.cuh -- arithmetic helpers of the softmax warps: a polynomial 2^x on the FMA pipe
// and the soft-cap's tanh, each on a pair of fp32 values packed in 64 bits.  Shared by the forward kernel and the device unit test of
// their error bounds (tests/cuda/math_check.cu).
#pragma once

#include <stdint.h>

#include "sm100_ptx.cuh"

namespace odf {

// 2^x for a pair on the FMA pipe.  At d = 64, and in the soft-capped variants whose MUFU unit
// also computes tanh, the MUFU unit (16 results per clock per SM) is the binding limit, so part
// of the columns take this path instead.  x is clamped to -127, split as
// x = j + f with j = rint(x) (by adding and subtracting 1.5 * 2^23) and f in [-0.5, 0.5]; 2^f
// comes from a degree-3 polynomial whose coefficients were fitted here for minimax relative
// error with p(0) = 1 (max relative error 1.0e-4), and j is added to the exponent field.
// x = -127 (so also -inf) gives exactly +0; other x below -126 give values in [0, 2^-126).
constexpr float kExp2C1 = 0.6932829022407532f;
constexpr float kExp2C2 = 0.2422109693288803f;
constexpr float kExp2C3 = 0.055009059607982635f;

__device__ __forceinline__ uint64_t exp2_poly2(uint64_t x) {
    const uint64_t xc = ptx::f32x2(fmaxf(ptx::lo_f32(x), -127.0f), fmaxf(ptx::hi_f32(x), -127.0f));
    const uint64_t t = ptx::fadd2(xc, ptx::f32x2(12582912.0f));   // 1.5 * 2^23 + rint(x)
    const uint64_t j = ptx::fadd2(t, ptx::f32x2(-12582912.0f));   // rint(x), exact
    const uint64_t f = ptx::ffma2(j, ptx::f32x2(-1.0f), xc);      // x - rint(x), exact
    uint64_t p = ptx::ffma2(ptx::f32x2(kExp2C3), f, ptx::f32x2(kExp2C2));
    p = ptx::ffma2(p, f, ptx::f32x2(kExp2C1));
    p = ptx::ffma2(p, f, ptx::f32x2(1.0f));
    // the low bits of t hold 1.5 * 2^23 + j; shifted left by 23 only j << 23 remains (mod 2^32)
    const uint32_t lo = static_cast<uint32_t>(p) + (static_cast<uint32_t>(t) << 23);
    const uint32_t hi = static_cast<uint32_t>(p >> 32) + (static_cast<uint32_t>(t >> 32) << 23);
    return (static_cast<uint64_t>(hi) << 32) | lo;
}

// tanh of a pair, for the soft-cap softcap * tanh(score / softcap): one MUFU tanh.approx per
// value (the same MUFU cost as one exponential, and no FMA-pipe work).  PTX documents a relative
// error bound of 2^-11 for tanh.approx.f32; on sm_100 its measured error over [-20, 20] is at most
// 9.9e-6 relative and 7.8e-6 absolute, and tests/test_math_check_gpu.py pins an absolute bound of
// 1e-5 (times softcap after scaling), which the attention parity tolerances rely on.
__device__ __forceinline__ uint64_t tanh2(uint64_t t) {
    return ptx::f32x2(ptx::tanh_approx(ptx::lo_f32(t)), ptx::tanh_approx(ptx::hi_f32(t)));
}

}  // namespace odf
