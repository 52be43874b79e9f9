// softmax_math.cuh -- arithmetic helpers of the softmax warps that are not single PTX
// instructions: a polynomial 2^x on the FMA pipe and the soft-cap's tanh, each on a pair of
// fp32 values packed in 64 bits.  Shared by the forward kernel and the device unit test of
// their error bounds (tests/cuda/math_check.cu).
#pragma once

#include <stdint.h>

#include "sm100_ptx.cuh"

namespace odf {

// 2^x for a pair on the FMA pipe.  At d = 64 the MUFU unit (16 ex2 per clock per SM) is the
// binding limit, so part of the columns take this path instead.  x is clamped to -127, split as
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

// softcap * tanh(t) * log2(e) for a pair of scores given u = 2 log2(e) t (t = score / softcap),
// from tanh|t| = 2 / (1 + e) - 1 with e = 2^(-|u|) in (0, 1]: no overflow for any |t|, the
// scale folded into one FMA and the sign restored from u.  e is one MUFU ex2 per score; the
// reciprocal r = 1 / (1 + e) stays off the MUFU pipe (the soft-capped kernel is bound by it):
// with d = 1 + e in (1, 2], a quadratic seed fitted here for minimax relative error on [1, 2]
// (r0 = 70/33 - 48/33 d + 32/99 d^2, relative error 1/99) and two Newton steps
// r <- r + r (1 - d r) (error squared each time) give r to fp32 rounding, on the FMA pipe only.
// Absolute error of the result: a few fp32 ulps of softcap * log2(e).
constexpr float kRcpSeedC0 = 70.0f / 33.0f;
constexpr float kRcpSeedC1 = 48.0f / 33.0f;  // the seed's linear term is -C1 d
constexpr float kRcpSeedC2 = 32.0f / 99.0f;

__device__ __forceinline__ uint64_t softcap2(uint64_t u, uint64_t cap2x, uint64_t neg_cap) {
    const float e0 = ptx::ex2(-fabsf(ptx::lo_f32(u)));
    const float e1 = ptx::ex2(-fabsf(ptx::hi_f32(u)));
    // nd = -(1 + e); the seed in nd: C0 + C1 nd + C2 nd^2
    const uint64_t nd = ptx::ffma2(ptx::f32x2(e0, e1), ptx::f32x2(-1.0f), ptx::f32x2(-1.0f));
    uint64_t r = ptx::ffma2(nd, ptx::f32x2(kRcpSeedC2), ptx::f32x2(kRcpSeedC1));
    r = ptx::ffma2(r, nd, ptx::f32x2(kRcpSeedC0));
    uint64_t err = ptx::ffma2(nd, r, ptx::f32x2(1.0f));  // 1 - d r
    r = ptx::ffma2(r, err, r);
    err = ptx::ffma2(nd, r, ptx::f32x2(1.0f));
    r = ptx::ffma2(r, err, r);
    return ptx::ffma2(r, cap2x, neg_cap) ^ (u & 0x8000000080000000ull);
}

}  // namespace odf
