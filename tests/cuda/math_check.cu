// math_check.cu -- test-only device wrappers around the softmax warps' arithmetic helpers
// (dnn-flash_b200/csrc/softmax_math.cuh), so their error bounds can be checked on the GPU
// against exact values computed on the host.  Built into tests/cuda/lib/libodf_math_check.so
// by dnn-flash_b200/build.py; not part of the library.
#include <cuda_runtime.h>
#include <stdint.h>

#include "odf_internal.h"
#include "softmax_math.cuh"

namespace {

// y_poly[i] = exp2_poly2(x[i]) and y_mufu[i] = ex2.approx(x[i]), pairs (2i, 2i+1) per thread.
__global__ void exp2_kernel(const float* __restrict__ x, float* __restrict__ y_poly, float* __restrict__ y_mufu,
                            int64_t n_pairs) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n_pairs) return;
    const float x0 = x[2 * i], x1 = x[2 * i + 1];
    const uint64_t p = odf::exp2_poly2(odf::ptx::f32x2(x0, x1));
    y_poly[2 * i] = odf::ptx::lo_f32(p);
    y_poly[2 * i + 1] = odf::ptx::hi_f32(p);
    y_mufu[2 * i] = odf::ptx::ex2(x0);
    y_mufu[2 * i + 1] = odf::ptx::ex2(x1);
}

// y[i] = softcap * tanh(s[i] / softcap) as the kernel forms it: t = s / softcap, tanh2(t), times
// softcap (the kernel folds softcap * log2 e into its exponent instead), pairs (2i, 2i+1).
__global__ void softcap_kernel(const float* __restrict__ s, float* __restrict__ y, int64_t n_pairs, float softcap) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n_pairs) return;
    const float inv = 1.0f / softcap;
    const uint64_t th = odf::tanh2(odf::ptx::f32x2(s[2 * i] * inv, s[2 * i + 1] * inv));
    y[2 * i] = odf::ptx::lo_f32(th) * softcap;
    y[2 * i + 1] = odf::ptx::hi_f32(th) * softcap;
}

// q[i] = x[i] / d through the kernels' invariant-divisor division (odf::fast_div).
__global__ void fastdiv_kernel(odf::FastDiv f, const uint32_t* __restrict__ x, uint32_t* __restrict__ q, int64_t n) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) q[i] = odf::fast_div(x[i], f);
}

}  // namespace

extern "C" {

// Host pointers; the host build of odf::make_fastdiv / odf::fast_div (no GPU needed).
void odf_math_check_fastdiv_host(uint32_t d, const uint32_t* x, uint32_t* q, int64_t n) {
    const odf::FastDiv f = odf::make_fastdiv(d);
    for (int64_t i = 0; i < n; ++i) q[i] = odf::fast_div(x[i], f);
}

// Device pointers; the device build (multiply-high instruction), synchronous.
int odf_math_check_fastdiv(uint32_t d, const uint32_t* x, uint32_t* q, int64_t n) {
    if (n <= 0 || d == 0) return static_cast<int>(cudaErrorInvalidValue);
    fastdiv_kernel<<<static_cast<unsigned>((n + 255) / 256), 256>>>(odf::make_fastdiv(d), x, q, n);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return static_cast<int>(e);
}


// Device pointers, n even; synchronous.  Returns a cudaError_t value (0 = success).
int odf_math_check_exp2(const float* x, float* y_poly, float* y_mufu, int64_t n) {
    if (n <= 0 || (n & 1)) return static_cast<int>(cudaErrorInvalidValue);
    const int64_t pairs = n / 2;
    exp2_kernel<<<static_cast<unsigned>((pairs + 255) / 256), 256>>>(x, y_poly, y_mufu, pairs);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return static_cast<int>(e);
}

int odf_math_check_softcap(const float* s, float* y, int64_t n, float softcap) {
    if (n <= 0 || (n & 1) || !(softcap > 0.0f)) return static_cast<int>(cudaErrorInvalidValue);
    const int64_t pairs = n / 2;
    softcap_kernel<<<static_cast<unsigned>((pairs + 255) / 256), 256>>>(s, y, pairs, softcap);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return static_cast<int>(e);
}

}  // extern "C"
