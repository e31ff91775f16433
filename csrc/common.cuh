// Shared helpers for the sm_100a kernels of primus_dlrm_b200.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

// Light ATen headers only (no torch/extension.h): keeps nvcc host passes fast.
#include <ATen/core/Tensor.h>
#include <ATen/ops/empty.h>
#include <ATen/ops/empty_like.h>
#include <ATen/ops/zeros.h>
#include <ATen/ops/zeros_like.h>
#include <ATen/ops/from_blob.h>
#include <c10/cuda/CUDAStream.h>
#include <c10/util/Exception.h>
#include <atomic>
#include <cstdio>
#include <optional>
#include <vector>

// Checks in the nvcc-compiled sources format their message with snprintf and
// hand TORCH_CHECK one C string: a message assembled by c10::str from several
// parts (C++ streams) crashed the process with SIGSEGV in these translation
// units when the check failed, instead of raising (a failing check with a
// single-string message raises normally).
#define PD_CHECK(cond, ...)                                                        \
  do {                                                                             \
    if (C10_UNLIKELY(!(cond))) {                                                   \
      char pd_msg__[512];                                                          \
      snprintf(pd_msg__, sizeof(pd_msg__), __VA_ARGS__);                           \
      TORCH_CHECK(false, static_cast<const char*>(pd_msg__));                      \
    }                                                                              \
  } while (0)

#define PD_CHECK_CUDA(expr)                                                        \
  do {                                                                             \
    cudaError_t err__ = (expr);                                                    \
    PD_CHECK(err__ == cudaSuccess, "CUDA error %s at %s:%d", cudaGetErrorString(err__), __FILE__, __LINE__); \
  } while (0)

#define PD_CHECK_LAUNCH() do { PD_CHECK_CUDA(cudaGetLastError()); ::pd::note_launch(); } while (0)

namespace pd {

// Error codes a kernel writes into the device error word instead of faulting.
enum ErrorCode : int {
  kOk = 0,
  kIdOutOfRange = 1,
  kWaitTimeout = 2,
  kBadShape = 3,
};

// Number of kernels this library has launched (read by benchmarks to report
// how many of their kernels ran inside a timed region).
inline std::atomic<long long>& launch_counter() {
  static std::atomic<long long> n{0};
  return n;
}
inline void note_launch(int k = 1) { launch_counter().fetch_add(k, std::memory_order_relaxed); }

inline cudaStream_t stream() { return c10::cuda::getCurrentCUDAStream().stream(); }

inline int num_sms() {
  static int n = -1;
  if (n < 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

__device__ __forceinline__ float bf16_to_f(__nv_bfloat16 v) { return __bfloat162float(v); }

__device__ __forceinline__ void store4_bf16(__nv_bfloat16* dst, float4 v) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y);
  __nv_bfloat162 b = __floats2bfloat162_rn(v.z, v.w);
  uint2 pk;
  pk.x = *reinterpret_cast<uint32_t*>(&a);
  pk.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(dst) = pk;
}

__device__ __forceinline__ float4 load4_bf16(const __nv_bfloat16* src) {
  uint2 pk = *reinterpret_cast<const uint2*>(src);
  __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&pk.x);
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&pk.y);
  float2 fa = __bfloat1622float2(a);
  float2 fb = __bfloat1622float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Record the first error code seen by any thread (never traps).
__device__ __forceinline__ void set_error(int* err, int code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ float exp2f_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// GELU(x) = x * Phi(x) (the exact, erf-based form used by nn.GELU()).
// Normal CDF with no division and no exponential, so the GELU epilogues do
// not queue on the MUFU pipe: Phi(x) = 1/2 + x R(t), t = 2 x^2 / c^2 - 1,
// x clamped to [-c, c], c = 4.5. R is a degree-9 polynomial in t: the
// L-infinity fit of the absolute error of x R(t) to Phi(x) - 1/2 on [0, c],
// computed by Lawson's iteratively reweighted least squares
// (csrc/gen_gelu_poly.py prints the coefficients and the error). Max |error|
// over all x in fp32: 3.7e-6 (beyond the clamp the tail 1 - Phi(c) = 3.4e-6 is dropped).
__device__ __forceinline__ float norm_cdf_poly(float x) {
  const float xc = fminf(fmaxf(x, -4.5f), 4.5f);
  const float t = fmaf(xc * xc, 0.0987654328f, -1.0f);
  float r = fmaf(-0.00193071156f, t, 0.00496269623f);
  r = fmaf(r, t, -0.00606983015f);
  r = fmaf(r, t, 0.00965323579f);
  r = fmaf(r, t, -0.0184842162f);
  r = fmaf(r, t, 0.0288576446f);
  r = fmaf(r, t, -0.0402369164f);
  r = fmaf(r, t, 0.0546374917f);
  r = fmaf(r, t, -0.0771858841f);
  r = fmaf(r, t, 0.156906039f);
  const float p = fmaf(xc, r, 0.5f);
  // beyond the clamp the tail is dropped (exactly 0 or 1), so GELU(x) -> 0 for x -> -inf
  return fabsf(x) < 4.5f ? p : (x > 0.f ? 1.f : 0.f);
}

struct GeluEval { float cdf, pdf; };
__device__ __forceinline__ GeluEval gelu_eval(float x) {
  // phi(x) = exp(-x^2 / 2) / sqrt(2 pi): one MUFU exponential, needed by GELU' only
  const float e = exp2f_approx(x * x * -0.72134752044448170f);
  return GeluEval{norm_cdf_poly(x), 0.3989422804014327f * e};
}
__device__ __forceinline__ float gelu_f(float x) { return x * norm_cdf_poly(x); }
__device__ __forceinline__ float gelu_grad_f(float x) {
  const GeluEval g = gelu_eval(x);
  return g.cdf + x * g.pdf;
}

}  // namespace pd
