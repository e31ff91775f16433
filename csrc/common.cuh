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
// not queue on the MUFU pipe:
//   Phi(x) = sat(1/2 + x R(t)),  t = min(2 x^2 / c^2 - 1, 1),  c = 4.5,
// sat clamping to [0, 1]. R is a degree-9 polynomial in t: the L-infinity fit
// of the absolute error of x R(t) to Phi(x) - 1/2 on [0, c] by Lawson's
// iteratively reweighted least squares, under the constraint c R(1) =
// 1/2 + 2e-6 -- so for |x| >= c (t held at 1) the saturation returns exactly 0
// or 1 (csrc/gen_gelu_poly.py prints the coefficients and the error). Max
// |error| over all x in fp32: 5.5e-6.
#define PD_CDF_T_SCALE 0.0987654328f
#define PD_CDF_HORNER(R, T, FMA, K)                                              \
  R = FMA(K(-0.00155825319f), T, K(0.00492038578f));                           \
  R = FMA(R, T, K(-0.00684563117f));                                             \
  R = FMA(R, T, K(0.00971821137f));                                              \
  R = FMA(R, T, K(-0.0179516189f));                                              \
  R = FMA(R, T, K(0.0288285892f));                                               \
  R = FMA(R, T, K(-0.0403702296f));                                              \
  R = FMA(R, T, K(0.0546411946f));                                               \
  R = FMA(R, T, K(-0.0771770775f));                                              \
  R = FMA(R, T, K(0.156905979f))
#define PD_ID(v) (v)

__device__ __forceinline__ float norm_cdf_poly(float x) {
  const float t = fminf(fmaf(x * x, PD_CDF_T_SCALE, -1.0f), 1.0f);
  float r;
  PD_CDF_HORNER(r, t, fmaf, PD_ID);
  return __saturatef(fmaf(x, r, 0.5f));
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic: one instruction for two values).
__device__ __forceinline__ uint64_t pk2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ uint64_t pk2s(float v) { return pk2(v, v); }
__device__ __forceinline__ void pk2_split(uint64_t r, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ uint64_t pk2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t pk2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Phi of two values (same polynomial as norm_cdf_poly, Horner on pairs); u = x^2.
__device__ __forceinline__ void norm_cdf_poly2(float x0, float x1, uint64_t u, float& p0, float& p1) {
  float t0, t1;
  pk2_split(pk2_fma(u, pk2s(PD_CDF_T_SCALE), pk2s(-1.0f)), t0, t1);
  const uint64_t t = pk2(fminf(t0, 1.0f), fminf(t1, 1.0f));
  uint64_t r;
  PD_CDF_HORNER(r, t, pk2_fma, pk2s);
  float r0, r1;
  pk2_split(r, r0, r1);
  p0 = __saturatef(fmaf(x0, r0, 0.5f));
  p1 = __saturatef(fmaf(x1, r1, 0.5f));
}

// GELU of two values.
__device__ __forceinline__ void gelu2(float& x0, float& x1) {
  float p0, p1;
  norm_cdf_poly2(x0, x1, pk2_mul(pk2(x0, x1), pk2(x0, x1)), p0, p1);
  pk2_split(pk2_mul(pk2(x0, x1), pk2(p0, p1)), x0, x1);
}

// GELU'(x) = Phi(x) + x phi(x) of two values, phi(x) = exp(-x^2 / 2) / sqrt(2 pi)
// (one MUFU exponential each); with_gelu also returns GELU in x0, x1.
template <bool with_gelu>
__device__ __forceinline__ void gelu_grad2(float& x0, float& x1, float& d0, float& d1) {
  const uint64_t x = pk2(x0, x1);
  const uint64_t u = pk2_mul(x, x);
  float p0, p1;
  norm_cdf_poly2(x0, x1, u, p0, p1);
  float a0, a1;
  pk2_split(pk2_mul(u, pk2s(-0.72134752044448170f)), a0, a1);               // -x^2 / (2 ln 2)
  const uint64_t e = pk2(exp2f_approx(a0), exp2f_approx(a1));
  const uint64_t p = pk2(p0, p1);
  pk2_split(pk2_fma(pk2_mul(x, pk2s(0.3989422804014327f)), e, p), d0, d1);  // Phi + x phi
  if (with_gelu) pk2_split(pk2_mul(x, p), x0, x1);
}

__device__ __forceinline__ float gelu_f(float x) { return x * norm_cdf_poly(x); }
__device__ __forceinline__ float gelu_grad_f(float x) {
  const float e = exp2f_approx(x * x * -0.72134752044448170f);
  return fmaf(x * 0.3989422804014327f, e, norm_cdf_poly(x));
}

}  // namespace pd
