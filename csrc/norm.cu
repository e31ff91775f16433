// RMSNorm / LayerNorm forward + backward (bf16 activations, fp32 math).
//
// RMSNorm matches primus_dlrm/models/onetrans.py:74-82 under bf16 autocast:
//   t = bf16(x * rsqrt(mean(x^2) + eps));  y = bf16(t * w)
// (the reference multiplies the bf16 normalised tensor by the fp32 weight and
// the next Linear casts the fp32 product back to bf16).
//
// One warp owns one row; a lane moves 8 bf16 (16 B) per vector access.
// The optional residual input fuses `z = a + b` into the same pass (the
// OneTrans block's attention residual feeds norm2): the kernel then writes z
// as well as y.  dW is reduced per block in shared memory and added to an
// fp32 accumulator with one atomic per column per block.
#include "common.cuh"

namespace pd {

constexpr int kNormMaxVec = 8;  // up to 8 x 8 = 64 elements per lane -> D <= 2048

struct alignas(16) Vec8 { __nv_bfloat162 h[4]; };

__device__ __forceinline__ void unpack8(const Vec8& v, float* f) {
#pragma unroll
  for (int k = 0; k < 4; ++k) { float2 t = __bfloat1622float2(v.h[k]); f[2 * k] = t.x; f[2 * k + 1] = t.y; }
}
__device__ __forceinline__ Vec8 pack8(const float* f) {
  Vec8 v;
#pragma unroll
  for (int k = 0; k < 4; ++k) v.h[k] = __floats2bfloat162_rn(f[2 * k], f[2 * k + 1]);
  return v;
}
__device__ __forceinline__ float rbf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// kind: 0 = RMSNorm (weight only), 1 = LayerNorm (weight + bias)
template <int KIND, int NV>
__global__ void __launch_bounds__(256) norm_fwd_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ res,
    const float* __restrict__ w, const float* __restrict__ b, __nv_bfloat16* __restrict__ y,
    __nv_bfloat16* __restrict__ z, float* __restrict__ stat_rstd, float* __restrict__ stat_mean,
    int64_t rows, int D, float eps, int64_t rpb, int64_t x_bstride, int64_t r_bstride) {
  const int lane = threadIdx.x & 31;
  const int nvec = D >> 3;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t r = warp; r < rows; r += nw) {
    float v[NV][8];
    const int64_t bb = r / rpb, ii = r - bb * rpb;
    const Vec8* xr = reinterpret_cast<const Vec8*>(x + bb * x_bstride + ii * D);
    const Vec8* rr = res ? reinterpret_cast<const Vec8*>(res + bb * r_bstride + ii * D) : nullptr;
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int c = lane + 32 * k;
      if (c < nvec) {
        unpack8(xr[c], v[k]);
        if (rr) {
          float t[8];
          unpack8(rr[c], t);
#pragma unroll
          for (int e = 0; e < 8; ++e) v[k][e] = rbf(v[k][e] + t[e]);
          reinterpret_cast<Vec8*>(z + r * D)[c] = pack8(v[k]);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) s += (KIND == 0) ? v[k][e] * v[k][e] : v[k][e];
      }
    }
    s = warp_sum(s);
    float mean = 0.f, rstd;
    if (KIND == 0) {
      rstd = rsqrtf(s / D + eps);
    } else {
      mean = s / D;
      float q = 0.f;
#pragma unroll
      for (int k = 0; k < NV; ++k)
        if (lane + 32 * k < nvec)
#pragma unroll
          for (int e = 0; e < 8; ++e) { const float d = v[k][e] - mean; q += d * d; }
      q = warp_sum(q);
      rstd = rsqrtf(q / D + eps);
    }
    if (lane == 0) { stat_rstd[r] = rstd; if (KIND == 1) stat_mean[r] = mean; }
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int c = lane + 32 * k;
      if (c < nvec) {
        float o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int col = 8 * c + e;
          if (KIND == 0) o[e] = rbf(v[k][e] * rstd) * w[col];
          else o[e] = (v[k][e] - mean) * rstd * w[col] + b[col];
        }
        reinterpret_cast<Vec8*>(y + r * D)[c] = pack8(o);
      }
    }
  }
}

// Backward. dy: grad of y; dz_extra (optional): grad arriving directly at z
// (the residual path), added to dx. Writes dx (bf16) and accumulates dw/db.
template <int KIND, int NV>
__global__ void __launch_bounds__(256) norm_bwd_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ dy,
    const __nv_bfloat16* __restrict__ dz_extra, const float* __restrict__ w,
    const float* __restrict__ stat_rstd, const float* __restrict__ stat_mean,
    __nv_bfloat16* __restrict__ dx, float* __restrict__ dw, float* __restrict__ db,
    int64_t rows, int D) {
  extern __shared__ float sm[];  // [2 * D]: dw, db partials
  for (int i = threadIdx.x; i < 2 * D; i += blockDim.x) sm[i] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int nvec = D >> 3;
  float pw[NV][8], pb[NV][8];
#pragma unroll
  for (int k = 0; k < NV; ++k)
#pragma unroll
    for (int e = 0; e < 8; ++e) { pw[k][e] = 0.f; pb[k][e] = 0.f; }
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t r = warp; r < rows; r += nw) {
    const float rstd = stat_rstd[r];
    const float mean = KIND == 1 ? stat_mean[r] : 0.f;
    float xh[NV][8], g[NV][8];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int c = lane + 32 * k;
      if (c < nvec) {
        float xv[8], dv[8];
        unpack8(reinterpret_cast<const Vec8*>(x + r * D)[c], xv);
        unpack8(reinterpret_cast<const Vec8*>(dy + r * D)[c], dv);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int col = 8 * c + e;
          xh[k][e] = (xv[e] - mean) * rstd;
          g[k][e] = dv[e] * w[col];
          pw[k][e] += dv[e] * xh[k][e];
          pb[k][e] += dv[e];
          s1 += g[k][e] * xh[k][e];
          s2 += g[k][e];
        }
      }
    }
    s1 = warp_sum(s1) / D;
    s2 = warp_sum(s2) / D;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int c = lane + 32 * k;
      if (c < nvec) {
        float o[8];
        float ex[8];
        if (dz_extra) unpack8(reinterpret_cast<const Vec8*>(dz_extra + r * D)[c], ex);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float d = (KIND == 0) ? rstd * (g[k][e] - xh[k][e] * s1)
                                : rstd * (g[k][e] - s2 - xh[k][e] * s1);
          o[e] = dz_extra ? d + ex[e] : d;
        }
        reinterpret_cast<Vec8*>(dx + r * D)[c] = pack8(o);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int c = lane + 32 * k;
    if (c < nvec)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        atomicAdd(&sm[8 * c + e], pw[k][e]);
        if (KIND == 1) atomicAdd(&sm[D + 8 * c + e], pb[k][e]);
      }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    atomicAdd(dw + i, sm[i]);
    if (KIND == 1) atomicAdd(db + i, sm[D + i]);
  }
}

static void check_rows(const at::Tensor& t, int64_t D) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous(),
              "norm tensors must be contiguous bf16 CUDA tensors");
  TORCH_CHECK(t.size(-1) == D);
}

// [B, R, D] view whose rows are contiguous within a batch (any batch stride).
static void check_batch_rows(const at::Tensor& t, int64_t D) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16, "norm inputs must be bf16 CUDA tensors");
  TORCH_CHECK(t.dim() == 3 && t.size(2) == D && t.stride(2) == 1 && (t.size(1) == 1 || t.stride(1) == D),
              "norm input must be [B, R, D] with contiguous rows");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0 && t.stride(0) % 8 == 0,
              "norm input rows must be 16-byte aligned");
}

// Returns {y, z_or_empty, rstd, mean_or_empty}
std::vector<at::Tensor> norm_fwd(at::Tensor x, c10::optional<at::Tensor> res, at::Tensor w,
                                 c10::optional<at::Tensor> b, double eps, int64_t kind) {
  const int64_t D = x.size(-1);
  TORCH_CHECK(D % 8 == 0 && D <= 256 * kNormMaxVec, "norm dim must be a multiple of 8 and <= 2048");
  at::Tensor x3 = x.dim() == 3 ? x : x.reshape({1, -1, D});
  check_batch_rows(x3, D);
  at::Tensor r3;
  if (res) {
    r3 = res->dim() == 3 ? *res : res->reshape({1, -1, D});
    check_batch_rows(r3, D);
    TORCH_CHECK(r3.size(0) == x3.size(0) && r3.size(1) == x3.size(1));
  }
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.numel() == D);
  const int64_t rows = x3.size(0) * x3.size(1);
  const int64_t rpb = x3.size(1) > 0 ? x3.size(1) : 1;
  auto y = at::empty(x.sizes(), x.options());
  at::Tensor z = res ? at::empty(x.sizes(), x.options()) : at::Tensor();
  auto rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  at::Tensor mean = kind == 1 ? at::empty({rows}, x.options().dtype(at::kFloat)) : at::Tensor();
  if (rows == 0) return {y, z, rstd, mean};
  int64_t blocks = (rows + 7) / 8;
  const int64_t cap = int64_t(num_sms()) * 8;
  if (blocks > cap) blocks = cap;
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x3.data_ptr());
  auto rp = res ? reinterpret_cast<const __nv_bfloat16*>(r3.data_ptr()) : nullptr;
  const int64_t xbs = x3.stride(0), rbs = res ? r3.stride(0) : 0;
  auto yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  auto zp = res ? reinterpret_cast<__nv_bfloat16*>(z.data_ptr()) : nullptr;
  const float* bp = kind == 1 ? b->data_ptr<float>() : nullptr;
  float* mp = kind == 1 ? mean.data_ptr<float>() : nullptr;
  const int nv = int((D / 8 + 31) / 32);
#define PD_NF(K, NVv) norm_fwd_kernel<K, NVv><<<blocks, 256, 0, stream()>>>(xp, rp, w.data_ptr<float>(), bp, yp, zp, \
                                                   rstd.data_ptr<float>(), mp, rows, int(D), float(eps), rpb, xbs, rbs)
#define PD_NF_K(K) if (nv <= 1) PD_NF(K, 1); else if (nv <= 2) PD_NF(K, 2); else if (nv <= 4) PD_NF(K, 4); else PD_NF(K, 8)
  if (kind == 0) { PD_NF_K(0); } else { PD_NF_K(1); }
#undef PD_NF_K
#undef PD_NF
  PD_CHECK_LAUNCH();
  return {y, z, rstd, mean};
}

// Returns {dx, dw, db_or_empty}. xin is the normalised input (z when fused).
std::vector<at::Tensor> norm_bwd(at::Tensor xin, at::Tensor dy, c10::optional<at::Tensor> dz_extra,
                                 at::Tensor w, at::Tensor rstd, c10::optional<at::Tensor> mean,
                                 int64_t kind) {
  const int64_t D = xin.size(-1);
  check_rows(xin, D);
  auto dyc = dy.contiguous();
  check_rows(dyc, D);
  at::Tensor ex;
  if (dz_extra) { ex = dz_extra->contiguous(); check_rows(ex, D); }
  const int64_t rows = xin.numel() / D;
  auto dx = at::empty_like(xin);
  auto dw = at::zeros({D}, w.options());
  at::Tensor db = kind == 1 ? at::zeros({D}, w.options()) : at::Tensor();
  if (rows == 0) return {dx, dw, db};
  int64_t blocks = (rows + 7) / 8;
  const int64_t cap = int64_t(num_sms()) * 4;
  if (blocks > cap) blocks = cap;
  const size_t smem = 2 * D * sizeof(float);
  auto xp = reinterpret_cast<const __nv_bfloat16*>(xin.data_ptr());
  auto dyp = reinterpret_cast<const __nv_bfloat16*>(dyc.data_ptr());
  auto exp_ = ex.defined() ? reinterpret_cast<const __nv_bfloat16*>(ex.data_ptr()) : nullptr;
  auto dxp = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
  const float* mp = kind == 1 ? mean->data_ptr<float>() : nullptr;
  float* dbp = kind == 1 ? db.data_ptr<float>() : nullptr;
  const int nv = int((D / 8 + 31) / 32);
#define PD_NB(K, NVv) norm_bwd_kernel<K, NVv><<<blocks, 256, smem, stream()>>>(xp, dyp, exp_, w.data_ptr<float>(), \
                                                   rstd.data_ptr<float>(), mp, dxp, dw.data_ptr<float>(), dbp, rows, int(D))
#define PD_NB_K(K) if (nv <= 1) PD_NB(K, 1); else if (nv <= 2) PD_NB(K, 2); else if (nv <= 4) PD_NB(K, 4); else PD_NB(K, 8)
  if (kind == 0) { PD_NB_K(0); } else { PD_NB_K(1); }
#undef PD_NB_K
#undef PD_NB
  PD_CHECK_LAUNCH();
  return {dx, dw, db};
}

}  // namespace pd
