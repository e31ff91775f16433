// RMSNorm / LayerNorm forward + backward (bf16 activations, fp32 math).
//
// RMSNorm matches primus_dlrm/models/onetrans.py:74-82 under bf16 autocast:
//   t = bf16(x * rsqrt(mean(x^2) + eps));  y = bf16(t * w)
// (the reference multiplies the bf16 normalised tensor by the fp32 weight and
// the next Linear casts the fp32 product back to bf16).
//
// One warp owns a group of rows (4 at D <= 256); a lane moves 8 bf16 (16 B)
// per vector access and the group's loads are all issued before its reductions.
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
__device__ __forceinline__ Vec8 as_vec8(uint4 u) { return *reinterpret_cast<const Vec8*>(&u); }
__device__ __forceinline__ float rbf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Rows per warp per loop iteration: the loads of all RPW rows are issued
// before any reduction, so a warp keeps RPW x NV x 16 B per lane in flight
// (one 512-byte row per warp was latency-bound at D = 256).  Rows stay in
// registers as packed bf16 and are unpacked again for each pass, which keeps
// the live state at 4 registers per row-vector.  Weights (and the dW / dB
// partials) live in registers when a lane owns at most 16 columns; wider rows
// read the weight through L1 and accumulate the partials in shared memory.
template <int NV> struct NormRows { static constexpr int value = NV == 1 ? 4 : (NV == 2 ? 2 : 1); };
// The backward keeps only the extra-gradient vector of a row in registers.
template <int NV> struct NormRowsBwd { static constexpr int value = NV == 1 ? 4 : (NV == 2 ? 2 : 1); };

// Batch/row split of a flat row index; 32-bit division whenever it fits.
__device__ __forceinline__ void split_row(int64_t r, int64_t rpb, bool small, int64_t& bb, int64_t& ii) {
  if (small) {
    const uint32_t q = uint32_t(r) / uint32_t(rpb);
    bb = q;
    ii = r - int64_t(q) * rpb;
  } else {
    bb = r / rpb;
    ii = r - bb * rpb;
  }
}

template <int N>
__device__ __forceinline__ void warp_sum_n(float (&v)[N]) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] += __shfl_xor_sync(0xffffffffu, v[j], o);
}

__device__ __forceinline__ void load_f8(const float* p, float* f) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

// Per-lane weight columns: held in registers (HOLD) or re-read through L1.
template <int NV, bool HOLD>
struct LaneCols {
  float v[HOLD ? NV : 1][8];
  __device__ __forceinline__ void init(const float* p, int lane, int nvec) {
    if (HOLD) {
#pragma unroll
      for (int k = 0; k < NV; ++k) {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[k][e] = 0.f;
        if (lane + 32 * k < nvec) load_f8(p + 8 * (lane + 32 * k), v[k]);
      }
    }
  }
  __device__ __forceinline__ void get(const float* p, int k, int c, float* f) const {
    if (HOLD) {
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = v[HOLD ? k : 0][e];
    } else {
      load_f8(p + 8 * c, f);
    }
  }
};

// kind: 0 = RMSNorm (weight only), 1 = LayerNorm (weight + bias)
template <int KIND, int NV>
__global__ void __launch_bounds__(256) norm_fwd_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ res,
    const float* __restrict__ w, const float* __restrict__ b, __nv_bfloat16* __restrict__ y,
    __nv_bfloat16* __restrict__ z, float* __restrict__ stat_rstd, float* __restrict__ stat_mean,
    int64_t rows, int D, float eps, int64_t rpb, int64_t x_bstride, int64_t r_bstride) {
  constexpr int RPW = NormRows<NV>::value;
  constexpr bool HOLD = NV <= 2;
  const int lane = threadIdx.x & 31;
  const int nvec = D >> 3;
  const bool small = rows < (int64_t(1) << 32);
  LaneCols<NV, HOLD> wc, bc;
  wc.init(w, lane, nvec);
  if (KIND == 1) bc.init(b, lane, nvec);
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t r0 = warp * RPW; r0 < rows; r0 += nw * RPW) {
    Vec8 xv[RPW][NV], rv[RPW][NV];
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
      const int64_t r = r0 + j;
      if (r < rows) {
        int64_t bb, ii;
        split_row(r, rpb, small, bb, ii);
        const Vec8* xr = reinterpret_cast<const Vec8*>(x + bb * x_bstride + ii * D);
        const Vec8* rr = res ? reinterpret_cast<const Vec8*>(res + bb * r_bstride + ii * D) : nullptr;
#pragma unroll
        for (int k = 0; k < NV; ++k) {
          const int c = lane + 32 * k;
          if (c < nvec) {
            xv[j][k] = xr[c];
            if (rr) rv[j][k] = rr[c];
          }
        }
      }
    }
    // pass 1: residual sum (exact in bf16 after rounding, so it replaces xv) and the row sums
    float s[RPW];
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
      const int64_t r = r0 + j;
      s[j] = 0.f;
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int c = lane + 32 * k;
        if (c < nvec && r < rows) {
          float f[8];
          unpack8(xv[j][k], f);
          if (res) {
            float t[8];
            unpack8(rv[j][k], t);
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = f[e] + t[e];
            xv[j][k] = pack8(f);
            unpack8(xv[j][k], f);
            reinterpret_cast<Vec8*>(z + r * D)[c] = xv[j][k];
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) s[j] += (KIND == 0) ? f[e] * f[e] : f[e];
        }
      }
    }
    warp_sum_n(s);
    float mean[RPW], rstd[RPW];
    if (KIND == 0) {
#pragma unroll
      for (int j = 0; j < RPW; ++j) { mean[j] = 0.f; rstd[j] = rsqrtf(s[j] / D + eps); }
    } else {
      float q[RPW];
#pragma unroll
      for (int j = 0; j < RPW; ++j) {
        mean[j] = s[j] / D;
        q[j] = 0.f;
#pragma unroll
        for (int k = 0; k < NV; ++k)
          if (lane + 32 * k < nvec && r0 + j < rows) {
            float f[8];
            unpack8(xv[j][k], f);
#pragma unroll
            for (int e = 0; e < 8; ++e) { const float d = f[e] - mean[j]; q[j] += d * d; }
          }
      }
      warp_sum_n(q);
#pragma unroll
      for (int j = 0; j < RPW; ++j) rstd[j] = rsqrtf(q[j] / D + eps);
    }
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
      const int64_t r = r0 + j;
      if (r >= rows) continue;
      if (lane == 0) { stat_rstd[r] = rstd[j]; if (KIND == 1) stat_mean[r] = mean[j]; }
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int c = lane + 32 * k;
        if (c < nvec) {
          float f[8], wk[8], bk[8], o[8];
          unpack8(xv[j][k], f);
          wc.get(w, k, c, wk);
          if (KIND == 1) bc.get(b, k, c, bk);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if (KIND == 0) o[e] = rbf(f[e] * rstd[j]) * wk[e];
            else o[e] = (f[e] - mean[j]) * rstd[j] * wk[e] + bk[e];
          }
          reinterpret_cast<Vec8*>(y + r * D)[c] = pack8(o);
        }
      }
    }
  }
}

// Backward. dy: grad of y; dz_extra (optional): grad arriving directly at the
// normalised input (the residual path), added to dx.  dz_extra may cover only
// the last (ex_rpb - ex_off) of every ex_rpb rows -- the tail of each sample
// that a pre-norm block carries on as its residual -- so the slice's gradient
// is added here instead of through a zero-filled full-size copy.  Writes dx
// (bf16) and accumulates dw/db.
//
// Pass 1 reads x and dy of RPW rows (all loads issued first, through L1) for
// the two row sums; pass 2 reads them again -- L1 hits -- so only the
// extra-gradient vectors stay in registers across the reductions.
template <int KIND, int NV>
__global__ void __launch_bounds__(256, 2) norm_bwd_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ dy,
    const __nv_bfloat16* __restrict__ dz_extra, const float* __restrict__ w,
    const float* __restrict__ stat_rstd, const float* __restrict__ stat_mean,
    __nv_bfloat16* __restrict__ dx, float* __restrict__ dw, float* __restrict__ db,
    int64_t rows, int D, int64_t ex_rpb, int64_t ex_off) {
  constexpr int RPW = NormRowsBwd<NV>::value;
  constexpr bool HOLD = NV <= 2;
  extern __shared__ float sm[];  // [2 * D]: dw, db partials
  for (int i = threadIdx.x; i < 2 * D; i += blockDim.x) sm[i] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int nvec = D >> 3;
  const bool small = rows < (int64_t(1) << 32);
  LaneCols<NV, HOLD> wc;
  wc.init(w, lane, nvec);
  float pw[HOLD ? NV : 1][8], pb[HOLD ? NV : 1][8];
#pragma unroll
  for (int k = 0; k < (HOLD ? NV : 1); ++k)
#pragma unroll
    for (int e = 0; e < 8; ++e) { pw[k][e] = 0.f; pb[k][e] = 0.f; }
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t r0 = warp * RPW; r0 < rows; r0 += nw * RPW) {
    Vec8 ev[RPW][NV];
    float rstd[RPW], mean[RPW], s1[RPW], s2[RPW];
    bool has_ex[RPW];
    // pass 1: issue every load of the group, then the row sums and the column partials
    {
      Vec8 xv[RPW][NV], dv[RPW][NV];
#pragma unroll
      for (int j = 0; j < RPW; ++j) {
        const int64_t r = r0 + j;
        rstd[j] = 0.f;
        mean[j] = 0.f;
        has_ex[j] = false;
        if (r < rows) {
          rstd[j] = __ldg(stat_rstd + r);
          if (KIND == 1) mean[j] = __ldg(stat_mean + r);
          const Vec8* er = nullptr;
          if (dz_extra) {
            int64_t bb, ii;
            split_row(r, ex_rpb, small, bb, ii);
            if (ii >= ex_off) er = reinterpret_cast<const Vec8*>(dz_extra + (bb * (ex_rpb - ex_off) + ii - ex_off) * D);
          }
          has_ex[j] = er != nullptr;
#pragma unroll
          for (int k = 0; k < NV; ++k) {
            const int c = lane + 32 * k;
            if (c < nvec) {
              xv[j][k] = as_vec8(__ldg(reinterpret_cast<const uint4*>(x + r * D) + c));
              dv[j][k] = as_vec8(__ldg(reinterpret_cast<const uint4*>(dy + r * D) + c));
              if (er) ev[j][k] = as_vec8(__ldcs(reinterpret_cast<const uint4*>(er) + c));
            }
          }
        }
      }
#pragma unroll
      for (int j = 0; j < RPW; ++j) {
        s1[j] = 0.f;
        s2[j] = 0.f;
        if (r0 + j >= rows) continue;
#pragma unroll
        for (int k = 0; k < NV; ++k) {
          const int c = lane + 32 * k;
          if (c < nvec) {
            float xf[8], df[8], wk[8];
            unpack8(xv[j][k], xf);
            unpack8(dv[j][k], df);
            wc.get(w, k, c, wk);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float xh = (xf[e] - mean[j]) * rstd[j];
              const float g = df[e] * wk[e];
              s1[j] += g * xh;
              s2[j] += g;
              if (HOLD) {
                pw[HOLD ? k : 0][e] += df[e] * xh;
                pb[HOLD ? k : 0][e] += df[e];
              } else {
                atomicAdd(&sm[8 * c + e], df[e] * xh);
                if (KIND == 1) atomicAdd(&sm[D + 8 * c + e], df[e]);
              }
            }
          }
        }
      }
    }
    warp_sum_n(s1);
    warp_sum_n(s2);
    // pass 2: x and dy again (L1), dx out
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
      const int64_t r = r0 + j;
      if (r >= rows) continue;
      const float m1 = s1[j] / D, m2 = s2[j] / D;
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int c = lane + 32 * k;
        if (c < nvec) {
          float xf[8], df[8], wk[8], ex[8], o[8];
          const uint4 xr = __ldg(reinterpret_cast<const uint4*>(x + r * D) + c);
          const uint4 dr = __ldg(reinterpret_cast<const uint4*>(dy + r * D) + c);
          unpack8(as_vec8(xr), xf);
          unpack8(as_vec8(dr), df);
          wc.get(w, k, c, wk);
          if (has_ex[j]) unpack8(ev[j][k], ex);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float xh = (xf[e] - mean[j]) * rstd[j];
            const float g = df[e] * wk[e];
            const float d = (KIND == 0) ? rstd[j] * (g - xh * m1) : rstd[j] * (g - m2 - xh * m1);
            o[e] = has_ex[j] ? d + ex[e] : d;
          }
          reinterpret_cast<Vec8*>(dx + r * D)[c] = pack8(o);
        }
      }
    }
  }
  if (HOLD) {
#pragma unroll
    for (int k = 0; k < (HOLD ? NV : 1); ++k) {
      const int c = lane + 32 * k;
      if (c < nvec)
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          atomicAdd(&sm[8 * c + e], pw[k][e]);
          if (KIND == 1) atomicAdd(&sm[D + 8 * c + e], pb[k][e]);
        }
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

// One full wave of 256-thread blocks of a grid-stride kernel (every SM at its
// register / shared-memory occupancy).
template <typename Kern>
static int64_t resident_grid(Kern kernel, size_t smem) {
  int per_sm = 0;
  PD_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 256, smem));
  return int64_t(num_sms()) * std::max(per_sm, 1);
}

// fp32 weight / bias: read as float4 pairs.
static void check_param(const at::Tensor& t, int64_t D) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat && t.is_contiguous() && t.numel() == D &&
                  reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
              "norm weight / bias must be contiguous 16-byte aligned fp32 CUDA tensors of the row size");
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
  check_param(w, D);
  if (kind == 1) check_param(*b, D);
  const int64_t rows = x3.size(0) * x3.size(1);
  const int64_t rpb = x3.size(1) > 0 ? x3.size(1) : 1;
  auto y = at::empty(x.sizes(), x.options());
  at::Tensor z = res ? at::empty(x.sizes(), x.options()) : at::Tensor();
  auto rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  at::Tensor mean = kind == 1 ? at::empty({rows}, x.options().dtype(at::kFloat)) : at::Tensor();
  if (rows == 0) return {y, z, rstd, mean};
  const int64_t want = (rows + 32 - 1) / 32;   // 8 warps x 4 rows at D <= 256
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x3.data_ptr());
  auto rp = res ? reinterpret_cast<const __nv_bfloat16*>(r3.data_ptr()) : nullptr;
  const int64_t xbs = x3.stride(0), rbs = res ? r3.stride(0) : 0;
  auto yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  auto zp = res ? reinterpret_cast<__nv_bfloat16*>(z.data_ptr()) : nullptr;
  const float* bp = kind == 1 ? b->data_ptr<float>() : nullptr;
  float* mp = kind == 1 ? mean.data_ptr<float>() : nullptr;
  const int nv = int((D / 8 + 31) / 32);
#define PD_NF(K, NVv) do { static const int64_t cap_ = resident_grid(norm_fwd_kernel<K, NVv>, 0); \
    norm_fwd_kernel<K, NVv><<<std::min(want, cap_), 256, 0, stream()>>>(xp, rp, w.data_ptr<float>(), bp, yp, zp, \
                                                   rstd.data_ptr<float>(), mp, rows, int(D), float(eps), rpb, xbs, rbs); } while (0)
#define PD_NF_K(K) if (nv <= 1) PD_NF(K, 1); else if (nv <= 2) PD_NF(K, 2); else if (nv <= 4) PD_NF(K, 4); else PD_NF(K, 8)
  if (kind == 0) { PD_NF_K(0); } else { PD_NF_K(1); }
#undef PD_NF_K
#undef PD_NF
  PD_CHECK_LAUNCH();
  return {y, z, rstd, mean};
}

// Returns {dx, dw, db_or_empty}. xin is the normalised input (z when fused).
// dz_extra: same shape as xin, or (ex_off > 0) [B, T - ex_off, D] for a
// [B, T, D] xin -- the gradient of the last T - ex_off rows of every sample.
std::vector<at::Tensor> norm_bwd(at::Tensor xin, at::Tensor dy, c10::optional<at::Tensor> dz_extra,
                                 at::Tensor w, at::Tensor rstd, c10::optional<at::Tensor> mean,
                                 int64_t kind, int64_t ex_off) {
  const int64_t D = xin.size(-1);
  check_rows(xin, D);
  auto dyc = dy.contiguous();
  check_rows(dyc, D);
  TORCH_CHECK(dyc.numel() == xin.numel(), "norm_bwd: dy must match the input");
  const int64_t rows = xin.numel() / D;
  at::Tensor ex;
  int64_t ex_rpb = rows > 0 ? rows : 1;
  if (dz_extra) {
    ex = dz_extra->contiguous();
    check_rows(ex, D);
    if (ex_off > 0) {
      TORCH_CHECK(xin.dim() == 3 && ex.dim() == 3 && ex.size(0) == xin.size(0) &&
                      ex.size(1) == xin.size(1) - ex_off && ex_off < xin.size(1),
                  "norm_bwd: a tail gradient must be [B, T - ex_off, D] for a [B, T, D] input");
      ex_rpb = xin.size(1);
    } else {
      TORCH_CHECK(ex_off == 0 && ex.numel() == xin.numel(), "norm_bwd: dz_extra must match the input");
    }
  }
  check_param(w, D);
  auto dx = at::empty_like(xin);
  auto dw = at::zeros({D}, w.options());
  at::Tensor db = kind == 1 ? at::zeros({D}, w.options()) : at::Tensor();
  if (rows == 0) return {dx, dw, db};
  const int64_t want = (rows + 32 - 1) / 32;   // 8 warps x 4 rows at D <= 256
  const size_t smem = 2 * D * sizeof(float);
  auto xp = reinterpret_cast<const __nv_bfloat16*>(xin.data_ptr());
  auto dyp = reinterpret_cast<const __nv_bfloat16*>(dyc.data_ptr());
  auto exp_ = ex.defined() ? reinterpret_cast<const __nv_bfloat16*>(ex.data_ptr()) : nullptr;
  auto dxp = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
  const float* mp = kind == 1 ? mean->data_ptr<float>() : nullptr;
  float* dbp = kind == 1 ? db.data_ptr<float>() : nullptr;
  const int nv = int((D / 8 + 31) / 32);
#define PD_NB(K, NVv) do { static const int64_t cap_ = resident_grid(norm_bwd_kernel<K, NVv>, 2 * 2048 * 4); \
    norm_bwd_kernel<K, NVv><<<std::min(want, cap_), 256, smem, stream()>>>(xp, dyp, exp_, w.data_ptr<float>(), \
                                                   rstd.data_ptr<float>(), mp, dxp, dw.data_ptr<float>(), dbp, rows, int(D), \
                                                   ex_rpb, ex.defined() ? ex_off : 0); } while (0)
#define PD_NB_K(K) if (nv <= 1) PD_NB(K, 1); else if (nv <= 2) PD_NB(K, 2); else if (nv <= 4) PD_NB(K, 4); else PD_NB(K, 8)
  if (kind == 0) { PD_NB_K(0); } else { PD_NB_K(1); }
#undef PD_NB_K
#undef PD_NB
  PD_CHECK_LAUNCH();
  return {dx, dw, db};
}

}  // namespace pd
