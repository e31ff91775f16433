// Dense optimizer: global-norm gradient clipping fused with AdamW over the
// flat fp32 parameter / gradient arena (one launch for the norm, one for the
// update; the clip coefficient is read on the device, so no host sync).
//
// Semantics follow torch.nn.utils.clip_grad_norm_ + torch.optim.AdamW used by
// primus_dlrm/training/dist_trainer.py:233,451-454:
//   coef = min(1, max_norm / (||g||_2 + 1e-6))
//   p   *= 1 - lr * wd
//   m    = b1 m + (1 - b1) g ;  v = b2 v + (1 - b2) g^2
//   p   -= (lr / bc1) * m / (sqrt(v) / sqrt(bc2) + eps)
#include "common.cuh"

namespace pd {

__global__ void __launch_bounds__(256) sqnorm_kernel(const float* __restrict__ g, int64_t n,
                                                     float* __restrict__ out) {
  float s = 0.f;
  const int64_t n4 = n >> 2;
  const float4* g4 = reinterpret_cast<const float4*>(g);
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += int64_t(gridDim.x) * blockDim.x) {
    const float4 v = g4[i];
    s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (int64_t i = 4 * n4 + int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    s += g[i] * g[i];
  s = warp_sum(s);
  __shared__ float ws[8];
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? ws[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) atomicAdd(out, t);
  }
}

__global__ void __launch_bounds__(256) adamw_kernel(float* __restrict__ p, const float* __restrict__ g,
                                                    float* __restrict__ m, float* __restrict__ v, int64_t n,
                                                    float lr, float b1, float b2, float eps, float wd,
                                                    float bc1, float bc2, float max_norm,
                                                    const float* __restrict__ sqnorm) {
  float coef = 1.f;
  if (max_norm > 0.f && sqnorm != nullptr) coef = fminf(1.f, max_norm / (sqrtf(*sqnorm) + 1e-6f));
  const float step = lr / bc1;
  const float isb2 = rsqrtf(bc2);
  const float decay = 1.f - lr * wd;
  const int64_t n4 = n >> 2;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += int64_t(gridDim.x) * blockDim.x) {
    float4 pv = reinterpret_cast<float4*>(p)[i];
    float4 gv = reinterpret_cast<const float4*>(g)[i];
    float4 mv = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float* pp = reinterpret_cast<float*>(&pv);
    float* gp = reinterpret_cast<float*>(&gv);
    float* mp = reinterpret_cast<float*>(&mv);
    float* vp = reinterpret_cast<float*>(&vv);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float gg = gp[e] * coef;
      mp[e] = b1 * mp[e] + (1.f - b1) * gg;
      vp[e] = b2 * vp[e] + (1.f - b2) * gg * gg;
      pp[e] = pp[e] * decay - step * mp[e] / (sqrtf(vp[e]) * isb2 + eps);
    }
    reinterpret_cast<float4*>(p)[i] = pv;
    reinterpret_cast<float4*>(m)[i] = mv;
    reinterpret_cast<float4*>(v)[i] = vv;
  }
  for (int64_t i = 4 * n4 + int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const float gg = g[i] * coef;
    m[i] = b1 * m[i] + (1.f - b1) * gg;
    v[i] = b2 * v[i] + (1.f - b2) * gg * gg;
    p[i] = p[i] * decay - step * m[i] / (sqrtf(v[i]) * isb2 + eps);
  }
}

// Scale a flat buffer in place by s / *denom (used for grad averaging).
__global__ void scale_kernel(float* __restrict__ x, int64_t n, float s) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    x[i] *= s;
}

static int64_t ew_blocks(int64_t n) {
  int64_t b = (n / 4 + 255) / 256;
  const int64_t cap = int64_t(num_sms()) * 8;
  if (b > cap) b = cap;
  return b < 1 ? 1 : b;
}

void grad_sqnorm(at::Tensor g, at::Tensor out) {
  TORCH_CHECK(g.is_cuda() && g.scalar_type() == at::kFloat && g.is_contiguous());
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.numel() >= 1);
  TORCH_CHECK(reinterpret_cast<uintptr_t>(g.data_ptr()) % 16 == 0);
  sqnorm_kernel<<<ew_blocks(g.numel()), 256, 0, stream()>>>(g.data_ptr<float>(), g.numel(), out.data_ptr<float>());
  PD_CHECK_LAUNCH();
}

void adamw_step(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v, double lr, double b1, double b2,
                double eps, double wd, double bc1, double bc2, double max_norm,
                c10::optional<at::Tensor> sqnorm) {
  for (auto* t : {&p, &g, &m, &v}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous());
    TORCH_CHECK(t->numel() == p.numel());
    TORCH_CHECK(reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0);
  }
  adamw_kernel<<<ew_blocks(p.numel()), 256, 0, stream()>>>(
      p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), p.numel(), float(lr),
      float(b1), float(b2), float(eps), float(wd), float(bc1), float(bc2), float(max_norm),
      sqnorm ? sqnorm->data_ptr<float>() : nullptr);
  PD_CHECK_LAUNCH();
}

void scale_(at::Tensor x, double s) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat && x.is_contiguous());
  scale_kernel<<<ew_blocks(x.numel() * 4), 256, 0, stream()>>>(x.data_ptr<float>(), x.numel(), float(s));
  PD_CHECK_LAUNCH();
}

long long launches() { return launch_counter().load(); }

}  // namespace pd
