// Fused multi-task heads + losses (BCE-with-logits / MSE), forward and backward.
//
// Replaces, in one launch each way, the per-task Linear(D, 1) heads of
// primus_dlrm/models/onetrans.py:368-371,608 (and dlrm.py heads) and the
// weighted MultiTaskLoss of primus_dlrm/training/losses.py:13-50:
//   logit[t, b] = <h[b], W[t]> + bias[t]
//   loss_t      = mean_b BCE(logit, y) | mean_b (logit - y)^2
//   total       = sum_t weight_t * loss_t
// The forward also stores dtotal/dlogit (for an upstream grad of 1), so the
// backward is a single pass: dh = g * dlogit^T W, dW = g * dlogit h, db = g * sum dlogit,
// with g read from device memory (no host sync).
#include "common.cuh"

namespace pd {

constexpr int kMaxTasks = 16;

struct HeadParams {
  int n_tasks;
  float weight[kMaxTasks];
  int regression[kMaxTasks];
};

// One warp per sample; lanes split D.
__global__ void __launch_bounds__(256) heads_loss_fwd_kernel(
    const __nv_bfloat16* __restrict__ h, const float* __restrict__ W, const float* __restrict__ bias,
    const float* __restrict__ labels /*[T, ldl]*/, int64_t ldl, HeadParams hp, int64_t B, int D,
    float* __restrict__ logits /*[T, B]*/, float* __restrict__ dlogit /*[T, B]*/,
    float* __restrict__ out /*[1 + T]: total, per-task*/) {
  __shared__ float part[kMaxTasks];
  if (threadIdx.x < kMaxTasks) part[threadIdx.x] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const float invB = 1.f / float(B);
  for (int64_t b = warp; b < B; b += nw) {
    const __nv_bfloat16* hr = h + b * D;
    for (int t = 0; t < hp.n_tasks; ++t) {
      float s = 0.f;
      for (int d = lane; d < D; d += 32) s += __bfloat162float(hr[d]) * W[t * D + d];
      s = warp_sum(s) + bias[t];
      if (lane == 0) {
        const float y = labels[t * ldl + b];
        float l, g;
        if (hp.regression[t]) {
          const float e = s - y;
          l = e * e;
          g = 2.f * e;
        } else {
          // BCE with logits, stable form: max(x,0) - x*y + log(1 + exp(-|x|))
          l = fmaxf(s, 0.f) - s * y + log1pf(__expf(-fabsf(s)));
          g = 1.f / (1.f + __expf(-s)) - y;
        }
        logits[t * B + b] = s;
        dlogit[t * B + b] = g * invB * hp.weight[t];
        atomicAdd(&part[t], l);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x < hp.n_tasks) {
    const float lt = part[threadIdx.x] * invB;
    atomicAdd(out + 1 + threadIdx.x, lt);
    atomicAdd(out, lt * hp.weight[threadIdx.x]);
  }
}

// Backward: dh [B, D] bf16; dW [T, D] fp32 (+=); db [T] fp32 (+=). g = *gscale.
__global__ void __launch_bounds__(256) heads_loss_bwd_kernel(
    const __nv_bfloat16* __restrict__ h, const float* __restrict__ W, const float* __restrict__ dlogit,
    const float* __restrict__ gscale, int T, int64_t B, int D, __nv_bfloat16* __restrict__ dh,
    float* __restrict__ dW, float* __restrict__ db) {
  extern __shared__ float sm[];  // [T * D + T]
  for (int i = threadIdx.x; i < T * D + T; i += blockDim.x) sm[i] = 0.f;
  __syncthreads();
  const float g = *gscale;
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t b = warp; b < B; b += nw) {
    float dl[kMaxTasks];
    for (int t = 0; t < T; ++t) dl[t] = dlogit[t * B + b] * g;
    if (lane < T) atomicAdd(&sm[T * D + lane], dl[lane]);
    for (int d = lane; d < D; d += 32) {
      const float hv = __bfloat162float(h[b * D + d]);
      float acc = 0.f;
      for (int t = 0; t < T; ++t) {
        acc += dl[t] * W[t * D + d];
        atomicAdd(&sm[t * D + d], dl[t] * hv);
      }
      dh[b * D + d] = __float2bfloat16_rn(acc);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < T * D; i += blockDim.x) atomicAdd(dW + i, sm[i]);
  for (int i = threadIdx.x; i < T; i += blockDim.x) atomicAdd(db + i, sm[T * D + i]);
}

// Returns {out [1+T] (total, per-task), logits [T, B], dlogit [T, B]}
std::vector<at::Tensor> heads_loss_fwd(at::Tensor h, at::Tensor W, at::Tensor bias, at::Tensor labels,
                                       std::vector<double> task_weight, std::vector<int64_t> regression) {
  TORCH_CHECK(h.is_cuda() && h.scalar_type() == at::kBFloat16 && h.dim() == 2 && h.is_contiguous());
  const int64_t B = h.size(0);
  const int D = int(h.size(1));
  const int T = int(W.size(0));
  TORCH_CHECK(T >= 1 && T <= kMaxTasks, "1..16 tasks supported");
  TORCH_CHECK(W.scalar_type() == at::kFloat && W.is_contiguous() && W.size(1) == D);
  TORCH_CHECK(labels.scalar_type() == at::kFloat && labels.dim() == 2 && labels.size(0) == T &&
              labels.size(1) == B && labels.stride(1) == 1);
  HeadParams hp;
  hp.n_tasks = T;
  for (int t = 0; t < T; ++t) { hp.weight[t] = float(task_weight[t]); hp.regression[t] = int(regression[t]); }
  auto out = at::zeros({1 + T}, h.options().dtype(at::kFloat));
  auto logits = at::empty({T, B}, h.options().dtype(at::kFloat));
  auto dlogit = at::empty({T, B}, h.options().dtype(at::kFloat));
  int64_t blocks = (B + 7) / 8;
  const int64_t cap = int64_t(num_sms()) * 4;
  if (blocks > cap) blocks = cap;
  heads_loss_fwd_kernel<<<blocks, 256, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(h.data_ptr()), W.data_ptr<float>(), bias.data_ptr<float>(),
      labels.data_ptr<float>(), labels.stride(0), hp, B, D, logits.data_ptr<float>(), dlogit.data_ptr<float>(),
      out.data_ptr<float>());
  PD_CHECK_LAUNCH();
  return {out, logits, dlogit};
}

// Returns {dh, dW, db}
std::vector<at::Tensor> heads_loss_bwd(at::Tensor h, at::Tensor W, at::Tensor dlogit, at::Tensor gscale) {
  const int64_t B = h.size(0);
  const int D = int(h.size(1));
  const int T = int(W.size(0));
  auto dh = at::empty_like(h);
  auto dW = at::zeros_like(W);
  auto db = at::zeros({T}, W.options());
  auto g = gscale.to(at::kFloat).contiguous();
  int64_t blocks = (B + 7) / 8;
  const int64_t cap = int64_t(num_sms()) * 2;
  if (blocks > cap) blocks = cap;
  const size_t smem = size_t(T * D + T) * sizeof(float);
  TORCH_CHECK(smem <= 200 * 1024, "heads too wide for the fused backward");
  if (smem > 48 * 1024)
    PD_CHECK_CUDA(cudaFuncSetAttribute(heads_loss_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  heads_loss_bwd_kernel<<<blocks, 256, smem, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(h.data_ptr()), W.data_ptr<float>(), dlogit.data_ptr<float>(),
      g.data_ptr<float>(), T, B, D, reinterpret_cast<__nv_bfloat16*>(dh.data_ptr()), dW.data_ptr<float>(),
      db.data_ptr<float>());
  PD_CHECK_LAUNCH();
  return {dh, dW, db};
}

}  // namespace pd
