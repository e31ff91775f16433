// tcgen05.mma throughput probe (sm_100a): cycles per instruction for the
// operand shapes and layouts the attention and GEMM kernels issue.
//
// One CTA per SM. Thread 0 issues `iters` back-to-back
//   tcgen05.mma.cta_group::1.kind::f16  (M = 128, N = n, K = 16, bf16 -> fp32)
// rotating over `nacc` accumulators, commits them to an mbarrier and waits;
// clock64() before the first issue, after the last issue and after the
// commit completes gives the issue time and the execution time. Operand
// values are a fixed hash pattern (their values do not change the timing).
//
// Modes: 0 = SS, A and B K-major; 1 = SS, A K-major, B MN-major;
//        2 = SS, A MN-major, B MN-major; 3 = TS (A from TMEM), B K-major;
//        4 = TS, B MN-major.
// swz: 2 = 128-byte swizzle, 4 = 64-byte swizzle (the row width of a
// d = 32 bf16 tile), applied to both shared-memory operands.
#include "common.cuh"

namespace pd {
namespace mrate {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t make_desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint64_t swz) {
  return uint64_t((addr >> 4) & 0x3FFF) | (uint64_t((lbo >> 4) & 0x3FFF) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFF) << 32) | (uint64_t(1) << 46) | (swz << 61);
}
__host__ __device__ constexpr uint32_t idesc(int m, int n, int a_mn, int b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(a_mn) << 15) | (uint32_t(b_mn) << 16) |
         (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

constexpr int kSmemBytes = 160 * 1024;  // A region 64 KB + B region 64 KB (+ alignment); forces one CTA per SM
constexpr uint64_t kWaitLimitNs = 1000000000ull;

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 rx;\n\t.reg .pred px;\n\t"
      "elect.sync rx|px, %1;\n\t"
      "selp.b32 %0, 1, 0, px;\n\t}"
      : "=r"(pred) : "r"(0xffffffffu));
  return pred != 0;
}

// issue: 0 = lane 0 alone runs the issue loop (the rest of its warp waits at
// the CTA barrier); 1 = the whole warp runs the loop and elect.sync picks the
// issuing lane for each instruction; 2 = as 1 with the disable-output-lane
// operand form of the instruction.
__global__ void __launch_bounds__(128, 1) mma_rate_kernel(int mode, int n, int iters, int nacc, int swz, int issue,
                                                          long long* out, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + 65536;
  __shared__ uint64_t done;
  __shared__ uint32_t tmem_slot;
  // operand pattern: bf16 values in [-1, 1) from a multiplicative hash
  for (int i = threadIdx.x; i < 65536; i += blockDim.x) {
    const uint32_t h = uint32_t(i) * 2654435761u + blockIdx.x;
    const float v = float(h >> 8) * (1.0f / 8388608.0f) - 1.0f;
    reinterpret_cast<__nv_bfloat16*>(smem)[i] = __float2bfloat16(v);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&done)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&tmem_slot))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_slot;
  if ((issue == 0 && threadIdx.x == 0) || (issue != 0 && warp == 0)) {
    const int a_mn = (mode == 2) ? 1 : 0;
    const int b_mn = (mode == 1 || mode == 2 || mode == 4) ? 1 : 0;
    const bool ts = (mode >= 3);
    const uint32_t id = idesc(128, n, a_mn, b_mn);
    const uint32_t row_b = (swz == 2) ? 128u : 64u;     // bytes per swizzle row
    const uint32_t atom = 8u * row_b;                   // one 8-row swizzle atom
    // K-major: 8-row groups of the M / N extent `atom` bytes apart; k-step at +32 B.
    // MN-major: one k-step = two 8-row atoms along K; atoms along M / N 16 * row_b * 2 apart.
    const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
    const uint64_t da_k = make_desc(a0, 16u, atom, uint64_t(swz));
    const uint64_t da_mn = make_desc(a0, 4u * atom, atom, uint64_t(swz));
    const uint64_t db_k = make_desc(b0, 16u, atom, uint64_t(swz));
    const uint64_t db_mn = make_desc(b0, 4u * atom, atom, uint64_t(swz));
    const uint64_t da = a_mn ? da_mn : da_k;
    const uint64_t db = b_mn ? db_mn : db_k;
    const uint32_t a_tmem = tmem + 448u;                // A (TS): 8 columns of packed bf16 pairs
    __syncwarp(issue == 0 ? 1u : 0xffffffffu);
    const long long t0 = clock64();
    const uint32_t z = 0u;
    for (int i = 0; i < iters; ++i) {
      const uint32_t d = tmem + uint32_t((i % nacc) * n);
      const uint32_t acc = (i >= nacc) ? 1u : 0u;
      if (issue != 0 && !elect_one()) continue;
      if (issue == 2) {
        if (ts)
          asm volatile(
              "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
              "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}"
              ::"r"(d), "r"(a_tmem), "l"(db), "r"(id), "r"(acc), "r"(z) : "memory");
        else
          asm volatile(
              "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
              "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
              ::"r"(d), "l"(da), "l"(db), "r"(id), "r"(acc), "r"(z) : "memory");
      } else if (ts) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
            ::"r"(d), "r"(a_tmem), "l"(db), "r"(id), "r"(acc) : "memory");
      } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
            ::"r"(d), "l"(da), "l"(db), "r"(id), "r"(acc) : "memory");
      }
    }
    __syncwarp(issue == 0 ? 1u : 0xffffffffu);
    const long long t1 = clock64();
    if (issue == 0 || elect_one()) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(&done))
                 : "memory");
    const uint64_t g0 = globaltimer_ns();
    uint32_t ok = 0;
    while (!ok) {
      asm volatile(
          "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\tselp.b32 %0, 1, 0, p;\n\t}"
          : "=r"(ok) : "r"(smem_u32(&done)) : "memory");
      if (!ok && globaltimer_ns() - g0 > kWaitLimitNs) {
        set_error(err, kWaitTimeout);
        break;
      }
    }
    const long long t2 = clock64();
    out[2 * blockIdx.x] = t1 - t0;
    out[2 * blockIdx.x + 1] = t2 - t0;
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
  }
}

// Unrolled variant: N is a compile-time constant and the body issues 16 MMAs
// in straight-line code (no per-instruction index arithmetic). `issuers`
// warps of the CTA (1 or 2) issue at the same time, each into its own
// accumulator, and the launch puts `per_sm` CTAs on each SM (1 or 2; each
// CTA then allocates 256 TMEM columns), so the tensor pipe's throughput can
// be told apart from the latency of one issuing thread.
// var: 0 identical operands every instruction; 1 the B descriptor advances one
// k-step (32 bytes) per instruction over 8 steps; 2 A advances (TS: 8 TMEM
// columns, SS: 32 bytes); 3 the accumulate flag is a run-time value; 4 the
// 16-instruction body is not unrolled; 5 = 1 + 2 + 3 (a k-loop as kernels issue it).
template <int N, int VAR>
__device__ __forceinline__ void burst_body(uint32_t d, uint32_t a_tmem, uint64_t da, uint64_t db, uint32_t id, int ts,
                                           int i) {
#pragma unroll
  for (int u = 0; u < 16; ++u) {
    const uint32_t k = uint32_t(u & 7);
    const uint64_t dbu = (VAR == 1 || VAR == 5) ? db + 2 * k : db;
    const uint64_t dau = (VAR == 2 || VAR == 5) ? da + 2 * k : da;
    const uint32_t atu = (VAR == 2 || VAR == 5) ? a_tmem + 8 * k : a_tmem;
    const uint32_t acc = (VAR == 3 || VAR == 5) ? ((i > 0 || u > 0) ? 1u : 0u) : 1u;
    if (ts)
      asm volatile(
          "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
          ::"r"(d), "r"(atu), "l"(dbu), "r"(id), "r"(acc) : "memory");
    else
      asm volatile(
          "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
          ::"r"(d), "l"(dau), "l"(dbu), "r"(id), "r"(acc) : "memory");
  }
}

template <int N>
__global__ void __launch_bounds__(512) mma_burst_kernel(int iters, int issuers, int wstride, int lanes, int ts,
                                                        int var, int tmem_cols, long long* out, int* err) {
  // (var may be rewritten below for the layout cases)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t done[4];
  __shared__ uint32_t tmem_slot;
  for (int i = threadIdx.x; i < 24576; i += blockDim.x) {
    const uint32_t h = uint32_t(i) * 2654435761u + blockIdx.x;
    reinterpret_cast<__nv_bfloat16*>(smem)[i] = __float2bfloat16(float(h >> 8) * (1.0f / 8388608.0f) - 1.0f);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int k = 0; k < 4; ++k) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&done[k])));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                 "r"(tmem_cols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_slot;
  const int me = warp / wstride;                 // issuer index of this warp
  if (warp % wstride == 0 && me < issuers && lane < lanes) {
    // var >= 10: operand layouts of the attention kernels (fixed operands):
    // 10 A K SW128 / B K SW128, 11 A K SW128 / B MN SW64, 12 A MN SW128 / B MN SW64,
    // 13 A K SW64 / B K SW64
    const int lay = var >= 10 ? var - 10 : 0;
    const uint32_t id = idesc(128, N, lay == 2 ? 1 : 0, (lay == 1 || lay == 2) ? 1 : 0);
    const uint32_t a0 = smem_u32(smem), b0 = smem_u32(smem + 16384);
    const uint64_t da = lay == 2 ? make_desc(a0, 8192u, 1024u, 2)
                      : lay == 3 ? make_desc(a0, 16u, 512u, 4) : make_desc(a0, 16u, 1024u, 2);
    const uint64_t db = (lay == 1 || lay == 2) ? make_desc(b0, 8192u, 512u, 4)
                      : lay == 3 ? make_desc(b0, 16u, 512u, 4) : make_desc(b0, 16u, 1024u, 2);
    if (var >= 10) var = 0;
    // accumulator of this issuer; TS operand A in the last 8 columns of the allocation
    const uint32_t d = tmem + uint32_t((me * lanes + lane) * (N <= 32 ? N : 0));
    const uint32_t a_tmem = tmem + uint32_t(tmem_cols - 64);
    const long long t0 = clock64();
    if (var == 4) {
      for (int i = 0; i < iters * 16; ++i) {
        if (ts)
          asm volatile(
              "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
              "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
              ::"r"(d), "r"(a_tmem), "l"(db), "r"(id), "r"(1u) : "memory");
        else
          asm volatile(
              "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
              "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
              ::"r"(d), "l"(da), "l"(db), "r"(id), "r"(1u) : "memory");
      }
    } else {
      for (int i = 0; i < iters; ++i) {
        switch (var) {
          case 1: burst_body<N, 1>(d, a_tmem, da, db, id, ts, i); break;
          case 2: burst_body<N, 2>(d, a_tmem, da, db, id, ts, i); break;
          case 3: burst_body<N, 3>(d, a_tmem, da, db, id, ts, i); break;
          case 5: burst_body<N, 5>(d, a_tmem, da, db, id, ts, i); break;
          default: burst_body<N, 0>(d, a_tmem, da, db, id, ts, i); break;
        }
      }
    }
    const long long t1 = clock64();
    if (lane == 0)
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                   ::"r"(smem_u32(&done[me])) : "memory");
    const uint64_t g0 = globaltimer_ns();
    uint32_t ok = 0;
    while (!ok) {
      asm volatile(
          "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\tselp.b32 %0, 1, 0, p;\n\t}"
          : "=r"(ok) : "r"(smem_u32(&done[me])) : "memory");
      if (!ok && globaltimer_ns() - g0 > kWaitLimitNs) {
        set_error(err, kWaitTimeout);
        break;
      }
    }
    const long long t2 = clock64();
    if (lane == 0) {
      out[8 * blockIdx.x + 2 * me] = t1 - t0;
      out[8 * blockIdx.x + 2 * me + 1] = t2 - t0;
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_cols) : "memory");
  }
}

}  // namespace mrate

// Returns int64 [grid, 2]: (issue cycles, issue + execution cycles) per CTA.
at::Tensor tc_mma_rate(int64_t mode, int64_t n, int64_t iters, int64_t nacc, int64_t swz, int64_t issue,
                       at::Tensor err) {
  TORCH_CHECK(issue >= 0 && issue <= 2, "issue in [0, 2]");
  TORCH_CHECK(mode >= 0 && mode <= 4, "mode in [0, 4]");
  TORCH_CHECK(n >= 16 && n <= 256 && n % 16 == 0, "n: a multiple of 16 in [16, 256]");
  TORCH_CHECK(nacc >= 1 && nacc * n <= 448, "nacc * n must leave TMEM columns [448, 512) for the TS operand");
  TORCH_CHECK(swz == 2 || swz == 4, "swz: 2 (128 B) or 4 (64 B)");
  TORCH_CHECK(iters >= 1 && iters <= (1 << 20), "iters in [1, 2^20]");
  TORCH_CHECK(err.is_cuda() && err.scalar_type() == at::kInt, "err: int32 CUDA tensor");
  const int grid = num_sms();
  auto out = at::zeros({grid, 2}, err.options().dtype(at::kLong));
  PD_CHECK_CUDA(cudaFuncSetAttribute(mrate::mma_rate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     mrate::kSmemBytes));
  mrate::mma_rate_kernel<<<grid, 128, mrate::kSmemBytes, stream()>>>(
      int(mode), int(n), int(iters), int(nacc), int(swz), int(issue), reinterpret_cast<long long*>(out.data_ptr()),
      err.data_ptr<int>());
  PD_CHECK_LAUNCH();
  return out;
}

// Unrolled probe: int64 [grid, 8] = per CTA, per issuing warp (issue cycles,
// issue + execution cycles) for iters x 16 MMAs of M = 128 x n x 16. The
// issuers are warps 0, wstride, 2 wstride, ... (warp w runs on sub-partition
// w % 4, so wstride 4 puts every issuer on the same one); in each, lanes
// 0 .. lanes-1 execute every tcgen05.mma (one instruction per lane).
at::Tensor tc_mma_burst(int64_t n, int64_t iters, int64_t issuers, int64_t per_sm, int64_t ts, int64_t wstride,
                        int64_t lanes, int64_t var, at::Tensor err) {
  TORCH_CHECK((var >= 0 && var <= 5) || (var >= 10 && var <= 13), "var in [0, 5] or [10, 13]");
  // A read from TMEM has no MN-major (transposed) form: that descriptor is an illegal instruction
  TORCH_CHECK(!(ts && var == 12), "an MN-major A operand needs the SS form (A in shared memory)");
  TORCH_CHECK(lanes >= 1 && lanes <= 4, "lanes in [1, 4]");
  TORCH_CHECK(n == 32 || n == 64 || n == 128 || n == 256, "n in {32, 64, 128, 256}");
  TORCH_CHECK(issuers >= 1 && issuers <= 4, "issuers in [1, 4]");
  TORCH_CHECK(wstride == 1 || wstride == 4, "wstride: 1 or 4");
  TORCH_CHECK(per_sm == 1 || per_sm == 2, "per_sm: 1 or 2");
  TORCH_CHECK(iters >= 1 && iters <= (1 << 16), "iters in [1, 2^16]");
  TORCH_CHECK(err.is_cuda() && err.scalar_type() == at::kInt, "err: int32 CUDA tensor");
  const int grid = num_sms() * int(per_sm);
  const int cols = per_sm == 1 ? 512 : 256;
  const int smem = per_sm == 1 ? 160 * 1024 : 100 * 1024;
  auto out = at::zeros({grid, 8}, err.options().dtype(at::kLong));
  auto go = [&](auto kern) {
    PD_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kern<<<grid, 512, smem, stream()>>>(int(iters), int(issuers), int(wstride), int(lanes), int(ts), int(var), cols,
                                        reinterpret_cast<long long*>(out.data_ptr()), err.data_ptr<int>());
  };
  if (n == 32) go(mrate::mma_burst_kernel<32>);
  else if (n == 64) go(mrate::mma_burst_kernel<64>);
  else if (n == 128) go(mrate::mma_burst_kernel<128>);
  else go(mrate::mma_burst_kernel<256>);
  PD_CHECK_LAUNCH();
  return out;
}

}  // namespace pd
