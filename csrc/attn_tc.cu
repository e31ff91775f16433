// Pyramid causal attention on the 5th-generation tensor cores (tcgen05 +
// TMEM + TMA) for sm_100a.
//
// Semantics (primus_dlrm/models/onetrans.py:62-67,146-166): the queries are
// the LAST q_len of the T tokens of a [B, T, 3, H, d] fused projection; query
// i (absolute position p = T - q_len + i) attends keys j <= p; scale 1/sqrt(d).
//
// Forward (fmha_fwd_tc_kernel): 128-query tiles, 64-key S tiles triple-
// buffered in TMEM with P written back over them, S issued two tiles ahead of
// the softmax; details at the kernel. Backward (fmha_bwd_tc_kernel, d = 32):
// one CTA per (b, h), one MMA-issuing warp per product stream; details at
// the kernel.
//
// Every wait is bounded (2 s on %globaltimer); on timeout the error word
// gets kWaitTimeout, the roles leave their loops, drain their own in-flight
// copies / MMAs (bounded) and the CTA frees TMEM and exits.
#include "common.cuh"
#include "driver_api.h"

#include <cuda.h>

namespace pd {
namespace atc {

constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr int kTile = 128;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
// try_wait with a suspend-time hint: a waiting warp sleeps (issuing nothing)
// until the phase completes or ~0.2 ms pass, instead of spinning and taking
// issue slots from the warps that do the work.
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(b)), "r"(parity), "r"(200000u) : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, int* err) {
  if (mbar_try(b, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try(b, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      set_error(err, kWaitTimeout);
      return false;
    }
  }
  return true;
}
// Non-blocking probe of an mbarrier phase.
__device__ __forceinline__ bool mbar_test(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(b)), "r"(parity) : "memory");
  return ok != 0;
}
// 5-D tiled TMA load into this CTA's shared memory, completing on an mbarrier.
__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6, %7}], "
      "[%2];" ::"r"(smem_u32(dst)), "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_u32(bar)) : "memory");
}
// D (tmem) (+)= A (smem desc) * B (smem desc)
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d), "l"(da), "l"(db), "r"(idesc), "r"(acc) : "memory");
}
// D (tmem) (+)= A (tmem, K-major packed bf16 pairs) * B (smem desc)
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a_tmem, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d), "r"(a_tmem), "l"(db), "r"(idesc), "r"(acc) : "memory");
}
// 32 lanes x 32 consecutive 32-bit columns: thread = lane, r[i] = column i.
__device__ __forceinline__ void tm_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tm_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// wait::ld that also names the 32 destination registers, so no use of them
// can be scheduled before the wait.
__device__ __forceinline__ void tm_ld_wait(uint32_t* r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :: "memory");
}
__device__ __forceinline__ void tm_ld_wait8(uint32_t* r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7])
               :: "memory");
}
__device__ __forceinline__ void tm_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
        "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
        "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tm_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tm_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Packed fp32 pairs (sm_100 f32x2 arithmetic: one instruction for two lanes'
// worth of FMA / add) and the three-input max.
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_split(uint64_t r, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ uint64_t fma_f2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add_f2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t sub_f2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t mul_f2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Shared-memory operand geometry for [rows][d] bf16 tiles as written by TMA
// with the d-wide swizzle: rows of 2d bytes, 8-row atoms (SWIZZLE_64B for
// d = 32, SWIZZLE_128B for d = 64).
template <int D>
struct Geo {
  static constexpr int RB = D * 2;                   // bytes per row
  static constexpr int kTileBytes = kTile * RB;      // one 128-row tile
  static constexpr uint64_t kSwz = (D == 32) ? 4 : 2;  // descriptor layout code
  static constexpr uint32_t kAtom = 8 * RB;          // bytes per 8-row atom
};
__device__ __forceinline__ uint64_t make_desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint64_t swz) {
  return uint64_t((addr >> 4) & 0x3FFF) | (uint64_t((lbo >> 4) & 0x3FFF) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFF) << 32) | (uint64_t(1) << 46) | (swz << 61);
}
// K-major operand (rows = M or N, d = K): k-step kk (16 elements) starts 32 B further.
template <int D>
__device__ __forceinline__ uint64_t desc_k(uint32_t tile, int kk) {
  return make_desc(tile + uint32_t(kk) * 32u, 16u, Geo<D>::kAtom, Geo<D>::kSwz);
}
// MN-major operand (rows = K, d = M or N, one swizzle atom wide): k-step kk
// covers rows [16 kk, 16 kk + 16), i.e. two 8-row atoms.
template <int D>
__device__ __forceinline__ uint64_t desc_mn(uint32_t tile, int kk) {
  return make_desc(tile + uint32_t(kk) * 2u * Geo<D>::kAtom, uint32_t(Geo<D>::kTileBytes), Geo<D>::kAtom,
                   Geo<D>::kSwz);
}
// kind::f16 instruction descriptor: f32 accumulate, bf16 A/B; majors per operand.
__host__ __device__ constexpr uint32_t idesc(int m, int n, int a_mn, int b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(a_mn) << 15) | (uint32_t(b_mn) << 16) |
         (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

struct FwdArgs {
  int B, H, T, q_len, nq, items;
  float c2;                 // softmax scale * log2(e)
  __nv_bfloat16* o;         // [B, q_len, H, D]
  float* lse;               // [B, H, q_len], log2 domain
  int* err;
};

constexpr int kFwdThreads = 192;
constexpr int kKT = 64;                  // keys per S tile
constexpr int kSBuf = 3;                 // S / P buffers in TMEM

// Tile enumeration shared by the roles: this CTA's items (b, h, 128-query
// tile), then the 64-key tiles the query tile sees.
struct FwdIt {
  int w, j, nkv, i0, b, h;
  __device__ void load(const FwdArgs& a) {
    const int bh = w / a.nq;
    i0 = (w - bh * a.nq) * kTile;
    b = bh / a.H;
    h = bh - b * a.H;
    const int last = min(a.T - 1, a.T - a.q_len + i0 + kTile - 1);
    nkv = last / kKT + 1;
  }
  __device__ void start(const FwdArgs& a, int wb, int we) { w = wb; j = 0; if (w < we) load(a); }
  __device__ bool last_of_item() const { return j == nkv - 1; }
  __device__ void next(const FwdArgs& a, int we) {
    if (++j < nkv) return;
    ++w; j = 0;
    if (w < we) load(a);
  }
};

// Forward: one CTA = one 128-query tile at a time (persistent over this CTA's
// contiguous item range), two CTAs per SM.
//   warp 0     TMA: the Q tile (double-buffered across items), 64-key K / V
//              tiles into a KST-deep ring
//   warp 1     TMEM owner + MMA issuer: S_t = Q K_t^T (SS) two tiles ahead of
//              the softmax, O += P_t V_t (TS: P from TMEM) as each P is ready
//   warps 2-5  softmax: thread = query row = TMEM lane; the 64-key S row is
//              read from TMEM once, its max and exponentials computed in
//              registers, and P (bf16 pairs) written back over the S columns
// TMEM (256 columns): S / P buffers [64 b, 64 b + 64) for b < 3 (P in the
// first 32 columns of its S tile), O [192, 192 + d).
// S of tile t goes to buffer t % 3; it is issued after PV(t - 2), once PV(t - 3)
// (the last reader of that buffer's P) completed. The running max is raised
// only when it grows by more than 2^8 (log2 domain), so O is rescaled rarely;
// a rescale first waits for the PV product of the previous tile.
template <int D, int KST>
__global__ void __launch_bounds__(kFwdThreads, 2) fmha_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                                                                     const __grid_constant__ CUtensorMap tm_kv,
                                                                     const FwdArgs a) {
  using G = Geo<D>;
  constexpr uint32_t kCols = 256;
  constexpr uint32_t cO = kSBuf * kKT;
  constexpr int kQBytes = kTile * G::RB;
  constexpr int kKVBytes = kKT * G::RB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                 // [2] Q tiles (next item's Q prefetched)
  uint8_t* sK = sQ + 2 * kQBytes;                     // [KST]
  uint8_t* sV = sK + KST * kKVBytes;                  // [KST]
  uint64_t* bar = reinterpret_cast<uint64_t*>(sV + KST * kKVBytes);
  uint64_t* q_full = bar;                 // [2]
  uint64_t* q_empty = bar + 2;            // [2]
  uint64_t* kv_full = bar + 4;            // [KST]
  uint64_t* kv_empty = kv_full + KST;     // [KST]
  uint64_t* s_full = kv_empty + KST;      // [3]
  uint64_t* p_full = s_full + kSBuf;      // [3]
  uint64_t* pv_done = p_full + kSBuf;     // [3]
  uint64_t* o_full = pv_done + kSBuf;
  uint64_t* o_free = o_full + 1;
  uint64_t* mma_done = o_free + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int k = 0; k < 2; ++k) { mbar_init(&q_full[k], 1); mbar_init(&q_empty[k], 1); }
    for (int k = 0; k < KST; ++k) { mbar_init(&kv_full[k], 1); mbar_init(&kv_empty[k], 1); }
    for (int k = 0; k < kSBuf; ++k) { mbar_init(&s_full[k], 1); mbar_init(&p_full[k], 128); mbar_init(&pv_done[k], 1); }
    mbar_init(o_full, 1); mbar_init(o_free, 128); mbar_init(mma_done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_q) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_kv) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(tmem_slot)), "r"(kCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int off = a.T - a.q_len;  // absolute position of query 0
  // contiguous item range per CTA: whole (b, h) groups (equal cost) and the
  // K / V tiles of a head reused from L2 by consecutive items
  const int per = (a.items + gridDim.x - 1) / gridDim.x;
  const int w_begin = blockIdx.x * per;
  const int w_end = min(a.items, w_begin + per);

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      FwdIt it;
      it.start(a, w_begin, w_end);
      int item = 0, kvc = 0;
      int issued_q[2] = {0, 0}, issued_kv[KST];
#pragma unroll
      for (int k = 0; k < KST; ++k) issued_kv[k] = 0;
      bool good = true;
      while (good && it.w < w_end && !*abort_flag) {
        if (it.j == 0) {
          const int qb = item & 1;
          if (!mbar_wait(&q_empty[qb], ((item >> 1) & 1) ^ 1, a.err)) { good = false; break; }
          mbar_expect_tx(&q_full[qb], kQBytes);
          tma_load_5d(sQ + qb * kQBytes, &tm_q, &q_full[qb], 0, it.h, 0, off + it.i0, it.b);
          ++issued_q[qb];
        }
        const int st = kvc % KST;
        if (!mbar_wait(&kv_empty[st], ((kvc / KST) & 1) ^ 1, a.err)) { good = false; break; }
        mbar_expect_tx(&kv_full[st], 2 * kKVBytes);
        tma_load_5d(sK + st * kKVBytes, &tm_kv, &kv_full[st], 0, it.h, 1, it.j * kKT, it.b);
        tma_load_5d(sV + st * kKVBytes, &tm_kv, &kv_full[st], 0, it.h, 2, it.j * kKT, it.b);
        ++issued_kv[st];
        ++kvc;
        if (it.last_of_item()) ++item;
        it.next(a, w_end);
      }
      if (!good) *abort_flag = 1;
      if (*abort_flag) {  // every issued copy lands before the CTA may exit
        for (int qb = 0; qb < 2; ++qb)
          if (issued_q[qb] > 0) (void)mbar_wait(&q_full[qb], uint32_t(issued_q[qb] - 1) & 1u, a.err);
#pragma unroll
        for (int s2 = 0; s2 < KST; ++s2)
          if (issued_kv[s2] > 0) (void)mbar_wait(&kv_full[s2], uint32_t(issued_kv[s2] - 1) & 1u, a.err);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t id_s = idesc(128, kKT, 0, 0);
      constexpr uint32_t id_pv = idesc(128, D, 0, 1);
      FwdIt si, pi;
      si.start(a, w_begin, w_end);
      pi.start(a, w_begin, w_end);
      int ts = 0, tp = 0, s_item = 0, p_item = 0;
      bool good = true;
      auto issue_s = [&]() {
        const int qb = s_item & 1;
        if (si.j == 0 && !mbar_wait(&q_full[qb], (s_item >> 1) & 1, a.err)) return false;
        const int st = ts % KST, buf = ts % kSBuf;
        if (!mbar_wait(&kv_full[st], (ts / KST) & 1, a.err)) return false;
        if (ts >= kSBuf && !mbar_wait(&pv_done[buf], uint32_t(ts / kSBuf - 1) & 1u, a.err)) return false;
        tc_fence_after();
        const uint32_t qt = smem_u32(sQ + qb * kQBytes), kt = smem_u32(sK + st * kKVBytes);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          mma_ss(tmem + uint32_t(kKT * buf), desc_k<D>(qt, kk), desc_k<D>(kt, kk), id_s, kk > 0 ? 1u : 0u);
        tc_commit(&s_full[buf]);
        if (si.last_of_item()) { tc_commit(&q_empty[qb]); ++s_item; }
        si.next(a, w_end);
        ++ts;
        return true;
      };
      auto issue_pv = [&]() {
        const int st = tp % KST, buf = tp % kSBuf;
        if (!mbar_wait(&p_full[buf], uint32_t(tp / kSBuf) & 1u, a.err)) return false;
        if (pi.j == 0 && !mbar_wait(o_free, (p_item & 1) ^ 1, a.err)) return false;
        tc_fence_after();
        const uint32_t vt = smem_u32(sV + st * kKVBytes);
#pragma unroll
        for (int kk = 0; kk < kKT / 16; ++kk)
          mma_ts(tmem + cO, tmem + uint32_t(kKT * buf + 8 * kk), desc_mn<D>(vt, kk), id_pv,
                 (pi.j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&kv_empty[st]);
        tc_commit(&pv_done[buf]);
        if (pi.last_of_item()) { tc_commit(o_full); ++p_item; }
        pi.next(a, w_end);
        ++tp;
        return true;
      };
      // S runs two tiles ahead of PV
      for (int k = 0; k < 2 && good && si.w < w_end; ++k) good = issue_s();
      while (good && pi.w < w_end && !*abort_flag) {
        good = issue_pv();
        if (good && si.w < w_end) good = issue_s();
      }
      if (!good) *abort_flag = 1;
      tc_commit(mma_done);
      (void)mbar_wait(mma_done, 0, a.err);
    }
  } else {
    // ---------------- softmax + epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;                      // row of the tile = TMEM lane
    const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
    FwdIt it;
    it.start(a, w_begin, w_end);
    int t = 0, item = 0;
    bool ok = true;
    while (ok && it.w < w_end && !*abort_flag) {
      const int p_abs = off + it.i0 + r;                    // this row's last visible key
      float m = -1e30f, l = 0.f;
      const int b = it.b, h = it.h, i0 = it.i0;
      for (;;) {
        const int buf = t % kSBuf, j = it.j;
        if (!mbar_wait(&s_full[buf], uint32_t(t / kSBuf) & 1u, a.err)) { ok = false; break; }
        tc_fence_after();
        uint32_t sr[64];
        tm_ld32(lane_base + uint32_t(kKT * buf), sr);
        tm_ld32(lane_base + uint32_t(kKT * buf + 32), sr + 32);
        tm_ld_wait();
        const int lim = p_abs - j * kKT;                    // keys c <= lim are visible
        const bool diag = __any_sync(0xffffffffu, lim < kKT - 1);   // warp-uniform masking
        if (diag) {
#pragma unroll
          for (int c = 0; c < 64; ++c) sr[c] = (c <= lim) ? sr[c] : __float_as_uint(-INFINITY);
        }
        // row max: four chains of three-input maxima
        float mxa = -INFINITY, mxb = -INFINITY, mxc = -INFINITY, mxd = -INFINITY;
#pragma unroll
        for (int c = 0; c < 64; c += 8) {
          mxa = max3(mxa, __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
          mxb = max3(mxb, __uint_as_float(sr[c + 2]), __uint_as_float(sr[c + 3]));
          mxc = max3(mxc, __uint_as_float(sr[c + 4]), __uint_as_float(sr[c + 5]));
          mxd = max3(mxd, __uint_as_float(sr[c + 6]), __uint_as_float(sr[c + 7]));
        }
        const float mx = fmaxf(fmaxf(mxa, mxb), fmaxf(mxc, mxd));
        const float m_new = fmaxf(m, mx * a.c2);
        const bool need = m_new > m + 8.0f;
        if (__any_sync(0xffffffffu, need && j > 0)) {
          // rescale O once the previous tile's PV product (the last writer) completed
          if (!mbar_wait(&pv_done[(t - 1) % kSBuf], uint32_t((t - 1) / kSBuf) & 1u, a.err)) { ok = false; break; }
          tc_fence_after();
          const float alpha = need ? ex2(m - m_new) : 1.f;
#pragma unroll
          for (int c0 = 0; c0 < D; c0 += 32) {
            uint32_t orr[32];
            tm_ld32(lane_base + cO + c0, orr);
            tm_ld_wait();
#pragma unroll
            for (int c = 0; c < 32; ++c) orr[c] = __float_as_uint(__uint_as_float(orr[c]) * alpha);
            tm_st32(lane_base + cO + c0, orr);
          }
          tm_st_wait();
        }
        if (need) {
          l *= ex2(m - m_new);
          m = m_new;
        }
        // P = exp2(S c - m) -> bf16 pairs over the S columns, with S c - m and
        // the row sums as packed pairs. All exponentials on the MUFU unit: this
        // loop is bound by instruction issue and latency, so moving some of
        // them to an FMA-pipe polynomial measured slower (v6 layer 0: 4.43 ms
        // with none, slower with 8, 16 or 24 of the 64 columns moved).
        // Masked columns hold -inf: ex2 -> 0.
        const uint64_t c2v = f2(a.c2, a.c2), nmv = f2(-m, -m);
        uint64_t acc0 = f2(0.f, 0.f), acc1 = acc0, acc2 = acc0, acc3 = acc0;
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 64; c += 2) {
          float x0, x1;
          f2_split(fma_f2(f2(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), c2v, nmv), x0, x1);
          const float p0 = ex2(x0), p1 = ex2(x1);
          const uint64_t pp = f2(p0, p1);
          switch ((c >> 1) & 3) {
            case 0: acc0 = add_f2(acc0, pp); break;
            case 1: acc1 = add_f2(acc1, pp); break;
            case 2: acc2 = add_f2(acc2, pp); break;
            default: acc3 = add_f2(acc3, pp); break;
          }
          pk[c >> 1] = pack_bf16(p0, p1);
        }
        {
          float u0, u1, u2, u3, u4, u5, u6, u7;
          f2_split(acc0, u0, u1); f2_split(acc1, u2, u3); f2_split(acc2, u4, u5); f2_split(acc3, u6, u7);
          l += ((u0 + u1) + (u2 + u3)) + ((u4 + u5) + (u6 + u7));
        }
        tm_st32(lane_base + uint32_t(kKT * buf), pk);
        tm_st_wait();
        tc_fence_before();
        mbar_arrive(&p_full[buf]);
        ++t;
        const bool last = it.last_of_item();
        it.next(a, w_end);
        if (last) break;
      }
      if (!ok || !mbar_wait(o_full, item & 1, a.err)) { ok = false; break; }
      tc_fence_after();
      const int qi = i0 + r;
      const float inv = 1.f / l;
      __nv_bfloat16* dst = a.o + ((int64_t(b) * a.q_len + qi) * a.H + h) * D;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t orr[32];
        tm_ld32(lane_base + cO + c0, orr);
        tm_ld_wait();
        if (qi < a.q_len) {
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            uint4 v;
            v.x = pack_bf16(__uint_as_float(orr[c]) * inv, __uint_as_float(orr[c + 1]) * inv);
            v.y = pack_bf16(__uint_as_float(orr[c + 2]) * inv, __uint_as_float(orr[c + 3]) * inv);
            v.z = pack_bf16(__uint_as_float(orr[c + 4]) * inv, __uint_as_float(orr[c + 5]) * inv);
            v.w = pack_bf16(__uint_as_float(orr[c + 6]) * inv, __uint_as_float(orr[c + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + c0 + c) = v;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(o_free);
      if (qi < a.q_len) a.lse[(int64_t(b) * a.H + h) * a.q_len + qi] = m + __log2f(l);
      ++item;
    }
    if (!ok) *abort_flag = 1;
  }
  // teardown: every role is out of its loop (all waits above are bounded)
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
  }
}

// ===========================================================================
// Backward (d = 32): one persistent CTA per (b, h) at a time.
//
//   for each 128-key tile j (K_j, V_j double-buffered in smem)
//     for each 128-query tile i that sees any key of j
//       S^T  = K_j Q_i^T      dP^T = V_j dO_i^T           (SS MMAs -> TMEM)
//       compute warps: P^T = exp2(S^T c - lse), dS^T = P^T (dP^T - delta)
//       dV_j += P^T dO_i      dK_j += dS^T Q_i            (TS: A = P^T / dS^T in TMEM)
//       dQ_i  = dS K_j                                     (SS: dS from a swizzled smem tile)
//       compute warps add dQ_i into an fp32 dQ block in shared memory
//   dQ, dK, dV are written once, in bf16, straight into the fused-QKV
//   gradient; the Q rows the pyramid pruned get zeros.
// One CTA owns every key tile of the head, so dQ accumulates in shared
// memory (no fp32 atomics, no accumulator buffer, no conversion pass) and
// delta = rowsum(dO * O) is computed in the CTA's prologue: one launch.
//
// Issue: a single thread that issues tcgen05.mma back to back waits about
// 100-120 cycles per instruction whatever N is, while the tensor pipe can
// take instructions from several warps at once (measured with
// scripts/bench_tcgen05_mma.py: an N = 32 TS product runs 4x faster from
// four issuing warps than from one; two lanes of one warp only 1.5x). With
// d = 32 a pair is 4 N = 128 and 24 N = 32 products, so each product stream
// has its own issuing warp:
//   warp 0  S^T and dP^T of the next pair (as soon as the compute warps
//           have read the current ones), warp 1 dV, warp 2 dK, warp 3 dQ.
// Warps 4..19 compute (warp w reads TMEM lanes 32 (w % 4)..+31 = key rows;
// (w - 4) / 4 selects 32 of the 128 query columns). 20 warps keep every
// sub-partition at 5 warps (96 registers per thread).
// The TMA loads (QST stages of Q / dO, two of K / V) are issued by lane 0
// of warp 4: it knows when a buffer is free because it has just waited for
// the products that read it (mma2_done), so its waits never block on work
// that itself waits for the compute warps.
// TMEM (512 columns): S^T [0,128), dP^T [128,256), P^T bf16 [256,320),
// dS^T bf16 [320,384), dV [384,416), dK [416,448), dQ [448,480).
// ===========================================================================
struct BwdArgs {
  int B, H, T, q_len, nq, nkv, items;
  float c2, scale;
  const __nv_bfloat16* o;     // [B, q_len, H, 32]
  const __nv_bfloat16* dout;  // [B, q_len, H, 32]
  const float* lse;           // [B, H, q_len]
  __nv_bfloat16* dqkv;        // [B, T, 3, H, 32]
  int* err;
  long long* dbg;             // optional per-stage clock stamps of CTA 0 (profiling aid), or null
};

constexpr int kBwdCompute = 16;                       // compute warps
constexpr int kBwdC0 = 4;                             // first compute warp
constexpr int kBwdThreads = 32 * (kBwdC0 + kBwdCompute);
constexpr int kBwdCT = 32 * kBwdCompute;              // compute threads
constexpr int kDbgPairs = 64, kDbgSlots = 16;

// Pair enumeration shared by every role: items (b, h) of this CTA, key tiles,
// then the query tiles that see the key tile. Only the cursor lives in
// registers; the shapes come from the kernel arguments.
struct PairIt {
  int w, jt, i, first_i;
  __device__ void first_q(const BwdArgs& a) {
    const int k0 = jt * kTile, off = a.T - a.q_len;
    first_i = k0 > off ? (k0 - off) / kTile : 0;
    i = first_i;
  }
  __device__ void start(const BwdArgs& a, int wb) { w = wb; jt = 0; first_q(a); }
  __device__ bool last_of_kv(const BwdArgs& a) const { return i == a.nq - 1; }
  __device__ bool first_of_kv() const { return i == first_i; }
  __device__ void next(const BwdArgs& a) {
    if (++i < a.nq) return;
    if (++jt < a.nkv) { first_q(a); return; }
    ++w; jt = 0; first_q(a);
  }
};
__device__ __forceinline__ void dbg_stamp(const BwdArgs& a, int pc, int slot) {
  if (a.dbg != nullptr && blockIdx.x == 0 && pc < kDbgPairs) a.dbg[pc * kDbgSlots + slot] = clock64();
}
__device__ __forceinline__ void tm_ld8(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tm_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// Wait for this thread's tcgen05 work committed to `bar` (bounded).
__device__ __forceinline__ void drain(uint64_t* bar, int* err) {
  tc_commit(bar);
  (void)mbar_wait(bar, 0, err);
}

template <int QST>
__global__ void __launch_bounds__(kBwdThreads, 1) fmha_bwd_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv,
                                                                    const __grid_constant__ CUtensorMap tm_do,
                                                                    const BwdArgs a) {
  constexpr int D = 32;
  using G = Geo<D>;
  constexpr uint32_t cS = 0, cdP = 128, cP = 256, cdS = 320, cdV = 384, cdK = 416, cdQ = 448;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;                                // [2] key tiles
  uint8_t* sV = sK + 2 * G::kTileBytes;              // [2]
  uint8_t* sQ = sV + 2 * G::kTileBytes;              // [QST] stages
  uint8_t* sdO = sQ + QST * G::kTileBytes;           // [QST] stages
  uint8_t* sdS = sdO + QST * G::kTileBytes;          // 128 x 128 bf16, MN-major SW128 for the dQ product
  float* sLSE = reinterpret_cast<float*>(sdS + 32768);          // [nq * 128]
  float* sDel = sLSE + a.nq * kTile;                             // [nq * 128]
  float* sdQ = sDel + a.nq * kTile;                              // [q_len(8)] x 32 fp32, 16B chunks swizzled
  const int qrows = (a.q_len + 7) & ~7;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sdQ + qrows * 32);
  uint64_t* kv_full = bar;               // [2]
  uint64_t* kv_empty = bar + 2;          // [2]   arrivals: the dQ issuer's commit
  uint64_t* qd_full = bar + 4;           // [QST]
  uint64_t* qd_empty = bar + 4 + QST;    // [QST] arrivals: the dV and dK issuers' commits
  uint64_t* s_full = bar + 4 + 2 * QST;
  uint64_t* s_free = s_full + 1;
  uint64_t* p_full = s_full + 2;
  uint64_t* mma2_done = s_full + 3;      // arrivals: dV, dK, dQ issuers
  uint64_t* drained = s_full + 4;        // [4] one per issuing warp
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int k = 0; k < 2; ++k) { mbar_init(&kv_full[k], 1); mbar_init(&kv_empty[k], 1); }
    for (int k = 0; k < QST; ++k) { mbar_init(&qd_full[k], 1); mbar_init(&qd_empty[k], 2); }
    mbar_init(s_full, 1); mbar_init(s_free, kBwdCT); mbar_init(p_full, kBwdCT); mbar_init(mma2_done, 3);
    for (int k = 0; k < 4; ++k) mbar_init(&drained[k], 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_qkv) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_do) : "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(tmem_slot)), "r"(512) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int per = (a.items + gridDim.x - 1) / gridDim.x;
  const int w_begin = blockIdx.x * per, w_end = min(a.items, w_begin + per);
  const int off = a.T - a.q_len;
  // registers: the issuing warpgroup (warps 0-3) needs few, the compute
  // warpgroups take them (640 x 96 at launch >= 128 x 56 + 512 x 104)
  if (warp < kBwdC0) asm volatile("setmaxnreg.dec.sync.aligned.u32 56;" ::: "memory");
  else asm volatile("setmaxnreg.inc.sync.aligned.u32 104;" ::: "memory");

  if (warp == 0) {
    // ---------------- TMA loads + S^T / dP^T issuer ----------------
    if (lane == 0) {
      constexpr uint32_t id_s = idesc(128, 128, 0, 0);
      PairIt it, ld;
      it.start(a, w_begin);
      ld.start(a, w_begin);
      int pc = 0, kc = 0;          // pairs issued, key tiles consumed
      int ldc = 0, kvc = 0;        // pairs loaded, key tiles loaded
      // Load pair ldc (and its K / V tile when it opens one). A Q / dO stage is
      // free once the dV / dK products of the pair QST back completed; a K / V
      // buffer once the dQ products of the tile two back completed. block:
      // wait for them (bounded); else only issue when both are already free.
      // Returns 1 issued, 0 not yet free, -1 wait timed out.
      auto load_one = [&](bool block) -> int {
        const int lb = ld.w / a.H, lh = ld.w - lb * a.H;
        const int st = ldc % QST;
        const uint32_t qpar = uint32_t((ldc / QST) & 1) ^ 1u;
        const bool opens = ld.first_of_kv();
        const int kb = kvc & 1;
        const uint32_t kpar = uint32_t((kvc >> 1) & 1) ^ 1u;
        if (!block && !(mbar_test(&qd_empty[st], qpar) && (!opens || mbar_test(&kv_empty[kb], kpar)))) return 0;
        if (opens) {
          if (!mbar_wait(&kv_empty[kb], kpar, a.err)) return -1;
          mbar_expect_tx(&kv_full[kb], 2 * G::kTileBytes);
          tma_load_5d(sK + kb * G::kTileBytes, &tm_qkv, &kv_full[kb], 0, lh, 1, ld.jt * kTile, lb);
          tma_load_5d(sV + kb * G::kTileBytes, &tm_qkv, &kv_full[kb], 0, lh, 2, ld.jt * kTile, lb);
          ++kvc;
        }
        if (!mbar_wait(&qd_empty[st], qpar, a.err)) return -1;
        mbar_expect_tx(&qd_full[st], 2 * G::kTileBytes);
        tma_load_5d(sQ + st * G::kTileBytes, &tm_qkv, &qd_full[st], 0, lh, 0, off + ld.i * kTile, lb);
        asm volatile(
            "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
            "[%2];" ::"r"(smem_u32(sdO + st * G::kTileBytes)), "l"(&tm_do), "r"(smem_u32(&qd_full[st])), "r"(0),
            "r"(lh), "r"(ld.i * kTile), "r"(lb) : "memory");
        ld.next(a);
        ++ldc;
        return 1;
      };
      bool good = true;
      for (; good && it.w < w_end && !*abort_flag; it.next(a), ++pc) {
        if (pc > 0) {
          // wait until the compute warps have read S^T / dP^T of the last pair,
          // issuing loads as their buffers free up meanwhile
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_test(s_free, uint32_t(pc - 1) & 1u)) {
            if (ld.w < w_end && ldc < pc + QST && load_one(false) < 0) { good = false; break; }
            if (globaltimer_ns() - t0 > kWaitLimitNs) { set_error(a.err, kWaitTimeout); good = false; break; }
            __nanosleep(64);
          }
          if (!good) break;
        }
        dbg_stamp(a, pc, 8);
        while (ld.w < w_end && ldc <= pc)                        // this pair's loads
          if (load_one(true) < 0) { good = false; break; }
        while (good && ld.w < w_end && ldc < pc + QST && load_one(false) == 1) {}
        if (!good) break;
        if (it.first_of_kv()) {
          if (!mbar_wait(&kv_full[kc & 1], (kc >> 1) & 1, a.err)) { good = false; break; }
          ++kc;
        }
        const int st = pc % QST;
        if (!mbar_wait(&qd_full[st], (pc / QST) & 1, a.err)) { good = false; break; }
        dbg_stamp(a, pc, 9);
        tc_fence_after();
        const int kb = (kc - 1) & 1;
        const uint32_t kt = smem_u32(sK + kb * G::kTileBytes), vt = smem_u32(sV + kb * G::kTileBytes);
        const uint32_t qt = smem_u32(sQ + st * G::kTileBytes), dt = smem_u32(sdO + st * G::kTileBytes);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) mma_ss(tmem + cS, desc_k<D>(kt, kk), desc_k<D>(qt, kk), id_s, kk > 0);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) mma_ss(tmem + cdP, desc_k<D>(vt, kk), desc_k<D>(dt, kk), id_s, kk > 0);
        tc_commit(s_full);
        dbg_stamp(a, pc, 10);
      }
      if (!good) {
        *abort_flag = 1;
        // every issued copy lands before the CTA may exit: loads into buffer k
        // were issued for counts k, k + n, k + 2n, ... below the total
        for (int k = 0; k < 2; ++k)
          if (kvc > k) (void)mbar_wait(&kv_full[k], uint32_t((kvc - 1 - k) / 2) & 1u, a.err);
        for (int k = 0; k < QST; ++k)
          if (ldc > k) (void)mbar_wait(&qd_full[k], uint32_t((ldc - 1 - k) / QST) & 1u, a.err);
      }
      drain(&drained[0], a.err);
    }
  } else if (warp < kBwdC0) {
    // ---------------- dV (warp 1), dK (warp 2), dQ (warp 3) issuers ----------------
    if (lane == 0) {
      const int role = warp - 1;
      constexpr uint32_t id_kv = idesc(128, D, 0, 1);        // A in TMEM, B (dO / Q) MN-major
      constexpr uint32_t id_q = idesc(128, D, 1, 1);         // A (dS) MN-major, B (K) MN-major
      PairIt it;
      it.start(a, w_begin);
      int pc = 0, kc = 0;
      const uint32_t ds = smem_u32(sdS);
      for (; it.w < w_end && !*abort_flag; it.next(a), ++pc) {
        if (it.first_of_kv()) ++kc;
        if (!mbar_wait(p_full, pc & 1, a.err)) { *abort_flag = 1; break; }
        if (role != 1) dbg_stamp(a, pc, role == 0 ? 11 : 14);
        tc_fence_after();
        const int st = pc % QST, kb = (kc - 1) & 1;
        const uint32_t acc0 = it.first_of_kv() ? 0u : 1u;
        if (role == 0) {
          const uint32_t dt = smem_u32(sdO + st * G::kTileBytes);
#pragma unroll
          for (int kk = 0; kk < kTile / 16; ++kk)
            mma_ts(tmem + cdV, tmem + cP + uint32_t(8 * kk), desc_mn<D>(dt, kk), id_kv, (kk > 0) ? 1u : acc0);
          tc_commit(&qd_empty[st]);
        } else if (role == 1) {
          const uint32_t qt = smem_u32(sQ + st * G::kTileBytes);
#pragma unroll
          for (int kk = 0; kk < kTile / 16; ++kk)
            mma_ts(tmem + cdK, tmem + cdS + uint32_t(8 * kk), desc_mn<D>(qt, kk), id_kv, (kk > 0) ? 1u : acc0);
          tc_commit(&qd_empty[st]);
        } else {
          const uint32_t kt = smem_u32(sK + kb * G::kTileBytes);
#pragma unroll
          for (int kk = 0; kk < kTile / 16; ++kk)
            mma_ss(tmem + cdQ, make_desc(ds + uint32_t(kk) * 2048u, 16384u, 1024u, 2), desc_mn<D>(kt, kk), id_q,
                   kk > 0 ? 1u : 0u);
          if (it.last_of_kv(a)) tc_commit(&kv_empty[kb]);
        }
        tc_commit(mma2_done);
        if (role != 1) dbg_stamp(a, pc, role == 0 ? 12 : 15);
      }
      drain(&drained[1 + role], a.err);
    }
  } else {
    // ---------------- compute warps ----------------
    const int ct = threadIdx.x - 32 * kBwdC0;          // 0 .. 511
    const int quarter = warp & 3;
    const int g = (warp - kBwdC0) >> 2;                // query columns [32 g, 32 g + 32)
    const int r = quarter * 32 + lane;                 // key row within the tile = TMEM lane
    const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
    const bool stamp = (warp == kBwdC0 && lane == 0);
    auto bar_compute = [&]() { asm volatile("bar.sync 1, %0;" ::"n"(kBwdCT) : "memory"); };
    // dQ of a finished pair (lanes = query rows, this warp's 8 columns) into
    // the smem block; `qr` was loaded from TMEM (tm_ld8) and waited for
    auto add_dq = [&](int qi, const uint32_t* qr) {
      const int qrow = qi * kTile + r;
      if (qrow < a.q_len) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int chunk = (2 * g + hh) ^ (qrow & 7);
          float4* dst = reinterpret_cast<float4*>(sdQ + qrow * 32) + chunk;
          float4 v = *dst;
          v.x += __uint_as_float(qr[4 * hh]); v.y += __uint_as_float(qr[4 * hh + 1]);
          v.z += __uint_as_float(qr[4 * hh + 2]); v.w += __uint_as_float(qr[4 * hh + 3]);
          *dst = v;
        }
      }
    };
    // dK, dV of a finished key tile: lanes = key rows, this warp's 8 columns
    auto write_dkv = [&](int b, int h, int jt) {
      uint32_t kr[8], vr[8];
      tm_ld8(lane_base + cdK + uint32_t(8 * g), kr);
      tm_ld8(lane_base + cdV + uint32_t(8 * g), vr);
      tm_ld_wait();
      const int krow = jt * kTile + r;
      if (krow < a.T) {
        __nv_bfloat16* dk = a.dqkv + ((int64_t(b) * a.T + krow) * 3 + 1) * a.H * D + h * D + 8 * g;
        __nv_bfloat16* dv = dk + a.H * D;
        uint4 u, v;
        u.x = pack_bf16(__uint_as_float(kr[0]) * a.scale, __uint_as_float(kr[1]) * a.scale);
        u.y = pack_bf16(__uint_as_float(kr[2]) * a.scale, __uint_as_float(kr[3]) * a.scale);
        u.z = pack_bf16(__uint_as_float(kr[4]) * a.scale, __uint_as_float(kr[5]) * a.scale);
        u.w = pack_bf16(__uint_as_float(kr[6]) * a.scale, __uint_as_float(kr[7]) * a.scale);
        v.x = pack_bf16(__uint_as_float(vr[0]), __uint_as_float(vr[1]));
        v.y = pack_bf16(__uint_as_float(vr[2]), __uint_as_float(vr[3]));
        v.z = pack_bf16(__uint_as_float(vr[4]), __uint_as_float(vr[5]));
        v.w = pack_bf16(__uint_as_float(vr[6]), __uint_as_float(vr[7]));
        *reinterpret_cast<uint4*>(dk) = u;
        *reinterpret_cast<uint4*>(dv) = v;
      }
    };
    PairIt it;
    it.start(a, w_begin);
    int pc = 0;
    bool ok = true;
    while (it.w < w_end && ok && !*abort_flag) {
      const int w = it.w;
      const int b = w / a.H, h = w - (w / a.H) * a.H;
      // ---- prologue: lse, delta = rowsum(dO * O), zero dQ ----
      for (int q = ct; q < a.nq * kTile; q += kBwdCT) {
        float lse = INFINITY, del = 0.f;
        if (q < a.q_len) {
          lse = a.lse[(int64_t(b) * a.H + h) * a.q_len + q];
          const int64_t base = ((int64_t(b) * a.q_len + q) * a.H + h) * D;
          const uint4* po = reinterpret_cast<const uint4*>(a.o + base);
          const uint4* pd = reinterpret_cast<const uint4*>(a.dout + base);
#pragma unroll
          for (int c = 0; c < D / 8; ++c) {
            const uint4 u = po[c], v = pd[c];
            const __nv_bfloat162* x = reinterpret_cast<const __nv_bfloat162*>(&u);
            const __nv_bfloat162* y = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 fx = __bfloat1622float2(x[e]), fy = __bfloat1622float2(y[e]);
              del = fmaf(fx.x, fy.x, fmaf(fx.y, fy.y, del));
            }
          }
        }
        sLSE[q] = lse;
        sDel[q] = del;
      }
      for (int k = ct; k < qrows * 8; k += kBwdCT) reinterpret_cast<float4*>(sdQ)[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      bar_compute();
      int prev_i = -1, prev_jt = -1;
      bool prev_last_kv = false;
      for (; it.w < w_end && it.w == w; it.next(a), ++pc) {
        if (stamp) dbg_stamp(a, pc, 0);
        if (!mbar_wait(s_full, pc & 1, a.err)) { ok = false; break; }
        if (stamp) dbg_stamp(a, pc, 1);
        tc_fence_after();
        // P^T, dS^T for key row r, queries q0 + c, in two halves of 16 columns
        // (the second half's S^T / dP^T are loaded after the first half is
        // done, which keeps the live registers low); S^T / dP^T are released
        // to the next pair's products once both halves are in registers
        const int q0 = it.i * kTile + 32 * g;
        const int key = it.jt * kTile + r;
        const int lim = key - off - q0;                    // query column c is visible iff c >= lim
        const int lim_hi = __reduce_max_sync(0xffffffffu, lim);
        const int lim_lo = __reduce_min_sync(0xffffffffu, lim);
        uint32_t pp[16], dd[16];
        // S c - lse, dP - delta and P (dP - delta) as packed fp32 pairs (one
        // instruction per two columns); exponentials on MUFU (this loop is
        // bound by instruction issue and latency, as in the forward)
        const uint64_t c2v = f2(a.c2, a.c2);
        auto half = [&](int h0, const uint32_t* sr, const uint32_t* dr) {
#pragma unroll
          for (int c = 0; c < 16; c += 4) {
            const int cc = h0 + c;
            const float4 l4 = *reinterpret_cast<const float4*>(sLSE + q0 + cc);
            const float4 d4 = *reinterpret_cast<const float4*>(sDel + q0 + cc);
            float x0, x1, x2, x3;
            f2_split(fma_f2(f2(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), c2v, f2(-l4.x, -l4.y)), x0, x1);
            f2_split(fma_f2(f2(__uint_as_float(sr[c + 2]), __uint_as_float(sr[c + 3])), c2v, f2(-l4.z, -l4.w)), x2, x3);
            float p0 = ex2(x0), p1 = ex2(x1), p2 = ex2(x2), p3 = ex2(x3);
            if (lim_hi > 0) {
              p0 = (cc >= lim) ? p0 : 0.f;
              p1 = (cc + 1 >= lim) ? p1 : 0.f;
              p2 = (cc + 2 >= lim) ? p2 : 0.f;
              p3 = (cc + 3 >= lim) ? p3 : 0.f;
            }
            pp[cc >> 1] = pack_bf16(p0, p1);
            pp[(cc >> 1) + 1] = pack_bf16(p2, p3);
            float e0, e1, e2, e3;
            f2_split(mul_f2(f2(p0, p1), sub_f2(f2(__uint_as_float(dr[c]), __uint_as_float(dr[c + 1])), f2(d4.x, d4.y))),
                     e0, e1);
            f2_split(mul_f2(f2(p2, p3),
                            sub_f2(f2(__uint_as_float(dr[c + 2]), __uint_as_float(dr[c + 3])), f2(d4.z, d4.w))),
                     e2, e3);
            dd[cc >> 1] = pack_bf16(e0, e1);
            dd[(cc >> 1) + 1] = pack_bf16(e2, e3);
          }
        };
        {
          uint32_t sr[16], dr[16];
          tm_ld16(lane_base + cS + uint32_t(32 * g), sr);
          tm_ld16(lane_base + cdP + uint32_t(32 * g), dr);
          tm_ld_wait();
          if (lim_lo <= 31) half(0, sr, dr);
        }
        {
          uint32_t sr[16], dr[16];
          tm_ld16(lane_base + cS + uint32_t(32 * g + 16), sr);
          tm_ld16(lane_base + cdP + uint32_t(32 * g + 16), dr);
          tm_ld_wait();
          tc_fence_before();
          mbar_arrive(s_free);
          if (stamp) dbg_stamp(a, pc, 2);
          if (lim_lo <= 31) half(16, sr, dr);
        }
        if (lim_lo > 31) {
#pragma unroll
          for (int c = 0; c < 16; ++c) { pp[c] = 0u; dd[c] = 0u; }
        }
        if (stamp) dbg_stamp(a, pc, 3);
        // the previous pair's products must be done before P / dS are overwritten
        uint32_t qr[8];
        if (prev_i >= 0) {
          if (!mbar_wait(mma2_done, (pc - 1) & 1, a.err)) { ok = false; break; }
          tc_fence_after();
          tm_ld8(lane_base + cdQ + uint32_t(8 * g), qr);      // the previous dQ, read while P / dS are stored
        }
        if (stamp) dbg_stamp(a, pc, 4);
        // P^T and dS^T into TMEM (A operands of dV / dK), dS^T into the swizzled smem tile (dQ)
        tm_st16(lane_base + cP + uint32_t(16 * g), pp);
        tm_st16(lane_base + cdS + uint32_t(16 * g), dd);
        {
          uint8_t* row = sdS + (g >> 1) * 16384 + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int chunk = (4 * (g & 1) + k) ^ (r & 7);
            *reinterpret_cast<uint4*>(row + chunk * 16) = make_uint4(dd[4 * k], dd[4 * k + 1], dd[4 * k + 2], dd[4 * k + 3]);
          }
        }
        if (prev_i >= 0) {
          tm_ld_wait8(qr);
          add_dq(prev_i, qr);
          if (prev_last_kv) write_dkv(b, h, prev_jt);
        }
        if (stamp) dbg_stamp(a, pc, 7);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tm_st_wait();
        tc_fence_before();
        mbar_arrive(p_full);
        if (stamp) dbg_stamp(a, pc, 13);
        prev_i = it.i;
        prev_jt = it.jt;
        prev_last_kv = it.last_of_kv(a);
      }
      if (!ok) break;
      // ---- item epilogue: the last pair's dQ / dK / dV, then dQ to global ----
      if (!mbar_wait(mma2_done, (pc - 1) & 1, a.err)) { ok = false; break; }
      tc_fence_after();
      {
        uint32_t qr[8];
        tm_ld8(lane_base + cdQ + uint32_t(8 * g), qr);
        tm_ld_wait8(qr);
        add_dq(prev_i, qr);
      }
      write_dkv(b, h, prev_jt);
      tc_fence_before();
      bar_compute();
      // dQ rows (scaled, bf16) into the Q part of dqkv; pruned rows [0, off) get zeros
      for (int t = ct; t < a.T; t += kBwdCT) {
        uint4* dst = reinterpret_cast<uint4*>(a.dqkv + ((int64_t(b) * a.T + t) * 3) * a.H * D + h * D);
        const int q = t - off;
        if (q < 0) {
#pragma unroll
          for (int c = 0; c < D / 8; ++c) dst[c] = make_uint4(0u, 0u, 0u, 0u);
        } else {
#pragma unroll
          for (int c = 0; c < D / 8; ++c) {
            const float4 x = reinterpret_cast<const float4*>(sdQ + q * 32)[(2 * c) ^ (q & 7)];
            const float4 y = reinterpret_cast<const float4*>(sdQ + q * 32)[(2 * c + 1) ^ (q & 7)];
            uint4 u;
            u.x = pack_bf16(x.x * a.scale, x.y * a.scale); u.y = pack_bf16(x.z * a.scale, x.w * a.scale);
            u.z = pack_bf16(y.x * a.scale, y.y * a.scale); u.w = pack_bf16(y.z * a.scale, y.w * a.scale);
            dst[c] = u;
          }
        }
      }
      bar_compute();
      tc_fence_after();
    }
    if (!ok) *abort_flag = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
  }
}

}  // namespace atc

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
namespace {

// 5-D map over a contiguous [B, T, 3, H, D] bf16 buffer; box = `rows` rows of
// one (b, part, head), swizzled by the row width (64 B for d = 32, 128 B for d = 64).
CUtensorMap qkv_map(const at::Tensor& qkv, int rows = atc::kTile) {
  const int64_t B = qkv.size(0), T = qkv.size(1), H = qkv.size(3), D = qkv.size(4);
  CUtensorMap m;
  cuuint64_t dims[5] = {cuuint64_t(D), cuuint64_t(H), 3, cuuint64_t(T), cuuint64_t(B)};
  cuuint64_t strides[4] = {cuuint64_t(D * 2), cuuint64_t(H * D * 2), cuuint64_t(3 * H * D * 2),
                           cuuint64_t(T * 3 * H * D * 2)};
  cuuint32_t box[5] = {cuuint32_t(D), 1, 1, cuuint32_t(rows), 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = tensor_map_encode_tiled(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, qkv.data_ptr(), dims, strides, box,
                                      estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                      D == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  PD_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled(qkv) failed: %d", int(r));
  return m;
}

void check_qkv5(const at::Tensor& qkv) {
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.dim() == 5 && qkv.is_contiguous(),
              "qkv must be a contiguous bf16 [B, T, 3, H, d] CUDA tensor");
  TORCH_CHECK(qkv.size(2) == 3 && (qkv.size(4) == 32 || qkv.size(4) == 64), "qkv: [B, T, 3, H, d] with d in {32, 64}");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(qkv.data_ptr()) % 16 == 0, "qkv must be 16-byte aligned");
}

// dynamic shared memory of the backward: K, V (two buffers each), Q, dO (`qst`
// stages each), the dS tile, lse / delta per query row (padded to whole
// tiles), the fp32 dQ block, barriers
size_t bwd_smem_bytes(int q_len, int qst) {
  const int nq = (q_len + atc::kTile - 1) / atc::kTile;
  const int qrows = (q_len + 7) & ~7;
  return 1024 + size_t(4 + 2 * qst) * atc::Geo<32>::kTileBytes + 32768 + 2 * size_t(nq) * atc::kTile * 4 +
         size_t(qrows) * 128 + 256;
}
constexpr size_t kSmemCap = 227 * 1024;

template <int D, int KST>
void launch_fwd(const CUtensorMap& tq, const CUtensorMap& tkv, const atc::FwdArgs& a) {
  constexpr size_t used = 1024 + 2 * atc::kTile * atc::Geo<D>::RB + 2 * KST * atc::kKT * atc::Geo<D>::RB + 256;
  // at least 80 KB, so at most two CTAs (two 256-column TMEM allocations) share an SM
  constexpr size_t smem = used > 81920 ? used : 81920;
  static bool attr = false;
  if (!attr) {
    PD_CHECK_CUDA(cudaFuncSetAttribute(atc::fmha_fwd_tc_kernel<D, KST>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    attr = true;
  }
  const int grid = a.items < 2 * num_sms() ? a.items : 2 * num_sms();
  atc::fmha_fwd_tc_kernel<D, KST><<<grid, atc::kFwdThreads, smem, stream()>>>(tq, tkv, a);
  PD_CHECK_LAUNCH();
}

}  // namespace

// largest q_len whose fp32 dQ block fits the 227 KB of shared memory
int64_t fmha_bwd_tc_max_q() {
  int q = 64;
  while (bwd_smem_bytes(q + 8, 2) <= kSmemCap) q += 8;
  return q;
}

// qkv [B, T, 3, H, d] (contiguous) -> (o [B, q_len, H, d], lse [B, H, q_len] log2 domain)
std::vector<at::Tensor> fmha_fwd_tc(at::Tensor qkv, int64_t q_len, double scale, at::Tensor err) {
  check_qkv5(qkv);
  const int B = int(qkv.size(0)), T = int(qkv.size(1)), H = int(qkv.size(3)), D = int(qkv.size(4));
  TORCH_CHECK(q_len >= 1 && q_len <= T, "q_len must be in [1, T]");
  auto o = at::empty({B, int64_t(q_len), H, D}, qkv.options());
  auto lse = at::empty({B, H, int64_t(q_len)}, qkv.options().dtype(at::kFloat));
  if (B == 0) return {o, lse};
  atc::FwdArgs a{};
  a.B = B; a.H = H; a.T = T; a.q_len = int(q_len);
  a.nq = int((q_len + atc::kTile - 1) / atc::kTile);
  a.items = B * H * a.nq;
  a.c2 = float(scale * 1.4426950408889634);
  a.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  a.lse = lse.data_ptr<float>();
  a.err = err.data_ptr<int>();
  const CUtensorMap tq = qkv_map(qkv, atc::kTile), tkv = qkv_map(qkv, atc::kKT);
  if (D == 32) launch_fwd<32, 6>(tq, tkv, a);
  else launch_fwd<64, 4>(tq, tkv, a);
  return {o, lse};
}

// Backward of fmha_fwd(_tc) for d = 32 into dqkv [B, T, 3, H, d] (fully written).
void fmha_bwd_tc(at::Tensor qkv, at::Tensor o, at::Tensor lse, at::Tensor dout, at::Tensor dqkv, int64_t q_len,
                 double scale, at::Tensor err, c10::optional<at::Tensor> dbg) {
  check_qkv5(qkv);
  const int B = int(qkv.size(0)), T = int(qkv.size(1)), H = int(qkv.size(3)), D = int(qkv.size(4));
  TORCH_CHECK(D == 32, "fmha_bwd_tc: head_dim 32 only");
  TORCH_CHECK(dqkv.sizes() == qkv.sizes() && dqkv.is_contiguous() && dqkv.scalar_type() == at::kBFloat16,
              "dqkv must be a contiguous bf16 tensor shaped like qkv");
  TORCH_CHECK(o.is_contiguous() && dout.is_contiguous() && o.dim() == 4 && o.size(0) == B && o.size(1) == q_len &&
              o.size(2) == H && o.size(3) == D && dout.sizes() == o.sizes() && dout.scalar_type() == at::kBFloat16,
              "o / dout must be contiguous [B, q_len, H, d]");
  TORCH_CHECK(lse.is_contiguous() && lse.scalar_type() == at::kFloat && lse.numel() == int64_t(B) * H * q_len);
  TORCH_CHECK(q_len >= 1 && q_len <= fmha_bwd_tc_max_q(), "fmha_bwd_tc: q_len above the shared-memory cap");
  if (B == 0) return;
  atc::BwdArgs a{};
  a.B = B; a.H = H; a.T = T; a.q_len = int(q_len);
  a.nq = int((q_len + atc::kTile - 1) / atc::kTile);
  a.nkv = (T + atc::kTile - 1) / atc::kTile;
  a.items = B * H;
  a.c2 = float(scale * 1.4426950408889634);
  a.scale = float(scale);
  a.o = reinterpret_cast<const __nv_bfloat16*>(o.data_ptr());
  a.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  a.lse = lse.data_ptr<float>();
  a.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  a.err = err.data_ptr<int>();
  a.dbg = nullptr;
  if (dbg && dbg->defined()) {
    TORCH_CHECK(dbg->is_cuda() && dbg->scalar_type() == at::kLong && dbg->numel() >= atc::kDbgPairs * atc::kDbgSlots,
                "dbg must be an int64 CUDA tensor of at least 1024 elements");
    a.dbg = reinterpret_cast<long long*>(dbg->data_ptr());
  }
  const CUtensorMap tq = qkv_map(qkv);
  CUtensorMap td;
  {
    cuuint64_t dims[4] = {cuuint64_t(D), cuuint64_t(H), cuuint64_t(q_len), cuuint64_t(B)};
    cuuint64_t strides[3] = {cuuint64_t(D * 2), cuuint64_t(H * D * 2), cuuint64_t(q_len * H * D * 2)};
    cuuint32_t box[4] = {cuuint32_t(D), 1, cuuint32_t(atc::kTile), 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = tensor_map_encode_tiled(&td, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, dout.data_ptr(), dims, strides, box,
                                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                                        CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    PD_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled(dout) failed: %d", int(r));
  }
  // three Q / dO stages where the dQ block leaves room for them, else two
  const int grid = a.items < num_sms() ? a.items : num_sms();
  auto go = [&](auto kern, int qst) {
    const size_t smem = bwd_smem_bytes(int(q_len), qst);
    PD_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    kern<<<grid, atc::kBwdThreads, smem, stream()>>>(tq, td, a);
  };
  if (bwd_smem_bytes(int(q_len), 3) <= kSmemCap) go(atc::fmha_bwd_tc_kernel<3>, 3);
  else go(atc::fmha_bwd_tc_kernel<2>, 2);
  PD_CHECK_LAUNCH();
}

}  // namespace pd
