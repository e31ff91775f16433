// Persistent tcgen05 GEMM for sm_100a with fused epilogues.
//
//   C[l, m, n] = epi( sum_k A[l, m, k] * B[l, n, k] )        (A, B K-major, bf16)
//
// Structure (one CTA per SM, 6 warps):
//   warp 0      TMA producer: A/B tiles (128 x 64 and BN x 64, 128-byte
//               swizzle) into a STAGES-deep shared-memory ring, one mbarrier
//               per stage with expected-transaction bytes; each CTA loads
//               its own tiles.
//   warp 1      allocates TMEM (2 x BN fp32 columns: a double-buffered
//               accumulator) and one elected lane issues tcgen05.mma
//               (M=128, N=BN, K=16 per instruction) for every k-step,
//               releasing each smem stage with tcgen05.commit.
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time (each thread owns
//               one accumulator row = one TMEM lane), apply the fused op,
//               convert to bf16 and store; then hand the accumulator buffer
//               back to the MMA warp.  The MMA of tile i+1 overlaps the
//               epilogue of tile i.
// Fused epilogues: none | GELU (optionally also storing the pre-activation) |
// GELU storing its derivative | residual add | GELU backward from the
// pre-activation (acc * gelu'(pre)) | product with a stored derivative. An addend R (residual, or
// a bias / positional table broadcast through zero strides) is added before
// the activation in every mode but the GELU backward, where R is the
// pre-activation.
//
// A and B are described by 3-D TMA maps {K, rows, L} with arbitrary row and
// batch strides, so strided views (e.g. the NS rows of every sample, one
// batch per NS token) are consumed in place; C / R / AUX take element strides.
//
// Every mbarrier wait is bounded (2 s on %globaltimer); on timeout the warp
// records kWaitTimeout in the error word, stops issuing work, drains its own
// in-flight operations (bounded) and the CTA frees its TMEM and exits.
#include "common.cuh"
#include "driver_api.h"

#include <cuda.h>

namespace pd {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kEpiWarps = 12;  // three warps per TMEM lane quarter, splitting the columns
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// kGeluD: C = GELU(x), AUX = GELU'(x) for x = acc + R in fp32 -- the derivative
// stored in the forward makes the backward's epilogue a plain product (kMul:
// C = acc * R), with no transcendental per element.
// kRelu: C = max(acc + R, 0) (R: a bias through a zero row stride);
// kMaskPos: C = acc where R > 0, else 0 (R: the ReLU layer's stored output,
// so the data gradient of the next layer leaves as the pre-activation
// gradient of this one); kMulAdd: C = R * (acc + b) + R2, with b added via
// the operands (an extra K row), AUX optionally storing acc (the DCNv2 cross
// layer: x_{l+1} = x0 * (t V + b) + x_l with R = x0, R2 = x_l).
enum Epi : int { kNone = 0, kGelu = 1, kResidual = 2, kDGelu = 3, kGeluD = 4, kMul = 5, kRelu = 6, kMaskPos = 7,
                 kMulAdd = 8 };

struct Params {
  int M, N, K, L;
  int m_blocks, n_blocks, k_blocks, tiles;
  __nv_bfloat16* C; int64_t c_ls, c_ms;
  const __nv_bfloat16* R; int64_t r_ls, r_ms;      // addend, pre-activation (kDGelu) or factor (kMul)
  __nv_bfloat16* AUX; int64_t aux_ls, aux_ms;       // pre-activation (kGelu, optional) or GELU' (kGeluD)
  const __nv_bfloat16* R2; int64_t r2_ls, r2_ms;    // second addend (kMulAdd)
  int epi;
  int a_mode, b_mode;   // TMA map dim order: 0 = {K, rows, L}, 1 = {K, L, rows}
  int c_mode, x_mode;   // store maps of C / AUX: 0 = {N, rows, L}, 1 = {N, L, rows}
  int r_tma, r_mode;    // R read by TMA (a full [L, M, N] view) and its map's dim order
  int b_shared;         // B has one batch shared by every l
  int b_kn;             // B stored [L, K, N] (N contiguous: a weight used transposed), loaded MN-major
  int* err;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier --------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
// try_wait with a suspend-time hint: a waiting warp sleeps until the phase
// completes or ~0.2 ms pass instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(b)), "r"(parity), "r"(200000u) : "memory");
  return ok != 0;
}
// Bounded wait: false (and the error word set) after kWaitLimitNs.
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

// ---- TMA -------------------------------------------------------------------
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2);
// Load rows [row, row + box) of batch l; mode 1 maps have dims {K, L, rows}.
__device__ __forceinline__ void tma_load_rows(void* dst, const CUtensorMap* map, uint64_t* bar, int mode, int k, int row,
                                              int l) {
  if (mode == 0) tma_load_3d(dst, map, bar, k, row, l);
  else tma_load_3d(dst, map, bar, k, l, row);
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2) : "memory");
}

// TMA store of one 32 x 32 bf16 block staged in shared memory (64-byte
// swizzle); mode 1 maps have dims {N, L, rows}.  Rows past the tensor's end
// are clipped by the copy engine.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];"
               ::"l"(map), "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2) : "memory");
}
__device__ __forceinline__ void tma_store_rows(const CUtensorMap* map, const void* src, int mode, int n, int row,
                                               int l) {
  if (mode == 0) tma_store_3d(map, src, n, row, l);
  else tma_store_3d(map, src, n, l, row);
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the staged source of every committed store has been read (the buffer may be rewritten)
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// generic-proxy shared-memory writes -> visible to the async proxy (TMA)
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---- tcgen05 ---------------------------------------------------------------
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major, 128-byte-swizzled operand tile: rows of 64 bf16 (128 B), 8-row
// atoms of 1024 B.  start advances by 32 B per 16-element k-step.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= uint64_t((addr >> 4) & 0x3FFF);        // start address
  d |= uint64_t(1) << 16;                       // leading byte offset (unused for swizzled K-major)
  d |= uint64_t(1024 >> 4) << 32;               // stride byte offset: 8 rows x 128 B
  d |= uint64_t(1) << 46;                       // descriptor version (sm_100)
  d |= uint64_t(2) << 61;                       // SWIZZLE_128B
  return d;
}
// MN-major, 128-byte-swizzled B tile: BN / 64 groups of [64 k-rows][64 n]
// (8 KB each, 128 B per k-row); a 16-row k-step starts 2048 B further, the
// groups are 8192 B apart (leading byte offset), 8-row atoms 1024 B apart.
__device__ __forceinline__ uint64_t smem_desc_mn(uint32_t addr) {
  uint64_t d = 0;
  d |= uint64_t((addr >> 4) & 0x3FFF);
  d |= uint64_t(8192 >> 4) << 16;
  d |= uint64_t(1024 >> 4) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}
// kind::f16 instruction descriptor: f32 accumulate, bf16 A/B, both K-major.
__host__ __device__ constexpr uint32_t instr_desc(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(acc) : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_u32(bar)) : "memory");
}
// tcgen05.ld of 32 columns without the wait (registers undefined until
// tc_ld_wait on the same array, which ties them to the wait instruction).
__device__ __forceinline__ void tc_ld32_issue(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr) : "memory");
}
__device__ __forceinline__ void tc_ld_wait(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :: "memory");
}
__device__ __forceinline__ void tc_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tile_coords(const Params& p, int t, int& l, int& mb, int& nb) {
  nb = t % p.n_blocks;
  const int r = t / p.n_blocks;
  mb = r % p.m_blocks;
  l = r / p.m_blocks;
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                                                           const __grid_constant__ CUtensorMap tmB,
                                                           const __grid_constant__ CUtensorMap tmC,
                                                           const __grid_constant__ CUtensorMap tmX,
                                                           const __grid_constant__ CUtensorMap tmR,
                                                           const Params p) {
  constexpr uint32_t kABytes = BM * BK * 2;
  constexpr uint32_t kBBytes = BN * BK * 2;
  constexpr uint32_t kTmemCols = 2 * BN;  // power of two for BN in {64, 128, 256}
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * kBBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;     // [2]
  uint64_t* tempty = tfull + 2;         // [2]
  uint64_t* mma_done = tempty + 2;      // [1]
  uint64_t* rbar_all = mma_done + 1;    // [kEpiWarps][2]: R blocks landed (TMA)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar_all + 2 * kEpiWarps);
  // per epilogue warp: 32 x 32 bf16 staging blocks for C and R / AUX (64-byte
  // rows, 16-byte chunks XOR-swizzled by (row >> 1) & 3: conflict-free both
  // when a thread writes its own row and when 4 lanes cover one row)
  // (the 64-byte swizzle of the TMA stores: buffers 512-byte aligned)
  uint8_t* stage_base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(tmem_slot) + 64 + 1023) & ~uintptr_t(1023));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(&tfull[a], 1); mbar_init(&tempty[a], kEpiWarps * 32); }
    mbar_init(mma_done, 1);
    for (int i = 0; i < 2 * kEpiWarps; ++i) mbar_init(&rbar_all[i], 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmA) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmB) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmC) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(tmem_slot)), "r"(kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 1;
      int issued = 0;
      int issued_on[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) issued_on[s] = 0;
      for (int t = blockIdx.x; t < p.tiles && !*abort_flag; t += gridDim.x) {
        int l, mb, nb;
        tile_coords(p, t, l, mb, nb);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase, p.err)) { *abort_flag = 1; break; }
          mbar_expect_tx(&full[stage], kABytes + kBBytes);
          tma_load_rows(sA + stage * kABytes, &tmA, &full[stage], p.a_mode, kb * BK, mb * BM, l);
          if (p.b_kn) {
#pragma unroll
            for (int g = 0; g < BN / 64; ++g)   // [64 k-rows][64 n] boxes
              tma_load_rows(sB + stage * kBBytes + g * 8192, &tmB, &full[stage], p.b_mode, nb * BN + 64 * g, kb * BK,
                            p.b_shared ? 0 : l);
          } else {
            tma_load_rows(sB + stage * kBBytes, &tmB, &full[stage], p.b_mode, kb * BK, nb * BN, p.b_shared ? 0 : l);
          }
          ++issued_on[stage];
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // drain: every issued load must have landed before the CTA can exit
      if (*abort_flag) {
#pragma unroll
        for (int s = 0; s < STAGES; ++s)
          if (issued_on[s] > 0) (void)mbar_wait(&full[s], uint32_t(issued_on[s] - 1) & 1u, p.err);
      }
      (void)issued;
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(BM, BN);
      const uint32_t idesc_run = idesc | (p.b_kn ? (1u << 16) : 0u);   // B MN-major
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int t = blockIdx.x; t < p.tiles && !*abort_flag; t += gridDim.x, ++local) {
        const int a = local & 1;
        const uint32_t ephase = ((local >> 1) & 1) ^ 1;
        if (!mbar_wait(&tempty[a], ephase, p.err)) { *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t d = tmem + uint32_t(a * BN);
        bool ok = true;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err)) { *abort_flag = 1; ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * kABytes);
          const uint32_t b_addr = smem_u32(sB + stage * kBBytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t db = p.b_kn ? smem_desc_mn(b_addr + k * 2048) : smem_desc(b_addr + k * 32);
            tc_mma(d, smem_desc(a_addr + k * 32), db, idesc_run, (kb | k) ? 1u : 0u);
          }
          tc_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit(&tfull[a]);
      }
      // all MMAs issued by this thread have finished before TMEM is freed
      tc_commit(mma_done);
      (void)mbar_wait(mma_done, 0, p.err);
    }
  } else {
    // ---------------- epilogue ----------------
    // Warp ew owns TMEM lane quarter q (rows q*32..q*32+31 of the tile) and the
    // 32-column chunks c with (c / 32) % 3 == part.  Per chunk: the R block
    // (residual, GELU' factor or pre-activation) arrives by TMA into a
    // two-deep ring, issued one chunk ahead (a broadcast addend -- bias or
    // positional table, zero strides -- is prefetched into registers
    // instead); tcgen05.ld the accumulator, apply the epilogue, stage the
    // bf16 block in swizzled smem and hand it to a TMA store (C, and AUX),
    // which runs while the next chunk is computed.
    const int ew = warp - 2;
    const int q = warp & 3;
    const int part = ew >> 2;
    constexpr int kParts = kEpiWarps / 4;
    uint8_t* stC = stage_base + ew * 3 * 2048;
    uint8_t* stR0 = stC + 2048;   // R ring: buffers stR0 and stR0 + 2048
    uint64_t* rbar = rbar_all + 2 * ew;
    const bool r_tma = p.r_tma != 0;
    int kc = 0;          // chunks processed by this warp (R ring position)
    int r_pending = 0;   // R blocks issued and not yet waited for
    const int cr = lane >> 2, cc = lane & 3;
    auto sw = [](int r, int c) { return r * 64 + ((c ^ ((r >> 1) & 3)) << 4); };
    const bool has_r = (p.R != nullptr);   // addend (bias / residual), or GELU's pre-activation for kDGelu
    // work items: (tile, chunk) in this warp's order
    auto first_chunk = [&]() { return part * 32; };
    auto next_work = [&](int& t, int& c) {
      c += kParts * 32;
      if (c >= BN) { c = first_chunk(); t += gridDim.x; }
    };
    auto load_r = [&](int t, int c, uint4* dst) {
      int l, mb, nb;
      tile_coords(p, t, l, mb, nb);
      const int m0 = mb * BM + q * 32;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = cr + 8 * i;
        dst[i] = (m0 + r < p.M)
                     ? __ldcs(reinterpret_cast<const uint4*>(p.R + l * p.r_ls + int64_t(m0 + r) * p.r_ms + nb * BN + c +
                                                             cc * 8))
                     : make_uint4(0, 0, 0, 0);
      }
    };
    auto issue_r = [&](int t, int c, int buf) {   // lane 0 only
      int l, mb, nb;
      tile_coords(p, t, l, mb, nb);
      mbar_expect_tx(&rbar[buf], 32 * 32 * 2);
      tma_load_rows(stR0 + (buf << 11), &tmR, &rbar[buf], p.r_mode, nb * BN + c, mb * BM + q * 32, l);
    };
    uint4 pref[4];
    if (has_r && first_chunk() < BN && blockIdx.x < p.tiles) {
      if (r_tma) {
        if (lane == 0) issue_r(blockIdx.x, first_chunk(), 0);
        r_pending = 1;
      } else {
        load_r(blockIdx.x, first_chunk(), pref);
      }
    }
    int local = 0;
    for (int t = blockIdx.x; t < p.tiles; t += gridDim.x, ++local) {
      const int a = local & 1;
      if (!mbar_wait(&tfull[a], (local >> 1) & 1, p.err)) { *abort_flag = 1; break; }
      tc_fence_after();
      int l, mb, nb;
      tile_coords(p, t, l, mb, nb);
      const int m0 = mb * BM + q * 32;
      const int n0 = nb * BN;
      const uint32_t tbase = tmem + (uint32_t(q * 32) << 16) + uint32_t(a * BN);
      // one chunk: 32 accumulator columns of this warp's 32 rows, already in r
      auto process = [&](uint32_t (&r)[32], int c) -> bool {
        // the previous chunk's TMA stores have read the staging blocks: waited
        // for here when an R block is about to land in one of them, else only
        // just before the first staging write (the math of this chunk overlaps
        // the stores' shared-memory reads)
        bool waited = false;
        auto wait_staging = [&]() {
          if (waited) return;
          if (lane == 0) bulk_wait_read_all();
          __syncwarp();
          waited = true;
        };
        if (has_r) wait_staging();
        uint8_t* stR = stR0 + (r_tma ? ((kc & 1) << 11) : 0);
        uint8_t* stX = stR;   // AUX staging reuses the R block once it has been consumed
        if (has_r) {
          int tn = t, cn = c;
          next_work(tn, cn);
          if (r_tma) {
            if (tn < p.tiles) {   // the next block lands in the other buffer while this chunk runs
              if (lane == 0) issue_r(tn, cn, (kc + 1) & 1);
              ++r_pending;
            }
            const bool ok = mbar_wait(&rbar[kc & 1], uint32_t(kc >> 1) & 1u, p.err);
            --r_pending;
            if (!ok) { *abort_flag = 1; return false; }
          } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) *reinterpret_cast<uint4*>(stR + sw(cr + 8 * i, cc)) = pref[i];
            __syncwarp();
            if (tn < p.tiles) load_r(tn, cn, pref);   // in flight during this chunk
          }
        }
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
        if (has_r && p.epi != kDGelu && p.epi != kMul && p.epi != kMaskPos && p.epi != kMulAdd) {
          // addend before the activation: residual, or a bias broadcast through a zero row stride
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 pk = *reinterpret_cast<const uint4*>(stR + sw(lane, j));
            const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&pk);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __bfloat1622float2(hh[e]);
              v[8 * j + 2 * e] += f.x;
              v[8 * j + 2 * e + 1] += f.y;
            }
          }
        }
        if (p.epi == kGelu && p.AUX) {
          wait_staging();
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint4 pk;
            __nv_bfloat162 h0 = __floats2bfloat162_rn(v[8 * j], v[8 * j + 1]);
            __nv_bfloat162 h1 = __floats2bfloat162_rn(v[8 * j + 2], v[8 * j + 3]);
            __nv_bfloat162 h2 = __floats2bfloat162_rn(v[8 * j + 4], v[8 * j + 5]);
            __nv_bfloat162 h3 = __floats2bfloat162_rn(v[8 * j + 6], v[8 * j + 7]);
            pk.x = *reinterpret_cast<uint32_t*>(&h0); pk.y = *reinterpret_cast<uint32_t*>(&h1);
            pk.z = *reinterpret_cast<uint32_t*>(&h2); pk.w = *reinterpret_cast<uint32_t*>(&h3);
            *reinterpret_cast<uint4*>(stX + sw(lane, j)) = pk;
          }
        }
        if (p.epi == kGelu) {
          // GELU of the bf16-rounded pre-activation (the value AUX stores)
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            float x0 = __bfloat162float(__float2bfloat16_rn(v[j]));
            float x1 = __bfloat162float(__float2bfloat16_rn(v[j + 1]));
            gelu2(x0, x1);
            v[j] = x0;
            v[j + 1] = x1;
          }
        } else if (p.epi == kGeluD) {
          uint4 dpk[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float d[8];
#pragma unroll
            for (int e = 0; e < 8; e += 2)       // the fp32 pre-activation (no bf16 round trip)
              gelu_grad2<true>(v[8 * j + e], v[8 * j + e + 1], d[e], d[e + 1]);
            __nv_bfloat162 h0 = __floats2bfloat162_rn(d[0], d[1]);
            __nv_bfloat162 h1 = __floats2bfloat162_rn(d[2], d[3]);
            __nv_bfloat162 h2 = __floats2bfloat162_rn(d[4], d[5]);
            __nv_bfloat162 h3 = __floats2bfloat162_rn(d[6], d[7]);
            dpk[j].x = *reinterpret_cast<uint32_t*>(&h0); dpk[j].y = *reinterpret_cast<uint32_t*>(&h1);
            dpk[j].z = *reinterpret_cast<uint32_t*>(&h2); dpk[j].w = *reinterpret_cast<uint32_t*>(&h3);
            // half of the math runs before the staging wait (register budget:
            // four warps per SMSP leave 128 registers a thread)
            if (j == 1) {
              wait_staging();
              *reinterpret_cast<uint4*>(stX + sw(lane, 0)) = dpk[0];
              *reinterpret_cast<uint4*>(stX + sw(lane, 1)) = dpk[1];
            } else if (j > 1) {
              *reinterpret_cast<uint4*>(stX + sw(lane, j)) = dpk[j];
            }
          }
        } else if (p.epi == kMul) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 pk = *reinterpret_cast<const uint4*>(stR + sw(lane, j));
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&pk);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __bfloat1622float2(h[e]);
              v[8 * j + 2 * e] *= f.x;
              v[8 * j + 2 * e + 1] *= f.y;
            }
          }
        } else if (p.epi == kRelu) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.f);
        } else if (p.epi == kMaskPos) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 pk = *reinterpret_cast<const uint4*>(stR + sw(lane, j));
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&pk);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __bfloat1622float2(h[e]);
              v[8 * j + 2 * e] = f.x > 0.f ? v[8 * j + 2 * e] : 0.f;
              v[8 * j + 2 * e + 1] = f.y > 0.f ? v[8 * j + 2 * e + 1] : 0.f;
            }
          }
        } else if (p.epi == kMulAdd) {
          // R2 row of this thread: 32 columns straight from global memory
          const int row = m0 + lane;
          uint4 q4[4] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0),
                         make_uint4(0, 0, 0, 0)};
          if (row < p.M) {
            const uint4* src = reinterpret_cast<const uint4*>(p.R2 + l * p.r2_ls + int64_t(row) * p.r2_ms + n0 + c);
#pragma unroll
            for (int j = 0; j < 4; ++j) q4[j] = __ldcs(src + j);
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 pk = *reinterpret_cast<const uint4*>(stR + sw(lane, j));
            if (p.AUX) {   // acc to AUX, in the 16 bytes of R this thread has just read
              uint4 ax;
              __nv_bfloat162 a0 = __floats2bfloat162_rn(v[8 * j], v[8 * j + 1]);
              __nv_bfloat162 a1 = __floats2bfloat162_rn(v[8 * j + 2], v[8 * j + 3]);
              __nv_bfloat162 a2 = __floats2bfloat162_rn(v[8 * j + 4], v[8 * j + 5]);
              __nv_bfloat162 a3 = __floats2bfloat162_rn(v[8 * j + 6], v[8 * j + 7]);
              ax.x = *reinterpret_cast<uint32_t*>(&a0); ax.y = *reinterpret_cast<uint32_t*>(&a1);
              ax.z = *reinterpret_cast<uint32_t*>(&a2); ax.w = *reinterpret_cast<uint32_t*>(&a3);
              *reinterpret_cast<uint4*>(stX + sw(lane, j)) = ax;
            }
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&pk);
            const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&q4[j]);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __bfloat1622float2(h[e]), g = __bfloat1622float2(h2[e]);
              v[8 * j + 2 * e] = fmaf(f.x, v[8 * j + 2 * e], g.x);
              v[8 * j + 2 * e + 1] = fmaf(f.y, v[8 * j + 2 * e + 1], g.y);
            }
          }
        } else if (p.epi == kDGelu) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 pk = *reinterpret_cast<const uint4*>(stR + sw(lane, j));
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&pk);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __bfloat1622float2(h[e]);
              float x0 = f.x, x1 = f.y, d0, d1;
              gelu_grad2<false>(x0, x1, d0, d1);
              v[8 * j + 2 * e] *= d0;
              v[8 * j + 2 * e + 1] *= d1;
            }
          }
        }
        wait_staging();
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 pk;
          __nv_bfloat162 h0 = __floats2bfloat162_rn(v[8 * j], v[8 * j + 1]);
          __nv_bfloat162 h1 = __floats2bfloat162_rn(v[8 * j + 2], v[8 * j + 3]);
          __nv_bfloat162 h2 = __floats2bfloat162_rn(v[8 * j + 4], v[8 * j + 5]);
          __nv_bfloat162 h3 = __floats2bfloat162_rn(v[8 * j + 6], v[8 * j + 7]);
          pk.x = *reinterpret_cast<uint32_t*>(&h0); pk.y = *reinterpret_cast<uint32_t*>(&h1);
          pk.z = *reinterpret_cast<uint32_t*>(&h2); pk.w = *reinterpret_cast<uint32_t*>(&h3);
          *reinterpret_cast<uint4*>(stC + sw(lane, j)) = pk;
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_rows(&tmC, stC, p.c_mode, n0 + c, m0, l);
          if ((p.epi == kGelu || p.epi == kGeluD || p.epi == kMulAdd) && p.AUX)
            tma_store_rows(&tmX, stX, p.x_mode, n0 + c, m0, l);
          bulk_commit();
        }
        ++kc;
        return true;
      };
      constexpr int kStep = kParts * 32;
      const int c0 = first_chunk();
      {
        bool ok = true;
#pragma unroll 1
        for (int c = c0; c < BN && ok; c += kStep) {
          uint32_t r0[32];
          tc_ld32_issue(tbase + c, r0);
          tc_ld_wait(r0);
          ok = process(r0, c);
        }
        if (!ok) break;
      }
      tc_fence_before();
      mbar_arrive(&tempty[a]);
    }
    // an R block still in flight (the loop ended early) lands before the CTA exits
    if (r_pending > 0) (void)mbar_wait(&rbar[kc & 1], uint32_t(kc >> 1) & 1u, p.err);
    if (lane == 0) bulk_wait_all();   // every store of this warp has completed
    __syncwarp();
  }
  // teardown: all roles are out of their loops (every wait above is bounded)
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}


// ---------------------------------------------------------------------------
// Weight gradient: C[l] (fp32, [M, N]) += sum over rows k of A[l][k, m] B[l][k, n]
// with A = dY [rows, M] and B = X [rows, N] both stored row-major, i.e. both
// operands MN-major (no transposes). The row dimension is long (every token of
// the batch) and the output small, so the work is split over K: a work item
// is (tile, k-range); items cycle over tiles first so concurrent CTAs hit
// different outputs. The epilogue adds its fp32 partial tile into C with
// vector reductions (red.global.add.v4.f32); C must be zeroed by the caller.
// Warp roles, TMEM double buffering and the bounded waits are those of
// gemm_kernel.
// ---------------------------------------------------------------------------
struct WgParams {
  int M, N, K, L;
  int m_blocks, n_blocks, k_blocks, tiles, splits, kb_per_split, items;
  int l_sum;        // 1: the L batches are part of the reduction (one output); k-blocks run over (l, k)
  int kb_per_l;     // k-blocks of one batch when l_sum
  float* C; int64_t c_ls, c_ms;
  int a_mode, b_mode;
  int* err;
};

__device__ __forceinline__ void wg_item(const WgParams& p, int w, int& l, int& mb, int& nb, int& kb0, int& kb1) {
  const int t = w % p.tiles;
  const int sp = w / p.tiles;
  nb = t % p.n_blocks;
  const int r = t / p.n_blocks;
  mb = r % p.m_blocks;
  l = p.l_sum ? 0 : r / p.m_blocks;
  kb0 = sp * p.kb_per_split;
  kb1 = min(kb0 + p.kb_per_split, p.k_blocks);
}

__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1) wgrad_kernel(const __grid_constant__ CUtensorMap tmA,
                                                            const __grid_constant__ CUtensorMap tmB,
                                                            const WgParams p) {
  constexpr uint32_t kABytes = BM * BK * 2;
  constexpr uint32_t kBBytes = BN * BK * 2;
  constexpr uint32_t kTmemCols = 2 * BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * kBBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;     // [2]
  uint64_t* tempty = tfull + 2;         // [2]
  uint64_t* mma_done = tempty + 2;      // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(&tfull[a], 1); mbar_init(&tempty[a], kEpiWarps * 32); }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmA) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmB) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(tmem_slot)), "r"(kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer: [64 k-rows][64 cols] boxes ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 1;
      int issued_on[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) issued_on[s] = 0;
      for (int w = blockIdx.x; w < p.items && !*abort_flag; w += gridDim.x) {
        int l, mb, nb, kb0, kb1;
        wg_item(p, w, l, mb, nb, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase, p.err)) { *abort_flag = 1; break; }
          mbar_expect_tx(&full[stage], kABytes + kBBytes);
          // with l_sum a k-block is (batch, block within the batch); rows past a batch's end load as zeros
          const int lb = p.l_sum ? kb / p.kb_per_l : l;
          const int kr = (p.l_sum ? kb % p.kb_per_l : kb) * BK;
#pragma unroll
          for (int g = 0; g < BM / 64; ++g)
            tma_load_rows(sA + stage * kABytes + g * 8192, &tmA, &full[stage], p.a_mode, mb * BM + 64 * g, kr, lb);
#pragma unroll
          for (int g = 0; g < BN / 64; ++g)
            tma_load_rows(sB + stage * kBBytes + g * 8192, &tmB, &full[stage], p.b_mode, nb * BN + 64 * g, kr, lb);
          ++issued_on[stage];
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (*abort_flag) {
#pragma unroll
        for (int s = 0; s < STAGES; ++s)
          if (issued_on[s] > 0) (void)mbar_wait(&full[s], uint32_t(issued_on[s] - 1) & 1u, p.err);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (A and B MN-major) ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(BM, BN) | (1u << 15) | (1u << 16);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int w = blockIdx.x; w < p.items && !*abort_flag; w += gridDim.x, ++local) {
        int l, mb, nb, kb0, kb1;
        wg_item(p, w, l, mb, nb, kb0, kb1);
        const int a = local & 1;
        const uint32_t ephase = ((local >> 1) & 1) ^ 1;
        if (!mbar_wait(&tempty[a], ephase, p.err)) { *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t d = tmem + uint32_t(a * BN);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err)) { *abort_flag = 1; ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * kABytes);
          const uint32_t b_addr = smem_u32(sB + stage * kBBytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            tc_mma(d, smem_desc_mn(a_addr + k * 2048), smem_desc_mn(b_addr + k * 2048), idesc,
                   (kb > kb0 || k > 0) ? 1u : 0u);
          tc_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit(&tfull[a]);
      }
      tc_commit(mma_done);
      (void)mbar_wait(mma_done, 0, p.err);
    }
  } else {
    // ---------------- epilogue: fp32 partial tile added into C ----------------
    const int ew = warp - 2;
    const int q = warp & 3;
    const int part = ew >> 2;
    constexpr int kParts = kEpiWarps / 4;
    int local = 0;
    for (int w = blockIdx.x; w < p.items; w += gridDim.x, ++local) {
      const int a = local & 1;
      if (!mbar_wait(&tfull[a], (local >> 1) & 1, p.err)) { *abort_flag = 1; break; }
      tc_fence_after();
      int l, mb, nb, kb0, kb1;
      wg_item(p, w, l, mb, nb, kb0, kb1);
      const int row = mb * BM + q * 32 + lane;
      const uint32_t tbase = tmem + (uint32_t(q * 32) << 16) + uint32_t(a * BN);
#pragma unroll 1
      for (int c = part * 32; c < BN; c += kParts * 32) {
        uint32_t r[32];
        tc_ld32_issue(tbase + c, r);
        tc_ld_wait(r);
        if (row < p.M && kb1 > kb0) {
          float* dst = p.C + l * p.c_ls + int64_t(row) * p.c_ms + nb * BN + c;
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            red_add_v4(dst + j, __uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                       __uint_as_float(r[j + 3]));
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[a]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

}  // namespace tc

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

// 3-D tensor map over bf16 rows of length K (strides in elements).  mode 0:
// dims {K, rows, L}; mode 1 (batch stride smaller than the row stride, e.g.
// one batch per NS token): dims {K, L, rows} so the strides stay ascending.
// Preconditions of cuTensorMapEncodeTiled checked on the host, so a bad view
// fails with a message instead of reaching the driver: 16-byte aligned base,
// extents in [1, 2^32), strides multiples of 16 bytes below 2^40, boxes of
// 1..256 elements.
void check_encode(const void* base, const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
                  int rank, const char* what) {
  PD_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "%s: base address not 16-byte aligned", what);
  for (int i = 0; i < rank; ++i) {
    PD_CHECK(dims[i] >= 1 && dims[i] < (cuuint64_t(1) << 32), "%s: extent %d out of range (%llu)", what, i,
             (unsigned long long)dims[i]);
    PD_CHECK(box[i] >= 1 && box[i] <= 256, "%s: box %d out of range (%u)", what, i, (unsigned)box[i]);
  }
  for (int i = 0; i + 1 < rank; ++i)
    PD_CHECK(strides[i] % 16 == 0 && strides[i] > 0 && strides[i] < (cuuint64_t(1) << 40),
             "%s: stride %d (%llu bytes) must be a positive multiple of 16 below 2^40", what, i,
             (unsigned long long)strides[i]);
}

// Every element a [L, rows, K] view addresses lies inside its storage (a TMA
// map of a view reaching past its allocation would read or write memory that
// is not the tensor's).
void check_extent(const at::Tensor& t, const char* name) {
  if (t.numel() == 0) return;
  int64_t last = t.storage_offset();
  for (int64_t d = 0; d < t.dim(); ++d) {
    PD_CHECK(t.stride(d) >= 0, "%s: negative strides are not supported", name);
    last += (t.size(d) - 1) * t.stride(d);
  }
  PD_CHECK(int64_t((last + 1) * t.element_size()) <= int64_t(t.storage().nbytes()),
           "%s: the view reaches past the end of its storage", name);
}

CUtensorMap make_map(const void* base, int64_t K, int64_t rows, int64_t L, int64_t row_stride, int64_t l_stride,
                     int box_rows, int& mode) {
  CUtensorMap m;
  if (L <= 1) l_stride = row_stride * rows;
  mode = (L > 1 && l_stride < row_stride) ? 1 : 0;
  cuuint64_t dims[3], strides[2];
  cuuint32_t box[3];
  if (mode == 0) {
    dims[0] = K; dims[1] = rows; dims[2] = L;
    strides[0] = row_stride * 2; strides[1] = l_stride * 2;
    box[0] = tc::BK; box[1] = box_rows; box[2] = 1;
  } else {
    dims[0] = K; dims[1] = L; dims[2] = rows;
    strides[0] = l_stride * 2; strides[1] = row_stride * 2;
    box[0] = tc::BK; box[1] = 1; box[2] = box_rows;
  }
  cuuint32_t estr[3] = {1, 1, 1};
  check_encode(base, dims, strides, box, 3, "operand map");
  CUresult r = tensor_map_encode_tiled(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                                      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  PD_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (%d): K=%lld rows=%lld L=%lld row_stride=%lld l_stride=%lld",
           int(r), (long long)K, (long long)rows, (long long)L, (long long)row_stride, (long long)l_stride);
  return m;
}

// Map of a [L, rows, N] bf16 epilogue operand (C / AUX stores, R loads):
// 32 x 32 boxes, 64-byte swizzle (the epilogue's staging layout); dim order
// as in make_map.
CUtensorMap make_store_map(const void* base, int64_t N, int64_t rows, int64_t L, int64_t row_stride,
                           int64_t l_stride, int& mode) {
  CUtensorMap m;
  if (L <= 1) l_stride = row_stride * rows;
  mode = (L > 1 && l_stride < row_stride) ? 1 : 0;
  cuuint64_t dims[3], strides[2];
  cuuint32_t box[3];
  if (mode == 0) {
    dims[0] = N; dims[1] = rows; dims[2] = L;
    strides[0] = row_stride * 2; strides[1] = l_stride * 2;
    box[0] = 32; box[1] = 32; box[2] = 1;
  } else {
    dims[0] = N; dims[1] = L; dims[2] = rows;
    strides[0] = l_stride * 2; strides[1] = row_stride * 2;
    box[0] = 32; box[1] = 1; box[2] = 32;
  }
  cuuint32_t estr[3] = {1, 1, 1};
  check_encode(base, dims, strides, box, 3, "epilogue map");
  CUresult r = tensor_map_encode_tiled(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                                      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                                      CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  PD_CHECK(r == CUDA_SUCCESS,
           "cuTensorMapEncodeTiled (store) failed (%d): N=%lld rows=%lld L=%lld row_stride=%lld l_stride=%lld",
           int(r), (long long)N, (long long)rows, (long long)L, (long long)row_stride, (long long)l_stride);
  return m;
}

// [L, rows, K] view (L may be 1): unit stride on K, 16-byte aligned rows.
void check_operand(const at::Tensor& t, const char* name) {
  PD_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16, "%s: bf16 CUDA tensor required", name);
  PD_CHECK(t.dim() == 3 && t.stride(2) == 1, "%s: [L, rows, K] with unit stride on K required", name);
  PD_CHECK(t.stride(1) % 8 == 0 && (t.size(0) == 1 || t.stride(0) % 8 == 0) &&
              reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, "%s: rows must be 16-byte aligned", name);
  PD_CHECK(t.size(2) % 8 == 0, "%s: K must be a multiple of 8", name);
  check_extent(t, name);
}

template <int BN, int STAGES>
void launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tcm, const CUtensorMap& txm,
            const CUtensorMap& trm, const tc::Params& p) {
  constexpr size_t smem = STAGES * (tc::BM * tc::BK * 2 + BN * tc::BK * 2) + 1024 + 1024 + tc::kEpiWarps * 3 * 2048;
  static_assert(smem <= 232448, "GEMM shared memory over the 227 KB per-block limit");
  static bool attr = false;
  if (!attr) {
    PD_CHECK_CUDA(cudaFuncSetAttribute(tc::gemm_kernel<BN, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(smem)));
    attr = true;
  }
  int grid = p.tiles < num_sms() ? p.tiles : num_sms();
  tc::gemm_kernel<BN, STAGES><<<grid, tc::kThreads, smem, stream()>>>(ta, tb, tcm, txm, trm, p);
  PD_CHECK_LAUNCH();
}

}  // namespace

// C[l, m, :N] = epi(A[l] @ B[l]^T).  A: [L, M, K], B: [L or 1, N, K] -- or, with b_kn,
// [L or 1, K, N] (a weight used transposed, read MN-major) -- C/R/AUX: [L, M, N] views
// (unit column stride).  epi: 0 none, 1 gelu (aux = pre-activation, optional), 2 residual (R),
// 3 dgelu (R = pre-activation), 4 gelu storing gelu' in AUX, 5 product with R, 6 relu (R = bias
// addend), 7 acc where R > 0, 8 R * acc + R2 (AUX: acc, optional).
void tc_gemm(at::Tensor A, at::Tensor B, at::Tensor C, int64_t epi, c10::optional<at::Tensor> R,
             c10::optional<at::Tensor> AUX, at::Tensor err, bool b_kn, c10::optional<at::Tensor> R2) {
  check_operand(A, "A");
  check_operand(B, "B");
  const int64_t L = A.size(0), M = A.size(1), K = A.size(2), N = b_kn ? B.size(2) : B.size(1);
  TORCH_CHECK((b_kn ? B.size(1) : B.size(2)) == K && (B.size(0) == L || B.size(0) == 1),
              b_kn ? "B must be [L or 1, K, N]" : "B must be [L or 1, N, K]");
  TORCH_CHECK(N % 64 == 0, "N must be a multiple of 64");
  TORCH_CHECK(C.dim() == 3 && C.size(0) == L && C.size(1) == M && C.size(2) == N && C.stride(2) == 1 &&
              C.scalar_type() == at::kBFloat16 && C.stride(1) % 8 == 0 && (C.size(0) == 1 || C.stride(0) % 8 == 0) &&
              reinterpret_cast<uintptr_t>(C.data_ptr()) % 16 == 0, "C must be a [L, M, N] bf16 view with aligned rows");
  check_extent(C, "C");
  if (R && R->defined()) check_extent(*R, "R");
  if (AUX && AUX->defined()) check_extent(*AUX, "AUX");
  tc::Params p{};
  p.M = int(M); p.N = int(N); p.K = int(K); p.L = int(L);
  p.m_blocks = int((M + tc::BM - 1) / tc::BM);
  p.k_blocks = int((K + tc::BK - 1) / tc::BK);
  p.C = reinterpret_cast<__nv_bfloat16*>(C.data_ptr()); p.c_ls = C.stride(0); p.c_ms = C.stride(1);
  p.epi = int(epi);
  p.err = err.data_ptr<int>();
  PD_CHECK(epi >= tc::kNone && epi <= tc::kMulAdd, "unknown epilogue %lld", (long long)epi);
  TORCH_CHECK(!(epi == tc::kResidual || epi == tc::kDGelu || epi == tc::kMul || epi == tc::kMaskPos ||
                epi == tc::kMulAdd) || (R && R->defined()),
              "this epilogue needs R");
  TORCH_CHECK(epi != tc::kMulAdd || (R2 && R2->defined()), "the multiply-add epilogue needs R2");
  if (epi == tc::kMulAdd) {
    TORCH_CHECK(R2->dim() == 3 && R2->sizes() == C.sizes() && R2->stride(2) == 1 && R2->stride(1) % 8 == 0 &&
                (R2->size(0) == 1 || R2->stride(0) % 8 == 0) && reinterpret_cast<uintptr_t>(R2->data_ptr()) % 16 == 0 &&
                R2->scalar_type() == at::kBFloat16, "R2 must match C (bf16, 16-byte aligned rows)");
    check_extent(*R2, "R2");
    p.R2 = reinterpret_cast<const __nv_bfloat16*>(R2->data_ptr()); p.r2_ls = R2->stride(0); p.r2_ms = R2->stride(1);
    TORCH_CHECK(R->stride(1) != 0 && (L == 1 || R->stride(0) != 0), "the multiply-add factor R must be a full matrix");
  }
  TORCH_CHECK(epi != tc::kGeluD || (AUX && AUX->defined()), "the GELU-derivative epilogue needs AUX");
  if (R && R->defined()) {
    // R: [L, M, N] view (stride 0 allowed on L and M: a bias or per-row-block addend)
    TORCH_CHECK(R->dim() == 3 && R->sizes() == C.sizes() && R->stride(2) == 1 && R->stride(1) % 8 == 0 &&
                (R->size(0) == 1 || R->stride(0) % 8 == 0) && reinterpret_cast<uintptr_t>(R->data_ptr()) % 16 == 0 &&
                R->scalar_type() == at::kBFloat16, "R must match C (bf16, 16-byte aligned rows)");
    p.R = reinterpret_cast<const __nv_bfloat16*>(R->data_ptr()); p.r_ls = R->stride(0); p.r_ms = R->stride(1);
  }
  if (AUX && AUX->defined()) {
    TORCH_CHECK(AUX->dim() == 3 && AUX->sizes() == C.sizes() && AUX->stride(2) == 1 && AUX->stride(1) % 8 == 0 &&
                (AUX->size(0) == 1 || AUX->stride(0) % 8 == 0) && reinterpret_cast<uintptr_t>(AUX->data_ptr()) % 16 == 0,
                "AUX must match C (16-byte aligned rows)");
    p.AUX = reinterpret_cast<__nv_bfloat16*>(AUX->data_ptr()); p.aux_ls = AUX->stride(0); p.aux_ms = AUX->stride(1);
  }
  if (M == 0 || L == 0) return;
  const int BN = (N % 256 == 0) ? 256 : (N % 128 == 0 ? 128 : 64);
  p.n_blocks = int(N / BN);
  p.tiles = int(L) * p.m_blocks * p.n_blocks;
  const CUtensorMap ta = make_map(A.data_ptr(), K, M, L, A.stride(1), A.stride(0), tc::BM, p.a_mode);
  p.b_kn = b_kn ? 1 : 0;
  // MN-major B: boxes of 64 n x 64 k-rows over dims {N, K, L}
  const CUtensorMap tb = b_kn ? make_map(B.data_ptr(), N, K, B.size(0), B.stride(1), B.stride(0), tc::BK, p.b_mode)
                              : make_map(B.data_ptr(), K, N, B.size(0), B.stride(1), B.stride(0), BN, p.b_mode);
  p.b_shared = (B.size(0) == 1) ? 1 : 0;
  const CUtensorMap tcm = make_store_map(C.data_ptr(), N, M, L, C.stride(1), C.stride(0), p.c_mode);
  p.x_mode = p.c_mode;
  const CUtensorMap txm = p.AUX ? make_store_map(AUX->data_ptr(), N, M, L, AUX->stride(1), AUX->stride(0), p.x_mode)
                                : tcm;
  // R by TMA unless it broadcasts through a zero stride (bias / positional addend)
  p.r_tma = (p.R && p.r_ms != 0 && (L == 1 || p.r_ls != 0)) ? 1 : 0;
  p.r_mode = 0;
  const CUtensorMap trm = p.r_tma ? make_store_map(R->data_ptr(), N, M, L, R->stride(1), R->stride(0), p.r_mode) : tcm;
  if (BN == 256) launch<256, 3>(ta, tb, tcm, txm, trm, p);
  else if (BN == 128) launch<128, 4>(ta, tb, tcm, txm, trm, p);
  else launch<64, 6>(ta, tb, tcm, txm, trm, p);
}


// C[l] (fp32 [M, N], zeroed by the caller) += A[l]^T B[l] over the rows:
// A [L, K, M], B [L, K, N] bf16 views with unit stride on the last dim.
// With l_sum, C is [1, M, N] and the sum runs over the batches as well.
void tc_wgrad(at::Tensor A, at::Tensor B, at::Tensor C, at::Tensor err, bool l_sum) {
  check_operand(A, "A");
  check_operand(B, "B");
  const int64_t L = A.size(0), K = A.size(1), M = A.size(2), N = B.size(2);
  TORCH_CHECK(B.size(0) == L && B.size(1) == K, "B must be [L, K, N] over the same rows as A");
  TORCH_CHECK(M % 64 == 0 && N % 64 == 0, "wgrad: M and N must be multiples of 64");
  const int64_t LC = l_sum ? 1 : L;
  TORCH_CHECK(C.scalar_type() == at::kFloat && C.dim() == 3 && C.size(0) == LC && C.size(1) == M && C.size(2) == N &&
                  C.stride(2) == 1 && C.stride(1) % 4 == 0 && (LC == 1 || C.stride(0) % 4 == 0) &&
                  reinterpret_cast<uintptr_t>(C.data_ptr()) % 16 == 0,
              "wgrad: C must be an fp32 [L, M, N] view with 16-byte aligned rows");
  if (K == 0 || L == 0) return;
  tc::WgParams p{};
  p.M = int(M); p.N = int(N); p.K = int(K); p.L = int(L);
  p.m_blocks = int((M + tc::BM - 1) / tc::BM);
  const int BN = (N % 256 == 0) ? 256 : (N % 128 == 0 ? 128 : 64);
  p.n_blocks = int(N / BN);
  p.l_sum = l_sum ? 1 : 0;
  p.kb_per_l = int((K + tc::BK - 1) / tc::BK);
  p.k_blocks = l_sum ? int(L) * p.kb_per_l : p.kb_per_l;
  p.tiles = int(LC) * p.m_blocks * p.n_blocks;
  // about two items per SM without a ragged last wave, each at least 8 k-blocks long
  int splits = std::max(1, (2 * num_sms()) / p.tiles);
  splits = std::min(splits, std::max(1, p.k_blocks / 8));
  p.kb_per_split = (p.k_blocks + splits - 1) / splits;
  p.splits = (p.k_blocks + p.kb_per_split - 1) / p.kb_per_split;
  p.items = p.tiles * p.splits;
  p.C = C.data_ptr<float>(); p.c_ls = C.stride(0); p.c_ms = C.stride(1);
  p.err = err.data_ptr<int>();
  // MN-major operands: [64 k-rows][64 cols] boxes over dims {cols, rows, L}
  const CUtensorMap ta = make_map(A.data_ptr(), M, K, L, A.stride(1), A.stride(0), tc::BK, p.a_mode);
  const CUtensorMap tb = make_map(B.data_ptr(), N, K, L, B.stride(1), B.stride(0), tc::BK, p.b_mode);
  auto go = [&](auto kern, int bn, int stages) {
    const size_t smem = size_t(stages) * (tc::BM * tc::BK * 2 + bn * tc::BK * 2) + 1024 + 1024;
    PD_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    const int grid = p.items < num_sms() ? p.items : num_sms();
    kern<<<grid, tc::kThreads, smem, stream()>>>(ta, tb, p);
  };
  if (BN == 256) go(tc::wgrad_kernel<256, 4>, 256, 4);
  else if (BN == 128) go(tc::wgrad_kernel<128, 6>, 128, 6);
  else go(tc::wgrad_kernel<64, 8>, 64, 8);
  PD_CHECK_LAUNCH();
}

}  // namespace pd
