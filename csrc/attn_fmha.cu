// Pyramid causal attention (OneTrans), forward + backward, for sm_100a.
//
// Semantics (primus_dlrm/models/onetrans.py:62-67,146-166): the queries are
// the LAST q_len of kv_len tokens; query i (absolute position
// p = kv_len - q_len + i) attends keys j <= p (causal mask aligned bottom-
// right); scale 1/sqrt(d).
//
// Why this shape of kernel: with head_dim 32 a 128x128 score tile needs 16K
// exponentials but only 2 MFLOP of matrix math, so on B200 the exp unit (16
// ex2 per clock per SM) is ~4x slower than the tensor pipe even at legacy
// mma.sync rates. The kernel is therefore built around keeping the exp pipe
// busy: scores and probabilities never leave registers (the accumulator
// fragment of QK^T is re-used as the A fragment of PV), the softmax scale and
// log2(e) are folded into one FMA, masking is applied only on tiles that cross
// the diagonal, and KV tiles beyond a query tile's last visible key are never
// loaded (pyramid + causal skipping).
//
// Layout: Q/K/V are read in place from the fused projection output
// [B, T, 3, H, d] (any batch / row stride, unit stride on d); O is written as
// [B, q_len, H, d]; LSE (log2 domain) as [B, H, q_len]. The backward writes
// dK/dV (and dQ after the fp32 accumulation pass) straight into the gradient
// of the fused QKV buffer, zero-filling the Q rows that the pyramid pruned.
#include "common.cuh"

#include <cstdlib>

namespace pd {
namespace attn {

struct alignas(16) U4 { uint32_t x, y, z, w; };

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void ldsm_x4(uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d) : "r"(smem_u32(p)));
}
// D(16x8 f32) += A(16x16 bf16, row) * B(16x8 bf16, col)
__device__ __forceinline__ void mma16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm volatile("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Swizzled smem tile of R rows x D bf16 (row = D*2 bytes, 16-byte chunks).
// Chunk c of row r lives at chunk (c ^ f(r)); f spreads the 8 rows read by
// one ldmatrix phase over all 32 banks.
template <int D>
struct Tile {
  static constexpr int kChunks = D / 8;  // 16-byte chunks per row
  __device__ static __forceinline__ int swz(int r, int c) {
    if constexpr (D == 32) return c ^ ((r >> 1) & 3);
    else return c ^ (r & 7);
  }
  __device__ static __forceinline__ int off(int r, int c) { return r * D + swz(r, c) * 8; }  // in elements
};

// Copy rows [r0, r0+R) of a [*, D] strided bf16 matrix into a swizzled tile;
// rows >= n_rows are zero-filled.
template <int D, int R, int NT>
__device__ __forceinline__ void load_tile(__nv_bfloat16* s, const __nv_bfloat16* g, int64_t rstride, int r0,
                                          int n_rows, int tid) {
  constexpr int C = D / 8;
#pragma unroll
  for (int i = tid; i < R * C; i += NT) {
    const int r = i / C, c = i % C;
    const bool ok = (r0 + r) < n_rows;
    const __nv_bfloat16* src = g + int64_t(ok ? r0 + r : 0) * rstride + c * 8;
    cp_async16(s + Tile<D>::off(r, c), src, ok);
  }
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
struct FwdArgs {
  const __nv_bfloat16* q; const __nv_bfloat16* k; const __nv_bfloat16* v;
  int64_t q_bs, q_rs, kv_bs, kv_rs;
  __nv_bfloat16* o; int64_t o_bs, o_rs;
  float* lse;  // [B, H, q_len] (log2 domain)
  int H, q_len, kv_len;
  float scale_log2;
};

constexpr int kFwdM = 128;  // queries per CTA (8 warps x 16)
constexpr int kFwdN = 64;   // keys per tile

// WARPS warps of 16 query rows each per CTA (8: 128 queries; 4: 64 queries,
// twice the CTAs, so a barrier stalls half as many warps).
template <int D, int WARPS = 8>
__global__ void __launch_bounds__(32 * WARPS, D == 32 ? 24 / WARPS : 1) fmha_fwd_kernel(const FwdArgs A) {
  constexpr int kFwdM = 16 * WARPS;
  constexpr int NT = 32 * WARPS;
  constexpr int NKS = D / 16;   // k-steps over d for QK^T
  constexpr int NDT = D / 8;    // n-tiles over d for PV
  __shared__ alignas(128) __nv_bfloat16 sQ[kFwdM * D];
  __shared__ alignas(128) __nv_bfloat16 sK[2][kFwdN * D];
  __shared__ alignas(128) __nv_bfloat16 sV[2][kFwdN * D];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.y, b = bh / A.H, h = bh % A.H;
  const int i0 = blockIdx.x * kFwdM;
  const int shift = A.kv_len - A.q_len;  // absolute position of query row 0
  const __nv_bfloat16* qg = A.q + b * A.q_bs + int64_t(h) * D;
  const __nv_bfloat16* kg = A.k + b * A.kv_bs + int64_t(h) * D;
  const __nv_bfloat16* vg = A.v + b * A.kv_bs + int64_t(h) * D;
  const int last_key = min(A.kv_len - 1, shift + min(i0 + kFwdM, A.q_len) - 1);
  const int n_tiles = last_key / kFwdN + 1;

  load_tile<D, kFwdM, NT>(sQ, qg, A.q_rs, i0, A.q_len, tid);
  load_tile<D, kFwdN, NT>(sK[0], kg, A.kv_rs, 0, A.kv_len, tid);
  load_tile<D, kFwdN, NT>(sV[0], vg, A.kv_rs, 0, A.kv_len, tid);
  cp_async_commit();

  // Q fragments (A operand) for this warp's 16 rows
  uint32_t qf[NKS][4];
  float o[NDT][4];
#pragma unroll
  for (int t = 0; t < NDT; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  const int g = lane >> 2, tq = lane & 3;
  const int row_a = i0 + warp * 16 + g;       // query rows held by this thread
  const int pos0 = shift + row_a, pos1 = pos0 + 8;
  const int warp_last = shift + i0 + warp * 16 + 15;

  for (int j = 0; j < n_tiles; ++j) {
    const int buf = j & 1;
    if (j + 1 < n_tiles) {
      load_tile<D, kFwdN, NT>(sK[buf ^ 1], kg, A.kv_rs, (j + 1) * kFwdN, A.kv_len, tid);
      load_tile<D, kFwdN, NT>(sV[buf ^ 1], vg, A.kv_rs, (j + 1) * kFwdN, A.kv_len, tid);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int ks = 0; ks < NKS; ++ks) {
        const int r = warp * 16 + (lane & 15);
        const int c = ks * 2 + (lane >> 4);
        ldsm_x4(qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], sQ + Tile<D>::off(r, c));
      }
    }
    const int k0 = j * kFwdN;
    if (k0 <= warp_last) {
      // S = Q K^T : 16 x 64 per warp
      float s[8][4];
#pragma unroll
      for (int t = 0; t < 8; ++t) s[t][0] = s[t][1] = s[t][2] = s[t][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < NKS; ++ks) {
#pragma unroll
        for (int tp = 0; tp < 4; ++tp) {  // pairs of n-tiles (16 keys)
          uint32_t b0, b1, b2, b3;
          const int r = tp * 16 + (lane & 7) + ((lane >> 4) << 3);
          const int c = ks * 2 + ((lane >> 3) & 1);
          ldsm_x4(b0, b1, b2, b3, sK[buf] + Tile<D>::off(r, c));
          mma16816(s[2 * tp], qf[ks], b0, b1);
          mma16816(s[2 * tp + 1], qf[ks], b2, b3);
        }
      }
      // mask: keys beyond the row's position (diagonal tiles) or beyond kv_len
      const bool need_mask = (k0 + kFwdN - 1 > shift + i0 + warp * 16) || (k0 + kFwdN > A.kv_len);
      if (need_mask) {
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const int c0 = k0 + t * 8 + 2 * tq;
          if (c0 > pos0 || c0 >= A.kv_len) s[t][0] = -INFINITY;
          if (c0 + 1 > pos0 || c0 + 1 >= A.kv_len) s[t][1] = -INFINITY;
          if (c0 > pos1 || c0 >= A.kv_len) s[t][2] = -INFINITY;
          if (c0 + 1 > pos1 || c0 + 1 >= A.kv_len) s[t][3] = -INFINITY;
        }
      }
      // online softmax (rows g and g+8 of the warp tile)
      float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        mx[0] = fmaxf(mx[0], fmaxf(s[t][0], s[t][1]));
        mx[1] = fmaxf(mx[1], fmaxf(s[t][2], s[t][3]));
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
        mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
      }
      float alpha[2], off[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        off[i] = mx[i] == -INFINITY ? 0.f : mx[i] * A.scale_log2;
        alpha[i] = ex2(m_r[i] * A.scale_log2 - off[i]);
        m_r[i] = mx[i];
      }
      float rs[2] = {0.f, 0.f};
      uint32_t pf[4][4];  // P as A fragments: 4 k-steps of 16 keys
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const float p0 = ex2(fmaf(s[t][0], A.scale_log2, -off[0]));
        const float p1 = ex2(fmaf(s[t][1], A.scale_log2, -off[0]));
        const float p2 = ex2(fmaf(s[t][2], A.scale_log2, -off[1]));
        const float p3 = ex2(fmaf(s[t][3], A.scale_log2, -off[1]));
        rs[0] += p0 + p1;
        rs[1] += p2 + p3;
        const int ks = t >> 1;
        if ((t & 1) == 0) { pf[ks][0] = pack_bf16(p0, p1); pf[ks][1] = pack_bf16(p2, p3); }
        else { pf[ks][2] = pack_bf16(p0, p1); pf[ks][3] = pack_bf16(p2, p3); }
      }
      l_r[0] = l_r[0] * alpha[0] + rs[0];
      l_r[1] = l_r[1] * alpha[1] + rs[1];
#pragma unroll
      for (int t = 0; t < NDT; ++t) {
        o[t][0] *= alpha[0]; o[t][1] *= alpha[0];
        o[t][2] *= alpha[1]; o[t][3] *= alpha[1];
      }
      // O += P V
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
        for (int tp = 0; tp < NDT / 2; ++tp) {
          uint32_t b0, b1, b2, b3;
          const int r = ks * 16 + (lane & 15);
          const int c = tp * 2 + (lane >> 4);
          ldsm_x4_t(b0, b1, b2, b3, sV[buf] + Tile<D>::off(r, c));
          mma16816(o[2 * tp], pf[ks], b0, b1);
          mma16816(o[2 * tp + 1], pf[ks], b2, b3);
        }
      }
    }
    __syncthreads();
  }
  // epilogue
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    l_r[i] += __shfl_xor_sync(0xffffffffu, l_r[i], 1);
    l_r[i] += __shfl_xor_sync(0xffffffffu, l_r[i], 2);
  }
  const float inv0 = l_r[0] > 0.f ? 1.f / l_r[0] : 0.f;
  const float inv1 = l_r[1] > 0.f ? 1.f / l_r[1] : 0.f;
  const int r0 = row_a, r1 = row_a + 8;
  __nv_bfloat16* og = A.o + b * A.o_bs + int64_t(h) * D;
#pragma unroll
  for (int t = 0; t < NDT; ++t) {
    const int c = t * 8 + 2 * tq;
    if (r0 < A.q_len)
      *reinterpret_cast<uint32_t*>(og + int64_t(r0) * A.o_rs + c) = pack_bf16(o[t][0] * inv0, o[t][1] * inv0);
    if (r1 < A.q_len)
      *reinterpret_cast<uint32_t*>(og + int64_t(r1) * A.o_rs + c) = pack_bf16(o[t][2] * inv1, o[t][3] * inv1);
  }
  if (tq == 0) {
    float* lg = A.lse + (int64_t(b) * A.H + h) * A.q_len;
    if (r0 < A.q_len) lg[r0] = l_r[0] > 0.f ? m_r[0] * A.scale_log2 + __log2f(l_r[0]) : INFINITY;
    if (r1 < A.q_len) lg[r1] = l_r[1] > 0.f ? m_r[1] * A.scale_log2 + __log2f(l_r[1]) : INFINITY;
  }
}

// ---------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------
struct BwdArgs {
  const __nv_bfloat16* q; const __nv_bfloat16* k; const __nv_bfloat16* v;
  int64_t q_bs, q_rs, kv_bs, kv_rs;
  const __nv_bfloat16* o; const __nv_bfloat16* dout; int64_t o_bs, o_rs;
  const float* lse; float* delta;        // [B, H, q_len]
  float* dq_acc;                          // [B, q_len, H, D] fp32
  __nv_bfloat16* dk; __nv_bfloat16* dv;   // strided like k / v (dqkv buffer)
  int64_t dkv_bs, dkv_rs;
  int H, q_len, kv_len;
  float scale_log2, scale;
};

// delta[b, h, i] = sum_d dO * O
template <int D>
__global__ void fmha_bwd_pre_kernel(const BwdArgs A) {
  const int bh = blockIdx.y, b = bh / A.H, h = bh % A.H;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < A.q_len; i += gridDim.x * blockDim.x) {
    const __nv_bfloat16* og = A.o + b * A.o_bs + int64_t(i) * A.o_rs + h * D;
    const __nv_bfloat16* dg = A.dout + b * A.o_bs + int64_t(i) * A.o_rs + h * D;
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < D; c += 8) {
      float4 a = load4_bf16(og + c), a2 = load4_bf16(og + c + 4);
      float4 d = load4_bf16(dg + c), d2 = load4_bf16(dg + c + 4);
      s += a.x * d.x + a.y * d.y + a.z * d.z + a.w * d.w + a2.x * d2.x + a2.y * d2.y + a2.z * d2.z + a2.w * d2.w;
    }
    A.delta[(int64_t(b) * A.H + h) * A.q_len + i] = s;
  }
}

constexpr int kBwdN = 64;  // keys per CTA (4 warps x 16)
constexpr int kBwdM = 64;  // queries per inner tile

template <int D>
__global__ void __launch_bounds__(128) fmha_bwd_kernel(const BwdArgs A) {
  constexpr int NKS = D / 16;
  constexpr int NDT = D / 8;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  __nv_bfloat16* sV = sK + kBwdN * D;
  __nv_bfloat16* sQb = sV + kBwdN * D;           // [2][kBwdM * D]
  __nv_bfloat16* sdOb = sQb + 2 * kBwdM * D;     // [2][kBwdM * D]
  __nv_bfloat16* sdS = sdOb + 2 * kBwdM * D;     // dS^T [kv][q], swizzled as 64-wide rows
  float* sLb = reinterpret_cast<float*>(sdS + kBwdN * kBwdM);  // [2][kBwdM]
  float* sDlb = sLb + 2 * kBwdM;                               // [2][kBwdM]
  auto sQ = [&](int i) { return sQb + i * kBwdM * D; };
  auto sdO = [&](int i) { return sdOb + i * kBwdM * D; };
  auto sL = [&](int i) { return sLb + i * kBwdM; };
  auto sDl = [&](int i) { return sDlb + i * kBwdM; };
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.y, b = bh / A.H, h = bh % A.H;
  const int j0 = blockIdx.x * kBwdN;
  const int shift = A.kv_len - A.q_len;
  const __nv_bfloat16* qg = A.q + b * A.q_bs + int64_t(h) * D;
  const __nv_bfloat16* kg = A.k + b * A.kv_bs + int64_t(h) * D;
  const __nv_bfloat16* vg = A.v + b * A.kv_bs + int64_t(h) * D;
  const __nv_bfloat16* dog = A.dout + b * A.o_bs + int64_t(h) * D;
  const float* lg = A.lse + (int64_t(b) * A.H + h) * A.q_len;
  const float* dlg = A.delta + (int64_t(b) * A.H + h) * A.q_len;
  // first query row that sees key j0: i >= j0 - shift
  const int i_first = max(0, j0 - shift);
  const int t_first = i_first / kBwdM;
  const int n_qt = (A.q_len + kBwdM - 1) / kBwdM;
  const int g = lane >> 2, tq = lane & 3;

  load_tile<D, kBwdN, 128>(sK, kg, A.kv_rs, j0, A.kv_len, tid);
  load_tile<D, kBwdN, 128>(sV, vg, A.kv_rs, j0, A.kv_len, tid);
  if (t_first < n_qt) {
    load_tile<D, kBwdM, 128>(sQ(0), qg, A.q_rs, t_first * kBwdM, A.q_len, tid);
    load_tile<D, kBwdM, 128>(sdO(0), dog, A.o_rs, t_first * kBwdM, A.q_len, tid);
  }
  cp_async_commit();

  float dk[NDT][4], dv[NDT][4];
#pragma unroll
  for (int t = 0; t < NDT; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) { dk[t][e] = 0.f; dv[t][e] = 0.f; }
  uint32_t kf[NKS][4], vf[NKS][4];
  const int key_a = j0 + warp * 16 + g;  // keys held by this thread (rows of S^T)

  for (int qt = t_first; qt < n_qt; ++qt) {
    const int buf = (qt - t_first) & 1;
    const int q0 = qt * kBwdM;
    if (tid < kBwdM) {
      const int i = q0 + tid;
      sL(buf)[tid] = i < A.q_len ? lg[i] : INFINITY;
      sDl(buf)[tid] = i < A.q_len ? dlg[i] : 0.f;
    }
    if (qt + 1 < n_qt) {
      load_tile<D, kBwdM, 128>(sQ(buf ^ 1), qg, A.q_rs, q0 + kBwdM, A.q_len, tid);
      load_tile<D, kBwdM, 128>(sdO(buf ^ 1), dog, A.o_rs, q0 + kBwdM, A.q_len, tid);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (qt == t_first) {
#pragma unroll
      for (int ks = 0; ks < NKS; ++ks) {
        const int r = warp * 16 + (lane & 15);
        const int c = ks * 2 + (lane >> 4);
        ldsm_x4(kf[ks][0], kf[ks][1], kf[ks][2], kf[ks][3], sK + Tile<D>::off(r, c));
        ldsm_x4(vf[ks][0], vf[ks][1], vf[ks][2], vf[ks][3], sV + Tile<D>::off(r, c));
      }
    }
    // S^T = K Q^T and dP^T = V dO^T : 16 keys x 64 queries per warp
    float s[8][4], dp[8][4];
#pragma unroll
    for (int t = 0; t < 8; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) { s[t][e] = 0.f; dp[t][e] = 0.f; }
#pragma unroll
    for (int ks = 0; ks < NKS; ++ks) {
#pragma unroll
      for (int tp = 0; tp < 4; ++tp) {
        uint32_t b0, b1, b2, b3;
        const int r = tp * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = ks * 2 + ((lane >> 3) & 1);
        ldsm_x4(b0, b1, b2, b3, sQ(buf) + Tile<D>::off(r, c));
        mma16816(s[2 * tp], kf[ks], b0, b1);
        mma16816(s[2 * tp + 1], kf[ks], b2, b3);
        ldsm_x4(b0, b1, b2, b3, sdO(buf) + Tile<D>::off(r, c));
        mma16816(dp[2 * tp], vf[ks], b0, b1);
        mma16816(dp[2 * tp + 1], vf[ks], b2, b3);
      }
    }
    // P^T = exp2(S^T * c - lse[q]) with the causal mask; dS^T = P^T (dP^T - delta[q])
    uint32_t pf[4][4], dsf[4][4];
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      float p[4], ds[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi = t * 8 + 2 * tq + (e & 1);          // query column within tile
        const int key = key_a + ((e >> 1) << 3);
        const int qa = q0 + qi;                            // query row
        const bool ok = qa < A.q_len && key < A.kv_len && key <= shift + qa;
        p[e] = ok ? ex2(fmaf(s[t][e], A.scale_log2, -sL(buf)[qi])) : 0.f;
        ds[e] = p[e] * (dp[t][e] - sDl(buf)[qi]);
      }
      const int ks = t >> 1;
      if ((t & 1) == 0) {
        pf[ks][0] = pack_bf16(p[0], p[1]); pf[ks][1] = pack_bf16(p[2], p[3]);
        dsf[ks][0] = pack_bf16(ds[0], ds[1]); dsf[ks][1] = pack_bf16(ds[2], ds[3]);
      } else {
        pf[ks][2] = pack_bf16(p[0], p[1]); pf[ks][3] = pack_bf16(p[2], p[3]);
        dsf[ks][2] = pack_bf16(ds[0], ds[1]); dsf[ks][3] = pack_bf16(ds[2], ds[3]);
      }
      // stash dS^T (bf16) for the dQ product: row = key (warp*16+g / +8), col = query
      const int rr = warp * 16 + g;
      const int cc = t * 8 + 2 * tq;
      *reinterpret_cast<uint32_t*>(sdS + Tile<64>::off(rr, cc >> 3) + (cc & 7)) = pack_bf16(ds[0], ds[1]);
      *reinterpret_cast<uint32_t*>(sdS + Tile<64>::off(rr + 8, cc >> 3) + (cc & 7)) = pack_bf16(ds[2], ds[3]);
    }
    // dV += P^T dO ; dK += dS^T Q   (B operands: dO / Q [q, d] via transposed ldmatrix)
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
      for (int tp = 0; tp < NDT / 2; ++tp) {
        uint32_t b0, b1, b2, b3;
        const int r = ks * 16 + (lane & 15);
        const int c = tp * 2 + (lane >> 4);
        ldsm_x4_t(b0, b1, b2, b3, sdO(buf) + Tile<D>::off(r, c));
        mma16816(dv[2 * tp], pf[ks], b0, b1);
        mma16816(dv[2 * tp + 1], pf[ks], b2, b3);
        ldsm_x4_t(b0, b1, b2, b3, sQ(buf) + Tile<D>::off(r, c));
        mma16816(dk[2 * tp], dsf[ks], b0, b1);
        mma16816(dk[2 * tp + 1], dsf[ks], b2, b3);
      }
    }
    __syncthreads();
    // dQ[q, d] += dS[q, kv] K[kv, d]: warp w takes queries 16w..16w+15
    {
      float dq[NDT][4];
#pragma unroll
      for (int t = 0; t < NDT; ++t) dq[t][0] = dq[t][1] = dq[t][2] = dq[t][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {  // 64 keys in 4 k-steps
        uint32_t a[4];
        // A = dS (q rows, kv cols) = transpose of sdS[kv][q]
        {
          const int r = ks * 16 + (lane & 7) + ((lane >> 4) << 3);   // kv row of sdS
          const int c = warp * 2 + ((lane >> 3) & 1);                // q chunk
          ldsm_x4_t(a[0], a[1], a[2], a[3], sdS + Tile<64>::off(r, c));
        }
#pragma unroll
        for (int tp = 0; tp < NDT / 2; ++tp) {
          uint32_t b0, b1, b2, b3;
          const int r = ks * 16 + (lane & 15);
          const int c = tp * 2 + (lane >> 4);
          ldsm_x4_t(b0, b1, b2, b3, sK + Tile<D>::off(r, c));
          mma16816(dq[2 * tp], a, b0, b1);
          mma16816(dq[2 * tp + 1], a, b2, b3);
        }
      }
      const int qa0 = q0 + warp * 16 + g, qa1 = qa0 + 8;
#pragma unroll
      for (int t = 0; t < NDT; ++t) {
        const int c = t * 8 + 2 * tq;
        if (qa0 < A.q_len) {
          float* p = A.dq_acc + ((int64_t(b) * A.q_len + qa0) * A.H + h) * D + c;
          atomicAdd(p, dq[t][0] * A.scale); atomicAdd(p + 1, dq[t][1] * A.scale);
        }
        if (qa1 < A.q_len) {
          float* p = A.dq_acc + ((int64_t(b) * A.q_len + qa1) * A.H + h) * D + c;
          atomicAdd(p, dq[t][2] * A.scale); atomicAdd(p + 1, dq[t][3] * A.scale);
        }
      }
    }
    __syncthreads();
  }
  // write dK (scaled), dV
  const int ka0 = key_a, ka1 = key_a + 8;
  __nv_bfloat16* dkg = A.dk + b * A.dkv_bs + int64_t(h) * D;
  __nv_bfloat16* dvg = A.dv + b * A.dkv_bs + int64_t(h) * D;
#pragma unroll
  for (int t = 0; t < NDT; ++t) {
    const int c = t * 8 + 2 * tq;
    if (ka0 < A.kv_len) {
      *reinterpret_cast<uint32_t*>(dkg + int64_t(ka0) * A.dkv_rs + c) = pack_bf16(dk[t][0] * A.scale, dk[t][1] * A.scale);
      *reinterpret_cast<uint32_t*>(dvg + int64_t(ka0) * A.dkv_rs + c) = pack_bf16(dv[t][0], dv[t][1]);
    }
    if (ka1 < A.kv_len) {
      *reinterpret_cast<uint32_t*>(dkg + int64_t(ka1) * A.dkv_rs + c) = pack_bf16(dk[t][2] * A.scale, dk[t][3] * A.scale);
      *reinterpret_cast<uint32_t*>(dvg + int64_t(ka1) * A.dkv_rs + c) = pack_bf16(dv[t][2], dv[t][3]);
    }
  }
}

// dQ (fp32 accumulator [B, q_len, H, D]) -> bf16 into the Q part of the dqkv
// buffer for the last q_len rows; the pruned rows [0, T - q_len) get zeros.
template <int D>
__global__ void fmha_bwd_dq_kernel(const float* __restrict__ dq_acc, __nv_bfloat16* __restrict__ dq,
                                   int64_t dq_bs, int64_t dq_rs, int B, int H, int q_len, int kv_len) {
  const int64_t rows = int64_t(B) * kv_len * H;
  for (int64_t r = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; r < rows; r += int64_t(gridDim.x) * blockDim.x) {
    const int h = int(r % H);
    const int64_t bt = r / H;
    const int t = int(bt % kv_len), b = int(bt / kv_len);
    __nv_bfloat16* dst = dq + b * dq_bs + int64_t(t) * dq_rs + int64_t(h) * D;
    const int i = t - (kv_len - q_len);
    if (i < 0) {
#pragma unroll
      for (int c = 0; c < D; c += 8) *reinterpret_cast<U4*>(dst + c) = U4{0, 0, 0, 0};
    } else {
      const float* src = dq_acc + ((int64_t(b) * q_len + i) * H + h) * D;
#pragma unroll
      for (int c = 0; c < D; c += 4) {
        float4 v = *reinterpret_cast<const float4*>(src + c);
        store4_bf16(dst + c, v);
      }
    }
  }
}

}  // namespace attn

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
static void check_qkv(const at::Tensor& t, const char* name) {
  PD_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16, "%s must be a bf16 CUDA tensor", name);
  PD_CHECK(t.dim() == 4 && t.stride(3) == 1, "%s must be [B, L, H, d] with unit stride on d", name);
  PD_CHECK(t.stride(2) == t.size(3), "%s: heads must be contiguous (stride d)", name);
  PD_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0 && t.stride(1) % 8 == 0 && t.stride(0) % 8 == 0,
           "%s: rows must be 16-byte aligned", name);
}

// q [B, q_len, H, d] (view), k/v [B, kv_len, H, d] (views) -> (o [B, q_len, H, d], lse [B, H, q_len])
std::vector<at::Tensor> fmha_fwd(at::Tensor q, at::Tensor k, at::Tensor v, double scale, int64_t warps_req) {
  check_qkv(q, "q"); check_qkv(k, "k"); check_qkv(v, "v");
  const int B = int(q.size(0)), ql = int(q.size(1)), H = int(q.size(2)), D = int(q.size(3));
  const int kl = int(k.size(1));
  TORCH_CHECK(D == 32 || D == 64, "head_dim must be 32 or 64");
  TORCH_CHECK(ql <= kl && k.size(0) == B && v.size(1) == kl && k.stride(0) == v.stride(0) && k.stride(1) == v.stride(1));
  auto o = at::empty({B, ql, H, D}, q.options());
  auto lse = at::empty({B, H, ql}, q.options().dtype(at::kFloat));
  if (B == 0 || ql == 0) return {o, lse};
  attn::FwdArgs A{reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(k.data_ptr()),
                  reinterpret_cast<const __nv_bfloat16*>(v.data_ptr()), q.stride(0), q.stride(1), k.stride(0), k.stride(1),
                  reinterpret_cast<__nv_bfloat16*>(o.data_ptr()), o.stride(0), o.stride(1), lse.data_ptr<float>(), H, ql, kl,
                  float(scale * 1.4426950408889634)};
  // d = 32: 64-query CTAs (4 warps, 6 per SM) by default -- v6 pyramid 18.06 ms
  // against 21.38 ms with 128-query CTAs and 18.26 ms with 32-query ones;
  // warps_req = 8 (or, when the caller passes 0, PD_FMHA_FWD_WARPS=8) selects
  // the 128-query CTAs.
  TORCH_CHECK(warps_req == 0 || warps_req == 4 || warps_req == 8, "warps: 0 (default), 4 or 8");
  int warps = int(warps_req);
  if (warps == 0) {
    const char* e = std::getenv("PD_FMHA_FWD_WARPS");
    warps = (e != nullptr && std::atoi(e) == 8) ? 8 : 4;
  }
  if (D == 32 && warps == 4) {
    dim3 grid4((ql + 63) / 64, B * H);
    attn::fmha_fwd_kernel<32, 4><<<grid4, 128, 0, stream()>>>(A);
  } else {
    dim3 grid((ql + attn::kFwdM - 1) / attn::kFwdM, B * H);
    if (D == 32) attn::fmha_fwd_kernel<32><<<grid, 256, 0, stream()>>>(A);
    else attn::fmha_fwd_kernel<64><<<grid, 256, 0, stream()>>>(A);
  }
  PD_CHECK_LAUNCH();
  return {o, lse};
}

// Backward. dqkv: the gradient buffer of the fused projection, [B, kv_len, 3, H, d];
// its Q/K/V parts are written completely (pruned Q rows zero-filled).
void fmha_bwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor lse, at::Tensor dout,
              at::Tensor dq, at::Tensor dk, at::Tensor dv, double scale) {
  check_qkv(q, "q"); check_qkv(k, "k"); check_qkv(v, "v"); check_qkv(dq, "dq"); check_qkv(dk, "dk"); check_qkv(dv, "dv");
  const int B = int(q.size(0)), ql = int(q.size(1)), H = int(q.size(2)), D = int(q.size(3));
  const int kl = int(k.size(1));
  TORCH_CHECK(o.is_contiguous() && dout.is_contiguous() && o.sizes() == dout.sizes() && o.size(1) == ql);
  TORCH_CHECK(dq.size(1) == kl && dk.size(1) == kl && dk.stride(1) == dv.stride(1) && dk.stride(0) == dv.stride(0));
  if (B == 0) return;
  auto delta = at::empty({B, H, ql}, lse.options());
  auto dq_acc = at::empty({B, ql, H, D}, lse.options());
  PD_CHECK_CUDA(cudaMemsetAsync(dq_acc.data_ptr(), 0, dq_acc.numel() * sizeof(float), stream()));
  attn::BwdArgs A{reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(k.data_ptr()),
                  reinterpret_cast<const __nv_bfloat16*>(v.data_ptr()), q.stride(0), q.stride(1), k.stride(0), k.stride(1),
                  reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
                  o.stride(0), o.stride(1), lse.data_ptr<float>(), delta.data_ptr<float>(), dq_acc.data_ptr<float>(),
                  reinterpret_cast<__nv_bfloat16*>(dk.data_ptr()), reinterpret_cast<__nv_bfloat16*>(dv.data_ptr()),
                  dk.stride(0), dk.stride(1), H, ql, kl, float(scale * 1.4426950408889634), float(scale)};
  dim3 gpre((ql + 255) / 256, B * H);
  dim3 gmain((kl + attn::kBwdN - 1) / attn::kBwdN, B * H);
  int64_t rows = int64_t(B) * kl * H;
  int64_t gq = (rows + 255) / 256;
  if (gq > int64_t(num_sms()) * 16) gq = int64_t(num_sms()) * 16;
  auto smem_bytes = [](int d) {
    return size_t((2 * attn::kBwdN * d + 4 * attn::kBwdM * d + attn::kBwdN * attn::kBwdM) * 2 + 4 * attn::kBwdM * 4);
  };
  static bool attr_set = false;
  if (!attr_set) {
    PD_CHECK_CUDA(cudaFuncSetAttribute(attn::fmha_bwd_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(smem_bytes(32))));
    PD_CHECK_CUDA(cudaFuncSetAttribute(attn::fmha_bwd_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(smem_bytes(64))));
    attr_set = true;
  }
  if (D == 32) {
    attn::fmha_bwd_pre_kernel<32><<<gpre, 256, 0, stream()>>>(A);
    attn::fmha_bwd_kernel<32><<<gmain, 128, smem_bytes(32), stream()>>>(A);
    attn::fmha_bwd_dq_kernel<32><<<gq, 256, 0, stream()>>>(dq_acc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()),
                                                       dq.stride(0), dq.stride(1), B, H, ql, kl);
  } else {
    attn::fmha_bwd_pre_kernel<64><<<gpre, 256, 0, stream()>>>(A);
    attn::fmha_bwd_kernel<64><<<gmain, 128, smem_bytes(64), stream()>>>(A);
    attn::fmha_bwd_dq_kernel<64><<<gq, 256, 0, stream()>>>(dq_acc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()),
                                                       dq.stride(0), dq.stride(1), B, H, ql, kl);
  }
  PD_CHECK_LAUNCH();
  note_launch(2);
}

}  // namespace pd
