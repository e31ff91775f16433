// Embedding lookup and fused sparse-optimizer backward for sm_100a.
//
// Replaces the FBGEMM TBE forward/backward the reference reaches through
// TorchRec (primus_dlrm/models/embedding.py:117-175 and the fused optimizer
// registered at primus_dlrm/distributed/wrapper.py:151-174).
//
// Design:
//  * One launch gathers every feature of one embedding dim. Each feature is a
//    "slot": ids + an output view (base pointer already offset to the slot's
//    column, row stride in elements). Writing a slot at column k*E of a
//    [B, L, G*E] buffer fuses the per-pool torch.cat of the tokenizer input;
//    writing bf16 fuses the autocast cast.
//  * Tables are read through an array of row-shard base pointers. A table on
//    one device has one shard. A row-wise sharded table has one shard per
//    rank, mapped into this process over NVLink (CUDA IPC), so the same
//    kernel is the cross-GPU lookup: rows are pulled straight from the
//    owner's HBM with peer loads, no id or row all-to-all.
//  * Backward sorts (table, row) keys, then one warp per chunk of 32 sorted
//    positions reduces each run of equal keys in registers and applies the
//    optimizer (SGD / Adagrad / row-wise Adagrad / Adam) to the touched row.
//    A run that crosses a chunk boundary (a hot Zipf row) is reduced by
//    every chunk it touches into a scratch row with fp32 atomics; the last
//    chunk to finish (per-row arrival counter) applies the update and clears
//    the scratch row and counter, so the scratch stays zero between calls.
//  * Nothing traps: an out-of-range id writes a zero row and records
//    kIdOutOfRange in the error word.
#include "common.cuh"

namespace pd {

constexpr int kMaxSlots = 48;
constexpr int kMaxTables = 32;
constexpr int kChunk = 32;  // sorted positions per warp in the backward

struct Slot {
  const void* ids;          // int32 or int64 ids, [n]
  void* io;                 // fwd: output view base; bwd: grad view base
  const int64_t* offsets;   // pooled jagged bags: [n_bags + 1]; nullptr = fixed bags
  int64_t n;                // number of ids
  int64_t io_stride;        // elements between consecutive output rows
  int32_t table;
  int32_t pool;             // 0 none, 1 sum, 2 mean
  int32_t bag_len;          // fixed bag length when pooled and offsets == nullptr
  int32_t pad_id;           // pooled: id excluded from the bag (-1 = none)
  int64_t n_bags;           // pooled: number of bags
};

struct Table {
  const float* const* shards;  // [n_shards] row-shard base pointers (device array)
  float* local;                // this rank's shard (updated in backward)
  float* state1;               // rowwise/adagrad accumulator or Adam m
  float* state2;               // Adam v
  int64_t rows;                // global rows
  int64_t chunk;               // rows per shard
  int64_t key_base;            // first sort key of this table
  int64_t local_row0;          // first global row owned by this rank
  int64_t local_rows;          // rows in this rank's shard
  int32_t n_shards;
  int32_t dim;
};

struct GatherParams {
  Slot slots[kMaxSlots];
  int64_t slot_off[kMaxSlots + 1];
  int64_t bag_off[kMaxSlots + 1];  // pooled: prefix of bag counts over slots
  Table tables[kMaxTables];
  int n_slots;
  int n_tables;
  int dim;
};

template <typename IdT>
__device__ __forceinline__ int64_t load_id(const void* p, int64_t i) {
  return static_cast<int64_t>(static_cast<const IdT*>(p)[i]);
}

__device__ __forceinline__ int find_slot(const int64_t* off, int n, int64_t p) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (off[mid] <= p) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Resolve a global row of table t to a readable pointer (local or peer).
__device__ __forceinline__ const float* row_ptr(const Table& t, int64_t g, bool& ok) {
  ok = (g >= 0 && g < t.rows);
  if (!ok) return nullptr;
  // owner = g / chunk; 32-bit division when both fit (tables below 2^32 rows)
  int64_t owner = 0;
  if (t.n_shards > 1)
    owner = (g < 0xffffffffll && t.chunk < 0xffffffffll) ? int64_t(uint32_t(g) / uint32_t(t.chunk)) : g / t.chunk;
  if (owner >= t.n_shards) owner = t.n_shards - 1;
  const int64_t r = g - owner * t.chunk;
  return t.shards[owner] + r * t.dim;
}

// ---------------------------------------------------------------------------
// Unpooled gather: out[slot][i] = W[table][ids[i]]
// Threads of a warp split into groups of `lanes` threads, each group owning a
// row; each thread moves `vpt` float4 of the row. A group handles kUnroll
// rows per iteration with all their id and row loads issued before any
// store, so several peer (NVLink) reads are in flight per thread.
// ---------------------------------------------------------------------------
constexpr int kGatherUnroll = 4;

template <typename IdT, typename OutT>
__global__ void __launch_bounds__(256) gather_kernel(const __grid_constant__ GatherParams P,
                                                     int64_t total, int* err) {
  const int nvec = P.dim >> 2;
  const int lanes = nvec < 32 ? nvec : 32;
  const int groups_per_warp = 32 / lanes;
  const int lane = threadIdx.x & 31;
  const int grp = lane / lanes;
  const int sub = lane % lanes;
  if (grp >= groups_per_warp) return;
  const int64_t warp_global = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int64_t stride = n_warps * groups_per_warp;
  for (int64_t r0 = warp_global * groups_per_warp + grp; r0 < total; r0 += stride * kGatherUnroll) {
    const float* src[kGatherUnroll];
    OutT* dst[kGatherUnroll];
    bool live[kGatherUnroll];
#pragma unroll
    for (int u = 0; u < kGatherUnroll; ++u) {
      const int64_t r = r0 + u * stride;
      live[u] = r < total;
      src[u] = nullptr;
      dst[u] = nullptr;
      if (live[u]) {
        const int s = find_slot(P.slot_off, P.n_slots, r);
        const Slot& sl = P.slots[s];
        const int64_t i = r - P.slot_off[s];
        const int64_t g = load_id<IdT>(sl.ids, i);
        bool ok;
        src[u] = row_ptr(P.tables[sl.table], g, ok);
        dst[u] = static_cast<OutT*>(sl.io) + i * sl.io_stride;
        if (!ok && sub == 0) set_error(err, kIdOutOfRange);
      }
    }
    for (int v = sub; v < nvec; v += lanes) {
      float4 x[kGatherUnroll];
#pragma unroll
      for (int u = 0; u < kGatherUnroll; ++u)
        x[u] = src[u] ? __ldcg(reinterpret_cast<const float4*>(src[u]) + v) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < kGatherUnroll; ++u) {
        if (!live[u]) continue;
        if constexpr (std::is_same<OutT, float>::value) {
          reinterpret_cast<float4*>(dst[u])[v] = x[u];
        } else {
          store4_bf16(dst[u] + 4 * v, x[u]);
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Deduplicated gather for sharded tables. The lookup's (table, row) keys,
// sorted by owner and row (the same sort the backward uses), are fetched once
// per unique key into a staging buffer -- peer reads walk each owner's shard
// in ascending address order and a hot Zipf row crosses NVLink once -- and
// then expanded to every position. The unique count is read on the device
// (seg of the last sorted key + 1), so nothing waits for the host.
// ---------------------------------------------------------------------------
__device__ __forceinline__ const float* key_row(const GatherParams& P, int64_t key, bool& ok) {
  int t = 0;
  while (t + 1 < P.n_tables && P.tables[t + 1].key_base <= key) ++t;
  const Table& T = P.tables[t];
  return row_ptr(T, key - T.key_base, ok);
}

template <typename OutT>
__global__ void __launch_bounds__(256) gather_unique_kernel(const __grid_constant__ GatherParams P,
                                                            const int64_t* __restrict__ uniq,
                                                            const int64_t* __restrict__ seg, int64_t n,
                                                            OutT* __restrict__ stage, int* err) {
  const int64_t U = seg[n - 1] + 1;
  const int nvec = P.dim >> 2;
  const int lanes = nvec < 32 ? nvec : 32;
  const int groups_per_warp = 32 / lanes;
  const int lane = threadIdx.x & 31;
  const int grp = lane / lanes;
  const int sub = lane % lanes;
  if (grp >= groups_per_warp) return;
  const int64_t warp_global = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int64_t stride = n_warps * groups_per_warp;
  for (int64_t u0 = warp_global * groups_per_warp + grp; u0 < U; u0 += stride * kGatherUnroll) {
    const float* src[kGatherUnroll];
#pragma unroll
    for (int u = 0; u < kGatherUnroll; ++u) {
      const int64_t r = u0 + u * stride;
      src[u] = nullptr;
      if (r < U) {
        bool ok;
        src[u] = key_row(P, uniq[r], ok);   // an out-of-range id's key resolves to no row: zeros
        if (!ok && sub == 0) set_error(err, kIdOutOfRange);
      }
    }
    for (int v = sub; v < nvec; v += lanes) {
      float4 x[kGatherUnroll];
#pragma unroll
      for (int u = 0; u < kGatherUnroll; ++u)
        x[u] = src[u] ? __ldcg(reinterpret_cast<const float4*>(src[u]) + v) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < kGatherUnroll; ++u) {
        const int64_t r = u0 + u * stride;
        if (r >= U) continue;
        OutT* dst = stage + r * P.dim;
        if constexpr (std::is_same<OutT, float>::value) {
          reinterpret_cast<float4*>(dst)[v] = x[u];
        } else {
          store4_bf16(dst + 4 * v, x[u]);
        }
      }
    }
  }
}

// Unique index of every position: u_of_pos[perm[p]] = seg[p].
__global__ void unique_of_position_kernel(const int64_t* __restrict__ perm, const int64_t* __restrict__ seg,
                                          int32_t* __restrict__ u_of_pos, int64_t n) {
  for (int64_t p = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; p < n; p += int64_t(gridDim.x) * blockDim.x)
    u_of_pos[perm[p]] = int32_t(seg[p]);
}

// out[j] = stage[u_of_pos[j]] in position order: the output rows are written
// in sequence (the random side is the staged rows, whose hot Zipf entries
// stay in L2). A group of threads per position, rows moved as 16-byte
// vectors, kGatherUnroll positions in flight per group.
template <typename OutT>
__global__ void __launch_bounds__(256, 4) expand_kernel(const __grid_constant__ GatherParams P,
                                                     const OutT* __restrict__ stage,
                                                     const int32_t* __restrict__ u_of_pos, int64_t n) {
  const int nvec = int(P.dim * sizeof(OutT) / 16);
  const int lanes = nvec < 32 ? nvec : 32;
  const int groups_per_warp = 32 / lanes;
  const int lane = threadIdx.x & 31;
  const int grp = lane / lanes;
  const int sub = lane % lanes;
  if (grp >= groups_per_warp) return;
  const int64_t warp_global = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int64_t stride = n_warps * groups_per_warp;
  for (int64_t j0 = warp_global * groups_per_warp + grp; j0 < n; j0 += stride * kGatherUnroll) {
    const uint4* src[kGatherUnroll];
    uint4* dst[kGatherUnroll];
#pragma unroll
    for (int u = 0; u < kGatherUnroll; ++u) {
      const int64_t j = j0 + u * stride;
      src[u] = nullptr;
      dst[u] = nullptr;
      if (j < n) {
        const int s = find_slot(P.slot_off, P.n_slots, j);
        const Slot& sl = P.slots[s];
        dst[u] = reinterpret_cast<uint4*>(static_cast<OutT*>(sl.io) + (j - P.slot_off[s]) * sl.io_stride);
        src[u] = reinterpret_cast<const uint4*>(stage + int64_t(u_of_pos[j]) * P.dim);
      }
    }
    for (int v = sub; v < nvec; v += lanes) {
      uint4 x[kGatherUnroll];
#pragma unroll
      for (int u = 0; u < kGatherUnroll; ++u) x[u] = src[u] ? src[u][v] : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int u = 0; u < kGatherUnroll; ++u)
        if (dst[u]) dst[u][v] = x[u];
    }
  }
}

// ---------------------------------------------------------------------------
// Pooled gather (sum / mean over a bag, pad id excluded): one warp per bag.
// ---------------------------------------------------------------------------
template <typename IdT, typename OutT>
__global__ void __launch_bounds__(256) pooled_kernel(const __grid_constant__ GatherParams P,
                                                     int64_t total_bags, int* err) {
  const int64_t* bag_off = P.bag_off;
  const int lane = threadIdx.x & 31;
  const int64_t warp_global = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int nvec = P.dim >> 2;
  for (int64_t b = warp_global; b < total_bags; b += n_warps) {
    const int s = find_slot(bag_off, P.n_slots, b);
    const Slot& sl = P.slots[s];
    const int64_t bag = b - bag_off[s];
    int64_t beg, end;
    if (sl.offsets) { beg = sl.offsets[bag]; end = sl.offsets[bag + 1]; }
    else { beg = bag * sl.bag_len; end = beg + sl.bag_len; }
    const Table& t = P.tables[sl.table];
    float4 acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    int cnt = 0;
    for (int64_t j = beg; j < end; ++j) {
      const int64_t g = load_id<IdT>(sl.ids, j);
      if (g == sl.pad_id) continue;
      bool ok;
      const float* src = row_ptr(t, g, ok);
      if (!ok) { if (lane == 0) set_error(err, kIdOutOfRange); continue; }
      ++cnt;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int v = lane + 32 * k;
        if (v < nvec) {
          float4 x = __ldg(reinterpret_cast<const float4*>(src) + v);
          acc[k].x += x.x; acc[k].y += x.y; acc[k].z += x.z; acc[k].w += x.w;
        }
      }
    }
    const float sc = (sl.pool == 2 && cnt > 0) ? 1.f / cnt : 1.f;
    OutT* dst = static_cast<OutT*>(sl.io) + bag * sl.io_stride;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int v = lane + 32 * k;
      if (v < nvec) {
        float4 x = make_float4(acc[k].x * sc, acc[k].y * sc, acc[k].z * sc, acc[k].w * sc);
        if constexpr (std::is_same<OutT, float>::value) reinterpret_cast<float4*>(dst)[v] = x;
        else store4_bf16(dst + 4 * v, x);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Backward step 1: sort keys. key = table.key_base + global row; positions
// that contribute nothing (pooled pad ids, out-of-range ids) get INT64_MAX.
// ---------------------------------------------------------------------------
template <typename IdT>
__global__ void keys_kernel(const __grid_constant__ GatherParams P, int64_t total, int64_t* keys) {
  for (int64_t p = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; p < total;
       p += int64_t(gridDim.x) * blockDim.x) {
    const int s = find_slot(P.slot_off, P.n_slots, p);
    const Slot& sl = P.slots[s];
    const int64_t g = load_id<IdT>(sl.ids, p - P.slot_off[s]);
    const Table& t = P.tables[sl.table];
    const bool skip = (sl.pool != 0 && g == sl.pad_id) || g < 0 || g >= t.rows;
    keys[p] = skip ? INT64_MAX : t.key_base + g;
  }
}

// Per-position gradient scale and row for pooled slots (bag -> row, 1/count).
template <typename IdT>
__global__ void pooled_scale_kernel(const __grid_constant__ GatherParams P, int64_t total,
                                    float* scale, int64_t* grad_row) {
  for (int64_t p = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; p < total;
       p += int64_t(gridDim.x) * blockDim.x) {
    const int s = find_slot(P.slot_off, P.n_slots, p);
    const Slot& sl = P.slots[s];
    const int64_t i = p - P.slot_off[s];
    if (sl.pool == 0) { scale[p] = 1.f; grad_row[p] = i; continue; }
    int64_t bag, beg, end;
    if (sl.offsets) {
      int64_t lo = 0, hi = sl.n_bags - 1;
      while (lo < hi) { int64_t m = (lo + hi + 1) >> 1; if (sl.offsets[m] <= i) lo = m; else hi = m - 1; }
      bag = lo; beg = sl.offsets[bag]; end = sl.offsets[bag + 1];
    } else {
      bag = i / sl.bag_len; beg = bag * sl.bag_len; end = beg + sl.bag_len;
    }
    float sc = 1.f;
    if (sl.pool == 2) {
      int cnt = 0;
      for (int64_t j = beg; j < end; ++j) cnt += (load_id<IdT>(sl.ids, j) != sl.pad_id);
      sc = cnt > 0 ? 1.f / cnt : 0.f;
    }
    scale[p] = sc;
    grad_row[p] = bag;
  }
}

// ---------------------------------------------------------------------------
// Backward step 2: reduce runs of equal sorted keys + apply the optimizer.
// ---------------------------------------------------------------------------
struct OptParams {
  int kind;        // 0 sgd, 1 adagrad, 2 rowwise_adagrad, 3 adam
  float lr;
  float eps;
  float weight_decay;
  float beta1, beta2;
  float bc1, bc2;  // Adam bias corrections 1 - beta^t
};

// Grad source: sorted position q -> (slot via perm) -> grad row pointer.
struct GradSrc {
  const int64_t* perm;      // sorted q -> original position p
  const float* scale;       // per original position (pooled); nullptr = 1
  const int64_t* grad_row;  // per original position: row within the slot's grad view; nullptr = i
  // Reduce-only mode: when out_rows != nullptr the summed gradient of the run
  // starting at sorted position q is stored to out_rows[seg[q]] (fp32 [U, dim])
  // instead of being applied to the table.
  float* out_rows;
  const int64_t* seg;
  // When > 0, perm values outside [0, perm_limit) are skipped and recorded as
  // kIdOutOfRange (the allocation-free entry point takes perm from its caller).
  int64_t perm_limit;
};

template <int KV = 8>
__device__ __forceinline__ void store_reduced(const GradSrc& src, int64_t q, const float4* acc, int nvec,
                                              int dim, int lane) {
  float4* o = reinterpret_cast<float4*>(src.out_rows + src.seg[q] * int64_t(dim));
#pragma unroll
  for (int k = 0; k < KV; ++k) {
    const int v = lane + 32 * k;
    if (v < nvec) o[v] = acc[k];
  }
}

template <typename GradT, int KV = 8>
__device__ __forceinline__ void accum_row(float4* acc, const GradT* src, int nvec, int lane, float sc) {
#pragma unroll
  for (int k = 0; k < KV; ++k) {
    const int v = lane + 32 * k;
    if (v < nvec) {
      float4 x;
      if constexpr (std::is_same<GradT, float>::value) x = reinterpret_cast<const float4*>(src)[v];
      else x = load4_bf16(src + 4 * v);
      acc[k].x += sc * x.x; acc[k].y += sc * x.y; acc[k].z += sc * x.z; acc[k].w += sc * x.w;
    }
  }
}

__device__ __forceinline__ int find_table(const GatherParams& P, int64_t key) {
  int lo = 0, hi = P.n_tables - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (P.tables[mid].key_base <= key) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Apply the optimizer to one row (this rank owns it). acc holds the summed grad.
template <int KV = 8>
__device__ void apply_update(const GatherParams& P, const OptParams& O, int64_t key,
                             float4* acc, int nvec, int lane, int* err) {
  const int ti = find_table(P, key);
  const Table& t = P.tables[ti];
  const int64_t g = key - t.key_base;
  const int64_t r = g - t.local_row0;
  if (r < 0 || r >= t.local_rows) { if (lane == 0) set_error(err, kIdOutOfRange); return; }
  float4* w = reinterpret_cast<float4*>(t.local + r * t.dim);
  float4 wv[KV];
#pragma unroll
  for (int k = 0; k < KV; ++k) {
    const int v = lane + 32 * k;
    wv[k] = v < nvec ? w[v] : make_float4(0.f, 0.f, 0.f, 0.f);
    if (O.weight_decay != 0.f && v < nvec) {
      acc[k].x += O.weight_decay * wv[k].x; acc[k].y += O.weight_decay * wv[k].y;
      acc[k].z += O.weight_decay * wv[k].z; acc[k].w += O.weight_decay * wv[k].w;
    }
  }
  if (O.kind == 2) {  // row-wise Adagrad: one accumulator per row, mean of g^2
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < KV; ++k)
      if (lane + 32 * k < nvec)
        ss += acc[k].x * acc[k].x + acc[k].y * acc[k].y + acc[k].z * acc[k].z + acc[k].w * acc[k].w;
    ss = warp_sum(ss) / float(t.dim);
    float G = 0.f;
    if (lane == 0) { G = t.state1[r] + ss; t.state1[r] = G; }
    G = __shfl_sync(0xffffffffu, G, 0);
    const float mul = O.lr / (sqrtf(G) + O.eps);
#pragma unroll
    for (int k = 0; k < KV; ++k) {
      const int v = lane + 32 * k;
      if (v < nvec) {
        wv[k].x -= mul * acc[k].x; wv[k].y -= mul * acc[k].y;
        wv[k].z -= mul * acc[k].z; wv[k].w -= mul * acc[k].w;
        w[v] = wv[k];
      }
    }
    return;
  }
#pragma unroll
  for (int k = 0; k < KV; ++k) {
    const int v = lane + 32 * k;
    if (v >= nvec) continue;
    float* gp = reinterpret_cast<float*>(&acc[k]);
    float* wp = reinterpret_cast<float*>(&wv[k]);
    if (O.kind == 0) {
#pragma unroll
      for (int e = 0; e < 4; ++e) wp[e] -= O.lr * gp[e];
    } else if (O.kind == 1) {
      float4 s = reinterpret_cast<float4*>(t.state1 + r * t.dim)[v];
      float* sp = reinterpret_cast<float*>(&s);
#pragma unroll
      for (int e = 0; e < 4; ++e) { sp[e] += gp[e] * gp[e]; wp[e] -= O.lr * gp[e] / (sqrtf(sp[e]) + O.eps); }
      reinterpret_cast<float4*>(t.state1 + r * t.dim)[v] = s;
    } else {
      float4 m = reinterpret_cast<float4*>(t.state1 + r * t.dim)[v];
      float4 vv = reinterpret_cast<float4*>(t.state2 + r * t.dim)[v];
      float* mp = reinterpret_cast<float*>(&m);
      float* vp = reinterpret_cast<float*>(&vv);
      const float step = O.lr / O.bc1;
      const float inv_sqrt_bc2 = rsqrtf(O.bc2);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        mp[e] = O.beta1 * mp[e] + (1.f - O.beta1) * gp[e];
        vp[e] = O.beta2 * vp[e] + (1.f - O.beta2) * gp[e] * gp[e];
        wp[e] -= step * mp[e] / (sqrtf(vp[e]) * inv_sqrt_bc2 + O.eps);
      }
      reinterpret_cast<float4*>(t.state1 + r * t.dim)[v] = m;
      reinterpret_cast<float4*>(t.state2 + r * t.dim)[v] = vv;
    }
    w[v] = wv[k];
  }
}

__device__ __forceinline__ int64_t lower_bound(const int64_t* a, int64_t n, int64_t key) {
  int64_t lo = 0, hi = n;
  while (lo < hi) { int64_t m = (lo + hi) >> 1; if (a[m] < key) lo = m + 1; else hi = m; }
  return lo;
}

// GradT: dtype of the grad views. Positions index the slots of P (or a flat
// receive buffer when P.n_slots == 1 and the slot covers it).
template <typename GradT>
__global__ void __launch_bounds__(256) reduce_update_kernel(
    const __grid_constant__ GatherParams P, OptParams O, const int64_t* __restrict__ skeys,
    GradSrc src, int64_t total, float* __restrict__ scratch, int* __restrict__ arrivals, int* err) {
  const int lane = threadIdx.x & 31;
  const int nvec = P.dim >> 2;
  const int64_t n_chunks = (total + kChunk - 1) / kChunk;
  const int64_t warp_global = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t c = warp_global; c < n_chunks; c += n_warps) {
    const int64_t c0 = c * kChunk;
    const int64_t c1 = min(c0 + kChunk, total);
    int64_t a = c0;
    while (a < c1) {
      const int64_t key = skeys[a];
      if (key == INT64_MAX) break;  // sentinel tail
      int64_t b = a + 1;
      while (b < c1 && skeys[b] == key) ++b;
      float4 acc[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int64_t q = a; q < b; ++q) {
        const int64_t p = src.perm[q];
        if (src.perm_limit > 0 && uint64_t(p) >= uint64_t(src.perm_limit)) {
          if (lane == 0) set_error(err, kIdOutOfRange);
          continue;
        }
        const int s = find_slot(P.slot_off, P.n_slots, p);
        const Slot& sl = P.slots[s];
        const int64_t i = p - P.slot_off[s];
        const int64_t row = src.grad_row ? src.grad_row[p] : i;
        const float sc = src.scale ? src.scale[p] : 1.f;
        accum_row<GradT>(acc, static_cast<const GradT*>(sl.io) + row * sl.io_stride, nvec, lane, sc);
      }
      const bool head = (a > 0) ? (skeys[a - 1] != key) : true;
      const bool tail = (b < total) ? (skeys[b] != key) : true;
      if (head && tail) {
        if (src.out_rows) store_reduced(src, a, acc, nvec, P.dim, lane);
        else apply_update(P, O, key, acc, nvec, lane, err);
      } else {
        // The run spans several chunks: accumulate into the head chunk's
        // scratch row; the last arriving chunk applies the update.
        const int64_t beg = head ? a : lower_bound(skeys, total, key);
        const int64_t end = tail ? b : lower_bound(skeys, total, key + 1);
        const int64_t hc = beg / kChunk;
        const int span = int((end - 1) / kChunk - hc + 1);
        float* srow = scratch + hc * int64_t(P.dim);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int v = lane + 32 * k;
          if (v < nvec) {
            atomicAdd(srow + 4 * v + 0, acc[k].x); atomicAdd(srow + 4 * v + 1, acc[k].y);
            atomicAdd(srow + 4 * v + 2, acc[k].z); atomicAdd(srow + 4 * v + 3, acc[k].w);
          }
        }
        __threadfence();
        __syncwarp();
        int prev = 0;
        if (lane == 0) prev = atomicAdd(arrivals + hc, 1);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev == span - 1) {
          __threadfence();
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int v = lane + 32 * k;
            if (v < nvec) {
              acc[k] = __ldcg(reinterpret_cast<const float4*>(srow) + v);
              reinterpret_cast<float4*>(srow)[v] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
          }
          if (lane == 0) arrivals[hc] = 0;
          if (src.out_rows) store_reduced(src, beg, acc, nvec, P.dim, lane);
          else apply_update(P, O, key, acc, nvec, lane, err);
        }
      }
      a = b;
    }
  }
}

// ---------------------------------------------------------------------------
// Same reduction with the chunk's gradient rows staged in shared memory.
// A warp first resolves the 32 positions of its chunk lane-parallel (key,
// perm, slot, row pointer, pooling scale), then copies all their rows into
// its shared-memory stage with cp.async (16-byte pieces, every piece of the
// chunk in flight at once), and reduces the runs of equal keys (found with a
// ballot) from shared memory. Loads are no longer serialised behind the
// previous position's perm lookup or the previous run's store.
// ---------------------------------------------------------------------------
constexpr int kStageMaxRowBytes = 512;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <typename GradT, int KV>
__global__ void __launch_bounds__(256) reduce_update_staged_kernel(
    const __grid_constant__ GatherParams P, OptParams O, const int64_t* __restrict__ skeys,
    GradSrc src, int64_t total, float* __restrict__ scratch, int* __restrict__ arrivals, int* err) {
  extern __shared__ __align__(16) unsigned char stage_smem[];
  const unsigned FULL = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const int nvec = P.dim >> 2;
  const int rb = P.dim * int(sizeof(GradT));
  const int v16 = rb >> 4;
  unsigned char* wstage = stage_smem + size_t(threadIdx.x >> 5) * kChunk * rb;
  const int64_t n_chunks = (total + kChunk - 1) / kChunk;
  const int64_t warp_global = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t c = warp_global; c < n_chunks; c += n_warps) {
    const int64_t c0 = c * kChunk;
    const int cn = int(min(int64_t(kChunk), total - c0));
    int64_t myk = INT64_MAX;
    unsigned long long gp = 0ull;
    float gs = 0.f;
    if (lane < cn) {
      myk = skeys[c0 + lane];
      if (myk != INT64_MAX) {
        const int64_t p = src.perm[c0 + lane];
        const int s = find_slot(P.slot_off, P.n_slots, p);
        const Slot& sl = P.slots[s];
        const int64_t row = src.grad_row ? src.grad_row[p] : p - P.slot_off[s];
        gs = src.scale ? src.scale[p] : 1.f;
        gp = reinterpret_cast<unsigned long long>(static_cast<const GradT*>(sl.io) + row * sl.io_stride);
      }
    }
    const int64_t before = c0 > 0 ? skeys[c0 - 1] : INT64_MIN;
    const int64_t after = c0 + cn < total ? skeys[c0 + cn] : INT64_MIN;
    const int n_live = __popc(__ballot_sync(FULL, gp != 0ull));  // padding keys sort last: a prefix
    const int pieces = n_live * v16;
    for (int base = 0; base < pieces; base += 32) {
      const int idx = base + lane;
      const int row = idx / v16;
      const unsigned long long rp = __shfl_sync(FULL, gp, row & 31);
      if (idx < pieces) cp_async16(wstage + size_t(idx) * 16, reinterpret_cast<const unsigned char*>(rp) + (idx - row * v16) * 16);
    }
    cp_async_wait_all();
    __syncwarp();
    const int64_t up = __shfl_up_sync(FULL, myk, 1);
    unsigned runs = __ballot_sync(FULL, lane < n_live && (lane == 0 || up != myk));
    while (runs) {
      const int ls = __ffs(runs) - 1;
      runs &= runs - 1;
      const int le = runs ? __ffs(runs) - 1 : n_live;
      const int64_t key = __shfl_sync(FULL, myk, ls);
      float4 acc[KV];
#pragma unroll
      for (int k = 0; k < KV; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int l = ls; l < le; ++l) {
        const float sc = __shfl_sync(FULL, gs, l);
        accum_row<GradT, KV>(acc, reinterpret_cast<const GradT*>(wstage + size_t(l) * rb), nvec, lane, sc);
      }
      const bool head = ls > 0 || before != key;
      const bool tail = le < cn || after != key;
      if (head && tail) {
        if (src.out_rows) store_reduced<KV>(src, c0 + ls, acc, nvec, P.dim, lane);
        else apply_update<KV>(P, O, key, acc, nvec, lane, err);
      } else {
        const int64_t beg = head ? c0 + ls : lower_bound(skeys, total, key);
        const int64_t end = tail ? c0 + le : lower_bound(skeys, total, key + 1);
        const int64_t hc = beg / kChunk;
        const int span = int((end - 1) / kChunk - hc + 1);
        float* srow = scratch + hc * int64_t(P.dim);
#pragma unroll
        for (int k = 0; k < KV; ++k) {
          const int v = lane + 32 * k;
          if (v < nvec) {
            atomicAdd(srow + 4 * v + 0, acc[k].x); atomicAdd(srow + 4 * v + 1, acc[k].y);
            atomicAdd(srow + 4 * v + 2, acc[k].z); atomicAdd(srow + 4 * v + 3, acc[k].w);
          }
        }
        __threadfence();
        __syncwarp();
        int prev = 0;
        if (lane == 0) prev = atomicAdd(arrivals + hc, 1);
        prev = __shfl_sync(FULL, prev, 0);
        if (prev == span - 1) {
          __threadfence();
#pragma unroll
          for (int k = 0; k < KV; ++k) {
            const int v = lane + 32 * k;
            if (v < nvec) {
              acc[k] = __ldcg(reinterpret_cast<const float4*>(srow) + v);
              reinterpret_cast<float4*>(srow)[v] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
          }
          if (lane == 0) arrivals[hc] = 0;
          if (src.out_rows) store_reduced<KV>(src, beg, acc, nvec, P.dim, lane);
          else apply_update<KV>(P, O, key, acc, nvec, lane, err);
        }
      }
    }
    __syncwarp();  // the stage is rewritten by the next chunk
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

static int64_t grid_for(int64_t work_items, int per_block) {
  int64_t blocks = (work_items + per_block - 1) / per_block;
  const int64_t cap = int64_t(num_sms()) * 16;
  if (blocks > cap) blocks = cap;
  return blocks < 1 ? 1 : blocks;
}

// tables: list of [weight(local shard, fp32 2D), shard_ptrs(int64 device tensor),
//          state1, state2] packed as tensors; meta: int64 [n_tables, 6] CPU tensor
//          (rows, chunk, key_base, local_row0, n_shards, dim).
static void fill_tables(GatherParams& P, const std::vector<at::Tensor>& weights,
                        const std::vector<at::Tensor>& shard_ptrs,
                        const std::vector<at::Tensor>& state1,
                        const std::vector<at::Tensor>& state2, const at::Tensor& meta) {
  const int nt = static_cast<int>(weights.size());
  PD_CHECK(nt <= kMaxTables, "too many tables in one launch: %d (at most %d)", nt, kMaxTables);
  TORCH_CHECK(meta.device().is_cpu() && meta.dtype() == at::kLong && meta.size(0) == nt && meta.size(1) == 6);
  auto m = meta.accessor<int64_t, 2>();
  P.n_tables = nt;
  for (int t = 0; t < nt; ++t) {
    Table& T = P.tables[t];
    TORCH_CHECK(weights[t].dtype() == at::kFloat && weights[t].is_contiguous(), "table must be fp32 contiguous");
    TORCH_CHECK(shard_ptrs[t].is_cuda() && shard_ptrs[t].dtype() == at::kLong);
    T.shards = reinterpret_cast<const float* const*>(shard_ptrs[t].data_ptr<int64_t>());
    T.local = weights[t].data_ptr<float>();
    T.state1 = state1[t].numel() ? state1[t].data_ptr<float>() : nullptr;
    T.state2 = state2[t].numel() ? state2[t].data_ptr<float>() : nullptr;
    T.rows = m[t][0]; T.chunk = m[t][1]; T.key_base = m[t][2];
    T.local_row0 = m[t][3]; T.n_shards = int(m[t][4]); T.dim = int(m[t][5]);
    T.local_rows = weights[t].size(0);
    TORCH_CHECK(T.dim == P.dim, "all tables of one launch must share the embedding dim");
    TORCH_CHECK(T.chunk > 0 && T.n_shards >= 1 && shard_ptrs[t].numel() == T.n_shards);
  }
}

static at::ScalarType fill_slots(GatherParams& P, const std::vector<at::Tensor>& ids,
                                 const std::vector<at::Tensor>& io, const at::Tensor& slot_meta,
                                 const std::vector<at::Tensor>& offsets, bool pooled_allowed) {
  const int ns = static_cast<int>(ids.size());
  PD_CHECK(ns >= 1 && ns <= kMaxSlots, "slot count out of range: %d (1 .. %d)", ns, kMaxSlots);
  TORCH_CHECK(io.size() == ids.size());
  TORCH_CHECK(slot_meta.device().is_cpu() && slot_meta.dtype() == at::kLong &&
              slot_meta.size(0) == ns && slot_meta.size(1) == 4);
  auto sm = slot_meta.accessor<int64_t, 2>();  // table, pool, bag_len, pad_id
  const at::ScalarType id_t = ids[0].scalar_type();
  P.n_slots = ns;
  P.slot_off[0] = 0;
  for (int s = 0; s < ns; ++s) {
    Slot& S = P.slots[s];
    TORCH_CHECK(ids[s].scalar_type() == id_t, "ids of one launch must share a dtype");
    TORCH_CHECK(id_t == at::kInt || id_t == at::kLong, "ids must be int32 or int64");
    TORCH_CHECK(ids[s].is_contiguous());
    TORCH_CHECK(io[s].dim() == 2 && io[s].stride(1) == 1 && io[s].size(1) == P.dim,
                "io view must be [rows, dim] with unit column stride");
    TORCH_CHECK((reinterpret_cast<uintptr_t>(io[s].data_ptr()) % 8) == 0 && io[s].stride(0) % 4 == 0,
                "io view must be 8-byte aligned with a row stride multiple of 4");
    S.ids = ids[s].data_ptr();
    S.io = io[s].data_ptr();
    S.n = ids[s].numel();
    S.io_stride = io[s].stride(0);
    S.table = int(sm[s][0]);
    S.pool = int(sm[s][1]);
    S.bag_len = int(sm[s][2]);
    S.pad_id = int(sm[s][3]);
    TORCH_CHECK(S.table >= 0 && S.table < P.n_tables);
    TORCH_CHECK(pooled_allowed || S.pool == 0);
    S.offsets = (offsets.size() > size_t(s) && offsets[s].numel()) ? offsets[s].data_ptr<int64_t>() : nullptr;
    if (S.pool) {
      S.n_bags = S.offsets ? offsets[s].numel() - 1 : (S.bag_len > 0 ? S.n / S.bag_len : 0);
      TORCH_CHECK(io[s].size(0) == S.n_bags, "pooled output rows must equal bag count");
    } else {
      S.n_bags = 0;
      TORCH_CHECK(io[s].size(0) == S.n, "unpooled output rows must equal id count");
    }
    P.slot_off[s + 1] = P.slot_off[s] + S.n;
  }
  return id_t;
}

// Forward gather (unpooled slots).
void emb_gather(std::vector<at::Tensor> ids, std::vector<at::Tensor> outs, at::Tensor slot_meta,
                std::vector<at::Tensor> weights, std::vector<at::Tensor> shard_ptrs,
                at::Tensor table_meta, int64_t dim, at::Tensor err) {
  GatherParams P;
  P.dim = int(dim);
  TORCH_CHECK(dim % 4 == 0 && dim <= 1024, "embedding dim must be a multiple of 4 and <= 1024");
  std::vector<at::Tensor> e1;
  for (size_t i = 0; i < weights.size(); ++i) e1.push_back(at::empty({0}, weights[i].options()));
  fill_tables(P, weights, shard_ptrs, e1, e1, table_meta);
  const auto id_t = fill_slots(P, ids, outs, slot_meta, {}, false);
  const int64_t total = P.slot_off[P.n_slots];
  if (total == 0) return;
  const at::ScalarType out_t = outs[0].scalar_type();
  for (auto& o : outs) TORCH_CHECK(o.scalar_type() == out_t, "outputs of one launch must share a dtype");
  const int nvec = P.dim / 4;
  const int rows_per_warp = nvec < 32 ? 32 / nvec : 1;
  const int64_t blocks = grid_for((total + 8 * rows_per_warp - 1) / (8 * rows_per_warp), 1);
  int* e = err.data_ptr<int>();
  auto s = stream();
#define PD_LAUNCH_GATHER(IDT, OT) gather_kernel<IDT, OT><<<blocks, 256, 0, s>>>(P, total, e)
  if (id_t == at::kInt) {
    if (out_t == at::kBFloat16) PD_LAUNCH_GATHER(int32_t, __nv_bfloat16); else PD_LAUNCH_GATHER(int32_t, float);
  } else {
    if (out_t == at::kBFloat16) PD_LAUNCH_GATHER(int64_t, __nv_bfloat16); else PD_LAUNCH_GATHER(int64_t, float);
  }
#undef PD_LAUNCH_GATHER
  PD_CHECK_LAUNCH();
}

// Deduplicated unpooled gather from a routing plan: skeys / perm are the
// owner-sorted keys and their source positions, seg the unique index of each
// sorted key, uniq[u] the (table key) of unique index u.
void emb_gather_planned(std::vector<at::Tensor> ids, std::vector<at::Tensor> outs, at::Tensor slot_meta,
                        std::vector<at::Tensor> weights, std::vector<at::Tensor> shard_ptrs,
                        at::Tensor table_meta, int64_t dim, at::Tensor skeys, at::Tensor perm, at::Tensor seg,
                        at::Tensor uniq, at::Tensor err) {
  GatherParams P;
  P.dim = int(dim);
  TORCH_CHECK(dim % 8 == 0 && dim <= 1024, "planned gather: embedding dim must be a multiple of 8 and <= 1024");
  std::vector<at::Tensor> e1;
  for (size_t i = 0; i < weights.size(); ++i) e1.push_back(at::empty({0}, weights[i].options()));
  fill_tables(P, weights, shard_ptrs, e1, e1, table_meta);
  fill_slots(P, ids, outs, slot_meta, {}, false);
  const int64_t total = P.slot_off[P.n_slots];
  if (total == 0) return;
  for (auto* t : {&skeys, &perm, &seg, &uniq})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kLong && t->is_contiguous() && t->numel() == total,
                "planned gather: plan tensors must be int64 [n] on the device");
  const at::ScalarType out_t = outs[0].scalar_type();
  for (auto& o : outs) {
    TORCH_CHECK(o.scalar_type() == out_t, "outputs of one launch must share a dtype");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(o.data_ptr()) % 16 == 0 && (o.stride(0) * o.element_size()) % 16 == 0,
                "planned gather: output rows must be 16-byte aligned");
  }
  auto stage = at::empty({total, dim}, outs[0].options());   // unique rows <= positions
  TORCH_CHECK(total < (int64_t(1) << 31), "planned gather: more than 2^31 positions in one launch");
  auto u_of_pos = at::empty({total}, skeys.options().dtype(at::kInt));
  const int nvec = P.dim / 4;
  const int rows_per_warp = nvec < 32 ? 32 / nvec : 1;
  const int64_t blocks = grid_for((total + 8 * rows_per_warp - 1) / (8 * rows_per_warp), 1);
  auto s = stream();
  const int64_t* sk = skeys.data_ptr<int64_t>();
  const int64_t* pm = perm.data_ptr<int64_t>();
  const int64_t* sg = seg.data_ptr<int64_t>();
  const int64_t* uq = uniq.data_ptr<int64_t>();
  (void)sk;
  int32_t* up = u_of_pos.data_ptr<int32_t>();
  unique_of_position_kernel<<<grid_for(total, 256), 256, 0, s>>>(pm, sg, up, total);
  PD_CHECK_LAUNCH();
  if (out_t == at::kBFloat16) {
    auto* st = reinterpret_cast<__nv_bfloat16*>(stage.data_ptr());
    gather_unique_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(P, uq, sg, total, st, err.data_ptr<int>());
    PD_CHECK_LAUNCH();
    expand_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(P, st, up, total);
  } else {
    TORCH_CHECK(out_t == at::kFloat, "planned gather: bf16 or fp32 outputs");
    auto* st = stage.data_ptr<float>();
    gather_unique_kernel<float><<<blocks, 256, 0, s>>>(P, uq, sg, total, st, err.data_ptr<int>());
    PD_CHECK_LAUNCH();
    expand_kernel<float><<<blocks, 256, 0, s>>>(P, st, up, total);
  }
  PD_CHECK_LAUNCH();
}

// Forward pooled gather (sum/mean bags).
void emb_pooled(std::vector<at::Tensor> ids, std::vector<at::Tensor> outs, at::Tensor slot_meta,
                std::vector<at::Tensor> offsets, std::vector<at::Tensor> weights,
                std::vector<at::Tensor> shard_ptrs, at::Tensor table_meta, int64_t dim, at::Tensor err) {
  GatherParams P;
  P.dim = int(dim);
  TORCH_CHECK(dim % 4 == 0 && dim <= 1024);
  std::vector<at::Tensor> e1;
  for (size_t i = 0; i < weights.size(); ++i) e1.push_back(at::empty({0}, weights[i].options()));
  fill_tables(P, weights, shard_ptrs, e1, e1, table_meta);
  const auto id_t = fill_slots(P, ids, outs, slot_meta, offsets, true);
  // bag offsets over slots (slot bag counts are known on the host)
  P.bag_off[0] = 0;
  for (int s = 0; s < P.n_slots; ++s) P.bag_off[s + 1] = P.bag_off[s] + P.slots[s].n_bags;
  const int64_t total_bags = P.bag_off[P.n_slots];
  if (total_bags == 0) return;
  const at::ScalarType out_t = outs[0].scalar_type();
  const int64_t blocks = grid_for((total_bags + 7) / 8, 1);
  int* e = err.data_ptr<int>();
  auto s = stream();
#define PD_LAUNCH_POOL(IDT, OT) \
  pooled_kernel<IDT, OT><<<blocks, 256, 0, s>>>(P, total_bags, e)
  if (id_t == at::kInt) {
    if (out_t == at::kBFloat16) PD_LAUNCH_POOL(int32_t, __nv_bfloat16); else PD_LAUNCH_POOL(int32_t, float);
  } else {
    if (out_t == at::kBFloat16) PD_LAUNCH_POOL(int64_t, __nv_bfloat16); else PD_LAUNCH_POOL(int64_t, float);
  }
#undef PD_LAUNCH_POOL
  PD_CHECK_LAUNCH();
}

// Sort keys for the backward (one key per id position over all slots).
at::Tensor emb_keys(std::vector<at::Tensor> ids, std::vector<at::Tensor> grads, at::Tensor slot_meta,
                    std::vector<at::Tensor> offsets, std::vector<at::Tensor> weights,
                    std::vector<at::Tensor> shard_ptrs, at::Tensor table_meta, int64_t dim) {
  GatherParams P;
  P.dim = int(dim);
  std::vector<at::Tensor> e1;
  for (size_t i = 0; i < weights.size(); ++i) e1.push_back(at::empty({0}, weights[i].options()));
  fill_tables(P, weights, shard_ptrs, e1, e1, table_meta);
  const auto id_t = fill_slots(P, ids, grads, slot_meta, offsets, true);
  const int64_t total = P.slot_off[P.n_slots];
  auto keys = at::empty({total}, ids[0].options().dtype(at::kLong));
  if (total == 0) return keys;
  const int64_t blocks = grid_for(total, 256);
  if (id_t == at::kInt) keys_kernel<int32_t><<<blocks, 256, 0, stream()>>>(P, total, keys.data_ptr<int64_t>());
  else keys_kernel<int64_t><<<blocks, 256, 0, stream()>>>(P, total, keys.data_ptr<int64_t>());
  PD_CHECK_LAUNCH();
  return keys;
}

// Per-position scale/row for pooled slots: returns (scale f32 [N], grad_row i64 [N]).
std::vector<at::Tensor> emb_pooled_scale(std::vector<at::Tensor> ids, std::vector<at::Tensor> grads,
                                         at::Tensor slot_meta, std::vector<at::Tensor> offsets,
                                         std::vector<at::Tensor> weights,
                                         std::vector<at::Tensor> shard_ptrs, at::Tensor table_meta,
                                         int64_t dim) {
  GatherParams P;
  P.dim = int(dim);
  std::vector<at::Tensor> e1;
  for (size_t i = 0; i < weights.size(); ++i) e1.push_back(at::empty({0}, weights[i].options()));
  fill_tables(P, weights, shard_ptrs, e1, e1, table_meta);
  const auto id_t = fill_slots(P, ids, grads, slot_meta, offsets, true);
  const int64_t total = P.slot_off[P.n_slots];
  auto scale = at::empty({total}, ids[0].options().dtype(at::kFloat));
  auto row = at::empty({total}, ids[0].options().dtype(at::kLong));
  if (total == 0) return {scale, row};
  const int64_t blocks = grid_for(total, 256);
  if (id_t == at::kInt)
    pooled_scale_kernel<int32_t><<<blocks, 256, 0, stream()>>>(P, total, scale.data_ptr<float>(), row.data_ptr<int64_t>());
  else
    pooled_scale_kernel<int64_t><<<blocks, 256, 0, stream()>>>(P, total, scale.data_ptr<float>(), row.data_ptr<int64_t>());
  PD_CHECK_LAUNCH();
  return {scale, row};
}

// Scratch for runs that cross chunk boundaries: one fp32 row and one arrival
// counter per chunk. Kept zero between calls by the kernel itself.
struct ScratchCache {
  at::Tensor rows, arrivals;
};
static ScratchCache& scratch_for(int device) {
  static ScratchCache caches[64];
  return caches[device];
}

void emb_reduce_update(std::vector<at::Tensor> grads, at::Tensor slot_meta,
                       std::vector<at::Tensor> weights, std::vector<at::Tensor> shard_ptrs,
                       std::vector<at::Tensor> state1, std::vector<at::Tensor> state2,
                       at::Tensor table_meta, int64_t dim, at::Tensor sorted_keys, at::Tensor perm,
                       c10::optional<at::Tensor> scale, c10::optional<at::Tensor> grad_row,
                       int64_t opt_kind, double lr, double eps, double weight_decay, double beta1,
                       double beta2, double bc1, double bc2, at::Tensor err,
                       c10::optional<at::Tensor> out_rows, c10::optional<at::Tensor> seg) {
  GatherParams P;
  P.dim = int(dim);
  fill_tables(P, weights, shard_ptrs, state1, state2, table_meta);
  // grads are described as slots whose ids are unused here: use the sorted
  // keys tensor as a dummy id array of the right length per slot.
  const int ns = int(grads.size());
  TORCH_CHECK(ns >= 1 && ns <= kMaxSlots);
  auto sm = slot_meta.accessor<int64_t, 2>();
  P.n_slots = ns;
  P.slot_off[0] = 0;
  TORCH_CHECK(slot_meta.size(1) == 5, "slot_meta for reduce_update: table, pool, bag_len, pad, n_ids");
  for (int s = 0; s < ns; ++s) {
    Slot& S = P.slots[s];
    TORCH_CHECK(grads[s].dim() == 2 && grads[s].stride(1) == 1 && grads[s].size(1) == dim);
    S.ids = nullptr;
    S.io = grads[s].data_ptr();
    S.io_stride = grads[s].stride(0);
    S.table = int(sm[s][0]); S.pool = int(sm[s][1]); S.bag_len = int(sm[s][2]); S.pad_id = int(sm[s][3]);
    S.n = sm[s][4];
    S.offsets = nullptr; S.n_bags = 0;
    P.slot_off[s + 1] = P.slot_off[s] + S.n;
  }
  const int64_t total = P.slot_off[ns];
  TORCH_CHECK(sorted_keys.numel() == total && perm.numel() == total);
  if (total == 0) return;
  const at::ScalarType gt = grads[0].scalar_type();
  for (auto& g : grads) TORCH_CHECK(g.scalar_type() == gt);
  OptParams O{int(opt_kind), float(lr), float(eps), float(weight_decay), float(beta1), float(beta2),
              float(bc1), float(bc2)};
  GradSrc src{perm.data_ptr<int64_t>(), scale ? scale->data_ptr<float>() : nullptr,
              grad_row ? grad_row->data_ptr<int64_t>() : nullptr, nullptr, nullptr};
  if (out_rows && out_rows->defined() && out_rows->numel() > 0) {
    TORCH_CHECK(seg && seg->numel() == total && out_rows->scalar_type() == at::kFloat &&
                out_rows->is_contiguous() && out_rows->size(-1) == dim,
                "reduce-only mode needs fp32 out_rows [U, dim] and seg [N]");
    src.out_rows = out_rows->data_ptr<float>();
    src.seg = seg->data_ptr<int64_t>();
  }
  const int64_t n_chunks = (total + kChunk - 1) / kChunk;
  const int dev = weights[0].get_device();
  ScratchCache& sc = scratch_for(dev);
  if (!sc.rows.defined() || sc.rows.numel() < n_chunks * dim) {
    sc.rows = at::zeros({n_chunks * dim + dim}, weights[0].options());
    sc.arrivals = at::zeros({n_chunks + 1}, weights[0].options().dtype(at::kInt));
  }
  // staged path: rows of at most 512 bytes, 16-byte aligned rows in every grad view
  const int64_t rb = dim * (gt == at::kBFloat16 ? 2 : 4);
  bool staged = rb % 16 == 0 && rb <= kStageMaxRowBytes;
  for (auto& g : grads)
    staged = staged && reinterpret_cast<uintptr_t>(g.data_ptr()) % 16 == 0 && (g.stride(0) * g.element_size()) % 16 == 0;
  if (staged) {
    const int threads = rb <= 256 ? 256 : 128;          // 64 KB of stage per block either way
    const size_t smem = size_t(threads / 32) * kChunk * rb;
    const int64_t blocks = grid_for((n_chunks + threads / 32 - 1) / (threads / 32), 1);
    auto launch = [&](auto kern) {
      PD_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
      kern<<<blocks, threads, smem, stream()>>>(P, O, sorted_keys.data_ptr<int64_t>(), src, total,
                                                sc.rows.data_ptr<float>(), sc.arrivals.data_ptr<int>(),
                                                err.data_ptr<int>());
    };
    // accumulators sized to the row: one float4 per lane per 128 columns
    const int64_t nv = dim / 4;
    if (gt == at::kBFloat16) {
      if (nv <= 32) launch(reduce_update_staged_kernel<__nv_bfloat16, 1>);
      else launch(reduce_update_staged_kernel<__nv_bfloat16, 2>);
    } else {
      launch(reduce_update_staged_kernel<float, 1>);   // fp32 rows of at most 512 bytes: dim <= 128
    }
    PD_CHECK_LAUNCH();
    return;
  }
  const int64_t blocks = grid_for((n_chunks + 7) / 8, 1);
  if (gt == at::kBFloat16)
    reduce_update_kernel<__nv_bfloat16><<<blocks, 256, 0, stream()>>>(
        P, O, sorted_keys.data_ptr<int64_t>(), src, total, sc.rows.data_ptr<float>(),
        sc.arrivals.data_ptr<int>(), err.data_ptr<int>());
  else
    reduce_update_kernel<float><<<blocks, 256, 0, stream()>>>(
        P, O, sorted_keys.data_ptr<int64_t>(), src, total, sc.rows.data_ptr<float>(),
        sc.arrivals.data_ptr<int>(), err.data_ptr<int>());
  PD_CHECK_LAUNCH();
}

}  // namespace pd

// ---------------------------------------------------------------------------
// Allocation-free variant of the fused sparse update (declared in noalloc.h).
// Same kernel as emb_reduce_update, for one table, with its scratch rows and
// arrival counters taken from fixed file-scope device arrays instead of the
// PyTorch allocator.
// ---------------------------------------------------------------------------
#include <mutex>

#include "noalloc.h"

namespace pd {
namespace {
constexpr int64_t kNaChunks = PD_NOALLOC_MAX_IDS / kChunk;
static __device__ __align__(256) float g_na_scratch[kNaChunks * PD_NOALLOC_MAX_DIM];
static __device__ __align__(256) int g_na_arrivals[kNaChunks];

struct NaDevice {
  bool ready = false;
  float* scratch = nullptr;
  int* arrivals = nullptr;
};
std::mutex g_na_mu;
NaDevice g_na_dev[128];
}  // namespace
}  // namespace pd

extern "C" int pd_emb_sparse_update_noalloc(
    const int64_t* sorted_keys, const int64_t* perm, int64_t n, const void* grads, int grad_dtype,
    int64_t grad_stride, float* weight, int64_t rows, int dim, float* state1, float* state2, int opt_kind,
    float lr, float eps, float weight_decay, float beta1, float beta2, float bc1, float bc2, int* err,
    cudaStream_t stream) {
  using namespace pd;
  if (n < 0 || dim <= 0) return PD_NOALLOC_BAD_ARG;
  if (n > PD_NOALLOC_MAX_IDS || dim > PD_NOALLOC_MAX_DIM) return PD_NOALLOC_TOO_LARGE;
  if (dim % 4 != 0 || opt_kind < 0 || opt_kind > 3 || (grad_dtype != 0 && grad_dtype != 1)) return PD_NOALLOC_BAD_ARG;
  if (n == 0) return 0;
  if (!sorted_keys || !perm || !grads || !weight || rows <= 0) return PD_NOALLOC_BAD_ARG;
  if ((opt_kind == 1 || opt_kind == 2) && !state1) return PD_NOALLOC_BAD_ARG;
  if (opt_kind == 3 && (!state1 || !state2)) return PD_NOALLOC_BAD_ARG;
  // The kernel reads a gradient row as 4-element vectors (16 bytes fp32, 8
  // bytes bf16) and the table / per-element state rows as float4.
  if (grad_stride < dim || grad_stride % 4 != 0) return PD_NOALLOC_BAD_ARG;
  auto misaligned = [](const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) != 0; };
  if (misaligned(grads, grad_dtype == 1 ? 8 : 16) || misaligned(weight, 16)) return PD_NOALLOC_BAD_ARG;
  if ((opt_kind == 1 || opt_kind == 3) && misaligned(state1, 16)) return PD_NOALLOC_BAD_ARG;
  if (opt_kind == 2 && misaligned(state1, 4)) return PD_NOALLOC_BAD_ARG;
  if (opt_kind == 3 && misaligned(state2, 16)) return PD_NOALLOC_BAD_ARG;
  if (misaligned(sorted_keys, 8) || misaligned(perm, 8) || (err && misaligned(err, 4))) return PD_NOALLOC_BAD_ARG;

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return int(e);
  if (dev < 0 || dev >= 128) return PD_NOALLOC_BAD_ARG;
  NaDevice* nd = &g_na_dev[dev];
  {
    std::lock_guard<std::mutex> lock(g_na_mu);
    if (!nd->ready) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_na_scratch);
      if (e != cudaSuccess) return int(e);
      nd->scratch = static_cast<float*>(p);
      e = cudaGetSymbolAddress(&p, g_na_arrivals);
      if (e != cudaSuccess) return int(e);
      nd->arrivals = static_cast<int*>(p);
      nd->ready = true;
    }
  }
  const int64_t n_chunks = (n + kChunk - 1) / kChunk;
  e = cudaMemsetAsync(nd->scratch, 0, size_t(n_chunks) * dim * sizeof(float), stream);
  if (e != cudaSuccess) return int(e);
  e = cudaMemsetAsync(nd->arrivals, 0, size_t(n_chunks) * sizeof(int), stream);
  if (e != cudaSuccess) return int(e);

  GatherParams P;
  memset(&P, 0, sizeof(P));
  P.dim = dim;
  P.n_slots = 1;
  P.slots[0].io = const_cast<void*>(grads);
  P.slots[0].io_stride = grad_stride;
  P.slots[0].n = n;
  P.slot_off[0] = 0;
  P.slot_off[1] = n;
  P.n_tables = 1;
  Table& T = P.tables[0];
  T.local = weight;
  T.state1 = state1;
  T.state2 = state2;
  T.rows = rows;
  T.chunk = rows;
  T.local_rows = rows;
  T.n_shards = 1;
  T.dim = dim;
  OptParams O{opt_kind, lr, eps, weight_decay, beta1, beta2, bc1, bc2};
  GradSrc src{perm, nullptr, nullptr, nullptr, nullptr, n};
  int64_t blocks = (n_chunks + 7) / 8;
  const int64_t cap = int64_t(num_sms()) * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  if (grad_dtype == 1)
    reduce_update_kernel<__nv_bfloat16><<<blocks, 256, 0, stream>>>(P, O, sorted_keys, src, n, nd->scratch,
                                                                    nd->arrivals, err);
  else
    reduce_update_kernel<float><<<blocks, 256, 0, stream>>>(P, O, sorted_keys, src, n, nd->scratch, nd->arrivals,
                                                            err);
  e = cudaGetLastError();
  if (e == cudaSuccess) note_launch();
  return int(e);
}
