// Peer-memory data plane over NVLink / NVSwitch (one process per GPU).
//
//  * alloc_shared / ipc_handle / ipc_open: device buffers whose handles are
//    exchanged over the process group (CUDA IPC), so every rank can load and
//    store another rank's buffer directly.
//  * push_rows: the backward half of the sparse embedding exchange. Each rank
//    has its gradient rows reduced per unique (table, row) key and grouped by
//    owner; one kernel writes every row straight into its owner's receive
//    slab (16-byte peer stores), at an offset the ranks agreed on from the
//    exchanged counts. Rows of replicated (data-parallel) tables go to every
//    rank.
//  * signal_barrier: each rank stores an epoch into a flag slot of every
//    peer's signal pad (system-scope release) and waits (bounded, on
//    %globaltimer) until all peers' epochs arrived in its own pad. On timeout
//    it records kWaitTimeout in the error word and returns: it never hangs.
#include "common.cuh"
#include "driver_api.h"

namespace pd {

// ---------------------------------------------------------------------------
// buffers and IPC
// ---------------------------------------------------------------------------

at::Tensor alloc_shared(int64_t nbytes, int64_t device) {
  TORCH_CHECK(nbytes > 0);
  int prev = 0;
  PD_CHECK_CUDA(cudaGetDevice(&prev));
  PD_CHECK_CUDA(cudaSetDevice(int(device)));
  void* p = nullptr;
  PD_CHECK_CUDA(cudaMalloc(&p, size_t(nbytes)));
  PD_CHECK_CUDA(cudaMemset(p, 0, size_t(nbytes)));
  PD_CHECK_CUDA(cudaSetDevice(prev));
  auto opts = at::TensorOptions().dtype(at::kByte).device(at::kCUDA, int(device));
  return at::from_blob(p, {nbytes}, [](void* q) { cudaFree(q); }, opts);
}

// Returns a CPU uint8 tensor: 64-byte cudaIpcMemHandle_t followed by the
// int64 byte offset of `t`'s data from the start of its allocation.
at::Tensor ipc_handle(at::Tensor t) {
  TORCH_CHECK(t.is_cuda());
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = mem_get_address_range(&base, &size, reinterpret_cast<CUdeviceptr>(t.data_ptr()));
  PD_CHECK(r == CUDA_SUCCESS, "cuMemGetAddressRange failed: %d", int(r));
  cudaIpcMemHandle_t h;
  PD_CHECK_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  auto out = at::empty({int64_t(sizeof(h) + 8)}, at::TensorOptions().dtype(at::kByte));
  memcpy(out.data_ptr(), &h, sizeof(h));
  int64_t off = int64_t(reinterpret_cast<CUdeviceptr>(t.data_ptr()) - base);
  memcpy(static_cast<uint8_t*>(out.data_ptr()) + sizeof(h), &off, 8);
  return out;
}

// Opens a peer handle on the current device; returns the mapped address of
// the peer tensor (allocation base + offset) and the base (for ipc_close).
std::vector<int64_t> ipc_open(at::Tensor handle) {
  TORCH_CHECK(handle.numel() == int64_t(sizeof(cudaIpcMemHandle_t) + 8));
  cudaIpcMemHandle_t h;
  memcpy(&h, handle.data_ptr(), sizeof(h));
  int64_t off = 0;
  memcpy(&off, static_cast<uint8_t*>(handle.data_ptr()) + sizeof(h), 8);
  void* p = nullptr;
  PD_CHECK_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return {int64_t(reinterpret_cast<uintptr_t>(p)) + off, int64_t(reinterpret_cast<uintptr_t>(p))};
}

void ipc_close(int64_t base) {
  PD_CHECK_CUDA(cudaIpcCloseMemHandle(reinterpret_cast<void*>(static_cast<uintptr_t>(base))));
}

// ---------------------------------------------------------------------------
// push of reduced gradient rows to their owners
// ---------------------------------------------------------------------------
// Receive slab layout on every rank: keys int64 [cap] then rows fp32 [cap, dim].
// Receive layout on rank d: rows it owns from source 0, 1, ..., W-1, then rows
// of replicated tables from source 0, 1, ..., W-1.
struct PushParams {
  int64_t* peer_keys[64];   // per rank: receive key array
  float* peer_rows[64];     // per rank: receive row array
  int64_t dst_off[64];      // per owner: first slot this rank writes at that owner
  int64_t bcast_off[64];    // per destination: first slot of this rank's replicated rows there
  int64_t seg_start[66];    // per owner 0..W (W = replicated): first unique index of its segment
  int world;
};

__global__ void __launch_bounds__(256) push_rows_kernel(const __grid_constant__ PushParams P,
                                                        const int64_t* __restrict__ keys,
                                                        const float* __restrict__ rows, int64_t n, int dim) {
  const int lane = threadIdx.x & 31;
  const int nvec = dim >> 2;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t u = warp; u < n; u += nw) {
    int o = 0;
    while (o < P.world && P.seg_start[o + 1] <= u) ++o;  // owner segment (<= 65 entries)
    const int64_t j = u - P.seg_start[o];
    const float4* src = reinterpret_cast<const float4*>(rows + u * dim);
    const int first = (o == P.world) ? 0 : o;
    const int last = (o == P.world) ? P.world - 1 : o;
    for (int d = first; d <= last; ++d) {
      const int64_t slot = (o == P.world ? P.bcast_off[d] : P.dst_off[o]) + j;
      int64_t* kd = P.peer_keys[d];
      float4* rd = reinterpret_cast<float4*>(P.peer_rows[d] + slot * dim);
      if (lane == 0) kd[slot] = keys[u];
      for (int v = lane; v < nvec; v += 32) rd[v] = src[v];
    }
  }
}

// keys/rows: this rank's unique keys (sorted by owner) and reduced rows.
// peer_keys / peer_rows: int64 CPU tensors [W] of mapped receive addresses.
// dst_off, bcast_off: int64 CPU [W]; seg_start: int64 CPU [W+2].
void push_rows(at::Tensor keys, at::Tensor rows, at::Tensor peer_keys, at::Tensor peer_rows,
               at::Tensor dst_off, at::Tensor bcast_off, at::Tensor seg_start) {
  const int W = int(peer_keys.numel());
  TORCH_CHECK(W >= 1 && W <= 64);
  TORCH_CHECK(rows.scalar_type() == at::kFloat && rows.is_contiguous() && rows.dim() == 2);
  TORCH_CHECK(keys.scalar_type() == at::kLong && keys.numel() == rows.size(0));
  const int dim = int(rows.size(1));
  TORCH_CHECK(dim % 4 == 0);
  PushParams P;
  P.world = W;
  auto pk = peer_keys.accessor<int64_t, 1>();
  auto pr = peer_rows.accessor<int64_t, 1>();
  for (int r = 0; r < W; ++r) {
    P.peer_keys[r] = reinterpret_cast<int64_t*>(static_cast<uintptr_t>(pk[r]));
    P.peer_rows[r] = reinterpret_cast<float*>(static_cast<uintptr_t>(pr[r]));
  }
  auto d = dst_off.accessor<int64_t, 1>();
  auto b = bcast_off.accessor<int64_t, 1>();
  auto s = seg_start.accessor<int64_t, 1>();
  for (int r = 0; r < W; ++r) { P.dst_off[r] = d[r]; P.bcast_off[r] = b[r]; }
  for (int r = 0; r <= W + 1; ++r) P.seg_start[r] = s[r];
  const int64_t n = keys.numel();
  if (n == 0) return;
  int64_t blocks = (n + 7) / 8;
  const int64_t cap = int64_t(num_sms()) * 8;
  if (blocks > cap) blocks = cap;
  push_rows_kernel<<<blocks, 256, 0, stream()>>>(P, keys.data_ptr<int64_t>(), rows.data_ptr<float>(), n, dim);
  PD_CHECK_LAUNCH();
}

// ---------------------------------------------------------------------------
// one small int64 row from this rank into a board on every rank
// ---------------------------------------------------------------------------
// Board on every rank: int64 [W, n]; this rank writes its row at index rank of
// every peer's board (the routing counts of the sparse exchange). A signal
// barrier after it publishes the rows.
struct PeerRowParams {
  int64_t* boards[64];
  int world;
  int rank;
};

__global__ void peer_put_row_kernel(const __grid_constant__ PeerRowParams P, const int64_t* __restrict__ src, int n) {
  for (int d = blockIdx.x; d < P.world; d += gridDim.x)
    for (int i = threadIdx.x; i < n; i += blockDim.x) P.boards[d][int64_t(P.rank) * n + i] = src[i];
}

void peer_put_row(at::Tensor src, at::Tensor boards, int64_t rank) {
  const int W = int(boards.numel());
  TORCH_CHECK(W >= 1 && W <= 64 && rank >= 0 && rank < W);
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == at::kLong && src.is_contiguous() && src.dim() == 1);
  PeerRowParams P;
  P.world = W;
  P.rank = int(rank);
  auto a = boards.accessor<int64_t, 1>();
  for (int r = 0; r < W; ++r) P.boards[r] = reinterpret_cast<int64_t*>(static_cast<uintptr_t>(a[r]));
  const int n = int(src.numel());
  if (n == 0) return;
  peer_put_row_kernel<<<W, 128, 0, stream()>>>(P, src.data_ptr<int64_t>(), n);
  PD_CHECK_LAUNCH();
}

// ---------------------------------------------------------------------------
// barrier over signal pads
// ---------------------------------------------------------------------------
struct BarrierParams {
  int64_t* pads[64];  // per rank: that rank's signal pad (int64 [64])
  int world;
  int rank;
};

__global__ void signal_barrier_kernel(const __grid_constant__ BarrierParams P, int64_t epoch,
                                      int64_t timeout_ns, int* err) {
  const int t = threadIdx.x;
  __threadfence_system();
  __syncthreads();
  if (t < P.world) {
    int64_t* slot = P.pads[t] + P.rank;
    asm volatile("st.release.sys.global.b64 [%0], %1;" ::"l"(slot), "l"(epoch) : "memory");
  }
  if (t < P.world) {
    const int64_t* mine = P.pads[P.rank] + t;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
      int64_t v;
      asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(mine) : "memory");
      if (v >= epoch) break;
      if (globaltimer_ns() - t0 > uint64_t(timeout_ns)) {
        set_error(err, kWaitTimeout);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  __threadfence_system();
}

void signal_barrier(at::Tensor pads, int64_t rank, int64_t epoch, int64_t timeout_ns, at::Tensor err) {
  const int W = int(pads.numel());
  TORCH_CHECK(W >= 1 && W <= 64 && rank >= 0 && rank < W);
  BarrierParams P;
  P.world = W;
  P.rank = int(rank);
  auto a = pads.accessor<int64_t, 1>();
  for (int r = 0; r < W; ++r) P.pads[r] = reinterpret_cast<int64_t*>(static_cast<uintptr_t>(a[r]));
  signal_barrier_kernel<<<1, 64, 0, stream()>>>(P, epoch, timeout_ns, err.data_ptr<int>());
  PD_CHECK_LAUNCH();
}

// ---------------------------------------------------------------------------
// dense gradient / parameter collectives over peer memory
//
// Every rank's flat fp32 buffer is mapped into every rank (CUDA IPC), and
// the buffer is split into W slices (64-element aligned). Between signal
// barriers:
//   peer_reduce_slice: this rank's slice = scale * sum over ranks of that
//     slice, read with L1-bypassing loads from each peer (NVLink P2P), written
//     into this rank's own buffer (two-shot reduce-scatter, first half);
//   peer_gather_slices: every other rank's (final) slice is copied from that
//     rank into this rank's buffer (second half, an all-gather).
// Slices are disjoint, so no rank writes memory another rank reads in the
// same phase; the barrier after the gather keeps a rank from reusing its
// buffer while peers still read it.
// ---------------------------------------------------------------------------
constexpr int kMaxPeers = 16;
struct PeerBufs {
  const float* buf[kMaxPeers];
  int world;
  int rank;
};

__global__ void __launch_bounds__(512) peer_reduce_slice_kernel(const __grid_constant__ PeerBufs P, float* __restrict__ own,
                                                                int64_t a, int64_t b, float scale) {
  const int64_t n4 = (b - a) >> 2;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const int64_t off = a + 4 * i;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (int p = 0; p < P.world; ++p) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(P.buf[p] + off));
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    acc.x *= scale; acc.y *= scale; acc.z *= scale; acc.w *= scale;
    *reinterpret_cast<float4*>(own + off) = acc;
  }
}

__global__ void __launch_bounds__(512) peer_gather_slices_kernel(const __grid_constant__ PeerBufs P, float* __restrict__ own,
                                                                 const int64_t* __restrict__ bounds) {
  // bounds: [world + 1] slice boundaries (elements); blockIdx.y = source rank
  const int src = blockIdx.y;
  if (src == P.rank) return;
  const int64_t a = bounds[src], b = bounds[src + 1];
  const int64_t n4 = (b - a) >> 2;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  const float* from = P.buf[src];
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const int64_t off = a + 4 * i;
    *reinterpret_cast<float4*>(own + off) = __ldcg(reinterpret_cast<const float4*>(from + off));
  }
}

static PeerBufs peer_bufs(const at::Tensor& ptrs, int64_t rank) {
  const int W = int(ptrs.numel());
  TORCH_CHECK(W >= 1 && W <= kMaxPeers && rank >= 0 && rank < W, "1..16 ranks");
  PeerBufs P;
  P.world = W;
  P.rank = int(rank);
  auto a = ptrs.accessor<int64_t, 1>();
  for (int r = 0; r < W; ++r) {
    P.buf[r] = reinterpret_cast<const float*>(static_cast<uintptr_t>(a[r]));
    TORCH_CHECK(a[r] % 16 == 0, "peer buffers must be 16-byte aligned");
  }
  return P;
}

// own[a:b) = scale * sum_r peer_r[a:b); a, b multiples of 4.
// max_blocks > 0 caps the grid (a collective overlapped with compute takes a
// few SMs' worth of CTAs instead of the whole GPU).
void peer_reduce_slice(at::Tensor ptrs, int64_t rank, at::Tensor own, int64_t a, int64_t b, double scale,
                       int64_t max_blocks) {
  TORCH_CHECK(own.is_cuda() && own.scalar_type() == at::kFloat && own.is_contiguous());
  TORCH_CHECK(a >= 0 && b <= own.numel() && a % 4 == 0 && b % 4 == 0 && a <= b, "slice must be 4-aligned");
  const PeerBufs P = peer_bufs(ptrs, rank);
  if (b == a) return;
  int64_t blocks = ((b - a) / 4 + 511) / 512;
  const int64_t cap = max_blocks > 0 ? max_blocks : int64_t(num_sms()) * 4;
  if (blocks > cap) blocks = cap;
  peer_reduce_slice_kernel<<<blocks, 512, 0, stream()>>>(P, own.data_ptr<float>(), a, b, float(scale));
  PD_CHECK_LAUNCH();
}

// own[slice q] = peer_q[slice q] for every q != rank; bounds: int64 CUDA [W + 1].
void peer_gather_slices(at::Tensor ptrs, int64_t rank, at::Tensor own, at::Tensor bounds, int64_t span,
                        int64_t max_blocks) {
  TORCH_CHECK(own.is_cuda() && own.scalar_type() == at::kFloat && own.is_contiguous());
  TORCH_CHECK(bounds.is_cuda() && bounds.scalar_type() == at::kLong && bounds.numel() == ptrs.numel() + 1);
  const PeerBufs P = peer_bufs(ptrs, rank);
  // span: elements the bounds cover (0: the whole buffer), sizes the grid
  const int64_t per = (span > 0 ? span : own.numel()) / P.world + 1;
  int64_t blocks = (per / 4 + 511) / 512;
  const int64_t cap = max_blocks > 0 ? (max_blocks + P.world - 2) / (P.world > 1 ? P.world - 1 : 1)
                                     : int64_t(num_sms()) * 4 / (P.world > 1 ? P.world - 1 : 1) + 1;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  peer_gather_slices_kernel<<<dim3(unsigned(blocks), unsigned(P.world)), 512, 0, stream()>>>(
      P, own.data_ptr<float>(), bounds.data_ptr<int64_t>());
  PD_CHECK_LAUNCH();
}

// ---------------------------------------------------------------------------
// owner of each (table, row) key; composite sort key = owner << 44 | key
// ---------------------------------------------------------------------------
constexpr int kMaxTablesComm = 32;
constexpr int kOwnerShift = 44;

struct OwnerParams {
  int64_t key_base[kMaxTablesComm + 1];
  int64_t chunk[kMaxTablesComm];
  int32_t kind[kMaxTablesComm];   // 0 row-wise, 1 fixed owner, 2 replicated (owner = W)
  int32_t owner[kMaxTablesComm];
  int n_tables;
  int world;
};

__global__ void owner_keys_kernel(const __grid_constant__ OwnerParams P, const int64_t* __restrict__ keys,
                                  int64_t* __restrict__ out, int64_t n) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t k = keys[i];
    if (k == INT64_MAX) { out[i] = INT64_MAX; continue; }
    int t = 0;
    while (t + 1 < P.n_tables && P.key_base[t + 1] <= k) ++t;
    int64_t o;
    if (P.kind[t] == 0) {
      o = (k - P.key_base[t]) / P.chunk[t];
      if (o >= P.world) o = P.world - 1;
    } else if (P.kind[t] == 1) {
      o = P.owner[t];
    } else {
      o = P.world;
    }
    out[i] = (o << kOwnerShift) | k;
  }
}

// meta: int64 CPU [n_tables, 4] = key_base, chunk, kind, owner.
at::Tensor owner_keys(at::Tensor keys, at::Tensor meta, int64_t world) {
  const int nt = int(meta.size(0));
  TORCH_CHECK(nt >= 1 && nt <= kMaxTablesComm && meta.size(1) == 4);
  OwnerParams P;
  auto m = meta.accessor<int64_t, 2>();
  for (int t = 0; t < nt; ++t) {
    P.key_base[t] = m[t][0]; P.chunk[t] = m[t][1] > 0 ? m[t][1] : 1;
    P.kind[t] = int(m[t][2]); P.owner[t] = int(m[t][3]);
  }
  P.n_tables = nt;
  P.world = int(world);
  auto out = at::empty_like(keys);
  const int64_t n = keys.numel();
  if (n == 0) return out;
  int64_t blocks = (n + 255) / 256;
  const int64_t cap = int64_t(num_sms()) * 16;
  if (blocks > cap) blocks = cap;
  owner_keys_kernel<<<blocks, 256, 0, stream()>>>(P, keys.data_ptr<int64_t>(), out.data_ptr<int64_t>(), n);
  PD_CHECK_LAUNCH();
  return out;
}

}  // namespace pd
