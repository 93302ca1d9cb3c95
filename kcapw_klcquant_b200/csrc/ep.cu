// Expert-parallel dispatch and combine over NVLink peer memory.
//
// Experts are sharded contiguously over the ranks of one node (rank r owns
// experts [r*epr, (r+1)*epr)).  Every rank owns an exchange arena in its own
// HBM that the other ranks map through CUDA IPC (plain peer mappings over
// NVLink/NVSwitch, no multicast objects):
//
//   flag_dispatch u32 [world]          written by source s: the epoch of its last dispatch
//   flag_combine  u32 [world]          written by destination d: the epoch of its last return
//   counts        i32 [world]          rows source s sent in its last dispatch
//   recv_meta     i32 [world][cap]     local expert id of each received row
//   recv_rows     bf16 [world][cap][H] token rows, one segment per source
//   back_rows     bf16 [world][cap][H] expert outputs, one segment per destination
//   --- local only ---
//   status, done counters, epoch (u32: forwards dispatched so far), recv_expert
//   i32 [world][cap] (expert id or -1 = empty slot)
//
// The epoch lives in device memory and every kernel reads it there (the send
// kernel's last CTA advances it), so a captured CUDA graph of forwards replays
// with fresh epochs.
//
// One layer forward on every rank, all stream-ordered, no host synchronisation:
//   1. dispatch: stable counting sort of the rank's (token, slot) pairs by
//      owner rank (the permute kernels), then ep_send_kernel stores each pair's
//      token row and expert id straight into the owner's arena, in the segment
//      of this source at the pair's position in the sorted order; its last CTA
//      writes the per-destination counts and then the dispatch flags.
//   2. experts: ep_fill_kernel waits (bounded) for every source's dispatch flag
//      and marks each received slot with its expert id or -1; the local expert
//      GEMMs run on the received rows (k = 1, empty slots skipped).  The down
//      GEMM's epilogue stores every expert output row straight into the
//      source's back_rows segment of this destination over NVLink, so the
//      return overlaps the GEMM tiles (weights-as-N kernels, up to 8 ranks;
//      otherwise ep_return_kernel copies the rows afterwards); then the
//      combine flags are raised.
//   3. combine: ep_wait_kernel waits (bounded) for every destination's combine
//      flag; the weighted combine (combine.cu) reads back_rows by the slot the
//      dispatch recorded for each pair, in top-k order: the reference's combine
//      order, so the result equals the single-GPU layer.
//
// Capacity: a source's segment holds cap = max_tokens * k rows, enough for all
// of its pairs going to one destination, so nothing can overflow.  Reuse is safe
// without further handshakes: a source starts its next dispatch only after its
// combine saw every destination's return, which each destination issues after
// its expert kernels finished reading the received rows; likewise for back_rows.
//
// Every wait is bounded (%globaltimer): on expiry the kernel records
// KLC_ERR_DEVICE_TIMEOUT with the waited-for rank in the arena's status word,
// treats the missing segment as empty and returns.
#include <cstring>
#include <mutex>
#include <vector>

#include "permute.cuh"

namespace klc {

namespace {

constexpr int kMaxRanks = 64;
constexpr uint64_t kDefaultWaitNs = 10ull * 1000000000ull;  // 10 s

struct ArenaLayout {
  size_t flag_dispatch, flag_combine, counts, recv_meta, recv_rows, back_rows;  // written by peers
  size_t status, done, epoch, recv_expert, ones;                              // local
  size_t total;
};

ArenaLayout arena_layout(int world, int64_t cap, int64_t hidden) {
  ArenaLayout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + (bytes > 0 ? bytes : 1), 256);
    return o;
  };
  const size_t slots = size_t(world) * size_t(cap);
  L.flag_dispatch = take(size_t(world) * 4);
  L.flag_combine = take(size_t(world) * 4);
  L.counts = take(size_t(world) * 4);
  L.recv_meta = take(slots * 4);
  L.recv_rows = take(slots * size_t(hidden) * 2);
  L.back_rows = take(slots * size_t(hidden) * 2);
  L.status = take(sizeof(DeviceStatus));
  L.done = take(2 * sizeof(unsigned int));
  L.epoch = take(sizeof(uint32_t));
  L.recv_expert = take(slots * 4);
  L.ones = take(slots * 2);
  L.total = off;
  return L;
}

struct PeerBases {
  char* base[kMaxRanks];
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// One warp copies a row of 16-byte chunks to (peer) memory with four loads in flight
// per lane before their stores, so the local reads do not serialise the remote writes.
__device__ __forceinline__ void copy_row(uint4* __restrict__ dst, const uint4* __restrict__ src, int chunks, int lane) {
  int c = lane;
  for (; c + 96 < chunks; c += 128) {
    const uint4 v0 = src[c], v1 = src[c + 32], v2 = src[c + 64], v3 = src[c + 96];
    dst[c] = v0;
    dst[c + 32] = v1;
    dst[c + 64] = v2;
    dst[c + 96] = v3;
  }
  for (; c < chunks; c += 32) dst[c] = src[c];
}

// Bounded wait until *flag >= epoch (wrap-aware); false on expiry.
__device__ bool wait_flag(const uint32_t* flag, uint32_t epoch, uint64_t limit_ns) {
  if (int32_t(ld_acquire_sys(flag) - epoch) >= 0) return true;
  const uint64_t t0 = gtimer();
  while (int32_t(ld_acquire_sys(flag) - epoch) < 0) {
    if (gtimer() - t0 > limit_ns) return false;
    __nanosleep(128);
  }
  return true;
}

// Last-CTA signal: every CTA makes its peer stores visible system-wide and
// counts itself done; the last one writes the counts (dispatch) and the flag
// of this rank into every peer's arena, then rearms the counter.
__device__ bool signal_peers(const PeerBases& peers, int world, int rank, unsigned int* done, size_t flag_off,
                             size_t counts_off, const int32_t* counts, uint32_t epoch) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x != 0) return false;
  const unsigned int prev = atomicAdd(done, 1u);
  if (prev != gridDim.x - 1) return false;
  __threadfence_system();
  for (int d = 0; d < world; ++d) {
    char* b = peers.base[d];
    if (counts != nullptr) reinterpret_cast<volatile int32_t*>(b + counts_off)[rank] = counts[d];
  }
  __threadfence_system();
  for (int d = 0; d < world; ++d) st_release_sys(reinterpret_cast<uint32_t*>(peers.base[d] + flag_off) + rank, epoch);
  *done = 0u;  // the next launch using this counter starts after this kernel ends
  return true;
}

// 1. token rows of every (token, slot) pair into the owner rank's arena
__global__ void __launch_bounds__(256)
    ep_send_kernel(const int32_t* __restrict__ idx, const int32_t* __restrict__ pair_pos, const int32_t* __restrict__ offsets,
                   const int32_t* __restrict__ counts, int64_t pairs, int k, int epr, int world, int rank, int64_t cap,
                   const uint16_t* __restrict__ x, int64_t hidden, int32_t* __restrict__ pair_slot, PeerBases peers,
                   ArenaLayout L, char* arena) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  const int chunks = int(hidden / 8);
  // this forward's epoch; the last CTA advances the stored one after every CTA read it
  uint32_t* epoch_p = reinterpret_cast<uint32_t*>(arena + L.epoch);
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(epoch_p) + 1u;
  unsigned int* done = reinterpret_cast<unsigned int*>(arena + L.done);
  for (int64_t p = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); p < pairs; p += warps) {
    const int v = idx[p];
    const int d = v / epr;  // validated by the permute (faults recorded, pair_pos -1)
    const int pp = pair_pos[p];
    if (pp < 0 || d < 0 || d >= world) {
      if (lane == 0) pair_slot[p] = -1;
      continue;
    }
    const int64_t pos = pp - offsets[d];
    const int64_t slot = int64_t(rank) * cap + pos;  // this source's segment in the owner's arena
    char* b = peers.base[d];
    const uint4* src = reinterpret_cast<const uint4*>(x + (p / k) * hidden);
    uint4* dst = reinterpret_cast<uint4*>(b + L.recv_rows + size_t(slot) * size_t(hidden) * 2);
    copy_row(dst, src, chunks, lane);
    if (lane == 0) {
      reinterpret_cast<int32_t*>(b + L.recv_meta)[slot] = v - d * epr;
      pair_slot[p] = int32_t(int64_t(d) * cap + pos);
    }
  }
  if (signal_peers(peers, world, rank, done, L.flag_dispatch, L.counts, counts, epoch)) *epoch_p = epoch;
}

// 2a. wait for every source's rows, mark the received slots
__global__ void __launch_bounds__(256)
    ep_fill_kernel(char* arena, ArenaLayout L, int64_t cap, uint64_t limit_ns) {
  const int s = blockIdx.y;
  const uint32_t epoch = *reinterpret_cast<const volatile uint32_t*>(arena + L.epoch);
  __shared__ int count;
  if (threadIdx.x == 0) {
    const uint32_t* flag = reinterpret_cast<const uint32_t*>(arena + L.flag_dispatch) + s;
    int c = 0;
    if (wait_flag(flag, epoch, limit_ns)) {
      c = reinterpret_cast<volatile const int32_t*>(arena + L.counts)[s];
      if (c < 0 || c > cap) {
        record_fault(reinterpret_cast<DeviceStatus*>(arena + L.status), KLC_ERR_DEVICE_FAULT, 200 + s, c);
        c = 0;
      }
    } else {
      record_fault(reinterpret_cast<DeviceStatus*>(arena + L.status), KLC_ERR_DEVICE_TIMEOUT, 100 + s, int(epoch));
    }
    count = c;
  }
  __syncthreads();
  const int c = count;
  const volatile int32_t* meta = reinterpret_cast<const volatile int32_t*>(arena + L.recv_meta) + int64_t(s) * cap;
  int32_t* out = reinterpret_cast<int32_t*>(arena + L.recv_expert) + int64_t(s) * cap;
  for (int64_t p = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; p < cap; p += int64_t(gridDim.x) * blockDim.x)
    out[p] = p < c ? meta[p] : -1;
}

// 2b. expert outputs back to their sources
__global__ void __launch_bounds__(256)
    ep_return_kernel(const int32_t* __restrict__ recv_expert, const int32_t* __restrict__ pair_pos,
                     const uint16_t* __restrict__ y, int64_t hidden, int world, int rank, int64_t cap, PeerBases peers,
                     ArenaLayout L, char* arena) {
  const int lane = threadIdx.x & 31;
  const uint32_t epoch = *reinterpret_cast<const volatile uint32_t*>(arena + L.epoch);
  unsigned int* done = reinterpret_cast<unsigned int*>(arena + L.done) + 1;
  const int64_t slots = int64_t(world) * cap;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  const int chunks = int(hidden / 8);
  for (int64_t q = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); q < slots; q += warps) {
    if (recv_expert[q] < 0) continue;
    const int row = pair_pos[q];
    if (row < 0) continue;
    const int s = int(q / cap);
    const int64_t pos = q - int64_t(s) * cap;
    const uint4* src = reinterpret_cast<const uint4*>(y + int64_t(row) * hidden);
    uint4* dst = reinterpret_cast<uint4*>(peers.base[s] + L.back_rows + size_t(int64_t(rank) * cap + pos) * size_t(hidden) * 2);
    copy_row(dst, src, chunks, lane);
  }
  signal_peers(peers, world, rank, done, L.flag_combine, 0, nullptr, epoch);
}

// 2b'. after a down kernel that stored the rows into the sources' arenas itself:
// only the combine flags (the rows were made visible system-wide by that kernel)
__global__ void ep_signal_kernel(int world, int rank, PeerBases peers, ArenaLayout L, char* arena) {
  const uint32_t epoch = *reinterpret_cast<const volatile uint32_t*>(arena + L.epoch);
  __threadfence_system();
  for (int d = threadIdx.x; d < world; d += blockDim.x)
    st_release_sys(reinterpret_cast<uint32_t*>(peers.base[d] + L.flag_combine) + rank, epoch);
}

// 3. wait for every destination's returned rows
__global__ void ep_wait_kernel(char* arena, ArenaLayout L, int world, uint64_t limit_ns) {
  const int d = threadIdx.x;
  if (d >= world) return;
  const uint32_t epoch = *reinterpret_cast<const volatile uint32_t*>(arena + L.epoch);
  const uint32_t* flag = reinterpret_cast<const uint32_t*>(arena + L.flag_combine) + d;
  if (!wait_flag(flag, epoch, limit_ns))
    record_fault(reinterpret_cast<DeviceStatus*>(arena + L.status), KLC_ERR_DEVICE_TIMEOUT, 300 + d, int(epoch));
}

__global__ void fill_ones_kernel(uint16_t* p, int64_t n) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    p[i] = 0x3F80u;  // bf16 1.0
}

}  // namespace

}  // namespace klc

struct klc_ep {
  int rank = 0, world = 1, device = 0, top_k = 1;
  int64_t max_tokens = 0, cap = 0, hidden = 0, epr = 1;
  klc::ArenaLayout L{};
  char* arena = nullptr;
  char* peer[klc::kMaxRanks] = {};
  bool opened[klc::kMaxRanks] = {};
  bool connected = false;
  uint64_t dispatches = 0;  // host count (the epoch itself lives in the arena)
  uint64_t wait_ns = klc::kDefaultWaitNs;
  // down epilogue stores rows to the sources (weights-as-N kernels).  On by default for two
  // ranks only: B200, config 3 (16 384 tokens), down + return + combine per rank measured
  // 0.87 ms fused against 0.94 copied at 2 ranks, but the down kernel itself slowed 1.8-2.2x
  // at 4 and 8 ranks when most of its stores went to peers
  bool fused_return = true;
};

namespace klc {
namespace {

PeerBases bases_of(const klc_ep* h) {
  PeerBases b{};
  for (int r = 0; r < h->world; ++r) b.base[r] = h->peer[r];
  return b;
}

int check_handle(const klc_ep* h, bool need_connected) {
  KLC_CHECK_ARG(h != nullptr, "null expert-parallel handle");
  if (need_connected && !h->connected) return fail(KLC_ERR_INVALID, "expert-parallel handle not connected (klc_ep_connect)");
  int dev = -1;
  KLC_CUDA(cudaGetDevice(&dev));
  if (dev != h->device) return fail(KLC_ERR_INVALID, "expert-parallel handle used on another device than it was created on");
  return KLC_OK;
}

klc_moe_dims local_dims(const klc_ep* h, const klc_moe_dims& d) {
  klc_moe_dims ld = d;
  ld.tokens = int64_t(h->world) * h->cap;  // every received slot of every source
  ld.top_k = 1;
  ld.hidden = h->hidden;
  return ld;
}

size_t dispatch_ws_bytes(const klc_ep* h) {
  klc_moe_dims d{h->max_tokens, 64, 64, h->world, h->top_k, KLC_PATH_SIMT};
  return workspace_layout(d, false).total;
}

}  // namespace
}  // namespace klc

using namespace klc;

extern "C" int klc_ep_create(int rank, int world, int64_t max_tokens, int top_k, int64_t hidden, int64_t experts_per_rank,
                             klc_ep** out) {
  KLC_CHECK_ARG(out != nullptr, "klc_ep_create: null output");
  *out = nullptr;
  KLC_CHECK_ARG(world >= 1 && world <= kMaxRanks && rank >= 0 && rank < world, "klc_ep_create: rank / world out of range");
  KLC_CHECK_ARG(max_tokens >= 1 && top_k >= 1 && top_k <= 8, "klc_ep_create: bad max_tokens / top_k");
  KLC_CHECK_ARG(hidden > 0 && hidden % 64 == 0 && hidden <= 65536, "klc_ep_create: hidden must be a positive multiple of 64");
  KLC_CHECK_ARG(experts_per_rank >= 1 && experts_per_rank * world <= 1024, "klc_ep_create: bad experts_per_rank");
  KLC_CHECK_ARG(max_tokens * top_k * int64_t(world) < (int64_t(1) << 31) - 1024 * 16, "klc_ep_create: max_tokens too large");
  klc_ep* h = new klc_ep();
  h->rank = rank;
  h->world = world;
  h->fused_return = world <= 2;
  h->top_k = top_k;
  h->max_tokens = max_tokens;
  h->cap = max_tokens * top_k;
  h->hidden = hidden;
  h->epr = experts_per_rank;
  h->L = arena_layout(world, h->cap, hidden);
  int st = KLC_OK;
  if ((st = cuda_check(cudaGetDevice(&h->device), "cudaGetDevice")) != KLC_OK ||
      (st = cuda_check(cudaMalloc(&h->arena, h->L.total), "klc_ep_create: cudaMalloc of the exchange arena")) != KLC_OK) {
    delete h;
    return st;
  }
  // flags start at epoch 0 (no dispatch yet), counters at 0, no status
  const size_t head = h->L.recv_meta;
  if ((st = cuda_check(cudaMemset(h->arena, 0, head), "klc_ep_create: cudaMemset")) != KLC_OK ||
      (st = cuda_check(cudaMemset(h->arena + h->L.status, 0, h->L.recv_expert - h->L.status), "klc_ep_create: cudaMemset")) != KLC_OK) {
    cudaFree(h->arena);
    delete h;
    return st;
  }
  const int64_t slots = int64_t(world) * h->cap;
  fill_ones_kernel<<<256, 256>>>(reinterpret_cast<uint16_t*>(h->arena + h->L.ones), slots);
  note_launch();
  if ((st = cuda_check(cudaDeviceSynchronize(), "klc_ep_create: arena initialisation")) != KLC_OK) {
    cudaFree(h->arena);
    delete h;
    return st;
  }
  h->peer[rank] = h->arena;
  *out = h;
  return KLC_OK;
}

extern "C" int klc_ep_arena_bytes(const klc_ep* h, size_t* out) {
  KLC_CHECK_ARG(h != nullptr && out != nullptr, "klc_ep_arena_bytes: null argument");
  *out = h->L.total;
  return KLC_OK;
}

extern "C" int klc_ep_ipc_handle(const klc_ep* h, void* out_bytes) {
  KLC_CHECK_ARG(h != nullptr && out_bytes != nullptr, "klc_ep_ipc_handle: null argument");
  cudaIpcMemHandle_t ih;
  KLC_CUDA(cudaIpcGetMemHandle(&ih, h->arena));
  std::memcpy(out_bytes, &ih, sizeof(ih));
  return KLC_OK;
}

extern "C" int klc_ep_connect(klc_ep* h, const void* handles) {
  int st = check_handle(h, false);
  if (st != KLC_OK) return st;
  KLC_CHECK_ARG(handles != nullptr, "klc_ep_connect: null handles");
  KLC_CHECK_ARG(!h->connected, "klc_ep_connect: already connected");
  cudaIpcMemHandle_t mine;
  KLC_CUDA(cudaIpcGetMemHandle(&mine, h->arena));
  const char* all = static_cast<const char*>(handles);
  for (int r = 0; r < h->world; ++r) {
    const char* hr = all + size_t(r) * sizeof(cudaIpcMemHandle_t);
    if (r == h->rank || std::memcmp(hr, &mine, sizeof(mine)) == 0) {
      h->peer[r] = h->arena;  // this rank's own arena (a handle equal to ours maps to it too)
      continue;
    }
    cudaIpcMemHandle_t ih;
    std::memcpy(&ih, hr, sizeof(ih));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, ih, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (h->opened[q]) {
          cudaIpcCloseMemHandle(h->peer[q]);
          h->opened[q] = false;
          h->peer[q] = nullptr;
        }
      return cuda_check(e, "klc_ep_connect: cudaIpcOpenMemHandle");
    }
    h->peer[r] = static_cast<char*>(p);
    h->opened[r] = true;
  }
  h->connected = true;
  return KLC_OK;
}

extern "C" int klc_ep_set_wait_limit_ns(klc_ep* h, uint64_t ns) {
  KLC_CHECK_ARG(h != nullptr && ns > 0, "klc_ep_set_wait_limit_ns: bad argument");
  h->wait_ns = ns;
  return KLC_OK;
}

extern "C" int klc_ep_set_fused_return(klc_ep* h, int enable) {
  KLC_CHECK_ARG(h != nullptr, "klc_ep_set_fused_return: null handle");
  h->fused_return = enable != 0;
  return KLC_OK;
}

extern "C" int klc_ep_workspace_size(const klc_ep* h, const klc_moe_dims* local, size_t* out) {
  KLC_CHECK_ARG(h != nullptr && local != nullptr && out != nullptr, "klc_ep_workspace_size: null argument");
  const klc_moe_dims ld = local_dims(h, *local);
  int st = validate_dims(&ld);
  if (st != KLC_OK) return st;
  KLC_CHECK_ARG(ld.experts == h->epr, "klc_ep_workspace_size: local experts must equal experts_per_rank");
  const size_t a = workspace_layout(ld, false).total, b = dispatch_ws_bytes(h);
  *out = a > b ? a : b;
  return KLC_OK;
}

extern "C" int klc_ep_dispatch(klc_ep* h, const int32_t* idx, int64_t tokens, const uint16_t* x, int32_t* pair_slot,
                               void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_handle(h, true);
  if (st != KLC_OK) return st;
  KLC_CHECK_ARG(tokens >= 0 && tokens <= h->max_tokens, "klc_ep_dispatch: tokens must be in [0, max_tokens]");
  KLC_CHECK_ARG(tokens == 0 || (idx && x && pair_slot), "klc_ep_dispatch: null pointer");
  KLC_CHECK_ARG((reinterpret_cast<uintptr_t>(x) & 15) == 0, "klc_ep_dispatch: x must be 16-byte aligned");
  const size_t need = dispatch_ws_bytes(h);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(KLC_ERR_WORKSPACE, "klc_ep_dispatch: workspace too small (need " + std::to_string(need) + " bytes)");
  cudaStream_t s = as_stream(stream);
  h->dispatches += 1;  // every rank dispatches once per forward, so the device epochs agree
  klc_moe_dims d{tokens, 64, 64, h->world, h->top_k, KLC_PATH_SIMT};
  const WorkspaceLayout W = workspace_layout(d, false);
  char* ws = static_cast<char*>(workspace);
  const int64_t pairs = tokens * h->top_k;
  if (pairs > 0) {
    // index faults of the dispatch go to the arena's status word (klc_ep_status)
    DeviceStatus* status = reinterpret_cast<DeviceStatus*>(h->arena + h->L.status);
    PermuteArgs pa{};
    pa.idx = idx;
    pa.tokens = tokens;
    pa.k = h->top_k;
    pa.experts = h->world;
    pa.pad = 1;
    pa.block_n = 1 << 24;
    pa.counts = reinterpret_cast<int32_t*>(ws + W.counts);
    pa.offsets = reinterpret_cast<int32_t*>(ws + W.offsets);
    pa.rows = reinterpret_cast<int32_t*>(ws + W.rows);
    pa.pair_pos = reinterpret_cast<int32_t*>(ws + W.pair_pos);
    pa.chunk_hist = reinterpret_cast<int32_t*>(ws + W.chunk_hist);
    pa.rowblocks = reinterpret_cast<int4*>(ws + W.rowblocks);
    pa.status = status;
    pa.hidden = h->hidden;
    pa.div = int(h->epr);
    st = launch_permute(pa, s);
    if (st != KLC_OK) return st;
  } else {
    KLC_CUDA(cudaMemsetAsync(ws + W.counts, 0, size_t(h->world) * 4, s));
  }
  const int64_t warps_needed = pairs > 0 ? pairs : 1;
  int64_t blocks = (warps_needed + 7) / 8;
  const int64_t max_blocks = int64_t(sm_count()) * 8;
  if (blocks > max_blocks) blocks = max_blocks;
  ep_send_kernel<<<unsigned(blocks), 256, 0, s>>>(
      idx, reinterpret_cast<const int32_t*>(ws + W.pair_pos), reinterpret_cast<const int32_t*>(ws + W.offsets),
      reinterpret_cast<const int32_t*>(ws + W.counts), pairs, h->top_k, int(h->epr), h->world, h->rank, h->cap, x,
      h->hidden, pair_slot, bases_of(h), h->L, h->arena);
  KLC_LAUNCH_CHECK("ep_send_kernel launch");
  return KLC_OK;
}

extern "C" int klc_ep_experts(klc_ep* h, const klc_moe_dims* local, const klc_moe_weights* wts, int precision, void* workspace,
                              size_t workspace_bytes, void* stream) {
  int st = check_handle(h, true);
  if (st != KLC_OK) return st;
  KLC_CHECK_ARG(local != nullptr, "klc_ep_experts: null dims");
  const klc_moe_dims ld = local_dims(h, *local);
  if ((st = validate_dims(&ld)) != KLC_OK) return st;
  if ((st = validate_weights(wts)) != KLC_OK) return st;
  KLC_CHECK_ARG(ld.experts == h->epr, "klc_ep_experts: local experts must equal experts_per_rank");
  KLC_CHECK_ARG(precision == KLC_PREC_FP32 || precision == KLC_PREC_BF16, "klc_ep_experts: bad precision");
  KLC_CHECK_ARG(h->dispatches > 0, "klc_ep_experts: no dispatch before");
  const WorkspaceLayout W = workspace_layout(ld, false);
  size_t need = W.total;
  if (need < dispatch_ws_bytes(h)) need = dispatch_ws_bytes(h);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(KLC_ERR_WORKSPACE, "klc_ep_experts: workspace too small (need " + std::to_string(need) + " bytes)");
  KLC_CHECK_ARG((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, "klc_ep_experts: workspace must be 256-byte aligned");
  cudaStream_t s = as_stream(stream);
  const int64_t fill_x = (h->cap + 255) / 256 < 64 ? (h->cap + 255) / 256 : 64;
  ep_fill_kernel<<<dim3(unsigned(fill_x), unsigned(h->world)), 256, 0, s>>>(h->arena, h->L, h->cap, h->wait_ns);
  KLC_LAUNCH_CHECK("ep_fill_kernel launch");
  char* ws = static_cast<char*>(workspace);
  const int32_t* recv_expert = reinterpret_cast<const int32_t*>(h->arena + h->L.recv_expert);
  // weights-as-N kernels: the down epilogue stores every output row straight into its
  // source's back_rows segment over NVLink, overlapping the transfer with the GEMM
  if (h->fused_return && h->world <= kMaxScatterSegments && use_tc_path(ld) &&
      experts_tc_can_scatter(*wts, ld.hidden, ld.intermediate, W.block_n)) {
    RowScatter sc{};
    const PeerBases pb = bases_of(h);
    for (int d = 0; d < h->world; ++d) sc.base[d] = pb.base[d] + h->L.back_rows;
    sc.seg_cap = h->cap;
    sc.slot0 = int64_t(h->rank) * h->cap;
    sc.world = h->world;
    st = run_expert_stage(ld, *wts, reinterpret_cast<const uint16_t*>(h->arena + h->L.recv_rows), recv_expert, precision,
                          nullptr, true, ws, W, s, &sc);
    if (st != KLC_OK) return st;
    ep_signal_kernel<<<1, ((h->world + 31) / 32) * 32, 0, s>>>(h->world, h->rank, pb, h->L, h->arena);
    KLC_LAUNCH_CHECK("ep_signal_kernel launch");
    return KLC_OK;
  }
  st = run_expert_stage(ld, *wts, reinterpret_cast<const uint16_t*>(h->arena + h->L.recv_rows), recv_expert, precision,
                        nullptr, true, ws, W, s);
  if (st != KLC_OK) return st;
  const int64_t slots = int64_t(h->world) * h->cap;
  int64_t blocks = (slots + 7) / 8;
  const int64_t max_blocks = int64_t(sm_count()) * 8;
  if (blocks > max_blocks) blocks = max_blocks;
  ep_return_kernel<<<unsigned(blocks), 256, 0, s>>>(recv_expert, reinterpret_cast<const int32_t*>(ws + W.pair_pos),
                                                    reinterpret_cast<const uint16_t*>(ws + W.y), h->hidden, h->world, h->rank,
                                                    h->cap, bases_of(h), h->L, h->arena);
  KLC_LAUNCH_CHECK("ep_return_kernel launch");
  return KLC_OK;
}

extern "C" int klc_ep_combine(klc_ep* h, const int32_t* pair_slot, const uint16_t* w, int64_t tokens,
                              const uint16_t* residual, const uint16_t* norm_w, float eps, uint16_t* out, uint16_t* normed,
                              void* stream) {
  int st = check_handle(h, true);
  if (st != KLC_OK) return st;
  KLC_CHECK_ARG(tokens >= 0 && tokens <= h->max_tokens, "klc_ep_combine: tokens must be in [0, max_tokens]");
  KLC_CHECK_ARG(tokens == 0 || (pair_slot && w && out), "klc_ep_combine: null pointer");
  KLC_CHECK_ARG((norm_w == nullptr) == (normed == nullptr), "klc_ep_combine: norm_w and normed go together");
  cudaStream_t s = as_stream(stream);
  ep_wait_kernel<<<1, ((h->world + 31) / 32) * 32, 0, s>>>(h->arena, h->L, h->world, h->wait_ns);
  KLC_LAUNCH_CHECK("ep_wait_kernel launch");
  if (tokens == 0) return KLC_OK;
  PostNorm post{norm_w, eps, normed};
  st = launch_combine(reinterpret_cast<const uint16_t*>(h->arena + h->L.back_rows), pair_slot, w, tokens, h->top_k,
                      h->hidden, residual, out, nullptr, nullptr, norm_w != nullptr ? &post : nullptr, s);
  stage_mark(kStageCombined, s);
  return st;
}

extern "C" int klc_ep_combine_route(klc_ep* h, const int32_t* pair_slot, const uint16_t* w, int64_t tokens,
                                    const uint16_t* residual, const uint16_t* norm_w, float eps, uint16_t* out,
                                    uint16_t* normed, const klc_next_router* next, void* stream) {
  int st = check_handle(h, true);
  if (st != KLC_OK) return st;
  KLC_CHECK_ARG(tokens >= 0 && tokens <= h->max_tokens, "klc_ep_combine_route: tokens must be in [0, max_tokens]");
  KLC_CHECK_ARG(tokens == 0 || (pair_slot && w && out && norm_w && normed), "klc_ep_combine_route: null pointer");
  KLC_CHECK_ARG(next != nullptr && next->router_w && next->experts >= 1 && next->experts <= 1024,
                "klc_ep_combine_route: bad next router");
  cudaStream_t s = as_stream(stream);
  ep_wait_kernel<<<1, ((h->world + 31) / 32) * 32, 0, s>>>(h->arena, h->L, h->world, h->wait_ns);
  KLC_LAUNCH_CHECK("ep_wait_kernel launch");
  if (tokens == 0) return KLC_OK;
  PostNorm post{norm_w, eps, normed};
  post.router_w = next->router_w;
  post.router_b = next->router_b;
  post.experts = int(next->experts);
  post.k = next->k;
  post.out_idx = next->out_idx;
  post.out_w = next->out_w;
  post.out_logits = next->out_logits;
  st = launch_combine(reinterpret_cast<const uint16_t*>(h->arena + h->L.back_rows), pair_slot, w, tokens, h->top_k,
                      h->hidden, residual, out, nullptr, nullptr, &post, s);
  stage_mark(kStageCombined, s);
  return st;
}

extern "C" int klc_ep_status(klc_ep* h, const void* workspace, int* code, int* where, void* stream) {
  KLC_CHECK_ARG(h != nullptr, "klc_ep_status: null handle");
  DeviceStatus d[2] = {};
  cudaStream_t s = as_stream(stream);
  KLC_CUDA(cudaMemcpyAsync(&d[0], h->arena + h->L.status, sizeof(DeviceStatus), cudaMemcpyDeviceToHost, s));
  // the workspace's own word: index checks of the last dispatch or local expert permute
  if (workspace != nullptr) KLC_CUDA(cudaMemcpyAsync(&d[1], workspace, sizeof(DeviceStatus), cudaMemcpyDeviceToHost, s));
  KLC_CUDA(cudaStreamSynchronize(s));
  const DeviceStatus& f = d[0].code != 0 ? d[0] : d[1];
  if (code) *code = f.code;
  if (where) *where = f.where;
  if (f.code != 0) {
    if (d[0].code != 0) {
      KLC_CUDA(cudaMemsetAsync(h->arena + h->L.status, 0, sizeof(DeviceStatus), s));
      KLC_CUDA(cudaStreamSynchronize(s));
    }
    return fail(f.code, "expert-parallel exchange: device status " + std::to_string(f.code) + " at site " +
                            std::to_string(f.where) + " (100+s: dispatch from rank s timed out, 300+d: return from rank d "
                            "timed out, 200+s: bad count, 1: expert id out of range)");
  }
  return KLC_OK;
}

extern "C" int klc_ep_forward(klc_ep* h, const klc_moe_dims* local, const klc_moe_weights* local_wts, const uint16_t* router_w,
                              const uint16_t* router_b, const uint16_t* x, int64_t tokens, int precision,
                              const uint16_t* residual, const uint16_t* norm_w, float eps, uint16_t* out, uint16_t* normed,
                              int32_t* out_idx, uint16_t* out_w, int32_t* pair_slot, void* workspace, size_t workspace_bytes,
                              void* stream) {
  int st = check_handle(h, true);
  if (st != KLC_OK) return st;
  KLC_CHECK_ARG(router_w && router_b, "klc_ep_forward: null router weights");
  KLC_CHECK_ARG(tokens == 0 || (out_idx && out_w && pair_slot), "klc_ep_forward: null routing buffers");
  if (tokens > 0) {
    stage_mark(kStageStart, as_stream(stream));
    st = launch_router(x, tokens, h->hidden, router_w, router_b, h->epr * h->world, h->top_k, nullptr, out_idx, out_w,
                       nullptr, as_stream(stream));
    if (st != KLC_OK) return st;
  }
  if ((st = klc_ep_dispatch(h, out_idx, tokens, x, pair_slot, workspace, workspace_bytes, stream)) != KLC_OK) return st;
  if ((st = klc_ep_experts(h, local, local_wts, precision, workspace, workspace_bytes, stream)) != KLC_OK) return st;
  return klc_ep_combine(h, pair_slot, out_w, tokens, residual, norm_w, eps, out, normed, stream);
}

extern "C" int klc_ep_received_rows(klc_ep* h, int64_t* out, void* stream) {
  KLC_CHECK_ARG(h != nullptr && out != nullptr, "klc_ep_received_rows: null argument");
  std::vector<int32_t> c(size_t(h->world), 0);
  cudaStream_t s = as_stream(stream);
  KLC_CUDA(cudaMemcpyAsync(c.data(), h->arena + h->L.counts, c.size() * 4, cudaMemcpyDeviceToHost, s));
  KLC_CUDA(cudaStreamSynchronize(s));
  int64_t n = 0;
  for (int32_t v : c) n += v;
  *out = n;
  return KLC_OK;
}

extern "C" int klc_ep_destroy(klc_ep* h) {
  if (h == nullptr) return KLC_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaSetDevice(h->device);
  cudaDeviceSynchronize();
  for (int r = 0; r < h->world; ++r)
    if (h->opened[r]) cudaIpcCloseMemHandle(h->peer[r]);
  cudaFree(h->arena);
  cudaSetDevice(dev);
  delete h;
  return KLC_OK;
}
