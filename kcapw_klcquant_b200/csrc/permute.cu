// Token dispatch: stable counting-sort of (token, slot) pairs by expert into
// contiguous, padded row groups, fused with the gather of each pair's
// activation row.
//
// The reference has no dispatch step: route() handles one token and loops
// over its k experts (streamed_moe_router.py:499).  Batched execution needs
// the pairs of each expert contiguous; the order inside a group is
// token-major, slot-minor (a stable sort of the flat expert ids), so results
// are deterministic and independent of the grid size.
//
// Up to 16384 pairs one fused launch does all three steps (below); larger
// batches use three launches, each a pass over the int32 index array:
//   1. per-chunk expert histograms (1024 pairs per CTA, shared-memory atomics)
//   2. one CTA: per-expert prefix over chunks, padded group offsets, and the
//      list of row-blocks (<= block_n rows of one expert) the GEMMs iterate
//   3. per chunk: stable rank of each pair among equal experts (warp
//      match_any + per-warp counts), scatter of rows/pair_pos, and the copy of
//      x[token] into its padded row.
//      A chunk is split over `split` CTAs: each ranks the whole chunk (a few
//      microseconds of shared-memory work) and copies 1/split of its rows, so
//      a decode batch of one or two chunks still spreads its row copies over
//      the SMs; only the first CTA of a chunk writes the index arrays.
#include "klc_common.cuh"
#include "permute.cuh"

namespace klc {

namespace {

constexpr int kChunk = 1024;

__global__ void __launch_bounds__(kChunk)
    hist_kernel(const int32_t* __restrict__ idx, int64_t pairs, int experts, int div, int32_t* __restrict__ chunk_hist) {
  pdl_wait();     // inputs written by the previous kernel of the chain
  pdl_trigger();  // the next kernel may launch and set up meanwhile
  extern __shared__ int32_t hist[];
  for (int e = threadIdx.x; e < experts; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int64_t p = int64_t(blockIdx.x) * kChunk + threadIdx.x;
  if (p < pairs) {
    const int v = idx[p];
    const int e = v >= 0 ? v / div : -1;
    if (e >= 0 && e < experts) atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < experts; e += blockDim.x) chunk_hist[int64_t(blockIdx.x) * experts + e] = hist[e];
}

// exclusive scan over a 1024-thread block; returns the block total in *total
__device__ int block_exclusive_scan(int v, int* tmp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) tmp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = (lane < int(blockDim.x >> 5)) ? tmp[lane] : 0;
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += n;
    }
    tmp[lane] = wi - w;  // exclusive warp prefix
    if (lane == 31) tmp[32] = wi;
  }
  __syncthreads();
  const int r = tmp[warp] + incl - v;
  *total = tmp[32];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(1024)
    scan_kernel(int32_t* __restrict__ chunk_hist, int nchunks, int experts, int pad, int block_n,
                int32_t* __restrict__ counts, int32_t* __restrict__ offsets, int32_t* __restrict__ rows,
                int4* __restrict__ rowblocks, int4* __restrict__ pairblocks, DeviceStatus* st) {
  pdl_wait();     // inputs written by the previous kernel of the chain
  pdl_trigger();  // the next kernel may launch and set up meanwhile
  __shared__ int tmp[33];
  const int e = threadIdx.x;
  int cnt = 0;
  if (e < experts) {
    for (int c = 0; c < nchunks; ++c) {
      const int h = chunk_hist[int64_t(c) * experts + e];
      chunk_hist[int64_t(c) * experts + e] = cnt;
      cnt += h;
    }
    counts[e] = cnt;
  }
  const int padded = (e < experts) ? (cnt + pad - 1) / pad * pad : 0;
  int total = 0;
  const int off = block_exclusive_scan(padded, tmp, &total);
  if (e < experts) {
    offsets[e] = off;
    for (int c = 0; c < nchunks; ++c) chunk_hist[int64_t(c) * experts + e] += off;
    for (int j = cnt; j < padded; ++j) rows[off + j] = -1;
  }
  if (e == 0) offsets[experts] = total;
  const int nb = (e < experts) ? (cnt + block_n - 1) / block_n : 0;
  int nblocks = 0;
  const int base = block_exclusive_scan(nb, tmp, &nblocks);
  for (int j = 0; j < nb; ++j) {
    const int r0 = j * block_n;
    rowblocks[base + j] = make_int4(e, off + r0, min(block_n, cnt - r0), 0);
  }
  if (e == 0) st->rowblocks = nblocks;
  if (pairblocks != nullptr) {
    const int np = (nb + 1) / 2;
    int npairs = 0;
    const int pbase = block_exclusive_scan(np, tmp, &npairs);
    for (int j = 0; j < np; ++j) {
      const int r0 = 2 * j * block_n;
      pairblocks[pbase + j] = make_int4(e, off + r0, min(2 * block_n, cnt - r0), base + 2 * j);
    }
    if (e == 0) st->pairblocks = npairs;
  }
}

__global__ void __launch_bounds__(kChunk)
    scatter_gather_kernel(const int32_t* __restrict__ idx, int64_t pairs, int k, int experts,
                          const int32_t* __restrict__ chunk_base, int32_t* __restrict__ rows,
                          int32_t* __restrict__ pair_pos, const uint16_t* __restrict__ x, int64_t hidden,
                          uint16_t* __restrict__ xp, int div, int32_t* __restrict__ aux_out,
                          int split, int empty_ok, DeviceStatus* st) {
  pdl_wait();     // inputs written by the previous kernel of the chain
  pdl_trigger();  // the next kernel may launch and set up meanwhile
  extern __shared__ int32_t sm[];
  int32_t* warp_cnt = sm;                      // [32][experts]
  int32_t* s_pos = sm + 32 * experts;          // [kChunk]
  int32_t* s_tok = s_pos + kChunk;             // [kChunk]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < 32 * experts; i += blockDim.x) warp_cnt[i] = 0;
  const int64_t chunk = blockIdx.x / split;
  const int sub = int(blockIdx.x % split);
  const bool writer = sub == 0;
  const int64_t p = chunk * kChunk + threadIdx.x;
  int e = -1, v = -1;
  if (p < pairs) {
    v = idx[p];
    e = v >= 0 ? v / div : -1;
    if (e >= experts || (e < 0 && !empty_ok)) {
      if (writer) record_fault(st, KLC_ERR_DEVICE_FAULT, 1, v);
      e = -1;
    }
  }
  __syncthreads();
  const unsigned same = __match_any_sync(0xffffffffu, e);
  const int rank = __popc(same & ((1u << lane) - 1u));
  if (e >= 0 && rank == 0) warp_cnt[warp * experts + e] = __popc(same);
  __syncthreads();
  for (int ex = threadIdx.x; ex < experts; ex += blockDim.x) {
    int run = 0;
    for (int w = 0; w < 32; ++w) {
      const int c = warp_cnt[w * experts + ex];
      warp_cnt[w * experts + ex] = run;
      run += c;
    }
  }
  __syncthreads();
  int pos = -1;
  if (e >= 0) {
    pos = chunk_base[chunk * experts + e] + warp_cnt[warp * experts + e] + rank;
    if (writer) {
      rows[pos] = int32_t(p);
      if (aux_out != nullptr) aux_out[pos] = v - e * div;
    }
  }
  if (writer && p < pairs) pair_pos[p] = pos;
  s_pos[threadIdx.x] = pos;
  s_tok[threadIdx.x] = (p < pairs) ? int32_t(p / k) : -1;
  __syncthreads();
  if (xp == nullptr) return;
  const int chunks = int(hidden / 8);
  const int per = (kChunk + split - 1) / split;
  const int i_end = min(kChunk, (sub + 1) * per);
  for (int i = sub * per + warp; i < i_end; i += 32) {
    const int dst = s_pos[i];
    if (dst < 0) continue;
    const uint4* src = reinterpret_cast<const uint4*>(x + int64_t(s_tok[i]) * hidden);
    uint4* out = reinterpret_cast<uint4*>(xp + int64_t(dst) * hidden);
    for (int c = lane; c < chunks; c += 32) {
      uint4 v = src[c];
      out[c] = v;
    }
  }
}

// Single-launch permute for batches of up to kFusedPairs pairs (decode).
// Every CTA histograms all pairs itself (shared-memory atomics over a few
// thousand indices), derives the padded group offsets and its chunk's base
// per expert, ranks its chunk like scatter_gather_kernel and copies its share
// of the rows.  CTA 0 alone writes counts, offsets, the padding markers and
// the row-block list; the first CTA of each chunk writes rows and pair_pos.
// Results are identical to the three-launch form.
constexpr int64_t kFusedPairs = 16 * kChunk;

__global__ void __launch_bounds__(kChunk)
    fused_permute_kernel(const int32_t* __restrict__ idx, int64_t pairs, int k, int experts, int pad, int block_n,
                         int32_t* __restrict__ counts, int32_t* __restrict__ offsets, int32_t* __restrict__ rows,
                         int4* __restrict__ rowblocks, int4* __restrict__ pairblocks, int32_t* __restrict__ pair_pos,
                         const uint16_t* __restrict__ x,
                         int64_t hidden, uint16_t* __restrict__ xp, int div, int32_t* __restrict__ aux_out,
                         int split, int empty_ok, DeviceStatus* st) {
  pdl_wait();     // inputs written by the previous kernel of the chain
  pdl_trigger();  // the next kernel may launch and set up meanwhile
  extern __shared__ int32_t sm[];
  int32_t* warp_cnt = sm;                    // [32][experts]
  int32_t* total = warp_cnt + 32 * experts;  // [experts]
  int32_t* before = total + experts;         // [experts]: pairs of earlier chunks
  int32_t* s_pos = before + experts;         // [kChunk]
  int32_t* s_tok = s_pos + kChunk;           // [kChunk]
  __shared__ int tmp[33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t chunk = blockIdx.x / split;
  const int sub = int(blockIdx.x % split);
  const bool writer = sub == 0;
  const int64_t c0 = chunk * kChunk;
  for (int i = threadIdx.x; i < 32 * experts; i += blockDim.x) warp_cnt[i] = 0;
  for (int i = threadIdx.x; i < experts; i += blockDim.x) {
    total[i] = 0;
    before[i] = 0;
  }
  __syncthreads();
  // warp-aggregated histogram; each 1024-pair pass lies wholly before or
  // at/after this chunk, so `earlier` is uniform across the block
  for (int64_t base = 0; base < pairs; base += kChunk) {
    const int64_t q = base + threadIdx.x;
    int e = -1;
    if (q < pairs) {
      const int v = idx[q];
      e = v >= 0 ? v / div : -1;
      if (e >= experts) e = -1;
    }
    const unsigned grp = __match_any_sync(0xffffffffu, e);
    if (e >= 0 && lane == __ffs(grp) - 1) {
      atomicAdd(&total[e], __popc(grp));
      if (base < c0) atomicAdd(&before[e], __popc(grp));
    }
  }
  __syncthreads();
  // padded group offsets (one thread per expert)
  const int e_t = threadIdx.x;
  const int cnt = e_t < experts ? total[e_t] : 0;
  const int padded = e_t < experts ? (cnt + pad - 1) / pad * pad : 0;
  int all = 0;
  const int off = block_exclusive_scan(padded, tmp, &all);
  if (blockIdx.x == 0) {
    if (e_t < experts) {
      counts[e_t] = cnt;
      offsets[e_t] = off;
      for (int j = cnt; j < padded; ++j) rows[off + j] = -1;
    }
    if (e_t == 0) offsets[experts] = all;
  }
  const int nb = e_t < experts ? (cnt + block_n - 1) / block_n : 0;
  int nblocks = 0;
  const int rb_base = block_exclusive_scan(nb, tmp, &nblocks);
  if (blockIdx.x == 0) {
    for (int j = 0; j < nb; ++j) {
      const int r0 = j * block_n;
      rowblocks[rb_base + j] = make_int4(e_t, off + r0, min(block_n, cnt - r0), 0);
    }
    if (e_t == 0) st->rowblocks = nblocks;
    if (pairblocks != nullptr) {  // uniform over the CTA: the scan's barriers are met by all threads
      const int np = (nb + 1) / 2;
      int npairs = 0;
      const int pbase = block_exclusive_scan(np, tmp, &npairs);
      for (int j = 0; j < np; ++j) {
        const int r0 = 2 * j * block_n;
        pairblocks[pbase + j] = make_int4(e_t, off + r0, min(2 * block_n, cnt - r0), rb_base + 2 * j);
      }
      if (e_t == 0) st->pairblocks = npairs;
    }
  }
  if (e_t < experts) before[e_t] += off;  // chunk base per expert
  // stable rank inside this chunk
  const int64_t p = c0 + threadIdx.x;
  int e = -1, v = -1;
  if (p < pairs) {
    v = idx[p];
    e = v >= 0 ? v / div : -1;
    if (e >= experts || (e < 0 && !empty_ok)) {
      if (writer) record_fault(st, KLC_ERR_DEVICE_FAULT, 1, v);
      e = -1;
    }
  }
  __syncthreads();
  const unsigned same = __match_any_sync(0xffffffffu, e);
  const int rank = __popc(same & ((1u << lane) - 1u));
  if (e >= 0 && rank == 0) warp_cnt[warp * experts + e] = __popc(same);
  __syncthreads();
  for (int ex = threadIdx.x; ex < experts; ex += blockDim.x) {
    int run = 0;
    for (int w = 0; w < 32; ++w) {
      const int c = warp_cnt[w * experts + ex];
      warp_cnt[w * experts + ex] = run;
      run += c;
    }
  }
  __syncthreads();
  int pos = -1;
  if (e >= 0) {
    pos = before[e] + warp_cnt[warp * experts + e] + rank;
    if (writer) {
      rows[pos] = int32_t(p);
      if (aux_out != nullptr) aux_out[pos] = v - e * div;
    }
  }
  if (writer && p < pairs) pair_pos[p] = pos;
  s_pos[threadIdx.x] = pos;
  s_tok[threadIdx.x] = (p < pairs) ? int32_t(p / k) : -1;
  __syncthreads();
  if (xp == nullptr) return;
  const int chunks = int(hidden / 8);
  const int per = (kChunk + split - 1) / split;
  const int i_end = min(kChunk, (sub + 1) * per);
  for (int i = sub * per + warp; i < i_end; i += 32) {
    const int dst = s_pos[i];
    if (dst < 0) continue;
    const uint4* src = reinterpret_cast<const uint4*>(x + int64_t(s_tok[i]) * hidden);
    uint4* out = reinterpret_cast<uint4*>(xp + int64_t(dst) * hidden);
    for (int c = lane; c < chunks; c += 32) {
      uint4 vv = src[c];
      out[c] = vv;
    }
  }
}

}  // namespace

int launch_permute(const PermuteArgs& a, cudaStream_t stream) {
  const int64_t pairs = a.tokens * a.k;
  if (pairs == 0) return KLC_OK;
  const int nchunks = int((pairs + kChunk - 1) / kChunk);
  const int E = int(a.experts);
  const int div = a.div > 0 ? a.div : 1;
  // split each chunk's row copies over enough CTAs to cover the SMs twice (at most 8 rows per CTA)
  int split = 1;
  if (a.xp != nullptr) {
    const int64_t want = (2 * int64_t(sm_count()) + nchunks - 1) / nchunks;
    split = int(want < kChunk / 8 ? want : kChunk / 8);
    if (split < 1) split = 1;
  }
  KLC_CHECK_ARG(int64_t(nchunks) * split <= 0x7fffffff, "permute: too many pairs");
  if (pairs <= kFusedPairs) {
    const size_t smem = (size_t(32) * E + 2 * E + 2 * kChunk) * sizeof(int32_t);
    KLC_CUDA(cudaFuncSetAttribute(fused_permute_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    KLC_CUDA(launch_chain(fused_permute_kernel, dim3(unsigned(int64_t(nchunks) * split)), dim3(kChunk), size_t(smem), stream, 0u, 
        a.idx, pairs, a.k, E, a.pad, a.block_n, a.counts, a.offsets, a.rows, a.rowblocks, a.pairblocks, a.pair_pos, a.x, a.hidden,
        a.xp, div, a.aux_out, split, a.empty_ok ? 1 : 0, a.status));
    KLC_LAUNCH_CHECK("permute (fused) launch");
    return KLC_OK;
  }
  KLC_CUDA(launch_chain(hist_kernel, dim3(nchunks), dim3(kChunk), size_t(E * sizeof(int32_t)), stream, 0u, a.idx, pairs, E, div, a.chunk_hist));
  KLC_LAUNCH_CHECK("permute hist launch");
  KLC_CUDA(launch_chain(scan_kernel, dim3(1), dim3(1024), size_t(0), stream, 0u, a.chunk_hist, nchunks, E, a.pad, a.block_n, a.counts, a.offsets, a.rows,
                                      a.rowblocks, a.pairblocks, a.status));
  KLC_LAUNCH_CHECK("permute scan launch");
  const size_t smem = (size_t(32) * E + 2 * kChunk) * sizeof(int32_t);
  KLC_CUDA(cudaFuncSetAttribute(scatter_gather_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  KLC_CUDA(launch_chain(scatter_gather_kernel, dim3(unsigned(int64_t(nchunks) * split)), dim3(kChunk), size_t(smem), stream, 0u, 
      a.idx, pairs, a.k, E, a.chunk_hist, a.rows, a.pair_pos, a.x, a.hidden, a.xp, div, a.aux_out, split,
      a.empty_ok ? 1 : 0, a.status));
  KLC_LAUNCH_CHECK("permute scatter launch");
  return KLC_OK;
}

}  // namespace klc
