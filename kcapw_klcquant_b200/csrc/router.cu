// Fused router: logits GEMV/GEMM + top-k + softmax over the selected experts.
//
// Replaces streamed_moe_router.py:269-284 (F.linear in bf16, topk of the
// fp32 logits, softmax of the selected fp32 scores cast to bf16).
//
// A thread-block cluster of C CTAs handles kTok tokens; CTA r of the cluster
// computes the logits of experts [r*epc, (r+1)*epc) for those tokens, so a
// decode batch of a few hundred tokens still spreads over every SM.  Each CTA
// stages the tokens' activations in shared memory (bf16); each warp streams
// router rows (E x H bf16, L2-resident after the first CTA) with 16-byte
// loads, four in flight per lane, and accumulates kTok dot products in fp32.
// A butterfly reduction finishes each dot product, the bias is added in fp32
// and the logit is rounded once to bf16.  After a cluster barrier, one warp
// per token gathers the token's E logits from the cluster's shared memory
// (distributed shared memory), then runs k rounds of a warp-wide arg-max
// (value descending, lower index on ties) and a k-way softmax.
//
// Tensor-core form (E <= 128, H a multiple of 64, H <= 3072): a cluster of C
// = ceil(H / 384) CTAs splits the reduction for a tile of NT tokens; CTA r
// multiplies the router rows [128 experts x 384 K] (rows past E zero) by the
// tokens' [NT x 384 K] slice with tcgen05.mma (bf16, fp32 accumulate in
// TMEM), leaves its partial logits in shared memory, and after a cluster
// barrier each token's logits are the partials summed in rank order (fixed,
// deterministic), the bias added in fp32 and rounded once to bf16.  Eight
// warps per CTA (one token each in the reduction): the kernel is latency-bound
// (one CTA per SM for its shared memory; 15 clusters of 8 resident), and
// eight warps took T = 4096 from 142 to 131 us.  The CUDA-core form above
// covers the other shapes.
#include <cooperative_groups.h>

#include "klc_common.cuh"
#include "permute.cuh"
#include "select.cuh"
#include "tc_common.cuh"

namespace klc {

namespace {

constexpr int kTok = 8;       // tokens per CTA
constexpr int kWarps = 8;     // warps per CTA
constexpr int kMaxK = 8;
constexpr int kMaxCluster = 8;  // portable cluster size
#ifndef KLC_ROUTER_GEMM_MIN_TOKENS
#define KLC_ROUTER_GEMM_MIN_TOKENS 1024
#endif
// 128-token tiles from here on (B200: 29 / 48 / 49 / 70 / 72 us at T = 1024 / 2048 / 4096 /
// 8192 / 16384); the tokens-as-N cluster form wins below (10 us at T = 1, 21 at 256, 29 at 512)
constexpr int64_t kRouterGemmMinTokens = KLC_ROUTER_GEMM_MIN_TOKENS;

// dot products of one router row with the kTok staged tokens; lanes split the
// 16-byte chunks of the row, four loads in flight per lane
__device__ __forceinline__ void router_row_dots(const uint16_t* __restrict__ wr, const uint16_t* xs, int64_t hidden,
                                                int chunks, float (&acc)[kTok]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int t = 0; t < kTok; ++t) acc[t] = 0.f;
  auto fma_chunk = [&](const uint4 wv, int c) {
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
    float wf[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      wf[2 * j] = __uint_as_float(ww[j] << 16);
      wf[2 * j + 1] = __uint_as_float(ww[j] & 0xffff0000u);
    }
#pragma unroll
    for (int t = 0; t < kTok; ++t) {
      const uint4 xv = reinterpret_cast<const uint4*>(xs + size_t(t) * hidden)[c];
      const uint32_t xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[t] = fmaf(wf[2 * j], __uint_as_float(xx[j] << 16), acc[t]);
        acc[t] = fmaf(wf[2 * j + 1], __uint_as_float(xx[j] & 0xffff0000u), acc[t]);
      }
    }
  };
  int c = lane;
  for (; c + 96 < chunks; c += 128) {
    uint4 wv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) wv[u] = ldg_nc_v4(wr + (c + 32 * u) * 8);
#pragma unroll
    for (int u = 0; u < 4; ++u) fma_chunk(wv[u], c + 32 * u);
  }
  for (; c < chunks; c += 32) fma_chunk(ldg_nc_v4(wr + c * 8), c);
#pragma unroll
  for (int t = 0; t < kTok; ++t) acc[t] = warp_sum(acc[t]);
}

__global__ void __launch_bounds__(kWarps * 32)
    router_kernel(const uint16_t* __restrict__ x, int64_t tokens, int64_t hidden, const uint16_t* __restrict__ w,
                  const uint16_t* __restrict__ b, int experts, int k, int epc, const float* __restrict__ adjust,
                  int32_t* __restrict__ out_idx, uint16_t* __restrict__ out_w, uint16_t* __restrict__ out_logits) {
  pdl_wait();     // inputs written by the previous kernel of the chain
  pdl_trigger();  // the next kernel may launch and set up meanwhile
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int C = int(cluster.num_blocks());
  const int crank = int(cluster.block_rank());
  extern __shared__ __align__(16) unsigned char smem[];
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem);                                   // [kTok][hidden]
  float* part = reinterpret_cast<float*>(smem + size_t(kTok) * hidden * 2);          // [kTok][epc]
  float* rows = part + size_t(kTok) * epc;                                           // [ceil(kTok/C)][experts]
  const int64_t t0 = int64_t(blockIdx.x / C) * kTok;
  const int ntok = int(tokens - t0 < kTok ? tokens - t0 : kTok);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

  // stage activations with asynchronous 16-byte copies (all in flight at
  // once); rows past the end are zero-filled (source size 0)
  const int chunks_per_row = int(hidden / 8);
  for (int i = threadIdx.x; i < kTok * chunks_per_row; i += blockDim.x) {
    const int r = i / chunks_per_row, c = i % chunks_per_row;
    const uint16_t* src = x + (t0 + (r < ntok ? r : 0)) * hidden + c * 8;
    const uint32_t dst = uint32_t(__cvta_generic_to_shared(xs + size_t(r) * hidden + c * 8));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(r < ntok ? 16 : 0)
                 : "memory");
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");
  __syncthreads();

  const int e_lo = crank * epc;
  const int e_hi = min(experts, e_lo + epc);
  for (int e = e_lo + warp; e < e_hi; e += kWarps) {
    float acc[kTok];
    router_row_dots(w + int64_t(e) * hidden, xs, hidden, chunks_per_row, acc);
    if (lane == 0) {
      const float bias = bf16_to_f32(b[e]);
      for (int t = 0; t < ntok; ++t) {
        const uint16_t lb = f32_to_bf16(acc[t] + bias);
        part[t * epc + (e - e_lo)] = bf16_to_f32(lb);
        if (out_logits) out_logits[(t0 + t) * experts + e] = lb;
      }
    }
  }
  cluster.sync();

  // top-k + softmax: token crank + C*j goes to warp j of CTA crank
  const int t = crank + C * warp;
  if (warp * C < kTok && t < ntok) {
    float* row = rows + size_t(warp) * experts;
    for (int e = lane; e < experts; e += 32) {
      const float* src = cluster.map_shared_rank(part, e / epc);
      float v = src[t * epc + e % epc];
      if (adjust) v += adjust[e];
      row[e] = v;
    }
    __syncwarp();
    select_softmax_warp(row, experts, k, false, out_idx + (t0 + t) * k, out_w + (t0 + t) * k);
  }
  cluster.sync();  // no CTA leaves while its logits may still be read
}

// ---------------------------------------------------------------------------
// tensor-core router
// ---------------------------------------------------------------------------
constexpr int kRtK = 384;  // reduction slice per cluster rank (6 swizzle atoms of 64 bf16)

__device__ DeviceStatus g_router_status;  // bounded-wait timeouts of the tensor-core router

template <int NT>
__global__ void __launch_bounds__(256, 1)
    router_tc_kernel(const uint16_t* __restrict__ x, int64_t tokens, int64_t hidden, const uint16_t* __restrict__ w,
                     const uint16_t* __restrict__ b, int experts, int k, const float* __restrict__ adjust,
                     int32_t* __restrict__ out_idx, uint16_t* __restrict__ out_w, uint16_t* __restrict__ out_logits) {
  pdl_wait();     // inputs written by the previous kernel of the chain
  pdl_trigger();  // the next kernel may launch and set up meanwhile
  namespace cg = cooperative_groups;
  using namespace tc;
  cg::cluster_group cluster = cg::this_cluster();
  const int C = int(cluster.num_blocks());
  const int crank = int(cluster.block_rank());
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  unsigned char* ws = smem;                      // router rows: 6 atoms x 128 rows x 128 B (later: partials)
  unsigned char* xs = smem + 6 * 16384;          // tokens: 6 atoms x NT rows x 128 B (later: per-warp rows)
  __shared__ __align__(8) uint64_t mma_bar;
  __shared__ uint32_t tmem_holder;
  __shared__ int failed;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t0 = int64_t(blockIdx.x / C) * NT;
  const int ntok = int(tokens - t0 < NT ? tokens - t0 : NT);
  const int k0 = crank * kRtK;
  const int kc = int(hidden - k0 < kRtK ? hidden - k0 : kRtK);  // a multiple of 64
  const int na = kc / 64;

  // stage both operands in the 128B-swizzled K-major layout (16-byte async
  // copies; rows past E / past the tokens are zero-filled)
  for (int i = threadIdx.x; i < na * 128 * 8; i += blockDim.x) {
    const int a = i / 1024, r = (i >> 3) & 127, c = i & 7;
    const uint16_t* src = w + int64_t(r < experts ? r : 0) * hidden + k0 + a * 64 + c * 8;
    const uint32_t dst = smem_u32(ws + a * 16384 + (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(r < experts ? 16 : 0)
                 : "memory");
  }
  for (int i = threadIdx.x; i < na * NT * 8; i += blockDim.x) {
    const int a = i / (NT * 8), t = (i >> 3) % NT, c = i & 7;
    const uint16_t* src = x + (t0 + (t < ntok ? t : 0)) * hidden + k0 + a * 64 + c * 8;
    const uint32_t dst = smem_u32(xs + a * (NT * 128) + (t >> 3) * 1024 + (t & 7) * 128 + ((c ^ (t & 7)) << 4));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(t < ntok ? 16 : 0)
                 : "memory");
  }
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&mma_bar), 1);
    failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_holder)),
                 "r"(NT < 32 ? 32 : NT));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_holder;
  if (threadIdx.x == 0) {
    // kind::f16: bf16 A and B, fp32 accumulate, both K-major, M = 128, N = NT
    const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(NT >> 3) << 17) | (uint32_t(128 >> 4) << 24);
    const uint64_t ad = sw128_desc(smem_u32(ws)), bd = sw128_desc(smem_u32(xs));
    for (int a = 0; a < na; ++a)
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t acc = (a | kk) ? 1u : 0u;
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
            "l"(ad + uint64_t((a * 16384 + kk * 32) >> 4)), "l"(bd + uint64_t((a * NT * 128 + kk * 32) >> 4)),
            "r"(idesc), "r"(acc));
      }
    tc_commit(smem_u32(&mma_bar));
  }
  // every thread waits for the accumulators (bounded)
  {
    bool ok = mbar_try_wait(smem_u32(&mma_bar), 0);
    const long long ts = clock64();
    while (!ok) {
      ok = mbar_try_wait(smem_u32(&mma_bar), 0);
      if (!ok && clock64() - ts > kWaitCycles) {
        failed = 1;
        record_fault(&g_router_status, KLC_ERR_DEVICE_TIMEOUT, 50, 0);
        break;
      }
    }
  }
  tc_fence_before();
  cluster.sync();  // every CTA's MMAs done: the operand space takes partial sums from the cluster
  tc_fence_after();
  // CTA r finishes tokens r, r + C, ... of the tile; every CTA stores its partial logits of
  // those tokens into that CTA's shared memory, slot (this rank, token / C): remote stores,
  // local reads.  Warps w and w + 4 share TMEM lane quarter w and split the token columns.
  const int tpc = (NT + C - 1) / C;  // tokens finished per CTA (at most)
  float* recv = reinterpret_cast<float*>(ws);  // [C][tpc][128 experts]
  {
    const int e = (warp & 3) * 32 + lane;
    for (int c0 = (warp >> 2) * 16; c0 < NT; c0 += 32) {
      uint32_t v[16];
      tmem_ld16(tmem + (uint32_t((warp & 3) * 32) << 16) + uint32_t(c0), v);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int tok = c0 + j;
        float* dst = C == 1 ? recv : cluster.map_shared_rank(recv, tok % C);
        dst[(crank * tpc + tok / C) * 128 + e] = __uint_as_float(v[j]);
      }
    }
  }
  tc_fence_before();
  cluster.sync();

  // local token j = tile token crank + C*j: the C partials summed in rank order, bias, one
  // bf16 rounding, then top-k + softmax (one warp per token)
  float* rows = reinterpret_cast<float*>(xs);  // [8 warps][experts]
  for (int j = warp; j < tpc; j += 8) {
    const int t = crank + C * j;
    if (t >= ntok || t >= NT) break;
    float* row = rows + warp * experts;
    for (int e = lane; e < experts; e += 32) {
      float acc = 0.f;
      for (int r = 0; r < C; ++r) acc += recv[(r * tpc + j) * 128 + e];
      const uint16_t lb = f32_to_bf16(acc + bf16_to_f32(b[e]));
      if (out_logits) out_logits[(t0 + t) * experts + e] = lb;
      row[e] = bf16_to_f32(lb) + (adjust ? adjust[e] : 0.f);
    }
    __syncwarp();
    if (!failed) select_softmax_warp(row, experts, k, false, out_idx + (t0 + t) * k, out_w + (t0 + t) * k);
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(NT < 32 ? 32 : NT));
}

template <int NT>
int launch_router_tc(const uint16_t* x, int64_t tokens, int64_t hidden, const uint16_t* w, const uint16_t* b,
                     int experts, int k, const float* adjust, int32_t* out_idx, uint16_t* out_w, uint16_t* out_logits,
                     cudaStream_t stream) {
  const int C = int((hidden + kRtK - 1) / kRtK);
  const int64_t tiles = (tokens + NT - 1) / NT;
  KLC_CHECK_ARG(tiles * C <= 0x7fffffff, "klc_router_topk: too many tokens");
  const size_t smem = 6 * 16384 + 6 * NT * 128 + 1024;
  KLC_CUDA(cudaFuncSetAttribute(router_tc_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  KLC_CUDA(launch_chain(router_tc_kernel<NT>, dim3(unsigned(tiles * C)), dim3(256), size_t(smem), stream, unsigned(C), x, tokens, hidden, w, b, experts, k, adjust, out_idx, out_w,
                              out_logits));
  KLC_LAUNCH_CHECK("klc_router_topk launch");
  return KLC_OK;
}

// Router for large batches: a tile of 128 tokens computes all E logits on the tensor
// cores (tcgen05 kind::f16, M = 128 tokens, N = E experts, fp32 accumulators in
// TMEM), the hidden dimension streamed through a TMA ring and split over a
// thread-block cluster of C = 1, 2, 4 or 8 CTAs (as many as keep the SMs covered
// once).  CTA r finishes tokens r, r + C, ... of the tile: once every CTA's MMAs are
// done, each stores its partial logits of those tokens into that CTA's shared
// memory (distributed shared memory stores; nobody waits on a remote load), and
// after a cluster barrier one warp per token sums the C partials in rank order
// (fixed, deterministic), adds the bias in fp32, rounds once to bf16 and runs the
// warp-wide top-k + softmax.  The split-K cluster
// form above, with tokens as N, serves small batches.
constexpr int kRgStages = 4;
constexpr int kRgThreads = 256;  // warp 0 TMA, warp 1 MMA, warps 4-7 TMEM -> shared; all 8 warps select

template <int EP>  // experts padded to a multiple of 16 (the MMA's N)
struct RgLayout {
  static constexpr int XBOX = 128 * 128, WBOX = EP * 128;  // bytes of one 64-K box of each operand
  static constexpr int RING = kRgStages * (XBOX + WBOX);
  static constexpr int PS = EP + 4;                        // partial row stride (floats), 16-byte rows
  static_assert(128 * PS * 4 <= RING, "partials fit in the drained ring");
  static constexpr int ROWS = RING;                        // per-warp selection rows [8][EP] floats
  static constexpr int BYTES = ROWS + 8 * EP * 4 + 1024;
  static constexpr uint32_t TMEM_COLS = EP <= 32 ? 32 : (EP <= 64 ? 64 : (EP <= 128 ? 128 : 256));
};

template <int EP>
__global__ void __launch_bounds__(kRgThreads, 1)
    router_gemm_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w, int64_t tokens,
                       int64_t hidden, const uint16_t* __restrict__ b, int experts, int k, const float* __restrict__ adjust,
                       int32_t* __restrict__ out_idx, uint16_t* __restrict__ out_w, uint16_t* __restrict__ out_logits) {
  pdl_wait();     // inputs written by the previous kernel of the chain
  pdl_trigger();  // the next kernel may launch and set up meanwhile
  namespace cg = cooperative_groups;
  using namespace tc;
  using Lay = RgLayout<EP>;
  cg::cluster_group cluster = cg::this_cluster();
  const int C = int(cluster.num_blocks());
  const int crank = int(cluster.block_rank());
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  unsigned char* xs = smem;
  unsigned char* wsm = smem + kRgStages * Lay::XBOX;
  __shared__ __align__(8) uint64_t bars[2 * kRgStages + 1];
  __shared__ uint32_t tmem_holder;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t0 = int64_t(blockIdx.x / C) * 128;
  const int nk = int(hidden / 64);
  const int kb0 = int(int64_t(crank) * nk / C), kb1 = int(int64_t(crank + 1) * nk / C);  // this CTA's 64-K steps
  auto full = [&](int s) { return smem_u32(&bars[s]); };
  auto empty = [&](int s) { return smem_u32(&bars[kRgStages + s]); };
  const uint32_t done = smem_u32(&bars[2 * kRgStages]);
  const Ctl ctl{reinterpret_cast<volatile int*>(&abort_flag), &g_router_status};
  if (threadIdx.x == 0) {
    for (int s = 0; s < kRgStages; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    mbar_init(done, 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_holder)),
                 "r"(Lay::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_holder;
  if (warp == 0 && lane == 0) {
    bool ok = true;
    uint32_t issued = 0;
    for (int kc = kb0; kc < kb1 && ok; ++kc) {
      const int i = kc - kb0, s = i % kRgStages;
      if (!(ok = wait_bar(empty(s), ((i / kRgStages) & 1) ^ 1, ctl, 60))) break;
      mbar_arrive_expect_tx(full(s), uint32_t(Lay::XBOX + Lay::WBOX));
      tma_load_2d(smem_u32(xs + s * Lay::XBOX), &map_x, kc * 64, int(t0), full(s));
      tma_load_2d(smem_u32(wsm + s * Lay::WBOX), &map_w, kc * 64, 0, full(s));
      ++issued;
    }
    if (!ok) drain_ring(full(0), kRgStages, issued);
  } else if (warp == 1 && lane == 0) {
    // kind::f16: bf16 A (tokens) and B (router rows), fp32 accumulate, K-major, M = 128, N = EP
    const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(EP >> 3) << 17) | (uint32_t(128 >> 4) << 24);
    bool ok = true;
    for (int kc = kb0; kc < kb1 && ok; ++kc) {
      const int i = kc - kb0, s = i % kRgStages;
      if (!(ok = wait_bar(full(s), (i / kRgStages) & 1, ctl, 61))) break;
      tc_fence_after();
      const uint64_t ad = sw128_desc(smem_u32(xs + s * Lay::XBOX)), bd = sw128_desc(smem_u32(wsm + s * Lay::WBOX));
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t acc = (i | kk) ? 1u : 0u;
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
            "l"(ad + uint64_t(kk * 2)), "l"(bd + uint64_t(kk * 2)), "r"(idesc), "r"(acc));
      }
      tc_commit(empty(s));
    }
    tc_commit(done);
  }
  if (C == 1) {
    if (warp >= 4) {
      // one thread per token: its logits from its TMEM lane, bias, one bf16 rounding,
      // top-k (value descending, lower index first) and the softmax of the selected
      const int q = warp & 3;
      const int tl = q * 32 + lane;
      const int64_t t = t0 + tl;
      bool ok = wait_bar_backoff(done, 0, ctl, 62);
      tc_fence_after();
      float sv[kMaxK];
      int si[kMaxK];
  #pragma unroll
      for (int r = 0; r < kMaxK; ++r) {
        sv[r] = -INFINITY;
        si[r] = -1;
      }
      for (int c0 = 0; c0 < EP; c0 += 16) {
        uint32_t raw[16];
        tmem_ld16(tmem + (uint32_t(q * 32) << 16) + uint32_t(c0), raw);
        tmem_wait_ld();
        uint32_t packed[8];
  #pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int e = c0 + j;
          uint16_t lb = 0;
          if (e < experts) {
            lb = f32_to_bf16(__uint_as_float(raw[j]) + bf16_to_f32(b[e]));
            const float v = bf16_to_f32(lb) + (adjust ? adjust[e] : 0.f);
            if (v == v) {  // NaN only fills slots nothing else takes (below)
              // insertion into the selection kept in (value descending, index ascending) order;
              // an element pushed down by the insertion keeps that order against equal values too
              float cv = v;
              int ci = e;
  #pragma unroll
              for (int r = 0; r < kMaxK; ++r) {
                if (r < k && ci >= 0 && (si[r] < 0 || cv > sv[r] || (cv == sv[r] && ci < si[r]))) {
                  const float tv = sv[r];
                  const int ti = si[r];
                  sv[r] = cv;
                  si[r] = ci;
                  cv = tv;
                  ci = ti;
                }
              }
            }
          }
          if (j & 1) packed[j >> 1] |= uint32_t(lb) << 16;
          else packed[j >> 1] = lb;
        }
        // 16-byte stores when the row and chunk start are 16-byte aligned (E a multiple of 8)
        if (out_logits != nullptr && t < tokens && c0 + 16 <= experts && (experts & 7) == 0 &&
            (reinterpret_cast<uintptr_t>(out_logits) & 15) == 0) {
          uint4* dst = reinterpret_cast<uint4*>(out_logits + t * experts + c0);
          dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
          dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
        } else if (out_logits != nullptr && t < tokens) {
          for (int j = 0; j < 16 && c0 + j < experts; ++j)
            out_logits[t * experts + c0 + j] = uint16_t((j & 1) ? (packed[j >> 1] >> 16) : (packed[j >> 1] & 0xFFFFu));
        }
      }
      // slots still empty: the lowest-index experts not taken (their scores NaN)
      for (int r = 0; r < k; ++r) {
        if (si[r] >= 0) continue;
        for (int e = 0; e < experts; ++e) {
          bool taken = false;
          for (int qq = 0; qq < r; ++qq) taken |= (si[qq] == e);
          if (!taken) {
            si[r] = e;
            sv[r] = __uint_as_float(0x7fc00000u);
            break;
          }
        }
      }
      if (ok && t < tokens) {
        float m = sv[0];
        for (int r = 1; r < k; ++r) m = fmaxf(m, sv[r]);
        float ex[kMaxK];
        float sum = 0.f;
        for (int r = 0; r < k; ++r) {
          ex[r] = expf(sv[r] - m);
          sum += ex[r];
        }
        for (int r = 0; r < k; ++r) {
          out_idx[t * k + r] = si[r];
          out_w[t * k + r] = f32_to_bf16(ex[r] / sum);
        }
      }
    }
  } else {
    // every CTA's MMAs done (the ring may then take partial sums from the cluster)
    const bool ok_done = warp < 4 ? true : wait_bar_backoff(done, 0, ctl, 62);
    (void)ok_done;
    __syncwarp();
    tc_fence_before();
    cluster.sync();
    tc_fence_after();
    // TMEM lane = token tl: its EP partial logits go to the CTA that finishes the token
    // (tl % C), into slot (this rank, tl / C) of that CTA's shared memory: remote stores,
    // local reads
    constexpr int kTokPer = 128;  // tokens of a tile; CTA r finishes tokens r, r + C, ...
    float* recv = reinterpret_cast<float*>(smem);
    if (warp >= 4) {
      const int q = warp & 3;
      const int tl = q * 32 + lane;
      const int owner = tl % C;
      float* dst_base = C == 1 ? recv : cluster.map_shared_rank(recv, owner);
      float* dst = dst_base + (crank * (kTokPer / C) + tl / C) * Lay::PS;
      for (int c0 = 0; c0 < EP; c0 += 16) {
        uint32_t raw[16];
        tmem_ld16(tmem + (uint32_t(q * 32) << 16) + uint32_t(c0), raw);
        tmem_wait_ld();
  #pragma unroll
        for (int j = 0; j < 16; j += 4)
          *reinterpret_cast<float4*>(dst + c0 + j) =
              make_float4(__uint_as_float(raw[j]), __uint_as_float(raw[j + 1]), __uint_as_float(raw[j + 2]), __uint_as_float(raw[j + 3]));
      }
    }
    __syncwarp();
    tc_fence_before();
    cluster.sync();
    const bool failed = abort_flag != 0;

    // local token j = tile token crank + C*j: the C partials summed in rank order, bias,
    // one bf16 rounding, locality adjustment, then top-k + softmax (one warp per token)
    float* row = reinterpret_cast<float*>(smem + Lay::ROWS) + warp * EP;
    for (int j = warp; j < kTokPer / C; j += kRgThreads / 32) {
      const int t = crank + C * j;
      const int64_t tg = t0 + t;
      if (tg >= tokens) break;
      for (int e = lane; e < experts; e += 32) {
        float acc = 0.f;
        for (int r = 0; r < C; ++r) acc += recv[(r * (kTokPer / C) + j) * Lay::PS + e];
        const uint16_t lb = f32_to_bf16(acc + bf16_to_f32(b[e]));
        if (out_logits) out_logits[tg * experts + e] = lb;
        row[e] = bf16_to_f32(lb) + (adjust ? adjust[e] : 0.f);
      }
      __syncwarp();
      if (!failed) select_softmax_warp(row, experts, k, false, out_idx + tg * k, out_w + tg * k);
      __syncwarp();
    }
  }
  tc_fence_before();
  __syncthreads();  // TMEM is freed once every warp is past its loads
  tc_fence_after();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Lay::TMEM_COLS));
}

__global__ void select_kernel(const float* __restrict__ scores, int64_t tokens, int experts, int k, int keep_order,
                              int32_t* __restrict__ out_idx, uint16_t* __restrict__ out_w) {
  const int lane = threadIdx.x & 31;
  const int64_t t = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= tokens) return;
  (void)lane;
  select_softmax_warp(scores + t * experts, experts, k, keep_order != 0, out_idx + t * k, out_w + t * k);
}

template <int EP>
int launch_router_gemm_ep(const CUtensorMap& mx, const CUtensorMap& mw, int64_t tokens, int64_t hidden, const uint16_t* b,
                          int experts, int k, const float* adjust, int32_t* out_idx, uint16_t* out_w, uint16_t* out_logits,
                          cudaStream_t stream) {
  const int smem = RgLayout<EP>::BYTES;
  KLC_CUDA(cudaFuncSetAttribute(router_gemm_kernel<EP>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int64_t tiles = (tokens + 127) / 128;
  const int nk = int(hidden / 64);
  // split the hidden dimension over a cluster while the CTAs still run in one wave (one
  // CTA per SM; B200 holds at most 15 clusters of 8 such CTAs at once)
  const int64_t sms = sm_count();
  int C = 1;
  if (tiles * 8 <= 15 * 8 && tiles * 8 <= sms && nk >= 8) C = 8;
  else if (tiles * 4 <= sms && nk >= 4) C = 4;  // pairs measured slower than whole tiles (86 against ~72 us at 64 tiles)
  KLC_CHECK_ARG(tiles * C <= 0x7fffffff, "klc_router_topk: too many tokens");
  KLC_CUDA(launch_chain(router_gemm_kernel<EP>, dim3(unsigned(tiles * C)), dim3(kRgThreads), size_t(size_t(smem)), stream, unsigned(C), mx, mw, tokens, hidden, b, experts, k, adjust, out_idx, out_w,
                              out_logits));
  KLC_LAUNCH_CHECK("klc_router_topk launch");
  return KLC_OK;
}

int launch_router_gemm(const uint16_t* x, int64_t tokens, int64_t hidden, const uint16_t* w, const uint16_t* b, int experts,
                       int k, const float* adjust, int32_t* out_idx, uint16_t* out_w, uint16_t* out_logits,
                       cudaStream_t stream) {
  const int ep = (experts + 15) / 16 * 16;
  CUtensorMap mx, mw;
  {
    const uint64_t dims[2] = {uint64_t(hidden), uint64_t(tokens)};
    const uint64_t strides[1] = {uint64_t(hidden) * 2};
    const uint32_t box[2] = {64, 128};
    int st = tc::make_map(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != KLC_OK) return st;
  }
  // the router-row box spans the kernel's padded expert count (rows past E read as zeros),
  // so every stage's transaction is XBOX + WBOX bytes
  const int ep_t = ep <= 64 ? 64 : (ep <= 128 ? 128 : 256);
  {
    const uint64_t dims[2] = {uint64_t(hidden), uint64_t(experts)};
    const uint64_t strides[1] = {uint64_t(hidden) * 2};
    const uint32_t box[2] = {64, uint32_t(ep_t)};
    int st = tc::make_map(&mw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != KLC_OK) return st;
  }
  if (ep <= 64) return launch_router_gemm_ep<64>(mx, mw, tokens, hidden, b, experts, k, adjust, out_idx, out_w, out_logits, stream);
  if (ep <= 128) return launch_router_gemm_ep<128>(mx, mw, tokens, hidden, b, experts, k, adjust, out_idx, out_w, out_logits, stream);
  return launch_router_gemm_ep<256>(mx, mw, tokens, hidden, b, experts, k, adjust, out_idx, out_w, out_logits, stream);
}

}  // namespace

int launch_router(const uint16_t* x, int64_t tokens, int64_t hidden, const uint16_t* w, const uint16_t* b,
                  int64_t experts, int k, const float* adjust, int32_t* out_idx, uint16_t* out_w,
                  uint16_t* out_logits, cudaStream_t stream) {
  KLC_CHECK_ARG(tokens >= 0 && hidden > 0 && experts > 0, "klc_router_topk: bad sizes");
  KLC_CHECK_ARG(hidden % 8 == 0, "klc_router_topk: hidden must be a multiple of 8");
  KLC_CHECK_ARG(k >= 1 && k <= kMaxK && k <= experts, "klc_router_topk: need 1 <= k <= min(8, experts)");
  KLC_CHECK_ARG(experts <= 1024, "klc_router_topk: at most 1024 experts");
  if (tokens == 0) return KLC_OK;
  KLC_CHECK_ARG(x && w && b && out_idx && out_w, "klc_router_topk: null pointer");
  KLC_CHECK_ARG((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0,
                "klc_router_topk: x and w must be 16-byte aligned");
  if (tokens >= kRouterGemmMinTokens && experts <= 256 && hidden % 64 == 0 && tc_path_supported(hidden, 64))
    return launch_router_gemm(x, tokens, hidden, w, b, int(experts), k, adjust, out_idx, out_w, out_logits, stream);
  if (experts <= 128 && hidden % 64 == 0 && hidden <= 8 * kRtK && tc_path_supported(hidden, 64)) {
    // token tile: as few router-weight passes as keep every SM busy
    const int C = int((hidden + kRtK - 1) / kRtK);
    const int64_t want = 2 * int64_t(sm_count());
    if ((tokens + 15) / 16 * C <= want)
      return launch_router_tc<16>(x, tokens, hidden, w, b, int(experts), k, adjust, out_idx, out_w, out_logits, stream);
    if ((tokens + 31) / 32 * C <= want)
      return launch_router_tc<32>(x, tokens, hidden, w, b, int(experts), k, adjust, out_idx, out_w, out_logits, stream);
    return launch_router_tc<64>(x, tokens, hidden, w, b, int(experts), k, adjust, out_idx, out_w, out_logits, stream);
  }
  // cluster size: enough CTAs to cover the SMs twice, at least 8 experts per CTA
  const int64_t nblocks = (tokens + kTok - 1) / kTok;
  int C = 1;
  while (C < kMaxCluster && nblocks * C < 2 * int64_t(sm_count()) && 2 * C * 8 <= experts) C *= 2;
  const int epc = int((experts + C - 1) / C);
  const size_t smem = size_t(kTok) * hidden * 2 + size_t(kTok) * epc * 4 + size_t((kTok + C - 1) / C) * experts * 4;
  KLC_CHECK_ARG(smem <= 200 * 1024, "klc_router_topk: hidden size too large for one CTA tile");
  KLC_CUDA(cudaFuncSetAttribute(router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  KLC_CHECK_ARG(nblocks * C <= 0x7fffffff, "klc_router_topk: too many tokens");
  KLC_CUDA(launch_chain(router_kernel, dim3(unsigned(nblocks * C)), dim3(kWarps * 32), size_t(smem), stream, unsigned(C), x, tokens, hidden, w, b, int(experts), k, epc, adjust, out_idx,
                              out_w, out_logits));
  KLC_LAUNCH_CHECK("klc_router_topk launch");
  return KLC_OK;
}

}  // namespace klc

extern "C" int klc_select_softmax(const float* scores, int64_t tokens, int64_t experts, int k, int keep_order,
                                  int32_t* out_idx, uint16_t* out_w, void* stream) {
  using namespace klc;
  KLC_CHECK_ARG(tokens >= 0 && experts >= 1 && k >= 1 && k <= 8 && k <= experts, "klc_select_softmax: bad sizes");
  KLC_CHECK_ARG(!keep_order || experts == k, "klc_select_softmax: keep_order needs experts == k");
  if (tokens == 0) return KLC_OK;
  KLC_CHECK_ARG(scores && out_w && (keep_order || out_idx), "klc_select_softmax: null pointer");
  const int64_t blocks = (tokens + 7) / 8;
  KLC_CHECK_ARG(blocks <= 0x7fffffff, "klc_select_softmax: too many tokens");
  select_kernel<<<unsigned(blocks), 256, 0, as_stream(stream)>>>(scores, tokens, int(experts), k, keep_order, out_idx, out_w);
  KLC_LAUNCH_CHECK("klc_select_softmax launch");
  return KLC_OK;
}

extern "C" int klc_router_status(int* code, int* where, void* stream) {
  using namespace klc;
  KLC_CUDA(cudaStreamSynchronize(as_stream(stream)));
  DeviceStatus st{};
  KLC_CUDA(cudaMemcpyFromSymbol(&st, g_router_status, sizeof(st)));
  if (code) *code = st.code;
  if (where) *where = st.where;
  if (st.code != 0) {
    const DeviceStatus zero{};
    KLC_CUDA(cudaMemcpyToSymbol(g_router_status, &zero, sizeof(zero)));
  }
  return st.code == 0 ? KLC_OK : st.code;
}

extern "C" int klc_router_topk(const uint16_t* x, int64_t tokens, int64_t hidden, const uint16_t* w,
                               const uint16_t* b, int64_t experts, int k, const float* adjust, int32_t* out_idx,
                               uint16_t* out_w, uint16_t* out_logits, void* stream) {
  return klc::launch_router(x, tokens, hidden, w, b, experts, k, adjust, out_idx, out_w, out_logits,
                            klc::as_stream(stream));
}
