// Tensor-core grouped expert GEMMs for sm_100a (tcgen05 + TMEM + TMA).
//
// Both expert GEMMs of the reference's _execute_mxfp4_experts
// (streamed_moe_router.py:500-511) for every (expert, row-block) of the
// permuted tokens, with the bias and the clamped SwiGLU (:524-529) fused
// into the epilogue.  "Swap-AB" orientation: the weights are the MMA's A
// operand (M = 128 output features of one expert), the tokens of a
// row-block are B (N = up to 256 rows), K is the reduction (H for gate_up,
// I for down).  One persistent CTA per SM walks the (row-block, m-tile)
// work list.
//
// Per CTA, warp-specialised (832 threads):
//   warps 0-3   MMA issuers, one thread each (warp 0 also allocates TMEM):
//               tcgen05.mma.cta_group::1.kind::f16, A from TMEM, B from smem;
//               K-stage `it` goes to issuer it % NP and its own accumulator
//   warps 4-19  four dequant warpgroups (K-stage `it` to warpgroup it % 4):
//               one thread per weight row converts 128 E2M1 values x
//               2^(s-127) to exact bf16 and writes them straight into the
//               warpgroup's TMEM A stage (tcgen05.st) -- the dequantized
//               weights never touch shared memory
//   warps 20-23 epilogue: tcgen05.ld of the fp32 accumulators (summed over
//               the pipelines in a fixed order), bias, SwiGLU (gate_up) or
//               bias (down), bf16 stores
//   warp 24     TMA producer: packed E2M1 nibbles (128 rows x 64 B, 64B
//               swizzle) + E8M0 scales (4 groups x 128 rows) into an A ring
//   warp 25     TMA producer: token rows (16-row boxes of 64 bf16, 128B
//               swizzle) into a B ring
// Inside every 8-element K chunk the dequant emits the order
// {0,4,1,5,2,6,3,7} (cheapest bit extraction); the activation rows are
// written in the same order by the permute/gather and by the gate_up
// epilogue, so the dot products are unchanged.
//
// Every mbarrier wait is bounded (SM cycle counter): after kWaitCycles the waiting
// role records KLC_ERR_DEVICE_TIMEOUT in the workspace status word, raises a
// CTA-wide abort flag, and all roles drain (TMA and MMA completion are
// awaited, again bounded) before the TMEM is freed and the CTA exits.
#include <cuda.h>

#include <mutex>

#include "permute.cuh"

namespace klc {

namespace {

constexpr int kMaxIssuers = 4;                   // MMA issuer warps 0..3 (one per SM sub-partition)
constexpr int kDqWGs = 4;                        // dequant warpgroups (warps 4..19)
constexpr int kEpiWarp0 = 4 + 4 * kDqWGs;        // first epilogue warp (20)
constexpr int kProdWarp0 = kEpiWarp0 + 4;        // TMA producers: A in warp 24, B in warp 25
constexpr int kThreads = (kProdWarp0 + 2) * 32;  // 832
constexpr int kBM = 128;                        // weight rows per tile (MMA M)
constexpr int kAtom = 64;                       // K per 128-byte swizzle atom of bf16
constexpr uint64_t kWaitNs = 2000000000ull;      // drain bound: 2 s of %globaltimer
constexpr long long kWaitCycles = 4000000000ll;  // wait bound: 4e9 SM cycles (2 s at 2 GHz)

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

struct Ctl {
  volatile int* abort;
  DeviceStatus* status;
};

// Bounded wait for the completion of phase `parity` of a barrier.  Returns
// false when the CTA is aborting (this wait timed out or another did).
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, const Ctl& c, int site) {
  if (mbar_try_wait(bar, parity)) return true;
  // slow path: the SM cycle counter is cheap to read (the global timer is
  // not); the bound is checked every 64 polls and is a few seconds at any clock
  const long long t0 = clock64();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0) {
      if (*c.abort) return false;
      if (clock64() - t0 > kWaitCycles) {
        *c.abort = 1;
        record_fault(c.status, KLC_ERR_DEVICE_TIMEOUT, site, 0);
        return false;
      }
    }
  }
}

// Drain-time wait: bounded, ignores the abort flag.
__device__ __noinline__ void drain_wait(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitNs) return;
    __nanosleep(64);
  }
}

// After an abort: wait (bounded) for the latest load issued into each slot of
// a ring of `n` full-barriers (8 bytes apart) that received `issued` loads in
// slot order (load i went to slot i % n, completing phase (i / n) & 1).
__device__ __noinline__ void drain_ring(uint32_t full0, int n, uint32_t issued) {
  for (int s = 0; s < n; ++s) {
    if (issued <= uint32_t(s)) break;
    const uint32_t last = issued - 1 - ((issued - 1 - uint32_t(s)) % uint32_t(n));
    drain_wait(full0 + 8u * s, (last / uint32_t(n)) & 1);
  }
}


__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accum));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}


__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), leading offset unused (1), descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return uint64_t((saddr & 0x3FFFFu) >> 4) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) | (uint64_t(1) << 46) |
         (uint64_t(2) << 61);
}

// kind::f16 instruction descriptor: fp32 accumulate, bf16 A and B, both
// K-major, M = 128, N = n.
__device__ __forceinline__ uint32_t make_idesc(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(kBM >> 4) << 24);
}

// One 16-byte MXFP4 group (32 E2M1 values, one E8M0 scale s) -> 16 bf16x2
// words, exact.  Each pair word holds nibbles (q, q+4) of a 32-bit nibble
// word, i.e. the K order {0,4,1,5,2,6,3,7} inside every 8 values.  The two
// nibbles are isolated with one AND and spread with one integer multiply
// (the two shifted copies do not overlap, so the multiply is a shift-OR) to
// a bf16 pair of value FP4 * 2^-126 (sign -> bit 15, e2m1 -> bits 8:6); a
// second AND drops the stray copies.  bf16 multiplies by exact powers of two
// then apply 2^(s-1) (split in two factors above s = 128 so no factor
// overflows).  Per 8 values: 9 ALU-pipe ops (1 shift, 8 AND) and 8 FMA-pipe
// ops (4 IMAD, 4 HMUL2).
template <bool kTwo>
__device__ __forceinline__ void dequant_group(uint4 c, uint32_t s, uint32_t* out) {
  const uint32_t lo = s < 128u ? s : 128u;
  const uint32_t f1 = ((lo + 126u) << 7) * 0x10001u;                   // 2^(min(s,128)-1)
  const uint32_t f2 = ((s > 128u ? s - 1u : 127u) << 7) * 0x10001u;     // 2^(s-128), or 1
  const uint32_t words[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t w = words[j], wh = w >> 8;
    uint32_t r[4];
    r[0] = ((w & 0x000F000Fu) * 0x1040u) & 0x81C081C0u;   // nibbles 0, 4
    r[1] = ((w & 0x00F000F0u) * 0x0104u) & 0x81C081C0u;   // nibbles 1, 5
    r[2] = ((wh & 0x000F000Fu) * 0x1040u) & 0x81C081C0u;  // nibbles 2, 6
    r[3] = ((wh & 0x00F000F0u) * 0x0104u) & 0x81C081C0u;  // nibbles 3, 7
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t v = bf16x2_mul(r[q], f1);
      if (kTwo) v = bf16x2_mul(v, f2);
      out[4 * j + q] = v;
    }
  }
}

struct TcParams {
  int n_out;          // weight rows of one expert (2I or H)
  int k_in;           // reduction length (H or I)
  int ksteps;         // ceil(k_in / stage K); the tail of the last stage is zero-filled by TMA
  int n_mtiles;       // ceil(n_out / 128)
  const int4* rowblocks;
  DeviceStatus* status;
  const int32_t* rows;
  const uint16_t* bias;  // [E, n_out]
  uint16_t* out;         // phase 1: [rows_cap, n_out/2] (K-order permuted); phase 2: [rows_cap, n_out]
  int out_ld;
  float* normsq;
  int precision;
  float limit, alpha;
};

// Tile / pipeline configuration.
//   BN    max token rows of a tile (MMA N <= BN)
//   NB    token (B) ring depth
//   NP    MMA pipelines: K-stage `it` goes to issuer warp it % NP, which
//         accumulates into its own fp32 accumulator; the epilogue sums the
//         NP accumulators in pipeline order (deterministic).  One thread
//         issuing tcgen05.mma at small N is latency-bound (about 60 cycles
//         per instruction alone, over 120 next to busy dequant warps), so
//         several issuers keep the tensor pipe fed
//   KA    64-wide K atoms per MMA stage (16 * KA MMAs per stage)
//   NT    TMEM A stages (KA * 32 columns each), one per active dequant warpgroup
//   NA    weight (A) ring depth; a weight slot holds SKA = 2 MMA stages (256 K:
//         128-byte nibble rows, which the copy engine streams from HBM about
//         twice as fast as 64-byte rows, and half the producer work per stage)
//   SKB   MMA stages per token (B) slot
//   ND    accumulator sets in flight (epilogue of one tile overlaps the next)
template <int BN_, int NB_, int NP_, int KA_, int NT_, int NA_, int ND_, int SKB_>
struct Cfg {
  static constexpr int BN = BN_, NB = NB_, NP = NP_, KA = KA_, NT = NT_, NA = NA_, ND = ND_, SKB = SKB_;
  static constexpr int SKA = 2;
  static constexpr int BK = kAtom * KA;         // K per MMA stage
  static constexpr int ACOLS = BK / 2;          // TMEM columns per A stage
  static constexpr int GROUPS = BK / 32;        // scale groups per MMA stage
  static constexpr int NIB = kBM * SKA * BK / 2;  // nibble bytes per weight slot (128 rows x 128 B)
  static constexpr int SCL = kBM * SKA * BK / 32; // scale bytes per weight slot
  static constexpr int BATOM = BN * kAtom * 2;  // bytes of one K atom of BN token rows
  static constexpr int BSLOT = SKB * KA * BATOM;
  // shared memory layout
  static constexpr int OFF_NIB = 0;
  static constexpr int OFF_SCL = OFF_NIB + NA * NIB;
  static constexpr int OFF_B = (OFF_SCL + NA * SCL + 1023) / 1024 * 1024;
  static constexpr int OFF_BAR = OFF_B + NB * BSLOT;
  static constexpr int NUM_BARS = 2 * NA + 2 * NB + 2 * NT + NP * ND + ND + 1;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  static_assert(NT * ACOLS + ND * NP * BN <= 512, "TMEM budget");
  static_assert(NT <= kDqWGs, "one dequant warpgroup per TMEM A stage");
  static_assert(NP >= 1 && NP <= kMaxIssuers, "issuer warps");
  static_assert(KA == 2 && (SKB == 1 || SKB == 2), "slot shapes");
  static_assert(BYTES + 1024 <= 227 * 1024, "shared memory budget");
};

template <int PHASE, class C>
__global__ void __launch_bounds__(kThreads, 1)
    tc_expert_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_s,
                     const __grid_constant__ CUtensorMap map_b, TcParams p) {
  constexpr int NA = C::NA, NB = C::NB, NT = C::NT, ND = C::ND, NP = C::NP, KA = C::KA, BN = C::BN;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // TMA destinations and swizzled operand tiles need 1024-byte alignment
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const uint32_t bar0 = smem_u32(smem + C::OFF_BAR);
  auto afull = [&](int s) { return bar0 + 8u * s; };
  auto aempty = [&](int s) { return bar0 + 8u * (NA + s); };
  auto bfull = [&](int s) { return bar0 + 8u * (2 * NA + s); };
  auto bempty = [&](int s) { return bar0 + 8u * (2 * NA + NB + s); };
  auto tfull = [&](int s) { return bar0 + 8u * (2 * NA + 2 * NB + s); };
  auto tempty = [&](int s) { return bar0 + 8u * (2 * NA + 2 * NB + NT + s); };
  auto dfull = [&](int pp, int s) { return bar0 + 8u * (2 * NA + 2 * NB + 2 * NT + pp * ND + s); };
  auto dempty = [&](int s) { return bar0 + 8u * (2 * NA + 2 * NB + 2 * NT + NP * ND + s); };
  const uint32_t mma_done = bar0 + 8u * (2 * NA + 2 * NB + 2 * NT + NP * ND + ND);
  // accumulator of pipeline pp for accumulator set d
  auto dcol = [&](int pp, int d) { return uint32_t(NT * C::ACOLS + (d * NP + pp) * BN); };
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const Ctl ctl{abort_flag, p.status};

  if (threadIdx.x == 0) {
    for (int s = 0; s < NA; ++s) {
      mbar_init(afull(s), 1);
      mbar_init(aempty(s), 4 * C::SKA);  // four dequant warps per MMA stage of the slot
    }
    for (int s = 0; s < NB; ++s) {
      mbar_init(bfull(s), 1);
      mbar_init(bempty(s), C::SKB);  // one MMA commit per MMA stage of the slot
    }
    for (int s = 0; s < NT; ++s) {
      mbar_init(tfull(s), 4);
      mbar_init(tempty(s), 1);
    }
    for (int s = 0; s < ND; ++s) {
      for (int pp = 0; pp < NP; ++pp) mbar_init(dfull(pp, s), 1);
      mbar_init(dempty(s), 4);
    }
    mbar_init(mma_done, NP);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_holder)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int nrb = p.status->rowblocks;
  const int total = nrb * p.n_mtiles;
  const int ks_n = p.ksteps;  // MMA stages per item
  // Ring slots hold SKA (weights) / SKB (tokens) consecutive MMA stages of one
  // item; an item with an odd stage count leaves the last weight slot half
  // used, and the consumers of that stage then arrive for both halves.
  const int spa = (ks_n + C::SKA - 1) / C::SKA;  // weight slots per item
  const int spb = (ks_n + C::SKB - 1) / C::SKB;  // token slots per item

  if (warp == kProdWarp0) {
    // ------------------------------------------------------------ A producer (weights)
    if (lane == 0) {
      uint32_t it = 0;  // loads issued so far
      bool ok = true;
      for (int item = blockIdx.x; item < total && ok; item += gridDim.x) {
        const int4 rb = p.rowblocks[item / p.n_mtiles];
        const int mt = item % p.n_mtiles;
        for (int j = 0; j < spa && ok; ++j, ++it) {
          const int sa = it % NA;
          if (!(ok = wait_bar(aempty(sa), ((it / NA) & 1) ^ 1, ctl, 10))) break;
          mbar_arrive_expect_tx(afull(sa), C::NIB + C::SCL);
          tma_load_3d(smem_u32(smem + C::OFF_NIB + sa * C::NIB), &map_a, j * (C::SKA * C::BK / 2), mt * kBM, rb.x,
                      afull(sa));
          tma_load_3d(smem_u32(smem + C::OFF_SCL + sa * C::SCL), &map_s, mt * kBM, j * (C::SKA * C::GROUPS), rb.x,
                      afull(sa));
        }
      }
      if (!ok) drain_ring(afull(0), NA, it);  // aborting: no bulk copy may still write shared memory
    }
  } else if (warp == kProdWarp0 + 1) {
    // ------------------------------------------------------------ B producer (token rows)
    // One copy per slot: the map views the rows as [K/64 atoms][rows][64] and
    // its box is SKB*KA atoms x BN rows, so the slot lands atom-major exactly
    // as the MMA descriptors address it.  Rows past the row-block (up to BN)
    // are loaded but not read by the MMA (N = the block's padded row count);
    // rows and atoms past the buffer are zero-filled.
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total && ok; item += gridDim.x) {
        const int4 rb = p.rowblocks[item / p.n_mtiles];
        for (int j = 0; j < spb && ok; ++j, ++it) {
          const int sb = it % NB;
          if (!(ok = wait_bar(bempty(sb), ((it / NB) & 1) ^ 1, ctl, 11))) break;
          mbar_arrive_expect_tx(bfull(sb), C::BSLOT);
          tma_load_3d(smem_u32(smem + C::OFF_B + sb * C::BSLOT), &map_b, 0, rb.y, j * (C::SKB * KA), bfull(sb));
        }
      }
      if (!ok) drain_ring(bfull(0), NB, it);
    }
  } else if (warp < NP) {
    // ------------------------------------------------------------ MMA issuers
    const int pp = warp;  // pipeline: K-stages with it % NP == pp
    if (lane == 0) {
      const int atoms_last = (p.k_in / kAtom) - (ks_n - 1) * KA;  // valid atoms in the last stage
      uint32_t it = 0, ic = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total && ok; item += gridDim.x, ++ic) {
        const int4 rb = p.rowblocks[item / p.n_mtiles];
        const int npad = (rb.z + 15) & ~15;
        const uint32_t idesc = make_idesc(npad);
        const int d = ic % ND;
        const uint32_t d_tmem = tmem + dcol(pp, d);
        if (!(ok = wait_bar(dempty(d), ((ic / ND) & 1) ^ 1, ctl, 20))) break;
        tc_fence_after();
        bool first = true;
        for (int ks = 0; ks < ks_n && ok; ++ks, ++it) {
          if (NP > 1 && int(it % NP) != pp) continue;
          const int st = it % NT;
          const uint32_t ib = ic * uint32_t(spb) + uint32_t(ks / C::SKB);  // token slot counter
          const int sb = ib % NB, hb = ks % C::SKB;
          if (!(ok = wait_bar(tfull(st), (it / NT) & 1, ctl, 21))) break;
          if (!(ok = wait_bar(bfull(sb), (ib / NB) & 1, ctl, 22))) break;
          tc_fence_after();
          const uint32_t a_tmem = tmem + uint32_t(st * C::ACOLS);
          // descriptors of the stage's K-slices differ only in the start-address field
          // (address >> 4, no carry out of the field below 256 KB of shared memory)
          const uint64_t bdesc0 = sw128_desc(smem_u32(smem + C::OFF_B + sb * C::BSLOT + hb * KA * C::BATOM));
          const int kk_n = 4 * ((ks == ks_n - 1) ? atoms_last : KA);
#pragma unroll
          for (int kk = 0; kk < 4 * KA; ++kk) {
            if (kk < kk_n)
              tc_mma_ts(d_tmem, a_tmem + kk * 8, bdesc0 + uint64_t(((kk >> 2) * C::BATOM + (kk & 3) * 32) >> 4), idesc,
                        (first && kk == 0) ? 0u : 1u);
          }
          first = false;
          tc_commit(tempty(st));
          tc_commit(bempty(sb));
          if (C::SKB == 2 && ks == ks_n - 1 && hb == 0) tc_commit(bempty(sb));  // no second stage in this slot
        }
        if (ok) tc_commit(dfull(pp, d));
      }
      tc_commit(mma_done);
      drain_wait(mma_done, 0);
    }
  } else if (warp >= 4 && warp < 4 + 4 * NT) {
    // ------------------------------------------------------------ dequant
    const int wg = (warp - 4) >> 2;  // K-stages with it % NT == wg, TMEM A stage wg
    const int q = warp & 3;          // TMEM lane quarter
    const int m = q * 32 + lane;     // weight row within the tile
    // 128-byte nibble rows, 128B swizzle: 16-byte chunk g of row m sits at chunk g ^ (m & 7)
    const int sw = m & 7;
    const uint32_t tbase = tmem + (uint32_t(q * 32) << 16) + uint32_t(wg * C::ACOLS);
    uint32_t it = 0, ic = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < total && ok; item += gridDim.x, ++ic) {
      for (int ks = 0; ks < ks_n; ++ks, ++it) {
        if (int(it % NT) != wg) continue;
        const uint32_t ia = ic * uint32_t(spa) + uint32_t(ks / C::SKA);  // weight slot counter
        const int sa = ia % NA, ha = ks % C::SKA;
        // every lane waits (acquire), the decision is made warp-uniform so the
        // .sync.aligned tcgen05 instructions below never run divergent
        ok = wait_bar(afull(sa), (ia / NA) & 1, ctl, 30);
        if (!(ok = __all_sync(0xffffffffu, ok))) break;
        const unsigned char* nib = smem + C::OFF_NIB + sa * C::NIB + m * (C::SKA * C::BK / 2);
        const unsigned char* scl = smem + C::OFF_SCL + sa * C::SCL + ha * C::GROUPS * kBM;
        uint4 c[C::GROUPS];
        uint32_t sc[C::GROUPS], smax = 0;
#pragma unroll
        for (int g = 0; g < C::GROUPS; ++g) {
          c[g] = *reinterpret_cast<const uint4*>(nib + (((ha * C::GROUPS + g) ^ sw) << 4));
          sc[g] = scl[g * kBM + m];
          smax = smax > sc[g] ? smax : sc[g];
        }
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(aempty(sa));
          if (ks == ks_n - 1 && ha == 0) mbar_arrive(aempty(sa));  // the slot's second half is past K
        }
        // scales above 128 need a second power-of-two factor; decided per warp
        const bool two = __any_sync(0xffffffffu, smax > 128u);
        ok = wait_bar(tempty(wg), ((it / NT) & 1) ^ 1, ctl, 31);
        if (!(ok = __all_sync(0xffffffffu, ok))) break;
        tc_fence_after();
#pragma unroll
        for (int h = 0; h < C::GROUPS / 2; ++h) {  // 32 columns at a time keeps the register footprint small
          uint32_t v[32];
          if (two) {
            dequant_group<true>(c[2 * h], sc[2 * h], v);
            dequant_group<true>(c[2 * h + 1], sc[2 * h + 1], v + 16);
          } else {
            dequant_group<false>(c[2 * h], sc[2 * h], v);
            dequant_group<false>(c[2 * h + 1], sc[2 * h + 1], v + 16);
          }
          tmem_st32(tbase + uint32_t(h * 32), v);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tfull(wg));
      }
    }
  } else if (warp >= kEpiWarp0) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int m = q * 32 + lane;
    uint32_t ic = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < total && ok; item += gridDim.x, ++ic) {
      const int4 rb = p.rowblocks[item / p.n_mtiles];
      const int mt = item % p.n_mtiles;
      const int e = rb.x, r0 = rb.y, nrows = rb.z;
      const int npad = (nrows + 15) & ~15;
      const int d = ic % ND;
      const int j = mt * kBM + m;  // output feature
      const bool jok = j < p.n_out;
      const float bias = jok ? bf16_to_f32(p.bias[int64_t(e) * p.n_out + j]) : 0.f;
      for (int pp = 0; pp < NP && ok; ++pp) ok = wait_bar(dfull(pp, d), (ic / ND) & 1, ctl, 40 + pp);
      if (!(ok = __all_sync(0xffffffffu, ok))) break;
      tc_fence_after();
      // pipeline pp received a K-stage of this item unless the item has fewer
      // stages than pipelines (stage `it` of the launch goes to it % NP)
      const uint32_t first_pp = uint32_t((uint64_t(ic) * uint64_t(ks_n)) % NP);
      const uint32_t lane_base = tmem + (uint32_t(q * 32) << 16);
      for (int c0 = 0; c0 < npad; c0 += 16) {
        uint32_t raw[16];
        tmem_ld16(lane_base + dcol(int(first_pp), d) + uint32_t(c0), raw);
        tmem_wait_ld();
        for (int j2 = 1; j2 < NP && j2 < ks_n; ++j2) {
          uint32_t raw2[16];
          tmem_ld16(lane_base + dcol(int((first_pp + j2) % NP), d) + uint32_t(c0), raw2);
          tmem_wait_ld();
#pragma unroll
          for (int cc = 0; cc < 16; ++cc) raw[cc] = __float_as_uint(__uint_as_float(raw[cc]) + __uint_as_float(raw2[cc]));
        }
        if (c0 + 16 >= npad) {
          // last accumulator columns read: hand the buffer back to the MMA warps early
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(dempty(d));
        }
#pragma unroll
        for (int cc = 0; cc < 16; ++cc) {
          const int n = c0 + cc;
          float v = __uint_as_float(raw[cc]);
          if (p.precision == KLC_PREC_BF16) v = round_bf16(v);
          v += bias;
          const bool nok = n < nrows;
          if (PHASE == 1) {
            const float up_raw = __shfl_xor_sync(0xffffffffu, v, 1);
            float g2 = 0.f;
            if ((lane & 1) == 0 && jok && nok) {
              const float gate = fminf(v, p.limit);
              const float up = fminf(fmaxf(up_raw, -p.limit), p.limit);
              const float glu = gate * (1.0f / (1.0f + expf(-(gate * p.alpha))));
              const float gated = (up + 1.0f) * glu;
              const uint16_t gb = f32_to_bf16(gated);
              const int i = j >> 1;
              const int pos = (i & ~7) | (((i & 3) << 1) | ((i >> 2) & 1));  // element i%8 -> slot {0,2,4,6,1,3,5,7}
              p.out[int64_t(r0 + n) * p.out_ld + pos] = gb;
              const float gr = bf16_to_f32(gb);
              g2 = (p.precision == KLC_PREC_BF16) ? gr * gr : gated * gated;
            }
            if (p.normsq != nullptr) {
              g2 = warp_sum(g2);
              if (lane == 0 && nok) atomicAdd(&p.normsq[int64_t(p.rows[r0 + n]) * 2 + 0], g2);
            }
          } else {
            float o2 = 0.f;
            if (jok && nok) {
              p.out[int64_t(r0 + n) * p.out_ld + j] = f32_to_bf16(v);
              o2 = v * v;
            }
            if (p.normsq != nullptr) {
              o2 = warp_sum(o2);
              if (lane == 0 && nok) atomicAdd(&p.normsq[int64_t(p.rows[r0 + n]) * 2 + 1], o2);
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_fn(EncodeTiledFn* out) {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (fn == nullptr) return fail(KLC_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  *out = fn;
  return KLC_OK;
}

int make_map(CUtensorMap* map, CUtensorMapDataType type, int rank, const void* base, const uint64_t* dims,
             const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = nullptr;
  int st = encode_fn(&fn);
  if (st != KLC_OK) return st;
  cuuint64_t gd[3], gs[2];
  cuuint32_t bx[3], es[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bx[i] = box[i];
  }
  for (int i = 0; i < rank - 1; ++i) gs[i] = strides_bytes[i];
  const CUresult r = fn(map, type, cuuint32_t(rank), const_cast<void*>(base), gd, gs, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(KLC_ERR_CUDA, "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(int(r)));
  return KLC_OK;
}

template <int PHASE, class C>
int launch_tc_phase(const uint8_t* blocks, const uint8_t* scales_t, const uint16_t* act, int64_t rows_cap, int experts,
                    TcParams p, int max_rowblocks, cudaStream_t stream) {
  CUtensorMap ma, ms, mb;
  const uint64_t K = uint64_t(p.k_in), N = uint64_t(p.n_out), G = K / 32;
  p.ksteps = int((K + C::BK - 1) / C::BK);
  {
    // packed nibbles [E][N][K/2] bytes; box = 128 rows x 128 bytes (one weight slot), 128B swizzle
    const uint64_t dims[3] = {K / 2, N, uint64_t(experts)};
    const uint64_t strides[2] = {K / 2, N * K / 2};
    const uint32_t box[3] = {uint32_t(C::SKA * C::BK / 2), kBM, 1};
    int st = make_map(&ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, blocks, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != KLC_OK) return st;
  }
  {
    // scales [E][G][N] bytes; box = (one weight slot's) 8 groups x 128 rows
    const uint64_t dims[3] = {N, G, uint64_t(experts)};
    const uint64_t strides[2] = {N, G * N};
    const uint32_t box[3] = {kBM, uint32_t(C::SKA * C::GROUPS), 1};
    int st = make_map(&ms, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, scales_t, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st != KLC_OK) return st;
  }
  {
    // token rows [rows_cap][K] bf16 viewed as [K/64 atoms][rows_cap][64]; box = SKB*KA atoms x BN rows x 64,
    // 128-byte swizzle (one copy per token slot)
    const uint64_t dims[3] = {kAtom, uint64_t(rows_cap), K / kAtom};
    const uint64_t strides[2] = {K * 2, kAtom * 2};
    const uint32_t box[3] = {kAtom, uint32_t(C::BN), uint32_t(C::SKB * C::KA)};
    int st = make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, act, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != KLC_OK) return st;
  }
  // >= 116 KB of shared memory keeps one CTA (and one 512-column TMEM allocation) per SM
  const int smem = (C::BYTES + 1024 > 118 * 1024) ? C::BYTES + 1024 : 118 * 1024;
  KLC_CUDA(cudaFuncSetAttribute(tc_expert_kernel<PHASE, C>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int64_t items = int64_t(max_rowblocks) * p.n_mtiles;
  const int grid = int(items < sm_count() ? items : sm_count());
  if (grid <= 0) return KLC_OK;
  tc_expert_kernel<PHASE, C><<<grid, kThreads, smem, stream>>>(ma, ms, mb, p);
  KLC_LAUNCH_CHECK("tcgen05 expert launch");
  return KLC_OK;
}

template <class C>
int launch_tc_both(const ExpertArgs& a, cudaStream_t stream) {
  const klc_moe_weights& w = *a.wts;
  TcParams p1{};
  p1.n_out = int(2 * a.inter);
  p1.k_in = int(a.hidden);
  p1.n_mtiles = (p1.n_out + kBM - 1) / kBM;
  p1.rowblocks = a.rowblocks;
  p1.status = a.status_rw;
  p1.rows = a.rows;
  p1.bias = w.gu_bias;
  p1.out = static_cast<uint16_t*>(a.gated);
  p1.out_ld = int(a.inter);
  p1.normsq = a.normsq;
  p1.precision = a.precision;
  p1.limit = w.swiglu_limit;
  p1.alpha = w.alpha;
  int st = launch_tc_phase<1, C>(w.gu_blocks, w.gu_scales_t, a.xp, a.rows_cap, int(a.experts), p1,
                                           a.max_rowblocks, stream);
  if (st != KLC_OK) return st;
  stage_mark(kStageGateUp, stream);
  TcParams p2 = p1;
  p2.n_out = int(a.hidden);
  p2.k_in = int(a.inter);
  p2.n_mtiles = (p2.n_out + kBM - 1) / kBM;
  p2.bias = w.dn_bias;
  p2.out = a.y;
  p2.out_ld = int(a.hidden);
  st = launch_tc_phase<2, C>(w.dn_blocks, w.dn_scales_t, static_cast<const uint16_t*>(a.gated), a.rows_cap,
                                       int(a.experts), p2, a.max_rowblocks, stream);
  stage_mark(kStageDown, stream);
  return st;
}

// Measured on B200 (decode, T=256): 128-K stages with four dequant
// warpgroups beat 256-K stages -- the dequant's TMEM writes and the MMA's
// TMEM reads of the A operand share TMEM bandwidth, so fewer, longer stages
// do not shorten the MMA chain.  The token (B) ring runs several stages
// per pipeline ahead: a slot is refilled only after the MMAs that read it
// complete, and the refill comes from L2 with a latency of about a
// microsecond.  TMEM: 4 A stages x 64 columns + ND x NP x BN accumulator
// columns = 512.
//                 BN   NB NP KA NT NA ND SKB
using CfgN32  = Cfg<32,  3, 4, 2, 4, 10, 2, 2>;
using CfgN64  = Cfg<64,  2, 2, 2, 4, 8,  2, 2>;
using CfgN128 = Cfg<128, 2, 2, 2, 4, 4,  1, 2>;
using CfgN256 = Cfg<256, 2, 1, 2, 4, 4,  1, 1>;

}  // namespace

bool tc_path_supported(int64_t hidden, int64_t inter) {
  int dev = 0, major = 0, minor = 0;
  if (hidden % kAtom != 0 || inter % kAtom != 0) return false;
  if (cudaGetDevice(&dev) != cudaSuccess) return true;  // no device: report the build's capability
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return true;
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  return major == 10 && minor == 0;
}

int launch_experts_tc(const ExpertArgs& a, cudaStream_t stream) {
  KLC_CHECK_ARG(a.hidden % kAtom == 0 && a.inter % kAtom == 0, "tensor-core path: hidden and intermediate must be multiples of 64");
  KLC_CHECK_ARG(a.rows_cap < (int64_t(1) << 31), "tensor-core path: too many rows");
  // block_n (the max rows of a row-block) decides the tile configuration
  switch (a.block_n) {
    case 32: return launch_tc_both<CfgN32>(a, stream);
    case 64: return launch_tc_both<CfgN64>(a, stream);
    case 128: return launch_tc_both<CfgN128>(a, stream);
    case 256: return launch_tc_both<CfgN256>(a, stream);
    default: return fail(KLC_ERR_INVALID, "tensor-core path: row-block size must be 32, 64, 128 or 256");
  }
}

}  // namespace klc
