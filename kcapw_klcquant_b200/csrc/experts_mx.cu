// Tensor-core grouped expert GEMMs for sm_100a on native MXFP4 weights.
//
// Both expert GEMMs of the reference's _execute_mxfp4_experts
// (streamed_moe_router.py:500-511) for every (expert, row-block) of the
// permuted tokens, with the bias and the clamped SwiGLU (:524-529) fused into
// the epilogue, computed by the block-scaled tensor-core MMA
// (tcgen05.mma.kind::mxf8f6f4.block_scale, M = 128, K = 32 per instruction):
//
//   A  the expert's packed E2M1 weights (128 output features of one m-tile),
//      read from shared memory, with their E8M0 scales (one per 32 K) copied
//      into TMEM -- the weights are never dequantized by the SM;
//   B  the row-block's activations, each bf16 row split into two E4M3 rows
//      (hi = the top 4 significant bits, lo = the next 4) with one E8M0 scale
//      per 32 K (mx_quant.cu); hi and lo are consecutive rows of B, so one
//      instruction computes both and the epilogue adds the column pair;
//   D  fp32 accumulators in TMEM.
// hi + lo reproduces every bf16 activation within 2^9 of its 32-block maximum
// exactly (smaller ones to within 2^-17 of that maximum), so each product is
// the bf16 product the reference forms, accumulated in fp32.
//
// The MMA reads E2M1 operands in the 16-byte-group layout (16 values in 8
// bytes, 8 bytes padding).  The weights stream from HBM packed, as 128-byte
// rows (256 K) through a TMA ring; repack warps copy each 8-byte group into
// its padded slot of a small staging ring (no bit manipulation).
//
// One persistent CTA per SM walks the (row-block, m-tile) work list;
// warp-specialised (544 threads; 672 with a second epilogue warpgroup):
//   warps 0,3   TMA producers: packed weights (128 rows x 128 B, 128B
//               swizzle) + the two 512-byte scale blocks of the slot (bulk
//               copy), even / odd slots
//   warps 1,16  TMA producers: hi/lo activation rows (N2 x 128 B) + their
//               scale blocks, even / odd stages
//   warp 2      the MMA issuer (one thread): 4 (or 8) MMAs and the commits
//               of each stage.  Every tcgen05 MMA and commit of the CTA comes
//               from this thread: with several threads issuing them at the
//               same time, B200 produced occasional wrong tiles.
//   warps 4-7   epilogue: TMEM loads, hi + lo, bias, SwiGLU (gate_up) or
//   (17-20)     bias (down), bf16 stores; 64-row tiles split each item's
//               8-token blocks between two epilogue warpgroups
//   warps 8-15  two repack warpgroups (stage `it` to warpgroup it % 2): the
//               padded E2M1 staging tile and, with tcgen05.st (each warp its
//               TMEM lane quarter), the stage's weight and activation scales
//
// Every mbarrier wait is bounded (tc_common.cuh): a timed-out role records
// KLC_ERR_DEVICE_TIMEOUT, raises the CTA abort flag, and all roles drain
// before the TMEM is freed and the CTA exits.
#include <mutex>

#include "permute.cuh"
#include "tc_common.cuh"

namespace klc {

using namespace tc;

namespace {

constexpr int kBM = 128;        // weight rows per tile (MMA M)
constexpr int kStageK = 128;    // K per MMA stage: 4 MMAs of K = 32 (4 scale blocks)
constexpr int kSlotK = 256;     // K per weight slot (128-byte packed rows)
constexpr int kWarpA = 0, kWarpB = 1, kWarpMma0 = 2, kWarpA2 = 3, kWarpEpi0 = 4, kWarpRep0 = 8, kWarpB2 = 16,
              kWarpEpi2 = 17;
constexpr int kRepWGs = 2;  // repack warpgroups: warps 8-11 and 12-15, stage s to warpgroup s % 2
__device__ __forceinline__ int repack_wg_of_warp(int warp) {  // repack warpgroup of a warp, or -1
  return (warp >= kWarpRep0 && warp < kWarpRep0 + 4 * kRepWGs) ? (warp - kWarpRep0) >> 2 : -1;
}
__device__ __forceinline__ int issuer_of_warp(int warp) {  // MMA pipeline of a warp, or -1
  return warp == kWarpMma0 ? 0 : -1;
}
constexpr int kTmemCols = 512;

// Tile / pipeline configuration.
//   BN  max token rows of a row-block (B holds N2 = 2*BN hi/lo rows; an MMA
//       covers at most 128 of them, NCH = ceil(N2 / 128) MMAs per K step)
//   NA  weight slots (256 K of packed E2M1, 16 KB + 1 KB of scales each)
//   NS  staging slots (one MMA stage of padded E2M1, 16 KB, + its TMEM scale set)
//   NB  activation slots (one MMA stage, N2 x 128 B + NCH x 512 B scales);
//       NB == NS, so one commit frees a stage's staging and activation slot
//   NP  MMA issuers, each with its own accumulators and scale TMEM
// A parity wait is only sound while the waiter is within one phase of the
// barrier (two ahead it passes on a stale phase; two behind it waits for a
// phase that needs the waiter itself).  So every waiter of a slot waits for
// every use of it in order, and every use needs every waiter: each staging
// and activation slot serves a single issuer (NS and NB are multiples of NP)
// and a single repack warpgroup.
//   ND  accumulator sets per issuer (the epilogue of one tile overlaps the next)
//   PF  weight slots prefetched into L2 beyond the shared-memory ring
//   EPI epilogue warpgroups (warps 4-7, and 17-20 for a second one), splitting
//       each item's 8-token blocks
template <int BN_, int NA_, int NS_, int NB_, int NP_, int ND_, int PF_, int EPI_>
struct MxCfg {
  static constexpr int BN = BN_, NA = NA_, NS = NS_, NB = NB_, NP = NP_, ND = ND_, PF = PF_, EPI = EPI_;
  static constexpr int THREADS = (EPI == 2 ? 21 : 17) * 32;
  static_assert(EPI == 1 || EPI == 2, "epilogue warpgroups");
  static constexpr int N2 = 2 * BN;
  static constexpr int NCH = (N2 + 127) / 128;
  static constexpr int ASLOT = kBM * kSlotK / 2;     // 16384 packed bytes
  static constexpr int SSLOT = kBM * kStageK;        // 16384 padded bytes
  static constexpr int BSLOT = N2 * kStageK;         // N2 rows x 128 B of E4M3
  // shared memory (swizzled tiles 1024-byte aligned)
  static constexpr int OFF_A = 0;
  static constexpr int OFF_S = OFF_A + NA * ASLOT;
  static constexpr int OFF_B = OFF_S + NS * SSLOT;
  static constexpr int OFF_ASF = OFF_B + NB * BSLOT;       // NA x 1024
  static constexpr int OFF_BSF = OFF_ASF + NA * 1024;      // NB x NCH x 512
  static constexpr int OFF_BAR = OFF_BSF + NB * NCH * 512;
  static constexpr int NUM_BARS = 2 * NA + 2 * NS + NB + NP * ND + ND + 1;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  // TMEM: accumulators, then per staging slot a scale set: 4 columns for A
  // and 4 per B chunk, lane r0 column r1 byte kb = scale of row r0 + 32 r1,
  // 32-K block kb, replicated in the four lane quarters.  The repack warps
  // write a stage's scales (tcgen05.st) together with its staging slot, so a
  // set is rewritten only after the MMAs of the slot's previous use completed.
  static constexpr int ACC_COLS = ND * NP * N2;
  static constexpr int SF_COLS = 4 + 4 * NCH;
  static_assert(ACC_COLS + NS * SF_COLS <= kTmemCols, "TMEM budget");
  static_assert((NP == 1 || NP == 2 || NP == 4) && N2 <= 256, "issuers / tile");
  static_assert(NS % kRepWGs == 0 && NS % NP == 0 && NB % NP == 0 && NB % 2 == 0 && NA % 2 == 0, "slot ownership");
  static constexpr int NSP = NS / NP;  // staging slots per issuer
  // concurrent tcgen05 issue from several threads gave occasional wrong tiles
  static_assert(NP == 1, "one MMA issuer");
  // Stage s uses staging slot and activation slot s % NS: the issuer's one
  // commit per stage (sempty) frees both, and the activation producers wait on
  // it.  (Releasing activation slots from the repack warps instead, with
  // NB >= 2 NS, gave nondeterministic wrong tiles on B200 in a 2-staging /
  // 6-activation layout; a second issuer commit per stage cost 12% at decode.)
  static_assert(NB == NS, "activation slots follow the staging slots");
  static_assert(BSLOT % 1024 == 0, "activation slots stay 1024-byte aligned");
  static_assert(BYTES + 1024 <= 227 * 1024, "shared memory budget");
};

// Staging slot of MMA stage s (issuer s % NP, its (s / NP)-th stage) and the
// mbarrier phase parity of that use.  Stages sharing a slot are congruent
// modulo NS (a multiple of kRepWGs and of NP), and the repack warpgroup of
// stage s is s % kRepWGs, so each slot is filled by one warpgroup and drained
// by one issuer, both in stage order.
template <class C>
__device__ __forceinline__ void staging_slot(uint32_t s, int& slot, uint32_t& parity) {
  const uint32_t pp = s % C::NP, li = s / C::NP;
  slot = int(pp * C::NSP + li % C::NSP);
  parity = (li / C::NSP) & 1;
}

// kind::mxf8f6f4 instruction descriptor: A E2M1, B E4M3, fp32 accumulate,
// both K-major, E8M0 scales, M = 128, N = n; scale-factor byte ids a_id/b_id.
__device__ __forceinline__ uint32_t mx_idesc(int n, uint32_t a_id, uint32_t b_id) {
  return (b_id << 4) | (5u << 7) | (0u << 10) | (uint32_t(n >> 3) << 17) | (1u << 23) | (uint32_t(kBM >> 4) << 24) |
         (a_id << 29);
}

__device__ __forceinline__ void mx_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t sfa, uint32_t sfb,
                                       uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb));
}

struct MxParams {
  int n_out;            // weight rows of one expert (2I or H)
  int k_in;             // reduction length (H or I), a multiple of 64
  int ksteps;           // ceil(k_in / 128) MMA stages per item
  int n_mtiles;         // ceil(n_out / 128)
  const int4* rowblocks;
  DeviceStatus* status;
  const int32_t* rows;
  const uint8_t* sfa;   // [E][n_mtiles][ksteps][512]
  const uint8_t* sfb;   // [max_rowblocks][ksteps][NCH][512]
  const uint16_t* bias; // [E, n_out]
  uint16_t* out;        // phase 1: gated [rows_cap, n_out/2]; phase 2: [rows_cap, n_out]
  int out_ld;
  float* normsq;
  int precision;
  float limit, alpha;
  RowScatter sc;        // phase 2 of the weights-as-N kernels: rows to other buffers (world 0: none)
  // phase 1 of the weights-as-N kernels, when not null: the epilogue writes the
  // down GEMM's operand itself (hi/lo E4M3 rows [rows_cap][2][n_out/2] and their
  // scale blocks, the layout of the activation quantize) instead of bf16 rows
  uint8_t* qout;
  uint8_t* qsf;
  int q_stages;         // ceil(n_out / 2 / 128): 128-K stages of a scale-block row
};

template <int PHASE, class C>
__global__ void __launch_bounds__(C::THREADS, 1)
    mx_expert_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, MxParams p) {
  pdl_wait();     // inputs written by the previous kernel of the chain
  pdl_trigger();  // the next kernel may launch and set up meanwhile
  constexpr int NA = C::NA, NS = C::NS, NB = C::NB, NP = C::NP, ND = C::ND, N2 = C::N2, NCH = C::NCH;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const uint32_t bar0 = smem_u32(smem + C::OFF_BAR);
  auto afull = [&](int s) { return bar0 + 8u * s; };
  auto aempty = [&](int s) { return bar0 + 8u * (NA + s); };
  auto sfull = [&](int s) { return bar0 + 8u * (2 * NA + s); };
  auto sempty = [&](int s) { return bar0 + 8u * (2 * NA + NS + s); };
  auto bfull = [&](int s) { return bar0 + 8u * (2 * NA + 2 * NS + s); };
  auto dfull = [&](int pp, int d) { return bar0 + 8u * (2 * NA + 2 * NS + NB + pp * ND + d); };
  auto dempty = [&](int d) { return bar0 + 8u * (2 * NA + 2 * NS + NB + NP * ND + d); };
  const uint32_t mma_done = bar0 + 8u * (2 * NA + 2 * NS + NB + NP * ND + ND);
  auto dcol = [&](int pp, int d) { return uint32_t((d * NP + pp) * N2); };
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const Ctl ctl{abort_flag, p.status};

  if (threadIdx.x == 0) {
    for (int s = 0; s < NA; ++s) {
      mbar_init(afull(s), 1);
      mbar_init(aempty(s), 8);  // a repack warpgroup (four warps) for each of the slot's two stages
    }
    for (int s = 0; s < NS; ++s) {
      mbar_init(sfull(s), 4);
      mbar_init(sempty(s), 1);
    }
    for (int s = 0; s < NB; ++s) mbar_init(bfull(s), 1);
    for (int d = 0; d < ND; ++d) {
      for (int pp = 0; pp < NP; ++pp) mbar_init(dfull(pp, d), 1);
      mbar_init(dempty(d), 4 * C::EPI);  // every epilogue warp
    }
    mbar_init(mma_done, NP);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kWarpMma0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int nrb = p.status->rowblocks;
  const int total = nrb * p.n_mtiles;
  const int ks_n = p.ksteps;
  const int spa = (ks_n + 1) / 2;  // weight slots per item (the last may hold one stage)

  if (warp == kWarpA || warp == kWarpA2) {
    // ------------------------------------------------------------ weights
    // Two producers (slot parity q; NA even, so each slot has one producer):
    // one thread's per-slot issue latency next to busy warps would otherwise
    // bound the stage rate.  The shared-memory ring holds NA slots; an L2
    // prefetch cursor runs PF slots further ahead (the same boxes, no shared
    // memory), so about (NA + PF) x 16 KB per SM are in flight to HBM.
    const uint32_t q = warp == kWarpA ? 0u : 1u;
    if (lane == 0) {
      uint32_t it = 0, mine = 0;
      bool ok = true;
      int pf_item = blockIdx.x, pf_j = 0;
      uint32_t pf_n = 0;
      int4 pf_rb = pf_item < total ? p.rowblocks[pf_item / p.n_mtiles] : make_int4(0, 0, 0, 0);
      auto prefetch_ahead = [&](uint32_t upto) {
        while (pf_n < upto && pf_item < total) {
          if ((pf_n & 1u) == q) {
            const int pmt = pf_item % p.n_mtiles;
            tma_prefetch_3d(&map_a, pf_j * (kSlotK / 2), pmt * kBM, pf_rb.x);
            const int pnsf = (2 * pf_j + 1 < ks_n) ? 2 : 1;
            bulk_prefetch_l2(p.sfa + ((int64_t(pf_rb.x) * p.n_mtiles + pmt) * ks_n + 2 * pf_j) * 512,
                             uint32_t(pnsf * 512));
          }
          ++pf_n;
          if (++pf_j == spa) {
            pf_j = 0;
            pf_item += gridDim.x;
            if (pf_item < total) pf_rb = p.rowblocks[pf_item / p.n_mtiles];
          }
        }
      };
      for (int item = blockIdx.x; item < total && ok; item += gridDim.x) {
        const int4 rb = p.rowblocks[item / p.n_mtiles];
        const int mt = item % p.n_mtiles;
        const uint8_t* sfa_item = p.sfa + (int64_t(rb.x) * p.n_mtiles + mt) * int64_t(ks_n) * 512;
        for (int j = 0; j < spa && ok; ++j, ++it) {
          if ((it & 1u) != q) continue;
          prefetch_ahead(it + NA + C::PF);
          const int sa = it % NA;
          if (!(ok = wait_bar(aempty(sa), ((it / NA) & 1) ^ 1, ctl, 10))) break;
          const int nsf = (2 * j + 1 < ks_n) ? 2 : 1;  // scale blocks of the slot's stages
          mbar_arrive_expect_tx(afull(sa), uint32_t(C::ASLOT + nsf * 512));
          tma_load_3d(smem_u32(smem + C::OFF_A + sa * C::ASLOT), &map_a, j * (kSlotK / 2), mt * kBM, rb.x, afull(sa));
          bulk_load(smem_u32(smem + C::OFF_ASF + sa * 1024), sfa_item + int64_t(2 * j) * 512, uint32_t(nsf * 512),
                    afull(sa));
          ++mine;
        }
      }
      if (!ok) {
        // aborting: no bulk copy may still write shared memory -- the latest load of each of
        // this producer's slots (slot counters q + 2i, i < mine)
        const uint32_t first = mine > uint32_t(NA / 2) ? mine - uint32_t(NA / 2) : 0u;
        for (uint32_t i = first; i < mine; ++i) {
          const uint32_t sl = q + 2 * i;
          drain_wait(afull(int(sl % NA)), (sl / NA) & 1);
        }
      }
    }
  } else if (warp == kWarpB || warp == kWarpB2) {
    // ------------------------------------------------------------ activations
    // Two producers (stage parity q), one copy each per stage, so the per-stage
    // issue latency of a single thread does not bound the stage rate; with NB
    // even, each slot is filled by one producer.  A slot is free again once the
    // MMAs of its previous stage completed (the staging slot's commit, sempty:
    // the two rings have the same depth).  Rows N2 past the row-block
    // are loaded but not read by the MMA (N = 2 x the block's rows rounded up
    // to 8); rows and K past the buffer are zero-filled.
    const uint32_t q = warp == kWarpB ? 0u : 1u;
    if (lane == 0) {
      uint32_t it = 0, mine = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total && ok; item += gridDim.x) {
        const int rbi = item / p.n_mtiles;
        const int4 rb = p.rowblocks[rbi];
        const uint8_t* sfb_rb = p.sfb + int64_t(rbi) * ks_n * NCH * 512;
        for (int ks = 0; ks < ks_n && ok; ++ks, ++it) {
          if ((it & 1u) != q) continue;
          const int sb = it % NB;
          if (!(ok = wait_bar(sempty(sb), ((it / NB) & 1) ^ 1, ctl, 11))) break;
          mbar_arrive_expect_tx(bfull(sb), uint32_t(C::BSLOT + NCH * 512));
          tma_load_2d(smem_u32(smem + C::OFF_B + sb * C::BSLOT), &map_b, ks * kStageK, 2 * rb.y, bfull(sb));
          bulk_load(smem_u32(smem + C::OFF_BSF + sb * NCH * 512), sfb_rb + int64_t(ks) * NCH * 512, uint32_t(NCH * 512),
                    bfull(sb));
          ++mine;
        }
      }
      if (!ok) {
        // the latest load of each of this producer's slots: stages q + 2i, i < mine
        const uint32_t first = mine > uint32_t(NB / 2) ? mine - uint32_t(NB / 2) : 0u;
        for (uint32_t i = first; i < mine; ++i) {
          const uint32_t st = q + 2 * i;
          drain_wait(bfull(int(st % NB)), (st / NB) & 1);
        }
      }
    }
  } else if (issuer_of_warp(warp) >= 0) {
    // ------------------------------------------------------------ MMA issuers
    const int pp = issuer_of_warp(warp);
    if (lane == 0 && pp < NP) {
      uint32_t it = 0, ic = 0;
      int ss = 0, sb = 0;     // staging / activation slot of stage `it`
      uint32_t sph = 0;       // phase parity of the staging slot's use
      bool ok = true;
      for (int item = blockIdx.x; item < total && ok; item += gridDim.x, ++ic) {
        const int4 rb = p.rowblocks[item / p.n_mtiles];
        const int n2 = 2 * ((rb.z + 7) & ~7);  // hi/lo rows the MMA reads
        const int d = ic % ND;
        const uint32_t d_tmem = tmem + dcol(pp, d);
        if (!(ok = wait_bar(dempty(d), ((ic / ND) & 1) ^ 1, ctl, 20))) break;
        tc_fence_after();
        bool first = true;
        for (int ks = 0; ks < ks_n && ok; ++ks) {
          // the repack warps signal a stage once its staging slot, its TMEM
          // scales and (waited for by them) its activation slot are ready
          if (!(ok = wait_bar(sfull(ss), sph, ctl, 21))) break;
          tc_fence_after();
          const uint32_t sfa_t = tmem + uint32_t(C::ACC_COLS + ss * C::SF_COLS);  // the staging slot's scale set
          const uint32_t sfb_t = sfa_t + 4;
          const uint64_t adesc0 = sw128_desc(smem_u32(smem + C::OFF_S + ss * C::SSLOT));
          const uint64_t bdesc0 = sw128_desc(smem_u32(smem + C::OFF_B + sb * C::BSLOT));
          const int kb_n = min(4, (p.k_in - ks * kStageK) / 32);  // 32-K blocks in this stage
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            if (kk < kb_n) {
              const uint32_t acc = (first && kk == 0) ? 0u : 1u;
#pragma unroll
              for (int ch = 0; ch < NCH; ++ch) {
                const int nn = min(128, n2 - 128 * ch);
                if (nn > 0)
                  // descriptor start addresses advance by 32 B per K block and by 16 KB per 128 B rows
                  mx_mma(d_tmem + uint32_t(128 * ch), adesc0 + uint64_t(kk * 2),
                         bdesc0 + uint64_t(kk * 2 + ch * (128 * kStageK >> 4)), mx_idesc(nn, kk, kk),
                         sfa_t | (uint32_t(kk) << 30), (sfb_t + 4 * ch) | (uint32_t(kk) << 30), acc);
              }
            }
          }
          first = false;
          tc_commit(sempty(ss));  // frees the staging slot and the activation slot
          ++it;
          if (++ss == NS) {
            ss = 0;
            sph ^= 1u;
          }
          if (++sb == NB) sb = 0;
        }
        if (ok) tc_commit(dfull(pp, d));
      }
      tc_commit(mma_done);
      drain_wait(mma_done, 0);
    }
  } else if (repack_wg_of_warp(warp) >= 0) {
    // ------------------------------------------------------------ repack
    const int wg = repack_wg_of_warp(warp);  // stages with it % kRepWGs == wg
    const int m = (warp & 3) * 32 + lane;
    const int sw = m & 7;
    bool ok = true;
    // own stages it = wg, wg + kRepWGs, ... over the CTA's items; the item
    // counter ic and the stage ks inside the item follow incrementally
    uint32_t it = uint32_t(wg), ic = 0;
    int ks = wg, item = blockIdx.x;
    while (ks >= ks_n) {
      ks -= ks_n;
      ++ic;
      item += gridDim.x;
    }
    for (; item < total; it += kRepWGs) {
      {
        const uint32_t ia = ic * uint32_t(spa) + uint32_t(ks >> 1);
        const int sa = ia % NA, h = ks & 1;
        int ss;
        uint32_t sph;
        staging_slot<C>(it, ss, sph);
        // every lane waits (acquire); the decision is warp-uniform.  The packed
        // half and its scales are read before waiting for the staging slot, so
        // only the stores follow the MMA that frees it.
        ok = wait_bar(afull(sa), (ia / NA) & 1, ctl, 30);
        if (!(ok = __all_sync(0xffffffffu, ok))) break;
        // packed row m, 64-byte half h: chunks 4h..4h+3 of the 128B-swizzled row
        const unsigned char* src = smem + C::OFF_A + sa * C::ASLOT + m * 128;
        uint4 c[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) c[i] = *reinterpret_cast<const uint4*>(src + (((4 * h + i) ^ sw) << 4));
        // scale-set line `lane` of the stage's weight scales (16 bytes; every warp reads the block)
        const uint4 sfa4 = *reinterpret_cast<const uint4*>(smem + C::OFF_ASF + sa * 1024 + h * 512 + lane * 16);
        __syncwarp();  // every lane's reads of the weight slot precede the release
        if (lane == 0) {
          mbar_arrive(aempty(sa));
          if (h == 0 && ks == ks_n - 1) mbar_arrive(aempty(sa));  // the slot has no second stage
        }
        ok = wait_bar(sempty(ss), sph ^ 1, ctl, 31);
        if (!(ok = __all_sync(0xffffffffu, ok))) break;
        tc_fence_after();  // the slot's TMEM scale set is rewritten after the MMAs that read it
        // padded row m: 8 groups of 16 values, group g in the first 8 bytes of 16-byte chunk g ^ (m & 7)
        unsigned char* dst = smem + C::OFF_S + ss * C::SSLOT + (m >> 3) * 1024 + (m & 7) * 128;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          *reinterpret_cast<uint4*>(dst + (((2 * i) ^ sw) << 4)) = make_uint4(c[i].x, c[i].y, 0u, 0u);
          *reinterpret_cast<uint4*>(dst + (((2 * i + 1) ^ sw) << 4)) = make_uint4(c[i].z, c[i].w, 0u, 0u);
        }
        // the activation slot of this stage, then both scale sets into TMEM
        // (this warp's lane quarter)
        const int sb = it % NB;
        ok = wait_bar(bfull(sb), (it / NB) & 1, ctl, 32);
        if (!(ok = __all_sync(0xffffffffu, ok))) break;
        const uint32_t sf_t = tmem + (uint32_t((warp & 3) * 32) << 16) + uint32_t(C::ACC_COLS + ss * C::SF_COLS);
        tmem_st4(sf_t, sfa4);
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch)
          tmem_st4(sf_t + 4 + 4 * ch,
                   *reinterpret_cast<const uint4*>(smem + C::OFF_BSF + (sb * NCH + ch) * 512 + lane * 16));
        tmem_wait_st();
        fence_proxy_async();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sfull(ss));
      }
      ks += kRepWGs;
      while (ks >= ks_n) {
        ks -= ks_n;
        ++ic;
        item += gridDim.x;
      }
    }
  } else if ((warp >= kWarpEpi0 && warp < kWarpEpi0 + 4) || (C::EPI == 2 && warp >= kWarpEpi2 && warp < kWarpEpi2 + 4)) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter of this warp
    const int m = q * 32 + lane;
    const int eg = warp >= kWarpEpi2 ? 1 : 0;  // epilogue warpgroup: 8-token blocks eg, eg + EPI, ...
    uint32_t ic = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < total && ok; item += gridDim.x, ++ic) {
      const int4 rb = p.rowblocks[item / p.n_mtiles];
      const int mt = item % p.n_mtiles;
      const int e = rb.x, r0 = rb.y, nrows = rb.z;
      const int npad = (nrows + 7) & ~7;
      const int d = ic % ND;
      const int j = mt * kBM + m;  // output feature
      const bool jok = j < p.n_out;
      const float bias = jok ? bf16_to_f32(p.bias[int64_t(e) * p.n_out + j]) : 0.f;
      for (int pp = 0; pp < NP && ok; ++pp) ok = wait_bar_backoff(dfull(pp, d), (ic / ND) & 1, ctl, 40 + pp);
      if (!(ok = __all_sync(0xffffffffu, ok))) break;
      tc_fence_after();
      // pipeline pp received a K-stage of this item unless the item has fewer
      // stages than pipelines (stage `it` of the launch goes to it % NP)
      const uint32_t first_pp = uint32_t((uint64_t(ic) * uint64_t(ks_n)) % NP);
      const uint32_t lane_base = tmem + (uint32_t(q * 32) << 16);
      if (8 * eg >= npad) {
        // no block of this item for this warpgroup: release the set at once
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dempty(d));
      }
      for (int t0 = 8 * eg; t0 < npad; t0 += 8 * C::EPI) {
        uint32_t raw[16];  // columns 2t (hi) and 2t+1 (lo) of tokens t0..t0+7
        tmem_ld16(lane_base + dcol(int(first_pp), d) + uint32_t(2 * t0), raw);
        tmem_wait_ld();
        float v8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v8[i] = __uint_as_float(raw[2 * i]) + __uint_as_float(raw[2 * i + 1]);
        for (int j2 = 1; j2 < NP && j2 < ks_n; ++j2) {
          tmem_ld16(lane_base + dcol(int((first_pp + j2) % NP), d) + uint32_t(2 * t0), raw);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 8; ++i) v8[i] += __uint_as_float(raw[2 * i]) + __uint_as_float(raw[2 * i + 1]);
        }
        if (t0 + 8 * C::EPI >= npad) {
          // last accumulator columns read: hand the set back to the MMA warps early
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(dempty(d));
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int n = t0 + i;
          float v = v8[i];
          if (p.precision == KLC_PREC_BF16) v = round_bf16(v);
          v += bias;
          const bool nok = n < nrows;
          if (PHASE == 1) {
            // rows 2i (gate) and 2i+1 (up) of the interleaved gate_up projection
            const float up_raw = __shfl_xor_sync(0xffffffffu, v, 1);
            float g2 = 0.f;
            if ((lane & 1) == 0 && jok && nok) {
              const float gate = fminf(v, p.limit);
              const float up = fminf(fmaxf(up_raw, -p.limit), p.limit);
              const float glu = gate * (1.0f / (1.0f + expf(-(gate * p.alpha))));
              const float gated = (up + 1.0f) * glu;
              const uint16_t gb = f32_to_bf16(gated);
              p.out[int64_t(r0 + n) * p.out_ld + (j >> 1)] = gb;
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
  if (warp == kWarpMma0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

// ---------------------------------------------------------------------------
// Direct-operand variant: the weights are loaded by TMA with the
// CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B element type, which writes each group
// of 16 packed E2M1 values (8 bytes) into a 16-byte slot -- the operand layout
// the MMA reads -- so the weight tile lands in shared memory ready to use and
// no warp copies it.  This needs each weight row's K padded to a multiple of
// 128 values (klc_mxfp4_pad_k128, once per layer).
//
// Warps: 0 weight TMA producer (+ L2 prefetch cursor), 1 activation TMA
// producer, 2 the MMA issuer (one thread), 4-7 (and 12-15) epilogue, 8-11 the
// scale warpgroup: each warp writes the stage's weight and activation E8M0
// scales into its TMEM lane quarter (tcgen05.st) once both TMA copies of the
// stage landed, then signals the issuer.  Per stage (SK = 128 or 256 K) the
// issuer waits once, issues SK/32 MMAs and one commit, which frees the stage's
// weight slot, activation slot and scale set together.
// ---------------------------------------------------------------------------
constexpr int kWarp2A = 0, kWarp2B = 1, kWarp2Mma = 2, kWarp2Epi0 = 4, kWarp2Sf0 = 8, kWarp2Epi2 = 12, kWarp2Sf1 = 16;

// tcgen05.cp of one 512-byte scale block (32 rows x 16 bytes in shared memory)
// into 4 TMEM columns of lanes 0-31, replicated to the four lane quarters
__device__ __forceinline__ void tc_cp_scales(uint32_t taddr, uint32_t saddr) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(plain_desc(saddr)) : "memory");
}

//   BN  max token rows of a row-block (N2 = 2*BN hi/lo rows, <= 128)
//   NS  pipeline stages (weight slot + activation slot + TMEM scale set each)
//   ND  accumulator sets (the epilogue of one item overlaps the next)
//   EPI epilogue warpgroups
//   SK  K per stage: SK/128 TMA boxes of each operand
//   PF  weight stages prefetched into L2 beyond the shared-memory ring
//   SFW scale writers: 1 or 2 scale warpgroups (tcgen05.st; stage parity picks
//       the warpgroup), or 0: the issuer copies the scales itself (tcgen05.cp)
template <int BN_, int NS_, int ND_, int EPI_, int SK_, int PF_, int SFW_ = 1>
struct Mx2Cfg {
  static constexpr int BN = BN_, NS = NS_, ND = ND_, EPI = EPI_, SK = SK_, PF = PF_, SFW = SFW_;
  static constexpr int N2 = 2 * BN;
  static_assert(N2 <= 128, "one MMA N chunk");
  static constexpr int SUB = SK / 128;  // 128-K boxes per stage
  static_assert(SK == 128 || SK == 256, "stage K");
  static_assert(SFW >= 0 && SFW <= 2 && (SFW < 2 || NS % 2 == 0), "scale warpgroups own slots by parity");
  static constexpr int THREADS = (SFW == 2 ? 20 : (EPI == 2 ? 16 : (SFW == 1 ? 12 : 8))) * 32;
  static constexpr int ABOX = kBM * 128;      // one 128-K box of padded E2M1: 128 rows x 128 B in shared memory
  static constexpr int ABOX_TX = ABOX / 2;    // ... whose TMA transaction counts the packed bytes it read (8 KB)
  static constexpr int BBOX = N2 * kStageK;   // one 128-K box of hi/lo E4M3 rows
  static constexpr int ASLOT = SUB * ABOX, BSLOT = SUB * BBOX;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + NS * ASLOT;
  static constexpr int OFF_ASF = OFF_B + NS * BSLOT;       // NS x SUB x 512
  static constexpr int OFF_BSF = OFF_ASF + NS * SUB * 512;  // NS x SUB x 512
  static constexpr int OFF_BAR = OFF_BSF + NS * SUB * 512;
  static constexpr int NUM_BARS = 4 * NS + 2 * ND + 1;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int ACC_COLS = ND * N2;
  static constexpr int SF_COLS = 8 * SUB;  // per scale set: 4 columns per box for A, 4 for B
  static_assert(ACC_COLS + NS * SF_COLS <= kTmemCols, "TMEM budget");
  static_assert(BSLOT % 1024 == 0 && ASLOT % 1024 == 0, "slots stay 1024-byte aligned");
  static_assert(BYTES + 1024 <= 227 * 1024, "shared memory budget");
};

template <int PHASE, class C>
__global__ void __launch_bounds__(C::THREADS, 1)
    mx2_expert_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, MxParams p) {
  pdl_wait();     // inputs written by the previous kernel of the chain
  pdl_trigger();  // the next kernel may launch and set up meanwhile
  constexpr int NS = C::NS, ND = C::ND, N2 = C::N2, SUB = C::SUB;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const uint32_t bar0 = smem_u32(smem + C::OFF_BAR);
  auto afull = [&](int s) { return bar0 + 8u * s; };
  auto bfull = [&](int s) { return bar0 + 8u * (NS + s); };
  auto sready = [&](int s) { return bar0 + 8u * (2 * NS + s); };
  auto sempty = [&](int s) { return bar0 + 8u * (3 * NS + s); };
  auto dfull = [&](int d) { return bar0 + 8u * (4 * NS + d); };
  auto dempty = [&](int d) { return bar0 + 8u * (4 * NS + ND + d); };
  const uint32_t mma_done = bar0 + 8u * (4 * NS + 2 * ND);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const Ctl ctl{abort_flag, p.status};

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(afull(s), 1);
      mbar_init(bfull(s), 1);
      mbar_init(sready(s), 4);  // the four warps of the slot's scale warpgroup
      mbar_init(sempty(s), 1);  // the issuer's commit
    }
    for (int d = 0; d < ND; ++d) {
      mbar_init(dfull(d), 1);
      mbar_init(dempty(d), 4 * C::EPI);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kWarp2Mma) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int nrb = p.status->rowblocks;
  const int total = nrb * p.n_mtiles;
  const int kb128 = p.ksteps;                 // 128-K boxes per item
  const int st_n = (kb128 + SUB - 1) / SUB;    // stages per item

  if (warp == kWarp2A) {
    // ------------------------------------------------------------ weights
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      int pf_item = blockIdx.x, pf_k = 0;
      uint32_t pf_n = 0;
      int4 pf_rb = pf_item < total ? p.rowblocks[pf_item / p.n_mtiles] : make_int4(0, 0, 0, 0);
      auto prefetch_ahead = [&](uint32_t upto) {  // upto: in 128-K boxes issued so far
        while (pf_n < upto && pf_item < total) {
          tma_prefetch_3d(&map_a, pf_k * 128, (pf_item % p.n_mtiles) * kBM, pf_rb.x);
          ++pf_n;
          if (++pf_k == kb128) {
            pf_k = 0;
            pf_item += gridDim.x;
            if (pf_item < total) pf_rb = p.rowblocks[pf_item / p.n_mtiles];
          }
        }
      };
      uint32_t boxes = 0;
      for (int item = blockIdx.x; item < total && ok; item += gridDim.x) {
        const int4 rb = p.rowblocks[item / p.n_mtiles];
        const int mt = item % p.n_mtiles;
        const uint8_t* sfa_item = p.sfa + (int64_t(rb.x) * p.n_mtiles + mt) * int64_t(kb128) * 512;
        for (int ks = 0; ks < st_n && ok; ++ks, ++it) {
          prefetch_ahead(boxes + uint32_t(NS * SUB + C::PF));
          const int s = int(it % NS);
          if (!(ok = wait_bar(sempty(s), ((it / NS) & 1) ^ 1, ctl, 50))) break;
          const int nb = min(SUB, kb128 - ks * SUB);
          mbar_arrive_expect_tx(afull(s), uint32_t(nb * (C::ABOX_TX + 512)));
          for (int j = 0; j < nb; ++j)
            tma_load_3d(smem_u32(smem + C::OFF_A + s * C::ASLOT + j * C::ABOX), &map_a, (ks * SUB + j) * 128, mt * kBM, rb.x,
                        afull(s));
          bulk_load(smem_u32(smem + C::OFF_ASF + s * SUB * 512), sfa_item + int64_t(ks * SUB) * 512, uint32_t(nb * 512),
                    afull(s));
          boxes += uint32_t(nb);
        }
      }
      if (!ok) drain_ring(afull(0), NS, it);
    }
  } else if (warp == kWarp2B) {
    // ------------------------------------------------------------ activations
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total && ok; item += gridDim.x) {
        const int rbi = item / p.n_mtiles;
        const int4 rb = p.rowblocks[rbi];
        const uint8_t* sfb_rb = p.sfb + int64_t(rbi) * kb128 * 512;
        for (int ks = 0; ks < st_n && ok; ++ks, ++it) {
          const int s = int(it % NS);
          if (!(ok = wait_bar(sempty(s), ((it / NS) & 1) ^ 1, ctl, 51))) break;
          const int nb = min(SUB, kb128 - ks * SUB);
          mbar_arrive_expect_tx(bfull(s), uint32_t(nb * (C::BBOX + 512)));
          for (int j = 0; j < nb; ++j)
            tma_load_2d(smem_u32(smem + C::OFF_B + s * C::BSLOT + j * C::BBOX), &map_b, (ks * SUB + j) * kStageK, 2 * rb.y,
                        bfull(s));
          bulk_load(smem_u32(smem + C::OFF_BSF + s * SUB * 512), sfb_rb + int64_t(ks * SUB) * 512, uint32_t(nb * 512),
                    bfull(s));
        }
      }
      if (!ok) drain_ring(bfull(0), NS, it);
    }
  } else if (C::SFW > 0 && ((warp >= kWarp2Sf0 && warp < kWarp2Sf0 + 4) || (C::SFW == 2 && warp >= kWarp2Sf1 && warp < kWarp2Sf1 + 4))) {
    // ------------------------------------------------------------ scales
    const int q = warp & 3;  // this warp's TMEM lane quarter
    const uint32_t wg = warp >= kWarp2Sf1 ? 1u : 0u;  // stages it with it % SFW == wg
    uint32_t it = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < total && ok; item += gridDim.x) {
      for (int ks = 0; ks < st_n; ++ks, ++it) {
        if (C::SFW == 2 && (it & 1u) != wg) continue;
        const int s = int(it % NS);
        const uint32_t ph = (it / NS) & 1;
        // lane 0 polls; then every lane observes the completed phases (acquire) once
        if (lane == 0) ok = wait_bar(afull(s), ph, ctl, 52) && wait_bar(bfull(s), ph, ctl, 53);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (ok && lane != 0) ok = mbar_try_wait(afull(s), ph) && mbar_try_wait(bfull(s), ph);
        if (!(ok = __all_sync(0xffffffffu, ok))) break;
        tc_fence_after();  // the set is rewritten after the MMAs of its previous use completed
        const int nb = min(SUB, kb128 - ks * SUB);
        const uint32_t sf_t = tmem + (uint32_t(q * 32) << 16) + uint32_t(C::ACC_COLS + s * C::SF_COLS);
        for (int j = 0; j < nb; ++j) {
          tmem_st4(sf_t + 4 * j, *reinterpret_cast<const uint4*>(smem + C::OFF_ASF + (s * SUB + j) * 512 + lane * 16));
          tmem_st4(sf_t + 4 * SUB + 4 * j, *reinterpret_cast<const uint4*>(smem + C::OFF_BSF + (s * SUB + j) * 512 + lane * 16));
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sready(s));
      }
    }
  } else if (warp == kWarp2Mma) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t it = 0, ic = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total && ok; item += gridDim.x, ++ic) {
        const int4 rb = p.rowblocks[item / p.n_mtiles];
        const int n2 = 2 * ((rb.z + 7) & ~7);  // hi/lo rows the MMA reads
        const uint32_t idesc = mx_idesc(n2, 0, 0);
        const int d = ic % ND;
        const uint32_t d_tmem = tmem + uint32_t(d * N2);
        if (!(ok = wait_bar(dempty(d), ((ic / ND) & 1) ^ 1, ctl, 60))) break;
        tc_fence_after();
        for (int ks = 0; ks < st_n && ok; ++ks, ++it) {
          const int s = int(it % NS);
          const uint32_t sfa_t = tmem + uint32_t(C::ACC_COLS + s * C::SF_COLS);
          const uint32_t sfb_t = sfa_t + 4 * SUB;
          if (C::SFW > 0) {
            if (!(ok = wait_bar(sready(s), (it / NS) & 1, ctl, 61))) break;
            tc_fence_after();
          } else {
            // both operands and their scale blocks landed: copy the scales into the
            // stage's set (ordered before this thread's MMAs that read them)
            if (!(ok = wait_bar(afull(s), (it / NS) & 1, ctl, 62) && wait_bar(bfull(s), (it / NS) & 1, ctl, 63))) break;
            tc_fence_after();
            const int nbx = min(SUB, kb128 - ks * SUB);
            for (int j = 0; j < nbx; ++j) {
              tc_cp_scales(sfa_t + 4 * j, smem_u32(smem + C::OFF_ASF + (s * SUB + j) * 512));
              tc_cp_scales(sfb_t + 4 * j, smem_u32(smem + C::OFF_BSF + (s * SUB + j) * 512));
            }
          }
          const uint64_t adesc0 = sw128_desc(smem_u32(smem + C::OFF_A + s * C::ASLOT));
          const uint64_t bdesc0 = sw128_desc(smem_u32(smem + C::OFF_B + s * C::BSLOT));
          const int kk_n = min(C::SK, p.k_in - ks * C::SK) / 32;  // 32-K blocks in this stage
#pragma unroll
          for (int kk = 0; kk < 4 * SUB; ++kk) {
            if (kk < kk_n) {
              const int j = kk >> 2, kb = kk & 3;
              // descriptor start addresses advance by 32 B per K block and by one box per 128 K
              mx_mma(d_tmem, adesc0 + uint64_t(j * (C::ABOX >> 4) + kb * 2), bdesc0 + uint64_t(j * (C::BBOX >> 4) + kb * 2),
                     idesc | (uint32_t(kb) << 4) | (uint32_t(kb) << 29), (sfa_t + 4 * j) | (uint32_t(kb) << 30),
                     (sfb_t + 4 * j) | (uint32_t(kb) << 30), (ks == 0 && kk == 0) ? 0u : 1u);
            }
          }
          tc_commit(sempty(s));  // frees the weight slot, the activation slot and the scale set
        }
        if (ok) tc_commit(dfull(d));
      }
      tc_commit(mma_done);
      drain_wait(mma_done, 0);
    }
  } else if ((warp >= kWarp2Epi0 && warp < kWarp2Epi0 + 4) || (C::EPI == 2 && warp >= kWarp2Epi2 && warp < kWarp2Epi2 + 4)) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int m = q * 32 + lane;
    const int eg = warp >= kWarp2Epi2 ? 1 : 0;
    uint32_t ic = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < total && ok; item += gridDim.x, ++ic) {
      const int4 rb = p.rowblocks[item / p.n_mtiles];
      const int mt = item % p.n_mtiles;
      const int e = rb.x, r0 = rb.y, nrows = rb.z;
      const int npad = (nrows + 7) & ~7;
      const int d = ic % ND;
      const int j = mt * kBM + m;
      const bool jok = j < p.n_out;
      const float bias = jok ? bf16_to_f32(p.bias[int64_t(e) * p.n_out + j]) : 0.f;
      ok = wait_bar_backoff(dfull(d), (ic / ND) & 1, ctl, 70);
      if (!(ok = __all_sync(0xffffffffu, ok))) break;
      tc_fence_after();
      const uint32_t lane_base = tmem + (uint32_t(q * 32) << 16) + uint32_t(d * N2);
      if (8 * eg >= npad) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dempty(d));
      }
      for (int t0 = 8 * eg; t0 < npad; t0 += 8 * C::EPI) {
        uint32_t raw[16];
        tmem_ld16(lane_base + uint32_t(2 * t0), raw);
        tmem_wait_ld();
        if (t0 + 8 * C::EPI >= npad) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(dempty(d));
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int n = t0 + i;
          float v = __uint_as_float(raw[2 * i]) + __uint_as_float(raw[2 * i + 1]);
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
              p.out[int64_t(r0 + n) * p.out_ld + (j >> 1)] = gb;
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
  if (warp == kWarp2Mma)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

// ---------------------------------------------------------------------------
// Swapped-operand variant: A = the row-block's hi/lo E4M3 activation rows (the
// MMA's M = 128 TMEM lanes; 2*BN rows are loaded and lanes past them are never
// read), B = kWN = 192 weight rows (N = 192) loaded by TMA's 4-bit unpacking
// copy.  One instruction then covers 192 weight rows x 32 K (3 KB of packed
// weights), 1.5x what the weights-as-A form covers with M = 128, so a stage needs
// fewer MMA issues per weight byte -- the limit of the decode kernel.  In D the
// lanes are activation rows (hi and lo of a token in lanes 2n, 2n+1) and the
// columns weight rows (gate and up of a feature in columns 2f, 2f+1): the
// epilogue adds hi + lo across a lane pair and applies the clamped SwiGLU across
// a column pair, both inside a thread's registers or one shuffle.
// Weight scales come in 192-row tiles (klc_mxfp4_scales_tile, two 512-byte
// blocks per 128-K stage: rows 0-127 and 128-191 of the tile).
// ---------------------------------------------------------------------------
constexpr int kWN = 192;

//   BN  max tokens of a row-block (2*BN <= 128 activation rows)
//   NS  pipeline stages, ND accumulator sets, SK K per stage, PF L2 prefetch depth (boxes)
//   EPI epilogue warpgroups (warps 4-7, 12-15): warpgroup g takes the 16-column
//       chunks c with c % EPI == g, so a decode tile (all tokens in lane quarter 0)
//       is still read by EPI warps at once
//   PAIR two-SM tiles: a cluster of two CTAs computes a paired row-block (two
//       consecutive 64-row blocks of one expert) with one M = 256 MMA
//       (cta_group::2) issued by the even CTA: each CTA loads its own 64 tokens
//       (A rows 0-127 / 128-255) and half of the weight tile (B rows 0-95 /
//       96-191), so every weight byte an SM loads feeds twice the rows; both
//       CTAs hold the full 128 x 192 accumulator of their own rows and all
//       weight scales, and each runs its own epilogue
template <int BN_, int NS_, int ND_, int SK_, int PF_, int EPI_ = 2, int PAIR_ = 0>
struct Mx3Cfg {
  static constexpr int BN = BN_, NS = NS_, ND = ND_, SK = SK_, PF = PF_, EPI = EPI_;
  static constexpr bool PAIR = PAIR_ != 0;
  static_assert(!PAIR || BN == 64, "two-SM tiles take 64 tokens per CTA");
  static constexpr int CTAS = PAIR ? 2 : 1;
  static constexpr int WNB = kWN / CTAS;             // weight rows one CTA loads per tile
  static constexpr int N2 = 2 * BN;
  static_assert(N2 <= 128, "activation rows fit the MMA's 128 lanes");
  static_assert(EPI == 1 || EPI == 2, "epilogue warpgroups");
  static constexpr int SUB = SK / 128;
  static_assert(SK == 128 || SK == 256, "stage K");
  static constexpr int THREADS = (EPI == 2 ? 16 : 12) * 32;
  static constexpr int ABOX = N2 * 128;              // activation box (= its transaction bytes)
  static constexpr int BBOX = WNB * 128;             // weight box in shared memory (16-byte groups)
  static constexpr int BBOX_TX = BBOX / 2;           // ... counted as the packed bytes read
  static constexpr int ASLOT = SUB * ABOX, BSLOT = SUB * BBOX;
  static constexpr int OFF_B = 0;
  static constexpr int OFF_A = OFF_B + NS * BSLOT;
  // the MMA reads 128 rows (16 KB) from every activation box start: keep 16 KB of
  // shared memory after the last box
  static constexpr int APAD = 16384 > ABOX ? 16384 - ABOX : 0;
  static constexpr int OFF_ASF = OFF_A + NS * ASLOT + APAD;   // NS x SUB x 512 (activation scales)
  static constexpr int OFF_BSF = OFF_ASF + NS * SUB * 512;    // NS x SUB x 1024 (weight scales, 2 chunks)
  static constexpr int OFF_BAR = OFF_BSF + NS * SUB * 1024;
  static constexpr int NUM_BARS = 4 * NS + 2 * ND + 1;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int OFF_XCH = OFF_MISC + 16;      // 2 x 4 x 64 block exponents (fused quantize)
  static constexpr int BYTES = OFF_XCH + 2048;
  static constexpr int ACC_COLS = ND * kWN;
  static constexpr int SF_COLS = 12 * SUB;  // per box: 4 columns of activation scales, 8 of weight scales
  static_assert(ACC_COLS + NS * SF_COLS <= kTmemCols, "TMEM budget");
  static_assert(ABOX % 1024 == 0 && BBOX % 1024 == 0, "boxes stay 1024-byte aligned");
  static_assert(BYTES + 1024 <= 227 * 1024, "shared memory budget");
};

// kind::mxf8f6f4 instruction descriptor: A E4M3 (activations), B E2M1 (weights),
// fp32 accumulate, both K-major, E8M0 scales, M = 128 (256 for a CTA pair),
// N = kWN; scale byte ids.
template <int M>
__device__ __forceinline__ uint32_t mx3_idesc(uint32_t a_id, uint32_t b_id) {
  return (b_id << 4) | (0u << 7) | (5u << 10) | (uint32_t(kWN >> 3) << 17) | (1u << 23) | (uint32_t(M >> 4) << 24) |
         (a_id << 29);
}

// two fp32 -> two E4M3 (satfinite, round to nearest): a -> lower byte, b -> upper
__device__ __forceinline__ uint32_t e4m3_pair(float a, float b) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(b), "f"(a));
  return r;
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// The two-SM forms of the MMA and of its commits (issued by the even CTA of
// the pair; the commit arrives on the barrier at the same offset in every CTA
// of `mask`).
__device__ __forceinline__ void mx_mma_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t sfa, uint32_t sfb,
                                            uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb));
}

__device__ __forceinline__ void tc_commit_pair(uint32_t bar, uint16_t mask) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
               "h"(mask)
               : "memory");
}

// Address of the same shared-memory variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}

// Arrive on a barrier of another CTA of the pair.  The plain form (release
// at CTA scope) is the one two-SM tcgen05 pipelines use for their peer
// arrivals: the tcgen05 fences around the arrive and the wait order the TMEM
// accesses.  A cluster-scope release here costs a memory barrier per stage
// (measured: the kernel ran at half speed, stalled on it).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

template <int PHASE, class C>
__global__ void __launch_bounds__(C::THREADS, 1)
    mx3_expert_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x, MxParams p) {
  pdl_wait();     // inputs written by the previous kernel of the chain
  pdl_trigger();  // the next kernel may launch and set up meanwhile
  constexpr int NS = C::NS, ND = C::ND, SUB = C::SUB;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const uint32_t bar0 = smem_u32(smem + C::OFF_BAR);
  auto wfull = [&](int s) { return bar0 + 8u * s; };
  auto xfull = [&](int s) { return bar0 + 8u * (NS + s); };
  auto sready = [&](int s) { return bar0 + 8u * (2 * NS + s); };
  auto sempty = [&](int s) { return bar0 + 8u * (3 * NS + s); };
  auto dfull = [&](int d) { return bar0 + 8u * (4 * NS + d); };
  auto dempty = [&](int d) { return bar0 + 8u * (4 * NS + ND + d); };
  const uint32_t mma_done = bar0 + 8u * (4 * NS + 2 * ND);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const Ctl ctl{abort_flag, p.status};
  // CTA pair: rank 0 issues the MMAs; sready and dempty of rank 0 count the
  // arrivals of both CTAs, the other barriers are per CTA
  uint32_t crank = 0;
  if constexpr (C::PAIR) asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(crank));
  const int cid = C::PAIR ? int(blockIdx.x >> 1) : int(blockIdx.x);
  const int ncl = C::PAIR ? int(gridDim.x >> 1) : int(gridDim.x);
  auto arrive_lead = [&](uint32_t bar) {
    if constexpr (C::PAIR) mbar_arrive_cluster(cluster_addr(bar, 0));
    else mbar_arrive(bar);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(wfull(s), 1);
      mbar_init(xfull(s), 1);
      mbar_init(sready(s), 4 * C::CTAS);
      mbar_init(sempty(s), 1);
    }
    for (int d = 0; d < ND; ++d) {
      mbar_init(dfull(d), 1);
      mbar_init(dempty(d), 4 * C::EPI * C::CTAS);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kWarp2Mma) {
    if constexpr (C::PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                   "r"(kTmemCols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                   "r"(kTmemCols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  tc_fence_before();
  if constexpr (C::PAIR) cluster_sync_all();  // the peer's barriers are initialised before any remote arrive
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  // items: (row-block, 192-row weight tile); for a pair, (paired row-block, tile)
  const int nrb = C::PAIR ? p.status->pairblocks : p.status->rowblocks;
  const int total = nrb * p.n_mtiles;
  const int kb128 = p.ksteps;
  const int st_n = (kb128 + SUB - 1) / SUB;

  if (warp == kWarp2A) {
    // ------------------------------------------------------------ weights (operand B)
    if (lane == 0) {
      uint32_t it = 0, boxes = 0;
      bool ok = true;
      int pf_item = cid, pf_k = 0;
      uint32_t pf_n = 0;
      int4 pf_rb = pf_item < total ? p.rowblocks[pf_item / p.n_mtiles] : make_int4(0, 0, 0, 0);
      auto prefetch_ahead = [&](uint32_t upto) {
        while (pf_n < upto && pf_item < total) {
          tma_prefetch_3d(&map_w, pf_k * 128, (pf_item % p.n_mtiles) * kWN + int(crank) * C::WNB, pf_rb.x);
          ++pf_n;
          if (++pf_k == kb128) {
            pf_k = 0;
            pf_item += ncl;
            if (pf_item < total) pf_rb = p.rowblocks[pf_item / p.n_mtiles];
          }
        }
      };
      for (int item = cid; item < total && ok; item += ncl) {
        const int4 rb = p.rowblocks[item / p.n_mtiles];
        const int nt = item % p.n_mtiles;
        const uint8_t* sfw_item = p.sfa + (int64_t(rb.x) * p.n_mtiles + nt) * int64_t(kb128) * 1024;
        for (int ks = 0; ks < st_n && ok; ++ks, ++it) {
          prefetch_ahead(boxes + uint32_t(NS * SUB + C::PF));
          const int s = int(it % NS);
          if (!(ok = wait_bar(sempty(s), ((it / NS) & 1) ^ 1, ctl, 80))) break;
          const int nb = min(SUB, kb128 - ks * SUB);
          mbar_arrive_expect_tx(wfull(s), uint32_t(nb * (C::BBOX_TX + 1024)));
          for (int j = 0; j < nb; ++j)
            tma_load_3d(smem_u32(smem + C::OFF_B + s * C::BSLOT + j * C::BBOX), &map_w, (ks * SUB + j) * 128,
                        nt * kWN + int(crank) * C::WNB, rb.x, wfull(s));
          bulk_load(smem_u32(smem + C::OFF_BSF + s * SUB * 1024), sfw_item + int64_t(ks * SUB) * 1024, uint32_t(nb * 1024),
                    wfull(s));
          boxes += uint32_t(nb);
        }
      }
      if (!ok) drain_ring(wfull(0), NS, it);
    }
  } else if (warp == kWarp2B) {
    // ------------------------------------------------------------ activations (operand A)
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int item = cid; item < total && ok; item += ncl) {
        const int rbi = item / p.n_mtiles;
        const int4 rb = p.rowblocks[rbi];
        // a pair's CTA takes the pair's row-block rb.w + crank (64 rows), which may be empty
        const int row0 = rb.y + int(crank) * 64;
        const bool load = !C::PAIR || rb.z > int(crank) * 64;
        const uint8_t* sfx_rb = p.sfb + int64_t(C::PAIR ? rb.w + int(crank) : rbi) * kb128 * 512;
        for (int ks = 0; ks < st_n && ok; ++ks, ++it) {
          const int s = int(it % NS);
          if (!(ok = wait_bar(sempty(s), ((it / NS) & 1) ^ 1, ctl, 81))) break;
          const int nb = min(SUB, kb128 - ks * SUB);
          if (!load) {  // no rows: the stage completes without data (its lanes are never read)
            mbar_arrive(xfull(s));
            continue;
          }
          mbar_arrive_expect_tx(xfull(s), uint32_t(nb * (C::ABOX + 512)));
          for (int j = 0; j < nb; ++j)
            tma_load_2d(smem_u32(smem + C::OFF_A + s * C::ASLOT + j * C::ABOX), &map_x, (ks * SUB + j) * kStageK, 2 * row0,
                        xfull(s));
          bulk_load(smem_u32(smem + C::OFF_ASF + s * SUB * 512), sfx_rb + int64_t(ks * SUB) * 512, uint32_t(nb * 512),
                    xfull(s));
        }
      }
      if (!ok) drain_ring(xfull(0), NS, it);
    }
  } else if (warp >= kWarp2Sf0 && warp < kWarp2Sf0 + 4) {
    // ------------------------------------------------------------ scales into TMEM
    const int q = warp & 3;
    uint32_t it = 0;
    bool ok = true;
    for (int item = cid; item < total && ok; item += ncl) {
      for (int ks = 0; ks < st_n; ++ks, ++it) {
        const int s = int(it % NS);
        const uint32_t ph = (it / NS) & 1;
        if (lane == 0) ok = wait_bar(wfull(s), ph, ctl, 82) && wait_bar(xfull(s), ph, ctl, 83);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (ok && lane != 0) ok = mbar_try_wait(wfull(s), ph) && mbar_try_wait(xfull(s), ph);
        if (!(ok = __all_sync(0xffffffffu, ok))) break;
        tc_fence_after();  // the set is rewritten after the MMAs of its previous use completed
        const int nb = min(SUB, kb128 - ks * SUB);
        const uint32_t sf_t = tmem + (uint32_t(q * 32) << 16) + uint32_t(C::ACC_COLS + s * C::SF_COLS);
        for (int j = 0; j < nb; ++j) {
          tmem_st4(sf_t + 12 * j, *reinterpret_cast<const uint4*>(smem + C::OFF_ASF + (s * SUB + j) * 512 + lane * 16));
          tmem_st4(sf_t + 12 * j + 4, *reinterpret_cast<const uint4*>(smem + C::OFF_BSF + (s * SUB + j) * 1024 + lane * 16));
          tmem_st4(sf_t + 12 * j + 8, *reinterpret_cast<const uint4*>(smem + C::OFF_BSF + (s * SUB + j) * 1024 + 512 + lane * 16));
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) arrive_lead(sready(s));
      }
    }
  } else if (warp == kWarp2Mma) {
    // ------------------------------------------------------------ MMA issuer (rank 0 of a pair)
    if (lane == 0 && crank == 0) {
      uint32_t it = 0, ic = 0;
      bool ok = true;
      for (int item = cid; item < total && ok; item += ncl, ++ic) {
        const int d = ic % ND;
        const uint32_t d_tmem = tmem + uint32_t(d * kWN);
        if (!(ok = wait_bar(dempty(d), ((ic / ND) & 1) ^ 1, ctl, 90))) break;
        tc_fence_after();
        for (int ks = 0; ks < st_n && ok; ++ks, ++it) {
          const int s = int(it % NS);
          if (!(ok = wait_bar(sready(s), (it / NS) & 1, ctl, 91))) break;
          tc_fence_after();
          const uint32_t sf_t = tmem + uint32_t(C::ACC_COLS + s * C::SF_COLS);
          const uint64_t xdesc0 = sw128_desc(smem_u32(smem + C::OFF_A + s * C::ASLOT));
          const uint64_t wdesc0 = sw128_desc(smem_u32(smem + C::OFF_B + s * C::BSLOT));
          const int kk_n = min(C::SK, p.k_in - ks * C::SK) / 32;
#pragma unroll
          for (int kk = 0; kk < 4 * SUB; ++kk) {
            if (kk < kk_n) {
              const int j = kk >> 2, kb = kk & 3;
              const uint64_t xd = xdesc0 + uint64_t(j * (C::ABOX >> 4) + kb * 2);
              const uint64_t wd = wdesc0 + uint64_t(j * (C::BBOX >> 4) + kb * 2);
              const uint32_t sfa = (sf_t + 12 * j) | (uint32_t(kb) << 30), sfb = (sf_t + 12 * j + 4) | (uint32_t(kb) << 30);
              const uint32_t acc = (ks == 0 && kk == 0) ? 0u : 1u;
              if constexpr (C::PAIR) mx_mma_pair(d_tmem, xd, wd, mx3_idesc<256>(uint32_t(kb), uint32_t(kb)), sfa, sfb, acc);
              else mx_mma(d_tmem, xd, wd, mx3_idesc<kBM>(uint32_t(kb), uint32_t(kb)), sfa, sfb, acc);
            }
          }
          if constexpr (C::PAIR) tc_commit_pair(sempty(s), 3);
          else tc_commit(sempty(s));
        }
        if (ok) {
          if constexpr (C::PAIR) tc_commit_pair(dfull(d), 3);
          else tc_commit(dfull(d));
        }
      }
      if constexpr (C::PAIR) tc_commit_pair(mma_done, 1);
      else tc_commit(mma_done);
      drain_wait(mma_done, 0);
    }
  } else if ((warp >= kWarp2Epi0 && warp < kWarp2Epi0 + 4) || (C::EPI == 2 && warp >= kWarp2Epi2 && warp < kWarp2Epi2 + 4)) {
    // ------------------------------------------------------------ epilogue
    // warp q reads TMEM lanes 32q..32q+31 = activation rows of tokens 16q..16q+15;
    // warpgroup eg takes the column chunks c with c % EPI == eg
    const int q = warp & 3;
    const int eg = warp >= kWarp2Epi2 ? 1 : 0;
    uint32_t ic = 0;
    uint32_t xk = 0;  // fused quantize: blocks exchanged so far (the exchange slot's parity)
    bool ok = true;
    for (int item = cid; item < total && ok; item += ncl, ++ic) {
      const int4 rb = p.rowblocks[item / p.n_mtiles];
      const int nt = item % p.n_mtiles;
      // a pair's CTA holds the accumulators of its own 64 rows
      const int e = rb.x, r0 = rb.y + int(crank) * 64;
      const int nrows = C::PAIR ? max(0, min(64, rb.z - int(crank) * 64)) : rb.z;
      const int d = ic % ND;
      ok = wait_bar_backoff(dfull(d), (ic / ND) & 1, ctl, 92);
      if (!(ok = __all_sync(0xffffffffu, ok))) break;
      tc_fence_after();
      const int n = 16 * q + (lane >> 1);     // this lane's token within the row-block
      const bool tok = n < nrows;
      const bool hi_lane = (lane & 1) == 0;   // even lane: hi row, holds the sum
      if (16 * q < nrows) {
        const uint32_t lane_base = tmem + (uint32_t(q * 32) << 16) + uint32_t(d * kWN);
        // destination row: dense, or (down pass with a scatter) its segment of another buffer
        uint16_t* drow = p.out + int64_t(r0 + n) * p.out_ld;
        if (PHASE == 2 && p.sc.world > 0 && tok) {
          const int pq = p.rows[r0 + n];
          const int seg = pq >= 0 ? int(pq / p.sc.seg_cap) : -1;
          drow = (seg >= 0 && seg < p.sc.world)
                     ? reinterpret_cast<uint16_t*>(p.sc.base[seg] +
                                                   (p.sc.slot0 + pq % p.sc.seg_cap) * int64_t(p.out_ld) * 2)
                     : nullptr;
        }
        float sq = 0.f;
        // bias of the first chunk, loaded before the accumulators are read; each
        // chunk then loads the next chunk's bias ahead of its own work
        const uint16_t* brow = p.bias + int64_t(e) * p.n_out;
        auto load_bias = [&](int c0, uint4& b0, uint4& b1) {
          const int j = nt * kWN + c0;
          if (c0 < kWN && j < p.n_out) {  // j is a multiple of 16; n_out a multiple of 64
            b0 = *reinterpret_cast<const uint4*>(brow + j);
            b1 = *reinterpret_cast<const uint4*>(brow + j + 8);
          }
        };
        uint4 nb0 = make_uint4(0, 0, 0, 0), nb1 = nb0;
        if (PHASE == 1 && C::EPI == 2 && p.qout != nullptr) {
          // Fused down-operand quantize: warpgroup eg takes features 16eg..16eg+15 of
          // each 32-feature block (column chunks 4b + 2eg, 4b + 2eg + 1); the two warps
          // of a lane quarter agree on the block's exponent through shared memory
          // (double-buffered by block parity, one named barrier per block).  Even
          // lanes store the hi row, odd lanes the lo row, each with its scale byte:
          // the bytes the activation quantize writes for the bf16 gated values.
          uint32_t* xch = reinterpret_cast<uint32_t*>(smem + C::OFF_XCH) + q * 64;
          const int rbq = C::PAIR ? rb.w + int(crank) : item / p.n_mtiles;  // scale tile's 64-row block
          const int kq = p.n_out >> 1;  // the down GEMM's K
          for (int b = 0; b < kWN / 64; ++b) {
            if (nt * kWN + 64 * b >= p.n_out) break;  // n_out is a multiple of 64: whole blocks
            uint16_t g[16];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int c0 = 64 * b + 32 * eg + 16 * h;
              const int j0 = nt * kWN + c0;
              uint32_t raw[16];
              tmem_ld16(lane_base + uint32_t(c0), raw);
              const uint4 b0 = *reinterpret_cast<const uint4*>(brow + j0);
              const uint4 b1 = *reinterpret_cast<const uint4*>(brow + j0 + 8);
              tmem_wait_ld();
              const uint32_t bw[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
              float v[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const float mine = __uint_as_float(raw[i]);
                float x = mine + __shfl_xor_sync(0xffffffffu, mine, 1);  // hi + lo
                if (p.precision == KLC_PREC_BF16) x = round_bf16(x);
                v[i] = x + bf16_to_f32(uint16_t((i & 1) ? (bw[i >> 1] >> 16) : (bw[i >> 1] & 0xFFFFu)));
              }
#pragma unroll
              for (int f = 0; f < 8; ++f) {
                const float gate = fminf(v[2 * f], p.limit);
                const float up = fminf(fmaxf(v[2 * f + 1], -p.limit), p.limit);
                const float glu = gate * (1.0f / (1.0f + expf(-(gate * p.alpha))));
                const float gated = (up + 1.0f) * glu;
                const uint16_t gb = f32_to_bf16(gated);
                const float gr = bf16_to_f32(gb);
                sq += (p.precision == KLC_PREC_BF16) ? gr * gr : gated * gated;
                g[8 * h + f] = gb;
              }
            }
            // the 32-value block's exponent: max over both halves, from the bf16 bits
            uint32_t emax = 0;
#pragma unroll
            for (int i = 0; i < 16; ++i) emax = max(emax, (uint32_t(g[i]) >> 7) & 0xFFu);
            // [parity][q][eg][lane]; the parity alternates over all blocks of all items, so a
            // slot is rewritten only after the partner passed the next barrier (its read done)
            uint32_t* slot = xch + (xk++ & 1u) * 256u;
            slot[eg * 32 + lane] = emax;
            named_bar_sync(1 + q, 64);
            emax = max(emax, slot[(1 - eg) * 32 + lane]);
            int S = emax == 0 ? 0 : int(emax) - 134;
            S = S < -126 ? -126 : (S > 126 ? 126 : S);
            const float inv = __uint_as_float(uint32_t(127 - S) << 23);  // 2^-S
            uint32_t qw[4];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const uint32_t a0 = g[2 * i], a1 = g[2 * i + 1];
              const float x0 = __uint_as_float(a0 << 16), x1 = __uint_as_float(a1 << 16);
              const float h0 = __uint_as_float((a0 & 0xFFF0u) << 16), h1 = __uint_as_float((a1 & 0xFFF0u) << 16);
              const uint32_t pr = hi_lane ? e4m3_pair(h0 * inv, h1 * inv) : e4m3_pair((x0 - h0) * inv, (x1 - h1) * inv);
              if (i & 1) qw[i >> 1] |= pr << 16;
              else qw[i >> 1] = pr;
            }
            if (tok) {
              const int64_t row = int64_t(r0 + n);
              const int f0 = (nt * kWN + 64 * b + 32 * eg) >> 1;  // first of the 16 features
              *reinterpret_cast<uint4*>(p.qout + row * 2 * kq + (hi_lane ? 0 : kq) + f0) =
                  make_uint4(qw[0], qw[1], qw[2], qw[3]);
              if (eg == 0) {
                const int kb = (nt * kWN + 64 * b) >> 6;  // 32-feature block index
                const int n2 = 2 * n + (hi_lane ? 0 : 1);
                uint8_t* blk = p.qsf + ((int64_t(rbq) * p.q_stages + kb / 4) + n2 / 128) * 512;
                blk[(n2 & 31) * 16 + ((n2 & 127) >> 5) * 4 + (kb & 3)] = uint8_t(S + 127);
              }
            }
          }
        } else {
        load_bias(16 * eg, nb0, nb1);
        for (int c0 = 16 * eg; c0 < kWN; c0 += 16 * C::EPI) {
          uint32_t raw[16];
          tmem_ld16(lane_base + uint32_t(c0), raw);
          const uint4 b0 = nb0, b1 = nb1;
          load_bias(c0 + 16 * C::EPI, nb0, nb1);
          tmem_wait_ld();
          const int j0 = nt * kWN + c0;  // first weight row of this chunk
          float v[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float mine = __uint_as_float(raw[i]);
            v[i] = mine + __shfl_xor_sync(0xffffffffu, mine, 1);  // hi + lo
          }
          if (j0 < p.n_out) {
            const uint32_t bw[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float x = v[i];
              if (p.precision == KLC_PREC_BF16) x = round_bf16(x);
              v[i] = x + bf16_to_f32(uint16_t((i & 1) ? (bw[i >> 1] >> 16) : (bw[i >> 1] & 0xFFFFu)));
            }
            if (tok && hi_lane && drow != nullptr) {
              uint16_t* orow = drow;
              if (PHASE == 1) {
                // columns 2f, 2f+1: gate and up of feature j0/2 + f
                uint32_t pk[4];
#pragma unroll
                for (int f = 0; f < 8; ++f) {
                  const float gate = fminf(v[2 * f], p.limit);
                  const float up = fminf(fmaxf(v[2 * f + 1], -p.limit), p.limit);
                  const float glu = gate * (1.0f / (1.0f + expf(-(gate * p.alpha))));
                  const float gated = (up + 1.0f) * glu;
                  const uint16_t gb = f32_to_bf16(gated);
                  const float gr = bf16_to_f32(gb);
                  sq += (p.precision == KLC_PREC_BF16) ? gr * gr : gated * gated;
                  if (f & 1) pk[f >> 1] |= uint32_t(gb) << 16;
                  else pk[f >> 1] = gb;
                }
                *reinterpret_cast<uint4*>(orow + (j0 >> 1)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
              } else {
                uint32_t pk[8];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  const uint16_t ob = f32_to_bf16(v[i]);
                  sq += v[i] * v[i];
                  if (i & 1) pk[i >> 1] |= uint32_t(ob) << 16;
                  else pk[i >> 1] = ob;
                }
                *reinterpret_cast<uint4*>(orow + j0) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                *reinterpret_cast<uint4*>(orow + j0 + 8) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
              }
            }
          }
        }
        }
        if (p.normsq != nullptr && tok && hi_lane)
          atomicAdd(&p.normsq[int64_t(p.rows[r0 + n]) * 2 + (PHASE == 1 ? 0 : 1)], sq);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) arrive_lead(dempty(d));
    }
    // scattered rows (peer memory) visible system-wide before the kernel that raises the flags
    if (PHASE == 2 && p.sc.world > 0) __threadfence_system();
  }

  tc_fence_before();
  // a pair: neither CTA leaves while the other's MMAs, arrivals or reads may still touch it
  if constexpr (C::PAIR) cluster_sync_all();
  else __syncthreads();
  tc_fence_after();
  if (warp == kWarp2Mma) {
    if constexpr (C::PAIR) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    else asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <int PHASE, class C>
int launch_mx_phase(const uint8_t* blocks, const uint8_t* act_q, int64_t rows_cap, int experts, MxParams p,
                    int max_rowblocks, cudaStream_t stream) {
  CUtensorMap ma, mb;
  const uint64_t K = uint64_t(p.k_in), N = uint64_t(p.n_out);
  p.ksteps = int((K + kStageK - 1) / kStageK);
  {
    // packed E2M1 [E][N][K/2] bytes; box = 128 rows x 128 bytes (one 256-K slot), 128B swizzle
    const uint64_t dims[3] = {K / 2, N, uint64_t(experts)};
    const uint64_t strides[2] = {K / 2, N * K / 2};
    const uint32_t box[3] = {kSlotK / 2, kBM, 1};
    int st = make_map(&ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, blocks, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != KLC_OK) return st;
  }
  {
    // hi/lo E4M3 rows [2 rows_cap][K] bytes; box = N2 rows x 128 bytes (one stage), 128B swizzle
    const uint64_t dims[2] = {K, 2 * uint64_t(rows_cap)};
    const uint64_t strides[1] = {K};
    const uint32_t box[2] = {kStageK, uint32_t(C::N2)};
    int st = make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, act_q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != KLC_OK) return st;
  }
  // >= 116 KB of shared memory keeps one CTA (and one 512-column TMEM allocation) per SM
  const int smem = (C::BYTES + 1024 > 118 * 1024) ? C::BYTES + 1024 : 118 * 1024;
  KLC_CUDA(cudaFuncSetAttribute(mx_expert_kernel<PHASE, C>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int64_t items = int64_t(max_rowblocks) * p.n_mtiles;
  const int grid = int(items < sm_count() ? items : sm_count());
  if (grid <= 0) return KLC_OK;
  KLC_CUDA(launch_chain(mx_expert_kernel<PHASE, C>, dim3(grid), dim3(C::THREADS), size_t(smem), stream, 0u, ma, mb, p));
  KLC_LAUNCH_CHECK("tcgen05 expert launch");
  return KLC_OK;
}

template <int PHASE, class C>
int launch_mx2_phase(const uint8_t* blocks_k128, const uint8_t* act_q, int64_t rows_cap, int experts, MxParams p,
                     int max_rowblocks, cudaStream_t stream) {
  CUtensorMap ma, mb;
  const uint64_t K = uint64_t(p.k_in), N = uint64_t(p.n_out);
  const uint64_t Kp = (K + 127) / 128 * 128;  // padded row length in E2M1 values
  p.ksteps = int(Kp / 128);
  KLC_CHECK_ARG((reinterpret_cast<uintptr_t>(blocks_k128) & 31) == 0, "tensor-core path: padded weight blocks must be 32-byte aligned");
  {
    // packed E2M1 [E][N][Kp] values (Kp/2 bytes per row); box = 128 values x 128 rows; each
    // 16-value group lands in a 16-byte shared-memory slot (16U4_ALIGN16B), 128B swizzle
    const uint64_t dims[3] = {Kp, N, uint64_t(experts)};
    const uint64_t strides[2] = {Kp / 2, N * Kp / 2};
    const uint32_t box[3] = {128, kBM, 1};
    int st = make_map(&ma, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 3, blocks_k128, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != KLC_OK) return st;
  }
  {
    // hi/lo E4M3 rows [2 rows_cap][K] bytes; box = N2 rows x 128 bytes, 128B swizzle
    const uint64_t dims[2] = {K, 2 * uint64_t(rows_cap)};
    const uint64_t strides[1] = {K};
    const uint32_t box[2] = {kStageK, uint32_t(C::N2)};
    int st = make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, act_q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != KLC_OK) return st;
  }
  const int smem = (C::BYTES + 1024 > 118 * 1024) ? C::BYTES + 1024 : 118 * 1024;  // one CTA per SM
  KLC_CUDA(cudaFuncSetAttribute(mx2_expert_kernel<PHASE, C>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int64_t items = int64_t(max_rowblocks) * p.n_mtiles;
  const int grid = int(items < sm_count() ? items : sm_count());
  if (grid <= 0) return KLC_OK;
  KLC_CUDA(launch_chain(mx2_expert_kernel<PHASE, C>, dim3(grid), dim3(C::THREADS), size_t(smem), stream, 0u, ma, mb, p));
  KLC_LAUNCH_CHECK("tcgen05 expert launch");
  return KLC_OK;
}

template <class C>
int launch_mx2_both(const ExpertArgs& a, const uint8_t* gu_k128, const uint8_t* dn_k128, cudaStream_t stream) {
  const klc_moe_weights& w = *a.wts;
  KLC_CHECK_ARG(w.gu_scales_mx != nullptr && w.dn_scales_mx != nullptr,
                "tensor-core path: gu_scales_mx / dn_scales_mx are required (klc_mxfp4_scales_mx)");
  MxParams p1{};
  p1.n_out = int(2 * a.inter);
  p1.k_in = int(a.hidden);
  p1.n_mtiles = (p1.n_out + kBM - 1) / kBM;
  p1.rowblocks = a.rowblocks;
  p1.status = a.status_rw;
  p1.rows = a.rows;
  p1.sfa = w.gu_scales_mx;
  p1.sfb = a.sfb1;
  p1.bias = w.gu_bias;
  p1.out = static_cast<uint16_t*>(a.gated);
  p1.out_ld = int(a.inter);
  p1.normsq = a.normsq;
  p1.precision = a.precision;
  p1.limit = w.swiglu_limit;
  p1.alpha = w.alpha;
  int st = launch_quantize_rows(a.x, a.hidden, a.rows, a.k, a.rowblocks, a.status, a.max_rowblocks, 1, a.xq, a.sfb1, stream);
  if (st != KLC_OK) return st;
  st = launch_mx2_phase<1, C>(gu_k128, a.xq, a.rows_cap, int(a.experts), p1, a.max_rowblocks, stream);
  if (st != KLC_OK) return st;
  stage_mark(kStageGateUp, stream);
  st = launch_quantize_rows(static_cast<const uint16_t*>(a.gated), a.inter, nullptr, 1, a.rowblocks, a.status,
                            a.max_rowblocks, 1, a.gq, a.sfb2, stream);
  if (st != KLC_OK) return st;
  MxParams p2 = p1;
  p2.n_out = int(a.hidden);
  p2.k_in = int(a.inter);
  p2.n_mtiles = (p2.n_out + kBM - 1) / kBM;
  p2.sfa = w.dn_scales_mx;
  p2.sfb = a.sfb2;
  p2.bias = w.dn_bias;
  p2.out = a.y;
  p2.out_ld = int(a.hidden);
  st = launch_mx2_phase<2, C>(dn_k128, a.gq, a.rows_cap, int(a.experts), p2, a.max_rowblocks, stream);
  stage_mark(kStageDown, stream);
  return st;
}

template <int PHASE, class C>
int launch_mx3_phase(const uint8_t* blocks_k128, const uint8_t* act_q, int64_t rows_cap, int experts, MxParams p,
                     int max_rowblocks, cudaStream_t stream) {
  CUtensorMap mw, mx;
  const uint64_t K = uint64_t(p.k_in), N = uint64_t(p.n_out);
  const uint64_t Kp = (K + 127) / 128 * 128;
  p.ksteps = int(Kp / 128);
  p.n_mtiles = int((N + kWN - 1) / kWN);  // 192-row weight tiles
  KLC_CHECK_ARG((reinterpret_cast<uintptr_t>(blocks_k128) & 31) == 0, "tensor-core path: padded weight blocks must be 32-byte aligned");
  {
    const uint64_t dims[3] = {Kp, N, uint64_t(experts)};
    const uint64_t strides[2] = {Kp / 2, N * Kp / 2};
    const uint32_t box[3] = {128, uint32_t(C::WNB), 1};
    int st = make_map(&mw, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 3, blocks_k128, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != KLC_OK) return st;
  }
  {
    const uint64_t dims[2] = {K, 2 * uint64_t(rows_cap)};
    const uint64_t strides[1] = {K};
    const uint32_t box[2] = {kStageK, uint32_t(C::N2)};
    int st = make_map(&mx, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, act_q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != KLC_OK) return st;
  }
  const int smem = (C::BYTES + 1024 > 118 * 1024) ? C::BYTES + 1024 : 118 * 1024;
  KLC_CUDA(cudaFuncSetAttribute(mx3_expert_kernel<PHASE, C>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int64_t items = int64_t(max_rowblocks) * p.n_mtiles;  // an upper bound: the count is on the device
  if constexpr (C::PAIR) {
    // one persistent pair per two SMs, as many as can be resident at once
    static int max_pairs = -1;
    static std::once_flag once;
    std::call_once(once, [&] {
      cudaLaunchConfig_t cfg{};
      cudaLaunchAttribute attr{};
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = 2;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.gridDim = dim3(unsigned(2 * (sm_count() / 2)));
      cfg.blockDim = dim3(C::THREADS);
      cfg.dynamicSmemBytes = size_t(smem);
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, mx3_expert_kernel<PHASE, C>, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = sm_count() / 2;
      }
      max_pairs = n;
    });
    const int64_t pairs = items < max_pairs ? items : max_pairs;
    if (pairs <= 0) return KLC_OK;
    KLC_CUDA(launch_chain(mx3_expert_kernel<PHASE, C>, dim3(unsigned(2 * pairs)), dim3(C::THREADS), size_t(smem), stream, 2u,
                          mw, mx, p));
    KLC_LAUNCH_CHECK("tcgen05 expert launch (two-SM tiles)");
    return KLC_OK;
  }
  const int grid = int(items < sm_count() ? items : sm_count());
  if (grid <= 0) return KLC_OK;
  KLC_CUDA(launch_chain(mx3_expert_kernel<PHASE, C>, dim3(grid), dim3(C::THREADS), size_t(smem), stream, 0u, mw, mx, p));
  KLC_LAUNCH_CHECK("tcgen05 expert launch");
  return KLC_OK;
}

template <class C>
int launch_mx3_both(const ExpertArgs& a, const uint8_t* gu_k128, const uint8_t* dn_k128, cudaStream_t stream) {
  const klc_moe_weights& w = *a.wts;
  MxParams p1{};
  p1.n_out = int(2 * a.inter);
  p1.k_in = int(a.hidden);
  p1.rowblocks = C::PAIR ? a.pairblocks : a.rowblocks;
  p1.status = a.status_rw;
  p1.rows = a.rows;
  p1.sfa = w.gu_scales_t192;
  p1.sfb = a.sfb1;
  p1.bias = w.gu_bias;
  p1.out = static_cast<uint16_t*>(a.gated);
  p1.out_ld = int(a.inter);
  p1.normsq = a.normsq;
  p1.precision = a.precision;
  p1.limit = w.swiglu_limit;
  p1.alpha = w.alpha;
  // the gate_up epilogue writes the down operand (hi/lo E4M3 + scales) itself.
  // Measured on one B200 (same box, A/B): config 2 prefill 1.538 -> 1.464 ms,
  // config 3 4.45 -> 4.43 ms; with 16-row decode tiles 0.483 -> 0.490 ms (the
  // heavier epilogue is on the decode critical path), so those keep the pass
  const bool fuse_q = C::EPI == 2 && C::BN >= 64 && fused_quantize_enabled();
  if (fuse_q) {
    p1.qout = a.gq;
    p1.qsf = a.sfb2;
    p1.q_stages = int((a.inter + 127) / 128);
  }
  int st = launch_quantize_rows(a.x, a.hidden, a.rows, a.k, a.rowblocks, a.status, a.max_rowblocks, 1, a.xq, a.sfb1, stream);
  if (st != KLC_OK) return st;
  st = launch_mx3_phase<1, C>(gu_k128, a.xq, a.rows_cap, int(a.experts), p1, a.max_rowblocks, stream);
  if (st != KLC_OK) return st;
  stage_mark(kStageGateUp, stream);
  if (!fuse_q) {
    st = launch_quantize_rows(static_cast<const uint16_t*>(a.gated), a.inter, nullptr, 1, a.rowblocks, a.status,
                              a.max_rowblocks, 1, a.gq, a.sfb2, stream);
    if (st != KLC_OK) return st;
  }
  MxParams p2 = p1;
  p2.qout = nullptr;
  p2.qsf = nullptr;
  p2.n_out = int(a.hidden);
  p2.k_in = int(a.inter);
  p2.sfa = w.dn_scales_t192;
  p2.sfb = a.sfb2;
  p2.bias = w.dn_bias;
  p2.out = a.y;
  p2.out_ld = int(a.hidden);
  if (a.scatter != nullptr) p2.sc = *a.scatter;
  st = launch_mx3_phase<2, C>(dn_k128, a.gq, a.rows_cap, int(a.experts), p2, a.max_rowblocks, stream);
  stage_mark(kStageDown, stream);
  return st;
}

template <class C>
int launch_mx_both(const ExpertArgs& a, cudaStream_t stream) {
  const klc_moe_weights& w = *a.wts;
  KLC_CHECK_ARG(w.gu_scales_mx != nullptr && w.dn_scales_mx != nullptr,
                "tensor-core path: gu_scales_mx / dn_scales_mx are required (klc_mxfp4_scales_mx)");
  MxParams p1{};
  p1.n_out = int(2 * a.inter);
  p1.k_in = int(a.hidden);
  p1.n_mtiles = (p1.n_out + kBM - 1) / kBM;
  p1.rowblocks = a.rowblocks;
  p1.status = a.status_rw;
  p1.rows = a.rows;
  p1.sfa = w.gu_scales_mx;
  p1.sfb = a.sfb1;
  p1.bias = w.gu_bias;
  p1.out = static_cast<uint16_t*>(a.gated);
  p1.out_ld = int(a.inter);
  p1.normsq = a.normsq;
  p1.precision = a.precision;
  p1.limit = w.swiglu_limit;
  p1.alpha = w.alpha;
  int st = launch_quantize_rows(a.x, a.hidden, a.rows, a.k, a.rowblocks, a.status, a.max_rowblocks, C::NCH, a.xq,
                                a.sfb1, stream);
  if (st != KLC_OK) return st;
  st = launch_mx_phase<1, C>(w.gu_blocks, a.xq, a.rows_cap, int(a.experts), p1, a.max_rowblocks, stream);
  if (st != KLC_OK) return st;
  stage_mark(kStageGateUp, stream);
  st = launch_quantize_rows(static_cast<const uint16_t*>(a.gated), a.inter, nullptr, 1, a.rowblocks, a.status,
                            a.max_rowblocks, C::NCH, a.gq, a.sfb2, stream);
  if (st != KLC_OK) return st;
  MxParams p2 = p1;
  p2.n_out = int(a.hidden);
  p2.k_in = int(a.inter);
  p2.n_mtiles = (p2.n_out + kBM - 1) / kBM;
  p2.sfa = w.dn_scales_mx;
  p2.sfb = a.sfb2;
  p2.bias = w.dn_bias;
  p2.out = a.y;
  p2.out_ld = int(a.hidden);
  st = launch_mx_phase<2, C>(w.dn_blocks, a.gq, a.rows_cap, int(a.experts), p2, a.max_rowblocks, stream);
  stage_mark(kStageDown, stream);
  return st;
}

// Two tile shapes.  Measured on B200 with one MMA issuer (gate_up + down,
// GPT-OSS-120B layer, rows per expert on average): 4 rows 0.53 ms (16-row
// tiles) vs 0.57 (64-row), 8 rows 0.54 vs 0.58, 16 rows 0.78 vs 0.60, 24 rows
// 1.04 vs 0.63, so 16-row tiles up to about 12 rows per expert and 64-row tiles
// with a 4-deep activation ring above (32- and 128-row tiles were slower in an
// earlier generation: T = 4096 3.42 / 3.59 ms vs 2.95 for 64 rows).  A 2-deep
// activation ring exposes a copy latency per slot reuse.
// One MMA issuer: with several threads issuing tcgen05 operations at the
// same time, B200 produced occasional wrong tiles (nondeterministic, about
// one 128 x 16 tile in 10^4 at T = 4096; never with a single issuer or with
// the issuers forced into one global order), so every tcgen05 MMA, scale copy
// and commit of a CTA comes from one thread.
// 64-row tiles get a second epilogue warpgroup: with one, the epilogue of an
// item (64 tokens x 128 features) took longer than the item's MMAs.
//                BN  NA NS NB NP ND PF EPI
using MxN16  = MxCfg<16, 4, 6, 6, 1, 2, 8, 1>;
using MxN64  = MxCfg<64, 4, 4, 4, 1, 2, 0, 2>;
// Direct-operand kernels (weights padded to K % 128 == 0):
//                 BN  NS ND EPI  SK  PF SFW
#ifndef KLC_MX2_N16
#define KLC_MX2_N16 16, 4, 2, 1, 256, 8, 1
#endif
#ifndef KLC_MX2_N64
#define KLC_MX2_N64 64, 3, 2, 2, 256, 0, 1
#endif
using Mx2N16 = Mx2Cfg<KLC_MX2_N16>;
using Mx2N64 = Mx2Cfg<KLC_MX2_N64>;
// Swapped-operand kernels (weights as N = 192, scales in 192-row tiles):
//                 BN  NS ND  SK  PF EPI
// (measured on B200, gate_up + down ms: decode T=256 0.290 + 0.146, config 3
// T=16384 2.76 + 1.35; 128-K stages win for 64-row tiles, 256-K stages for 16-row)
#ifndef KLC_MX3_N16
#define KLC_MX3_N16 16, 3, 2, 256, 0, 2
#endif
#ifndef KLC_MX3_N64
#define KLC_MX3_N64 64, 4, 2, 128, 0, 2
#endif
// Two-SM tiles (64 tokens per CTA, half of each weight tile per CTA): the
// half-size weight boxes leave room for three 256-K stages (one-SM tiles fit
// only two), which halves the stage hops per item.  Measured on B200, config 3
// (T = 16384, 512 rows per expert), gate_up + down ms: one-SM 128-K x 4 3.05 +
// 1.50; pair 128-K x 6 3.18 + 1.56, 128-K x 7 3.15 + 1.56, 256-K x 3 2.86 + 1.36.
//                 BN  NS ND  SK  PF EPI PAIR
#ifndef KLC_MX3_P64
#define KLC_MX3_P64 64, 3, 2, 256, 0, 2, 1
#endif
using Mx3N16 = Mx3Cfg<KLC_MX3_N16>;
using Mx3N64 = Mx3Cfg<KLC_MX3_N64>;
using Mx3P64 = Mx3Cfg<KLC_MX3_P64>;

}  // namespace

namespace tc {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static int encode_fn(EncodeTiledFn* out) {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
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
  cuuint64_t gd[5], gs[4];
  cuuint32_t bx[5], es[5] = {1, 1, 1, 1, 1};
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

}  // namespace tc

bool tc_path_supported(int64_t hidden, int64_t inter) {
  int dev = 0, major = 0, minor = 0;
  if (hidden % 64 != 0 || inter % 64 != 0) return false;
  if (cudaGetDevice(&dev) != cudaSuccess) return true;  // no device: report the build's capability
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return true;
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  return major == 10 && minor == 0;
}

int mx_sfb_chunks(int block_n) { return (2 * block_n + 127) / 128; }

namespace {
// padded (K multiple of 128) weight blocks for the direct-operand kernels, or null
const uint8_t* gu_k128_of(const klc_moe_weights& w, int64_t hidden) {
  return w.gu_blocks_k128 != nullptr ? w.gu_blocks_k128 : (hidden % 128 == 0 ? w.gu_blocks : nullptr);
}
const uint8_t* dn_k128_of(const klc_moe_weights& w, int64_t inter) {
  return w.dn_blocks_k128 != nullptr ? w.dn_blocks_k128 : (inter % 128 == 0 ? w.dn_blocks : nullptr);
}
bool mx3_usable(const klc_moe_weights& w, int64_t hidden, int64_t inter) {
  const bool bias16 = ((reinterpret_cast<uintptr_t>(w.gu_bias) | reinterpret_cast<uintptr_t>(w.dn_bias)) & 15) == 0;
  return gu_k128_of(w, hidden) != nullptr && dn_k128_of(w, inter) != nullptr && w.gu_scales_t192 != nullptr &&
         w.dn_scales_t192 != nullptr && bias16;
}
}  // namespace

bool experts_tc_can_scatter(const klc_moe_weights& w, int64_t hidden, int64_t inter, int block_n) {
  return hidden % 64 == 0 && inter % 64 == 0 && (block_n == 16 || block_n == 64) && mx3_usable(w, hidden, inter);
}

int launch_experts_tc(const ExpertArgs& a, cudaStream_t stream) {
  KLC_CHECK_ARG(a.hidden % 64 == 0 && a.inter % 64 == 0, "tensor-core path: hidden and intermediate must be multiples of 64");
  KLC_CHECK_ARG(2 * a.rows_cap < (int64_t(1) << 31), "tensor-core path: too many rows");
  // direct-operand kernels when the weights are available with K padded to a multiple of 128
  const klc_moe_weights& w = *a.wts;
  const uint8_t* gu = gu_k128_of(w, a.hidden);
  const uint8_t* dn = dn_k128_of(w, a.inter);
  KLC_CHECK_ARG(a.scatter == nullptr || mx3_usable(w, a.hidden, a.inter),
                "tensor-core path: row scatter needs the weights-as-N kernels");
  if (mx3_usable(w, a.hidden, a.inter)) {
    switch (a.block_n) {
      case 16: return launch_mx3_both<Mx3N16>(a, gu, dn, stream);
      case 64:
        if (a.pairblocks != nullptr) return launch_mx3_both<Mx3P64>(a, gu, dn, stream);
        return launch_mx3_both<Mx3N64>(a, gu, dn, stream);
      default: return fail(KLC_ERR_INVALID, "tensor-core path: row-block size must be 16 or 64");
    }
  }
  if (gu != nullptr && dn != nullptr) {
    switch (a.block_n) {
      case 16: return launch_mx2_both<Mx2N16>(a, gu, dn, stream);
      case 64: return launch_mx2_both<Mx2N64>(a, gu, dn, stream);
      default: return fail(KLC_ERR_INVALID, "tensor-core path: row-block size must be 16 or 64");
    }
  }
  switch (a.block_n) {
    case 16: return launch_mx_both<MxN16>(a, stream);
    case 64: return launch_mx_both<MxN64>(a, stream);
    default: return fail(KLC_ERR_INVALID, "tensor-core path: row-block size must be 16 or 64");
  }
}

}  // namespace klc
