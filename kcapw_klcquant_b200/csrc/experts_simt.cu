// CUDA-core expert kernels: MXFP4 dequant in registers + fp32 FMA.
//
// The reference's per-expert math (streamed_moe_router.py:500-511, 524-529):
//   gu    = x @ Wgu + b_gu          (fp32; 'bf16' precision rounds x@Wgu to bf16 first)
//   gated = (clamp(up,-L,L) + 1) * g * sigmoid(alpha g),  g = min(gate, L)
//   out   = gated @ Wd + b_d        (fp32; 'bf16' rounds gated and the product to bf16)
//
// Mapping: one thread per output feature (weight row), a CTA covers 128 rows
// of one row-block (<= kTok tokens of one expert at a time).  Each thread
// streams its row's packed nibbles (16 B per 32-value group) and the group's
// E8M0 scale, builds exact fp32 weights, and FMAs them against the row-block's
// activations, which every thread of the warp reads from shared memory as a
// broadcast.  Exact in fp32 up to the summation order, which makes this path
// the closest restatement of the reference's 'fp32' precision; it serves the
// smallest token counts and is the cross-check of the tensor-core path.
#include "permute.cuh"

namespace klc {

namespace {

constexpr int kRows = 128;  // output rows per CTA (one per thread)
constexpr int kTok = 8;     // tokens per pass

struct SimtParams {
  const uint8_t* blocks;    // [E, N, G, 16]
  const uint8_t* scales_t;  // [E, G, N]
  const uint16_t* bias;     // [E, N]
  int64_t n_out, k_in;      // N rows, K = G*32
  const int4* rowblocks;
  const DeviceStatus* status;
  const int32_t* rows;
  const void* in;           // phase 1: bf16 [rows_cap, K];  phase 2: fp32 [rows_cap, K]
  void* out;                // phase 1: fp32 [rows_cap, N/2]; phase 2: bf16 [rows_cap, N]
  float* normsq;            // [pairs, 2] or null
  int precision;
  float limit, alpha;
};

template <int PHASE>
__global__ void __launch_bounds__(kRows) simt_expert_kernel(SimtParams p) {
  pdl_wait();     // inputs written by the previous kernel of the chain
  pdl_trigger();  // the next kernel may launch and set up meanwhile
  extern __shared__ __align__(16) float xs[];  // [kTok][K]
  const int rb_index = blockIdx.y;
  if (rb_index >= p.status->rowblocks) return;
  const int4 rb = p.rowblocks[rb_index];
  const int e = rb.x, r0 = rb.y, nrows = rb.z;
  const int64_t K = p.k_in, N = p.n_out, G = K / 32;
  const int64_t m = int64_t(blockIdx.x) * kRows + threadIdx.x;
  const bool row_ok = m < N;
  const int lane = threadIdx.x & 31;

  const uint8_t* wrow = p.blocks + (int64_t(e) * N + (row_ok ? m : 0)) * G * 16;
  const uint8_t* srow = p.scales_t + int64_t(e) * G * N + (row_ok ? m : 0);
  const float bias = row_ok ? bf16_to_f32(p.bias[int64_t(e) * N + m]) : 0.f;

  for (int t0 = 0; t0 < nrows; t0 += kTok) {
    const int nt = min(kTok, nrows - t0);
    __syncthreads();
    // stage activations as fp32
    for (int64_t i = threadIdx.x; i < int64_t(kTok) * K; i += blockDim.x) {
      const int t = int(i / K);
      const int64_t kk = i - int64_t(t) * K;
      float v = 0.f;
      if (t < nt) {
        const int64_t r = int64_t(r0 + t0 + t);
        if (PHASE == 1) {
          v = bf16_to_f32(static_cast<const uint16_t*>(p.in)[r * K + kk]);
        } else {
          v = static_cast<const float*>(p.in)[r * K + kk];
          if (p.precision == KLC_PREC_BF16) v = round_bf16(v);  // gated.to(bf16) @ down (:508)
        }
      }
      xs[i] = v;
    }
    __syncthreads();
    float acc[kTok];
#pragma unroll
    for (int t = 0; t < kTok; ++t) acc[t] = 0.f;
    if (row_ok) {
      for (int64_t g = 0; g < G; ++g) {
        const uint4 nb = ldg_nc_v4(wrow + g * 16);
        const uint32_t s = srow[g * N];
        const uint32_t words[4] = {nb.x, nb.y, nb.z, nb.w};
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
          float wv[8];
#pragma unroll
          for (int n = 0; n < 8; ++n) wv[n] = e8m0_scale(fp4_to_f32((words[wi] >> (4 * n)) & 0xFu), s);
          const int64_t kb = g * 32 + wi * 8;
#pragma unroll
          for (int t = 0; t < kTok; ++t) {
            if (t < nt) {
              const float4 xa = *reinterpret_cast<const float4*>(xs + t * K + kb);
              const float4 xb = *reinterpret_cast<const float4*>(xs + t * K + kb + 4);
              float a = acc[t];
              a = fmaf(wv[0], xa.x, a);
              a = fmaf(wv[1], xa.y, a);
              a = fmaf(wv[2], xa.z, a);
              a = fmaf(wv[3], xa.w, a);
              a = fmaf(wv[4], xb.x, a);
              a = fmaf(wv[5], xb.y, a);
              a = fmaf(wv[6], xb.z, a);
              a = fmaf(wv[7], xb.w, a);
              acc[t] = a;
            }
          }
        }
      }
    }
    // epilogue
#pragma unroll
    for (int t = 0; t < kTok; ++t) {
      float v = acc[t];
      if (p.precision == KLC_PREC_BF16) v = round_bf16(v);
      v += bias;
      const int64_t r = int64_t(r0 + t0 + t);
      const bool tok_ok = t < nt;
      if (PHASE == 1) {
        const float partner = __shfl_xor_sync(0xffffffffu, v, 1);
        float gsq = 0.f;
        if ((lane & 1) == 0 && row_ok && tok_ok) {
          const float gate = fminf(v, p.limit);
          const float up = fminf(fmaxf(partner, -p.limit), p.limit);
          const float glu = gate * (1.0f / (1.0f + expf(-(gate * p.alpha))));
          const float gated = (up + 1.0f) * glu;
          static_cast<float*>(p.out)[r * (N / 2) + m / 2] = gated;
          gsq = gated * gated;
        }
        if (p.normsq != nullptr) {
          gsq = warp_sum(gsq);
          if (lane == 0 && tok_ok) atomicAdd(&p.normsq[int64_t(p.rows[r]) * 2 + 0], gsq);
        }
      } else {
        float osq = 0.f;
        if (row_ok && tok_ok) {
          static_cast<uint16_t*>(p.out)[r * N + m] = f32_to_bf16(v);
          osq = v * v;
        }
        if (p.normsq != nullptr) {
          osq = warp_sum(osq);
          if (lane == 0 && tok_ok) atomicAdd(&p.normsq[int64_t(p.rows[r]) * 2 + 1], osq);
        }
      }
    }
  }
}

template <int PHASE>
int launch_phase(const SimtParams& p, int max_rowblocks, cudaStream_t stream) {
  const size_t smem = size_t(kTok) * p.k_in * sizeof(float);
  KLC_CHECK_ARG(smem <= 200 * 1024, "SIMT expert path: reduction size too large for shared memory");
  KLC_CUDA(cudaFuncSetAttribute(simt_expert_kernel<PHASE>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  dim3 grid(unsigned((p.n_out + kRows - 1) / kRows), unsigned(max_rowblocks));
  KLC_CHECK_ARG(max_rowblocks <= 65535, "SIMT expert path: too many row-blocks");
  KLC_CUDA(launch_chain(simt_expert_kernel<PHASE>, dim3(grid), dim3(kRows), size_t(smem), stream, 0u, p));
  KLC_LAUNCH_CHECK("SIMT expert launch");
  return KLC_OK;
}

}  // namespace

int launch_experts_simt(const ExpertArgs& a, cudaStream_t stream) {
  const klc_moe_weights& w = *a.wts;
  SimtParams p1{};
  p1.blocks = w.gu_blocks;
  p1.scales_t = w.gu_scales_t;
  p1.bias = w.gu_bias;
  p1.n_out = 2 * a.inter;
  p1.k_in = a.hidden;
  p1.rowblocks = a.rowblocks;
  p1.status = a.status;
  p1.rows = a.rows;
  p1.in = a.xp;
  p1.out = a.gated;
  p1.normsq = a.normsq;
  p1.precision = a.precision;
  p1.limit = w.swiglu_limit;
  p1.alpha = w.alpha;
  int st = launch_phase<1>(p1, a.max_rowblocks, stream);
  if (st != KLC_OK) return st;
  stage_mark(kStageGateUp, stream);
  SimtParams p2 = p1;
  p2.blocks = w.dn_blocks;
  p2.scales_t = w.dn_scales_t;
  p2.bias = w.dn_bias;
  p2.n_out = a.hidden;
  p2.k_in = a.inter;
  p2.in = a.gated;
  p2.out = a.y;
  st = launch_phase<2>(p2, a.max_rowblocks, stream);
  stage_mark(kStageDown, stream);
  return st;
}

}  // namespace klc
