// Un-permute + weighted combine, the bias-only MoE path and RMSNorm.
//
// Combine restates streamed_moe_router.py:497,512-513 exactly:
//   output = zeros_like(hidden)                       (bf16)
//   for each selected expert, in top-k order:
//       output += out.to(bf16) * w                    (bf16 product, bf16 sum)
// so the result is bit-identical to the reference's for identical expert
// outputs.  One CTA per token; each thread owns 8 hidden elements and
// gathers them (16-byte loads) from the k permuted rows of the token.
// Memory-bound: k*H*2 bytes read + H*2 written per token.
//
// The fused form (kNorm) also applies the next layer's input RMSNorm to the
// residual sum, the executor's `hidden += moe_out` (streamed_transformer_
// executor.py:260) followed by `rms_norm(hidden, input_layernorm.weight)`
// (:235, streamed_attention.py:27-28): the token's sum of squares is taken
// from the bf16 values as they are stored, and each thread re-reads only the
// chunks it stored itself, so no second kernel re-reads the hidden state.
#include "permute.cuh"
#include "select.cuh"

namespace klc {

namespace {

constexpr int kMaxTopK = 8;

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float u = (lane < int(blockDim.x >> 5)) ? red[lane] : 0.f;
    u = warp_sum(u);
    if (lane == 0) red[0] = u;
  }
  __syncthreads();
  return red[0];
}

// 64 registers at most: four 256-thread CTAs (tokens) per SM keep enough row
// gathers in flight (the fused form needs 75 otherwise and ran 20 % slower).
template <bool kNorm>
__global__ void __launch_bounds__(256, 4) combine_kernel(const uint16_t* __restrict__ y, const int32_t* __restrict__ pair_pos,
                               const uint16_t* __restrict__ w, int k, int64_t hidden,
                               const uint16_t* __restrict__ residual, uint16_t* __restrict__ out,
                               const float* __restrict__ normsq, float* __restrict__ norms,
                               const uint16_t* __restrict__ norm_w, float eps, uint16_t* __restrict__ normed) {
  pdl_wait();     // inputs written by the previous kernel of the chain
  pdl_trigger();  // the next kernel may launch and set up meanwhile
  const int64_t t = blockIdx.x;
  float ss = 0.f;  // sum of squares of the stored row (kNorm)
  const int chunks = int(hidden / 8);
  if (norms != nullptr && threadIdx.x < 2 * k) {
    const int64_t q = t * k * 2 + threadIdx.x;
    norms[q] = sqrtf(normsq[q]);
  }
  int pos[kMaxTopK];
  float wsel[kMaxTopK];
#pragma unroll
  for (int s = 0; s < kMaxTopK; ++s) {
    pos[s] = s < k ? pair_pos[t * k + s] : -1;
    wsel[s] = s < k ? bf16_to_f32(w[t * k + s]) : 0.f;
  }
  for (int c = threadIdx.x; c < chunks; c += blockDim.x) {
    // all k rows in flight before the dependent bf16 chain
    uint4 v[kMaxTopK];
#pragma unroll
    for (int s = 0; s < kMaxTopK; ++s)
      v[s] = pos[s] >= 0 ? reinterpret_cast<const uint4*>(y + int64_t(pos[s]) * hidden)[c] : make_uint4(0, 0, 0, 0);
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
    for (int s = 0; s < kMaxTopK; ++s) {
      if (pos[s] < 0) continue;  // past k, or a pair dropped by the permute's index check (recorded in the status word)
      const float ws = wsel[s];
      const uint32_t vv[4] = {v[s].x, v[s].y, v[s].z, v[s].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float lo = __uint_as_float(vv[j] << 16), hi = __uint_as_float(vv[j] & 0xffff0000u);
        acc[2 * j] = round_bf16(acc[2 * j] + round_bf16(lo * ws));
        acc[2 * j + 1] = round_bf16(acc[2 * j + 1] + round_bf16(hi * ws));
      }
    }
    if (residual != nullptr) {
      const uint4 r = reinterpret_cast<const uint4*>(residual + t * hidden)[c];
      const uint32_t rr[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] = round_bf16(__uint_as_float(rr[j] << 16) + acc[2 * j]);
        acc[2 * j + 1] = round_bf16(__uint_as_float(rr[j] & 0xffff0000u) + acc[2 * j + 1]);
      }
    }
    uint4 o;
    o.x = uint32_t(f32_to_bf16(acc[0])) | (uint32_t(f32_to_bf16(acc[1])) << 16);
    o.y = uint32_t(f32_to_bf16(acc[2])) | (uint32_t(f32_to_bf16(acc[3])) << 16);
    o.z = uint32_t(f32_to_bf16(acc[4])) | (uint32_t(f32_to_bf16(acc[5])) << 16);
    o.w = uint32_t(f32_to_bf16(acc[6])) | (uint32_t(f32_to_bf16(acc[7])) << 16);
    reinterpret_cast<uint4*>(out + t * hidden)[c] = o;
    if (kNorm) {
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(acc[j], acc[j], ss);  // acc holds the stored bf16 values
    }
  }
  if (kNorm) {
    __shared__ float red[32];
    const float total = block_sum(ss, red);
    const float inv = round_bf16(1.0f / sqrtf(total / float(hidden) + eps));
    for (int c = threadIdx.x; c < chunks; c += blockDim.x) {
      const uint4 o = reinterpret_cast<const uint4*>(out + t * hidden)[c];  // this thread's own store
      const uint4 g = reinterpret_cast<const uint4*>(norm_w)[c];
      const uint32_t oo[4] = {o.x, o.y, o.z, o.w}, gg[4] = {g.x, g.y, g.z, g.w};
      uint32_t r[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float lo = round_bf16(__uint_as_float(oo[j] << 16) * inv) * __uint_as_float(gg[j] << 16);
        const float hi = round_bf16(__uint_as_float(oo[j] & 0xffff0000u) * inv) * __uint_as_float(gg[j] & 0xffff0000u);
        r[j] = uint32_t(f32_to_bf16(lo)) | (uint32_t(f32_to_bf16(hi)) << 16);
      }
      reinterpret_cast<uint4*>(normed + t * hidden)[c] = make_uint4(r[0], r[1], r[2], r[3]);
    }
  }
}

// execute_experts=False (streamed_moe_router.py:317-329):
//   contribution = sum(down_bias[experts].to(bf16) * weights[:, None], dim=0)
// products rounded to bf16, the k-term sum accumulated in fp32, rounded once.
__global__ void bias_only_kernel(const uint16_t* __restrict__ bias, int64_t hidden, int k,
                                 const int32_t* __restrict__ idx, const uint16_t* __restrict__ w,
                                 uint16_t* __restrict__ y) {
  const int64_t t = blockIdx.x;
  for (int64_t h = threadIdx.x; h < hidden; h += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < k; ++s) {
      const int e = idx[t * k + s];
      acc += round_bf16(bf16_to_f32(bias[int64_t(e) * hidden + h]) * bf16_to_f32(w[t * k + s]));
    }
    y[t * hidden + h] = f32_to_bf16(acc);
  }
}

// rms_norm (streamed_attention.py:27-28):
//   x * rsqrt(mean(x.float()^2) + eps).to(bf16) * weight   (bf16 products)
__global__ void rms_norm_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ wt, int64_t hidden,
                                float eps, uint16_t* __restrict__ y) {
  pdl_wait();     // inputs written by the previous kernel of the chain
  pdl_trigger();  // the next kernel may launch and set up meanwhile
  __shared__ float red[32];
  const int64_t r = blockIdx.x;
  const uint16_t* xr = x + r * hidden;
  float ss = 0.f;
  for (int64_t h = threadIdx.x; h < hidden; h += blockDim.x) {
    const float v = bf16_to_f32(xr[h]);
    ss = fmaf(v, v, ss);
  }
  const float mean = block_sum(ss, red) / float(hidden);
  const float inv = round_bf16(1.0f / sqrtf(mean + eps));
  for (int64_t h = threadIdx.x; h < hidden; h += blockDim.x) {
    const float v = round_bf16(bf16_to_f32(xr[h]) * inv);
    y[r * hidden + h] = f32_to_bf16(v * bf16_to_f32(wt[h]));
  }
}

}  // namespace

int launch_combine(const uint16_t* y, const int32_t* pair_pos, const uint16_t* w, int64_t tokens, int k,
                   int64_t hidden, const uint16_t* residual, uint16_t* out, const float* normsq, float* norms,
                   const PostNorm* post, cudaStream_t stream) {
  if (tokens == 0) return KLC_OK;
  KLC_CHECK_ARG(tokens <= 0x7fffffff, "combine: too many tokens");
  KLC_CHECK_ARG(k >= 1 && k <= kMaxTopK, "combine: need 1 <= k <= 8");
  int64_t threads = (hidden / 8 + 31) / 32 * 32;
  threads = threads < 64 ? 64 : (threads > 256 ? 256 : threads);
  if (post != nullptr) {
    KLC_CHECK_ARG(post->weight && post->normed, "combine: null RMSNorm weight or output");
    KLC_CHECK_ARG((reinterpret_cast<uintptr_t>(post->weight) & 15) == 0 && (reinterpret_cast<uintptr_t>(post->normed) & 15) == 0,
                  "combine: RMSNorm weight and output must be 16-byte aligned");
    if (post->router_w != nullptr) {
      // the next layer's router on the normalised rows, right behind the combine in the same
      // call (computing the logits inside the combine, one CTA per token streaming all E router
      // rows from L2, measured slower than the router kernels: 84 against 73 us per layer at
      // T = 1, 336 against 309 at T = 32, B200, GPT-OSS-120B layers)
      KLC_CHECK_ARG(post->router_b && post->out_idx && post->out_w, "combine: null next-layer router argument");
      KLC_CHECK_ARG(post->experts >= 1 && post->experts <= 1024 && post->k >= 1 && post->k <= kSelMaxK && post->k <= post->experts,
                    "combine: next-layer router needs 1 <= k <= min(8, experts), experts <= 1024");
      KLC_CUDA(launch_chain(combine_kernel<true>, dim3(unsigned(tokens)), dim3(threads), size_t(0), stream, 0u, y, pair_pos, w, k, hidden, residual, out, normsq,
                                                                      norms, post->weight, post->eps, post->normed));
      KLC_LAUNCH_CHECK("combine launch");
      return launch_router(post->normed, tokens, hidden, post->router_w, post->router_b, post->experts, post->k, nullptr,
                           post->out_idx, post->out_w, post->out_logits, stream);
    }
    KLC_CUDA(launch_chain(combine_kernel<true>, dim3(unsigned(tokens)), dim3(threads), size_t(0), stream, 0u, y, pair_pos, w, k, hidden, residual, out, normsq,
                                                                    norms, post->weight, post->eps, post->normed));
  } else {
    KLC_CUDA(launch_chain(combine_kernel<false>, dim3(unsigned(tokens)), dim3(threads), size_t(0), stream, 0u, y, pair_pos, w, k, hidden, residual, out, normsq,
                                                                     norms, nullptr, 0.f, nullptr));
  }
  KLC_LAUNCH_CHECK("combine launch");
  return KLC_OK;
}

}  // namespace klc

extern "C" int klc_moe_bias_only(const uint16_t* dn_bias, int64_t tokens, int64_t hidden, int k, const int32_t* idx,
                                 const uint16_t* w, uint16_t* y, void* stream) {
  using namespace klc;
  KLC_CHECK_ARG(tokens >= 0 && hidden > 0 && k >= 1, "klc_moe_bias_only: bad sizes");
  if (tokens == 0) return KLC_OK;
  KLC_CHECK_ARG(dn_bias && idx && w && y, "klc_moe_bias_only: null pointer");
  KLC_CHECK_ARG(tokens <= 0x7fffffff, "klc_moe_bias_only: too many tokens");
  bias_only_kernel<<<unsigned(tokens), 256, 0, as_stream(stream)>>>(dn_bias, hidden, k, idx, w, y);
  KLC_LAUNCH_CHECK("klc_moe_bias_only launch");
  return KLC_OK;
}

extern "C" int klc_rms_norm(const uint16_t* x, const uint16_t* w, int64_t rows, int64_t hidden, float eps,
                            uint16_t* y, void* stream) {
  using namespace klc;
  KLC_CHECK_ARG(rows >= 0 && hidden > 0, "klc_rms_norm: bad sizes");
  if (rows == 0) return KLC_OK;
  KLC_CHECK_ARG(x && w && y, "klc_rms_norm: null pointer");
  KLC_CHECK_ARG(rows <= 0x7fffffff, "klc_rms_norm: too many rows");
  KLC_CUDA(launch_chain(rms_norm_kernel, dim3(unsigned(rows)), dim3(256), size_t(0), as_stream(stream), 0u, x, w, hidden, eps, y));
  KLC_LAUNCH_CHECK("klc_rms_norm launch");
  return KLC_OK;
}

extern "C" int klc_moe_combine(const uint16_t* y_rows, const int32_t* pair_pos, const uint16_t* w, int64_t tokens,
                               int k, int64_t hidden, const uint16_t* residual, uint16_t* out, void* stream) {
  using namespace klc;
  KLC_CHECK_ARG(tokens >= 0 && k >= 1 && hidden > 0 && hidden % 8 == 0, "klc_moe_combine: bad sizes");
  if (tokens == 0) return KLC_OK;
  KLC_CHECK_ARG(y_rows && pair_pos && w && out, "klc_moe_combine: null pointer");
  return launch_combine(y_rows, pair_pos, w, tokens, k, hidden, residual, out, nullptr, nullptr, nullptr,
                        as_stream(stream));
}

extern "C" int klc_moe_combine_rmsnorm(const uint16_t* y_rows, const int32_t* pair_pos, const uint16_t* w,
                                       int64_t tokens, int k, int64_t hidden, const uint16_t* residual,
                                       const uint16_t* norm_w, float eps, uint16_t* out, uint16_t* normed,
                                       void* stream) {
  using namespace klc;
  KLC_CHECK_ARG(tokens >= 0 && k >= 1 && hidden > 0 && hidden % 8 == 0, "klc_moe_combine_rmsnorm: bad sizes");
  if (tokens == 0) return KLC_OK;
  KLC_CHECK_ARG(y_rows && pair_pos && w && out && norm_w && normed, "klc_moe_combine_rmsnorm: null pointer");
  const PostNorm post{norm_w, eps, normed};
  return launch_combine(y_rows, pair_pos, w, tokens, k, hidden, residual, out, nullptr, nullptr, &post,
                        as_stream(stream));
}

extern "C" int klc_moe_combine_rmsnorm_route(const uint16_t* y_rows, const int32_t* pair_pos, const uint16_t* w,
                                             int64_t tokens, int k, int64_t hidden, const uint16_t* residual,
                                             const uint16_t* norm_w, float eps, uint16_t* out, uint16_t* normed,
                                             const klc_next_router* next, void* stream) {
  using namespace klc;
  KLC_CHECK_ARG(tokens >= 0 && k >= 1 && hidden > 0 && hidden % 8 == 0, "klc_moe_combine_rmsnorm_route: bad sizes");
  KLC_CHECK_ARG(next != nullptr && next->experts >= 1 && next->experts <= 1024, "klc_moe_combine_rmsnorm_route: bad next router");
  if (tokens == 0) return KLC_OK;
  KLC_CHECK_ARG(y_rows && pair_pos && w && out && norm_w && normed, "klc_moe_combine_rmsnorm_route: null pointer");
  PostNorm post{norm_w, eps, normed};
  post.router_w = next->router_w;
  post.router_b = next->router_b;
  post.experts = int(next->experts);
  post.k = next->k;
  post.out_idx = next->out_idx;
  post.out_w = next->out_w;
  post.out_logits = next->out_logits;
  KLC_CHECK_ARG(post.router_w != nullptr, "klc_moe_combine_rmsnorm_route: null router weight");
  return launch_combine(y_rows, pair_pos, w, tokens, k, hidden, residual, out, nullptr, nullptr, &post, as_stream(stream));
}
