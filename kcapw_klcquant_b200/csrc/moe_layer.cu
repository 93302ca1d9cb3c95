// MoE layer orchestration behind the C ABI: workspace layout, permute ->
// expert GEMMs -> combine, and the router + experts entry point.
#include <algorithm>

#include "permute.cuh"

namespace klc {

// Stage timing: when enabled on a host thread, the layer entry points record
// a CUDA event on the caller's stream at each stage boundary; klc_stage_times
// returns the elapsed milliseconds between consecutive marks of the last call.
namespace {
struct StageTimer {
  bool enabled = false;
  cudaEvent_t ev[kStageCount] = {};
  bool marked[kStageCount] = {};
};
thread_local StageTimer g_timer;
}  // namespace

void stage_mark(int stage, cudaStream_t stream) {
  StageTimer& t = g_timer;
  if (!t.enabled || stage < 0 || stage >= kStageCount) return;
  if (t.ev[stage] == nullptr && cudaEventCreate(&t.ev[stage]) != cudaSuccess) return;
  if (cudaEventRecord(t.ev[stage], stream) == cudaSuccess) t.marked[stage] = true;
}

namespace {

constexpr int kPad = 16;  // rows of each expert group are padded to 16 (MMA N granularity)
// two-SM tiles by default from this many routed rows per expert on average
// (the row-block pairs of an expert then rarely have an empty half)
constexpr int64_t kPairMinRows = 192;

int pick_block_n(const klc_moe_dims& d, bool tc) {
  if (!tc) return 64;
  // tokens per expert on average; row-blocks hold up to block_n rows (one
  // weight pass each).  The tensor-core kernels have 16- and 64-row tiles;
  // 16-row tiles win up to about 12 rows per expert (experts_mx.cu has the
  // timings)
  const int64_t per_expert = (d.tokens * d.top_k + d.experts - 1) / std::max<int64_t>(d.experts, 1);
  return per_expert <= 12 ? 16 : 64;
}

}  // namespace

bool use_tc_path(const klc_moe_dims& d) {
  if (d.path == KLC_PATH_SIMT) return false;
  if (d.path == KLC_PATH_TC) return true;
  return tc_path_supported(d.hidden, d.intermediate);
}

WorkspaceLayout workspace_layout(const klc_moe_dims& d, bool need_routing_buffers) {
  WorkspaceLayout L{};
  const bool tc = use_tc_path(d);
  L.pad = kPad;
  L.block_n = pick_block_n(d, tc);
  L.pairs = d.tokens * d.top_k;
  L.rows_cap = L.pairs + d.experts * (kPad - 1);
  L.max_rowblocks = (L.pairs + L.block_n - 1) / L.block_n + d.experts;
  L.nchunks = (L.pairs + 1023) / 1024;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + std::max<size_t>(bytes, 1), 256);
    return o;
  };
  L.status = take(sizeof(DeviceStatus));
  L.counts = take(size_t(d.experts) * 4);
  L.offsets = take(size_t(d.experts + 1) * 4);
  L.chunk_hist = take(size_t(std::max<int64_t>(L.nchunks, 1)) * d.experts * 4);
  L.rows = take(size_t(L.rows_cap) * 4);
  L.pair_pos = take(size_t(L.pairs) * 4);
  L.rowblocks = take(size_t(L.max_rowblocks) * sizeof(int4));
  L.normsq = take(size_t(L.pairs) * 2 * 4);
  L.xp = take(size_t(L.rows_cap) * d.hidden * 2);  // SIMT: bf16 rows; TC: hi/lo E4M3 rows (same size)
  L.gated = take(size_t(L.rows_cap) * d.intermediate * (tc ? 2 : 4));
  L.y = take(size_t(L.rows_cap) * d.hidden * 2);
  if (tc) {
    const size_t nch = size_t(mx_sfb_chunks(L.block_n));
    L.gq = take(size_t(L.rows_cap) * 2 * d.intermediate);
    L.sfb1 = take(size_t(L.max_rowblocks) * size_t((d.hidden + 127) / 128) * nch * 512);
    L.sfb2 = take(size_t(L.max_rowblocks) * size_t((d.intermediate + 127) / 128) * nch * 512);
    if (L.block_n == 64) L.pairblocks = take(size_t(L.max_rowblocks) * sizeof(int4));
  }
  if (need_routing_buffers) {
    L.idx = take(size_t(L.pairs) * 4);
    L.w = take(size_t(L.pairs) * 2);
  }
  L.total = off;
  return L;
}

int validate_dims(const klc_moe_dims* d) {
  KLC_CHECK_ARG(d != nullptr, "null dims");
  KLC_CHECK_ARG(d->tokens >= 0, "tokens must be >= 0");
  KLC_CHECK_ARG(d->hidden > 0 && d->hidden % 64 == 0 && d->hidden <= 65536, "hidden must be a positive multiple of 64, at most 65536");
  KLC_CHECK_ARG(d->intermediate > 0 && d->intermediate % 64 == 0 && d->intermediate <= 65536,
                "intermediate must be a positive multiple of 64, at most 65536");
  KLC_CHECK_ARG(d->experts > 0 && d->experts <= 1024, "experts must be in [1, 1024]");
  KLC_CHECK_ARG(d->top_k >= 1 && d->top_k <= 8 && d->top_k <= d->experts, "top_k must be in [1, min(8, experts)]");
  KLC_CHECK_ARG(d->path >= KLC_PATH_AUTO && d->path <= KLC_PATH_TC, "unknown expert path");
  KLC_CHECK_ARG(d->tokens * d->top_k < (int64_t(1) << 31) - d->experts * kPad, "too many tokens");
  return KLC_OK;
}

int validate_weights(const klc_moe_weights* w) {
  KLC_CHECK_ARG(w != nullptr, "null weights");
  KLC_CHECK_ARG(w->gu_blocks && w->gu_scales_t && w->gu_bias && w->dn_blocks && w->dn_scales_t && w->dn_bias,
                "null expert weight pointer");
  KLC_CHECK_ARG((reinterpret_cast<uintptr_t>(w->gu_blocks) & 15) == 0 && (reinterpret_cast<uintptr_t>(w->dn_blocks) & 15) == 0,
                "expert blocks must be 16-byte aligned");
  return KLC_OK;
}

int run_expert_stage(const klc_moe_dims& d, const klc_moe_weights& wts, const uint16_t* x, const int32_t* idx, int precision,
                     float* normsq, bool empty_ok, char* ws, const WorkspaceLayout& L, cudaStream_t stream,
                     const RowScatter* scatter) {
  const bool tc = use_tc_path(d);
  KLC_CHECK_ARG(scatter == nullptr || (tc && experts_tc_can_scatter(wts, d.hidden, d.intermediate, L.block_n)),
                "expert stage: row scatter needs the weights-as-N tensor-core kernels");
  DeviceStatus* status = reinterpret_cast<DeviceStatus*>(ws + L.status);
  KLC_CUDA(cudaMemsetAsync(status, 0, sizeof(DeviceStatus), stream));
  PermuteArgs pa{};
  pa.idx = idx;
  pa.tokens = d.tokens;
  pa.k = d.top_k;
  pa.experts = d.experts;
  pa.pad = L.pad;
  pa.block_n = L.block_n;
  pa.counts = reinterpret_cast<int32_t*>(ws + L.counts);
  pa.offsets = reinterpret_cast<int32_t*>(ws + L.offsets);
  pa.rows = reinterpret_cast<int32_t*>(ws + L.rows);
  pa.pair_pos = reinterpret_cast<int32_t*>(ws + L.pair_pos);
  pa.chunk_hist = reinterpret_cast<int32_t*>(ws + L.chunk_hist);
  pa.rowblocks = reinterpret_cast<int4*>(ws + L.rowblocks);
  pa.status = status;
  pa.x = x;
  pa.hidden = d.hidden;
  pa.empty_ok = empty_ok;
  // SIMT gathers bf16 rows here; the tensor-core path quantizes straight from x per row-block
  pa.xp = tc ? nullptr : reinterpret_cast<uint16_t*>(ws + L.xp);
  // two-SM tiles: row-blocks paired by the permute (klc_set_pair_tiles)
  const int pair_mode = pair_tiles_mode();
  const int64_t rows_per_expert = d.tokens * d.top_k / std::max<int64_t>(d.experts, 1);
  if (tc && L.pairblocks != 0 && (pair_mode == 2 || (pair_mode == 1 && rows_per_expert >= kPairMinRows)))
    pa.pairblocks = reinterpret_cast<int4*>(ws + L.pairblocks);
  stage_mark(kStageRouted, stream);
  int st = launch_permute(pa, stream);
  if (st != KLC_OK) return st;
  stage_mark(kStagePermuted, stream);

  ExpertArgs ea{};
  ea.wts = &wts;
  ea.hidden = d.hidden;
  ea.inter = d.intermediate;
  ea.experts = d.experts;
  ea.k = d.top_k;
  ea.precision = precision;
  ea.rowblocks = pa.rowblocks;
  ea.pairblocks = pa.pairblocks;
  ea.max_rowblocks = int(L.max_rowblocks);
  ea.rows = pa.rows;
  ea.status = status;
  ea.status_rw = status;
  ea.xp = pa.xp;
  ea.x = x;
  if (tc) {
    ea.xq = reinterpret_cast<uint8_t*>(ws + L.xp);
    ea.gq = reinterpret_cast<uint8_t*>(ws + L.gq);
    ea.sfb1 = reinterpret_cast<uint8_t*>(ws + L.sfb1);
    ea.sfb2 = reinterpret_cast<uint8_t*>(ws + L.sfb2);
  }
  ea.gated = ws + L.gated;
  ea.y = reinterpret_cast<uint16_t*>(ws + L.y);
  ea.normsq = normsq;
  ea.rows_cap = L.rows_cap;
  ea.block_n = L.block_n;
  ea.scatter = scatter;
  return tc ? launch_experts_tc(ea, stream) : launch_experts_simt(ea, stream);
}

// Permute, expert GEMMs and combine for given routing; `post` (or null) fuses
// the next layer's input RMSNorm into the combine.
static int run_experts_post(const klc_moe_dims& d, const klc_moe_weights& wts, const uint16_t* x, const int32_t* idx,
                            const uint16_t* w, int precision, uint16_t* y, float* norms, const uint16_t* residual,
                            const PostNorm* post, char* ws, const WorkspaceLayout& L, cudaStream_t stream) {
  float* normsq = nullptr;
  if (norms != nullptr) {
    normsq = reinterpret_cast<float*>(ws + L.normsq);
    KLC_CUDA(cudaMemsetAsync(normsq, 0, size_t(L.pairs) * 2 * 4, stream));
  }
  int st = run_expert_stage(d, wts, x, idx, precision, normsq, false, ws, L, stream);
  if (st != KLC_OK) return st;
  st = launch_combine(reinterpret_cast<const uint16_t*>(ws + L.y), reinterpret_cast<const int32_t*>(ws + L.pair_pos), w,
                      d.tokens, d.top_k, d.hidden, residual, y, normsq, norms, post, stream);
  stage_mark(kStageCombined, stream);
  return st;
}

int run_experts(const klc_moe_dims& d, const klc_moe_weights& wts, const uint16_t* x, const int32_t* idx,
                const uint16_t* w, int precision, uint16_t* y, float* norms, const uint16_t* residual, char* ws,
                const WorkspaceLayout& L, cudaStream_t stream) {
  return run_experts_post(d, wts, x, idx, w, precision, y, norms, residual, nullptr, ws, L, stream);
}

// klc_moe_experts, with the optional fused RMSNorm of klc_moe_forward_rmsnorm.
static int experts_entry(const klc_moe_dims* dims, const klc_moe_weights* wts, const uint16_t* x, const int32_t* idx,
                         const uint16_t* w, int precision, uint16_t* y, float* norms, const uint16_t* residual,
                         const PostNorm* post, void* workspace, size_t workspace_bytes, void* stream) {
  int st = validate_dims(dims);
  if (st != KLC_OK) return st;
  st = validate_weights(wts);
  if (st != KLC_OK) return st;
  KLC_CHECK_ARG(precision == KLC_PREC_FP32 || precision == KLC_PREC_BF16, "precision must be KLC_PREC_FP32 or KLC_PREC_BF16");
  if (dims->tokens == 0) return KLC_OK;
  KLC_CHECK_ARG(x && idx && w && y, "klc_moe_experts: null pointer");
  const WorkspaceLayout L = workspace_layout(*dims, false);
  if (workspace == nullptr || workspace_bytes < L.total)
    return fail(KLC_ERR_WORKSPACE, "klc_moe_experts: workspace too small (need " + std::to_string(L.total) + " bytes)");
  KLC_CHECK_ARG((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, "workspace must be 256-byte aligned");
  return run_experts_post(*dims, *wts, x, idx, w, precision, y, norms, residual, post, static_cast<char*>(workspace), L,
                          as_stream(stream));
}

// klc_moe_forward: router, then experts_entry on its routing.
static int forward_entry(const klc_moe_dims* dims, const klc_moe_weights* wts, const uint16_t* x, const float* adjust,
                         int precision, uint16_t* y, int32_t* out_idx, uint16_t* out_w, uint16_t* out_logits,
                         float* norms, const uint16_t* residual, const PostNorm* post, void* workspace,
                         size_t workspace_bytes, void* stream) {
  int st = validate_dims(dims);
  if (st != KLC_OK) return st;
  st = validate_weights(wts);
  if (st != KLC_OK) return st;
  KLC_CHECK_ARG(wts->router_w && wts->router_b, "klc_moe_forward: null router weights");
  KLC_CHECK_ARG(out_idx && out_w, "klc_moe_forward: null routing outputs");
  if (dims->tokens == 0) return KLC_OK;
  stage_mark(kStageStart, as_stream(stream));
  st = launch_router(x, dims->tokens, dims->hidden, wts->router_w, wts->router_b, dims->experts, dims->top_k, adjust,
                     out_idx, out_w, out_logits, as_stream(stream));
  if (st != KLC_OK) return st;
  return experts_entry(dims, wts, x, out_idx, out_w, precision, y, norms, residual, post, workspace, workspace_bytes,
                       stream);
}

}  // namespace klc

using namespace klc;

extern "C" int klc_moe_workspace_size(const klc_moe_dims* dims, size_t* out_bytes) {
  int st = validate_dims(dims);
  if (st != KLC_OK) return st;
  KLC_CHECK_ARG(out_bytes != nullptr, "klc_moe_workspace_size: null output");
  *out_bytes = workspace_layout(*dims, false).total;
  return KLC_OK;
}

extern "C" int klc_moe_experts(const klc_moe_dims* dims, const klc_moe_weights* wts, const uint16_t* x,
                               const int32_t* idx, const uint16_t* w, int precision, uint16_t* y, float* norms,
                               const uint16_t* residual, void* workspace, size_t workspace_bytes, void* stream) {
  return experts_entry(dims, wts, x, idx, w, precision, y, norms, residual, nullptr, workspace, workspace_bytes, stream);
}

extern "C" int klc_moe_forward(const klc_moe_dims* dims, const klc_moe_weights* wts, const uint16_t* x,
                               const float* adjust, int precision, uint16_t* y, int32_t* out_idx, uint16_t* out_w,
                               uint16_t* out_logits, float* norms, const uint16_t* residual, void* workspace,
                               size_t workspace_bytes, void* stream) {
  return forward_entry(dims, wts, x, adjust, precision, y, out_idx, out_w, out_logits, norms, residual, nullptr,
                       workspace, workspace_bytes, stream);
}

extern "C" int klc_moe_forward_rmsnorm(const klc_moe_dims* dims, const klc_moe_weights* wts, const uint16_t* x,
                                       const float* adjust, int precision, uint16_t* y, int32_t* out_idx,
                                       uint16_t* out_w, uint16_t* out_logits, float* norms, const uint16_t* residual,
                                       const uint16_t* norm_w, float eps, uint16_t* normed, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  KLC_CHECK_ARG(norm_w && normed, "klc_moe_forward_rmsnorm: null RMSNorm weight or output");
  const PostNorm post{norm_w, eps, normed};
  return forward_entry(dims, wts, x, adjust, precision, y, out_idx, out_w, out_logits, norms, residual, &post,
                       workspace, workspace_bytes, stream);
}

namespace {
PostNorm post_with_router(const uint16_t* norm_w, float eps, uint16_t* normed, const klc_next_router* next) {
  PostNorm post{norm_w, eps, normed};
  if (next != nullptr) {
    post.router_w = next->router_w;
    post.router_b = next->router_b;
    post.experts = int(next->experts);
    post.k = next->k;
    post.out_idx = next->out_idx;
    post.out_w = next->out_w;
    post.out_logits = next->out_logits;
  }
  return post;
}
}  // namespace

extern "C" int klc_moe_forward_rmsnorm_route(const klc_moe_dims* dims, const klc_moe_weights* wts, const uint16_t* x,
                                             const float* adjust, int precision, uint16_t* y, int32_t* out_idx,
                                             uint16_t* out_w, uint16_t* out_logits, float* norms, const uint16_t* residual,
                                             const uint16_t* norm_w, float eps, uint16_t* normed,
                                             const klc_next_router* next, void* workspace, size_t workspace_bytes,
                                             void* stream) {
  KLC_CHECK_ARG(norm_w && normed && next && next->router_w, "klc_moe_forward_rmsnorm_route: null argument");
  KLC_CHECK_ARG(next->experts >= 1 && next->experts <= 1024, "klc_moe_forward_rmsnorm_route: next experts out of range");
  const PostNorm post = post_with_router(norm_w, eps, normed, next);
  return forward_entry(dims, wts, x, adjust, precision, y, out_idx, out_w, out_logits, norms, residual, &post,
                       workspace, workspace_bytes, stream);
}

extern "C" int klc_moe_experts_rmsnorm_route(const klc_moe_dims* dims, const klc_moe_weights* wts, const uint16_t* x,
                                             const int32_t* idx, const uint16_t* w, int precision, uint16_t* y,
                                             float* norms, const uint16_t* residual, const uint16_t* norm_w, float eps,
                                             uint16_t* normed, const klc_next_router* next, void* workspace,
                                             size_t workspace_bytes, void* stream) {
  KLC_CHECK_ARG(norm_w && normed && next && next->router_w, "klc_moe_experts_rmsnorm_route: null argument");
  KLC_CHECK_ARG(next->experts >= 1 && next->experts <= 1024, "klc_moe_experts_rmsnorm_route: next experts out of range");
  const PostNorm post = post_with_router(norm_w, eps, normed, next);
  return experts_entry(dims, wts, x, idx, w, precision, y, norms, residual, &post, workspace, workspace_bytes, stream);
}

extern "C" int klc_moe_permute(const int32_t* idx, int64_t tokens, int k, int64_t experts, int pad, int32_t* pair_pos,
                               int32_t* counts, int32_t* offsets, int32_t* rows, int64_t rows_cap, void* workspace,
                               size_t workspace_bytes, void* stream) {
  KLC_CHECK_ARG(tokens >= 0 && k >= 1 && experts >= 1 && experts <= 1024 && pad >= 1, "klc_moe_permute: bad sizes");
  if (tokens == 0) return KLC_OK;
  KLC_CHECK_ARG(idx && pair_pos && counts && offsets && rows, "klc_moe_permute: null pointer");
  const int64_t pairs = tokens * k;
  KLC_CHECK_ARG(rows_cap >= pairs + experts * (pad - 1), "klc_moe_permute: rows_cap too small");
  klc_moe_dims d{tokens, 64, 64, experts, k, KLC_PATH_SIMT};
  const WorkspaceLayout L = workspace_layout(d, false);
  if (workspace == nullptr || workspace_bytes < L.total)
    return fail(KLC_ERR_WORKSPACE, "klc_moe_permute: workspace too small (need " + std::to_string(L.total) + " bytes)");
  char* ws = static_cast<char*>(workspace);
  DeviceStatus* status = reinterpret_cast<DeviceStatus*>(ws + L.status);
  KLC_CUDA(cudaMemsetAsync(status, 0, sizeof(DeviceStatus), as_stream(stream)));
  PermuteArgs pa{};
  pa.idx = idx;
  pa.tokens = tokens;
  pa.k = k;
  pa.experts = experts;
  pa.pad = pad;
  pa.block_n = 1 << 24;
  pa.counts = counts;
  pa.offsets = offsets;
  pa.rows = rows;
  pa.pair_pos = pair_pos;
  pa.chunk_hist = reinterpret_cast<int32_t*>(ws + L.chunk_hist);
  pa.rowblocks = reinterpret_cast<int4*>(ws + L.rowblocks);
  pa.status = status;
  return launch_permute(pa, as_stream(stream));
}

extern "C" int klc_workspace_status(const void* workspace, int* code, int* where, int* detail, void* stream) {
  KLC_CHECK_ARG(workspace != nullptr, "klc_workspace_status: null workspace");
  DeviceStatus h{};
  KLC_CUDA(cudaMemcpyAsync(&h, workspace, sizeof(h), cudaMemcpyDeviceToHost, as_stream(stream)));
  KLC_CUDA(cudaStreamSynchronize(as_stream(stream)));
  if (code) *code = h.code;
  if (where) *where = h.where;
  if (detail) *detail = h.detail;
  return h.code == 0 ? KLC_OK : fail(h.code, "device-side check failed at site " + std::to_string(h.where) +
                                                 " (detail " + std::to_string(h.detail) + ")");
}

extern "C" int klc_stage_timing(int enable) {
  for (int i = 0; i < kStageCount; ++i) g_timer.marked[i] = false;
  g_timer.enabled = enable != 0;
  return KLC_OK;
}

extern "C" int klc_stage_times(float* ms, int max_stages, int* n_out) {
  KLC_CHECK_ARG(ms != nullptr && max_stages >= kStageCount - 1, "klc_stage_times: need room for 5 stages");
  StageTimer& t = g_timer;
  int n = 0;
  for (int i = 1; i < kStageCount; ++i) {
    ms[i - 1] = -1.0f;
    if (t.marked[i] && t.marked[i - 1]) {
      KLC_CUDA(cudaEventSynchronize(t.ev[i]));
      float v = 0.f;
      KLC_CUDA(cudaEventElapsedTime(&v, t.ev[i - 1], t.ev[i]));
      ms[i - 1] = v;
      ++n;
    }
  }
  for (int i = 0; i < kStageCount; ++i) t.marked[i] = false;
  if (n_out) *n_out = n;
  return KLC_OK;
}

extern "C" int klc_ep_pack(const int32_t* idx, int64_t tokens, int k, int64_t experts_per_rank, int nranks,
                           const uint16_t* x, int64_t hidden, uint16_t* send_rows, int32_t* send_expert,
                           int32_t* send_counts, int32_t* pair_pos, void* workspace, size_t workspace_bytes,
                           void* stream) {
  KLC_CHECK_ARG(tokens >= 0 && k >= 1 && experts_per_rank >= 1 && nranks >= 1 && nranks <= 1024 && hidden > 0 &&
                    hidden % 8 == 0,
                "klc_ep_pack: bad sizes");
  if (tokens == 0) {
    if (send_counts) KLC_CUDA(cudaMemsetAsync(send_counts, 0, size_t(nranks) * 4, as_stream(stream)));
    return KLC_OK;
  }
  KLC_CHECK_ARG(idx && x && send_rows && send_expert && send_counts && pair_pos, "klc_ep_pack: null pointer");
  klc_moe_dims d{tokens, 64, 64, nranks, k, KLC_PATH_SIMT};
  const WorkspaceLayout L = workspace_layout(d, false);
  if (workspace == nullptr || workspace_bytes < L.total)
    return fail(KLC_ERR_WORKSPACE, "klc_ep_pack: workspace too small (need " + std::to_string(L.total) + " bytes)");
  char* ws = static_cast<char*>(workspace);
  DeviceStatus* status = reinterpret_cast<DeviceStatus*>(ws + L.status);
  KLC_CUDA(cudaMemsetAsync(status, 0, sizeof(DeviceStatus), as_stream(stream)));
  PermuteArgs pa{};
  pa.idx = idx;
  pa.tokens = tokens;
  pa.k = k;
  pa.experts = nranks;
  pa.pad = 1;
  pa.block_n = 1 << 24;
  pa.counts = send_counts;
  pa.offsets = reinterpret_cast<int32_t*>(ws + L.offsets);
  pa.rows = reinterpret_cast<int32_t*>(ws + L.rows);
  pa.pair_pos = pair_pos;
  pa.chunk_hist = reinterpret_cast<int32_t*>(ws + L.chunk_hist);
  pa.rowblocks = reinterpret_cast<int4*>(ws + L.rowblocks);
  pa.status = status;
  pa.x = x;
  pa.hidden = hidden;
  pa.xp = send_rows;
  pa.div = int(experts_per_rank);
  pa.aux_out = send_expert;
  return launch_permute(pa, as_stream(stream));
}
