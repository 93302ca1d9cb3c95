// Locality-aware routing on the device: the per-token steps that
// StreamedMoERouter.route runs on the host when RoutingLocalityConfig.enabled
// (streamed_moe_router.py:270-302): raw top-k, the locality bias
// (_apply_locality_bias :331-363: sticky bonus, hot-expert mask, cache-aware
// bonus), the adjusted top-k, the semantic guard (_guarded_expert_selection
// :365-394), the softmax of the selected scores, the prediction of the next
// experts (predict_experts :426-440, taken before the state update as route()
// does) and the state updates (_update_sticky_scores / _update_workload_scores
// :396-424).  The sticky and workload scores and the recent-expert history live
// in a caller-owned device buffer, so consecutive calls (tokens, or batches of
// tokens processed in order) continue one policy state without a host hop.
//
// Exactness.  The reference does this with torch tensors and Python dicts, so
// every tie and rounding follows from those:
//   * torch.topk on a CPU fp32 tensor is libstdc++'s std::nth_element followed
//     by std::sort of the first k-1 elements (or std::partial_sort when
//     k * 64 <= n), with the comparator "x NaN and y not, or x > y" on
//     (value, index) pairs; topk_cpu below restates those algorithms step by
//     step (introselect with median-of-three pivots, heap select, insertion
//     sort), which gives the same order among equal values;
//   * bonuses, margins and thresholds are fp32 tensor arithmetic (a Python
//     float operand is rounded to fp32 first); the scores themselves are
//     Python floats (fp64), decayed and summed in fp64;
//   * dict iteration order (insertion order; a deleted key re-enters at the
//     end) decides ties in the stable sorts of the hot-expert set, of the
//     sticky trim and of Counter.most_common: every entry carries the stamp of
//     its insertion.
// One warp runs the call; lane 0 walks the tokens in order.  It is a latency
// kernel (tens of microseconds per token) meant for decode batches.
#include <cmath>

#include "klc_common.cuh"
#include "klc_moe.h"

namespace klc {
namespace {

constexpr int kLocMaxK = 8;

struct LocHeader {
  long long sticky_clock, workload_clock;
  int hist_len, hist_head, window, experts;
  long long pad[4];
};
static_assert(sizeof(LocHeader) == 64, "state header");

struct LocState {
  LocHeader* h;
  double* sticky;         // [E]
  double* workload;       // [E]
  long long* sticky_at;   // [E] insertion stamp, 0 = absent
  long long* workload_at; // [E]
  int* hist;              // [window] ring, oldest at hist_head
};

__host__ __device__ inline size_t loc_state_bytes(int64_t E, int window) {
  return sizeof(LocHeader) + size_t(E) * (8 + 8 + 8 + 8) + size_t(window) * 4;
}

__device__ LocState loc_view(char* base, int E, int window) {
  LocState s;
  s.h = reinterpret_cast<LocHeader*>(base);
  char* p = base + sizeof(LocHeader);
  s.sticky = reinterpret_cast<double*>(p);
  p += size_t(E) * 8;
  s.workload = reinterpret_cast<double*>(p);
  p += size_t(E) * 8;
  s.sticky_at = reinterpret_cast<long long*>(p);
  p += size_t(E) * 8;
  s.workload_at = reinterpret_cast<long long*>(p);
  p += size_t(E) * 8;
  s.hist = reinterpret_cast<int*>(p);
  return s;
}

// ---------------------------------------------------------------------------
// torch.topk (CPU, largest, sorted) restated: libstdc++ algorithms on
// (value, index) pairs with comp(x, y) = (isnan(x) && !isnan(y)) || x > y
// ---------------------------------------------------------------------------
struct VI {
  float v;
  int i;
};

__device__ __forceinline__ bool tk_comp(const VI& x, const VI& y) {
  const bool xn = x.v != x.v, yn = y.v != y.v;
  return (xn && !yn) || (x.v > y.v);
}

__device__ void tk_insertion_sort(VI* a, int first, int last) {
  if (first == last) return;
  for (int i = first + 1; i < last; ++i) {
    const VI val = a[i];
    if (tk_comp(val, a[first])) {
      for (int j = i; j > first; --j) a[j] = a[j - 1];
      a[first] = val;
    } else {
      int j = i;
      while (tk_comp(val, a[j - 1])) {
        a[j] = a[j - 1];
        --j;
      }
      a[j] = val;
    }
  }
}

__device__ __forceinline__ void tk_swap(VI* a, int x, int y) {
  const VI t = a[x];
  a[x] = a[y];
  a[y] = t;
}

__device__ void tk_move_median_to_first(VI* a, int result, int x, int y, int z) {
  if (tk_comp(a[x], a[y])) {
    if (tk_comp(a[y], a[z])) tk_swap(a, result, y);
    else if (tk_comp(a[x], a[z])) tk_swap(a, result, z);
    else tk_swap(a, result, x);
  } else if (tk_comp(a[x], a[z])) {
    tk_swap(a, result, x);
  } else if (tk_comp(a[y], a[z])) {
    tk_swap(a, result, z);
  } else {
    tk_swap(a, result, y);
  }
}

__device__ int tk_unguarded_partition(VI* a, int first, int last, int pivot) {
  while (true) {
    while (tk_comp(a[first], a[pivot])) ++first;
    --last;
    while (tk_comp(a[pivot], a[last])) --last;
    if (!(first < last)) return first;
    tk_swap(a, first, last);
    ++first;
  }
}

__device__ void tk_adjust_heap(VI* a, int first, int hole, int len, VI value) {
  const int top = hole;
  int second = hole;
  while (second < (len - 1) / 2) {
    second = 2 * (second + 1);
    if (tk_comp(a[first + second], a[first + second - 1])) --second;
    a[first + hole] = a[first + second];
    hole = second;
  }
  if ((len & 1) == 0 && second == (len - 2) / 2) {
    second = 2 * (second + 1);
    a[first + hole] = a[first + second - 1];
    hole = second - 1;
  }
  int parent = (hole - 1) / 2;
  while (hole > top && tk_comp(a[first + parent], value)) {
    a[first + hole] = a[first + parent];
    hole = parent;
    parent = (hole - 1) / 2;
  }
  a[first + hole] = value;
}

__device__ void tk_make_heap(VI* a, int first, int last) {
  const int len = last - first;
  if (len < 2) return;
  int parent = (len - 2) / 2;
  while (true) {
    tk_adjust_heap(a, first, parent, len, a[first + parent]);
    if (parent == 0) return;
    --parent;
  }
}

__device__ void tk_pop_heap(VI* a, int first, int last, int result) {
  const VI value = a[result];
  a[result] = a[first];
  tk_adjust_heap(a, first, 0, last - first, value);
}

__device__ void tk_heap_select(VI* a, int first, int middle, int last) {
  tk_make_heap(a, first, middle);
  for (int i = middle; i < last; ++i)
    if (tk_comp(a[i], a[first])) tk_pop_heap(a, first, middle, i);
}

__device__ void tk_sort_heap(VI* a, int first, int last) {
  while (last - first > 1) {
    --last;
    tk_pop_heap(a, first, last, last);
  }
}

__device__ __forceinline__ int floor_log2(int n) { return 31 - __clz(n); }

__device__ void tk_introselect(VI* a, int first, int nth, int last, int depth) {
  while (last - first > 3) {
    if (depth == 0) {
      tk_heap_select(a, first, nth + 1, last);
      tk_swap(a, first, nth);
      return;
    }
    --depth;
    const int mid = first + (last - first) / 2;
    tk_move_median_to_first(a, first, first + 1, mid, last - 1);
    const int cut = tk_unguarded_partition(a, first + 1, last, first);
    if (cut <= nth) first = cut;
    else last = cut;
  }
  tk_insertion_sort(a, first, last);
}

// the k largest of v[0..n) in torch.topk's order (indices into out)
__device__ void topk_cpu(const float* v, int n, int k, VI* scratch, int* out_idx, float* out_val) {
  for (int i = 0; i < n; ++i) scratch[i] = VI{v[i], i};
  if (int64_t(k) * 64 <= n) {
    tk_heap_select(scratch, 0, k, n);
    tk_sort_heap(scratch, 0, k);
  } else {
    tk_introselect(scratch, 0, k - 1, n, 2 * floor_log2(n));
    tk_insertion_sort(scratch, 0, k - 1);  // std::sort of [0, k-1): below its 16-element threshold
  }
  for (int r = 0; r < k; ++r) {
    out_idx[r] = scratch[r].i;
    if (out_val) out_val[r] = scratch[r].v;
  }
}

// entries of a stamped score table ordered like a stable sort of the dict by
// value descending: value first, then insertion stamp; `skip` marks chosen ones
__device__ int best_entry(const double* score, const long long* at, int E, const unsigned char* skip) {
  int best = -1;
  for (int e = 0; e < E; ++e) {
    if (at[e] == 0 || (skip && skip[e])) continue;
    if (best < 0 || score[e] > score[best] || (score[e] == score[best] && at[e] < at[best])) best = e;
  }
  return best;
}


// Python floats as the reference uses them: fp32 where they meet fp32 tensors,
// fp64 in the dict arithmetic, and the Python-side comparisons done on the host
struct LocCfg {
  float sticky_strength, sticky_margin, max_bonus, explore_margin, cache_strength;
  double sticky_decay, workload_decay;
  int semantic_guard, min_raw_overlap, max_hot, window, predictive, experts_per_token;
  int sticky_positive, max_bonus_positive, cache_positive;
};

__device__ __forceinline__ void st_remove(double* val, long long* at, int e) {
  val[e] = 0.0;
  at[e] = 0;
}

// One warp; lane 0 walks the tokens (each token's steps depend on the state the
// previous one left).
__global__ void __launch_bounds__(32) locality_route_kernel(LocCfg c, const uint16_t* __restrict__ logits, int64_t T, int E,
                                                            int k, const uint8_t* __restrict__ resident, int64_t res_stride,
                                                            char* state, int32_t* __restrict__ out_exp,
                                                            uint16_t* __restrict__ out_w, int32_t* __restrict__ out_raw,
                                                            int32_t* __restrict__ out_pred, int32_t* __restrict__ out_npred,
                                                            uint8_t* __restrict__ out_flags) {
  extern __shared__ __align__(16) unsigned char loc_smem[];
  if (threadIdx.x != 0) return;
  double* cnt = reinterpret_cast<double*>(loc_smem);           // [E] Counter values (predictions)
  long long* rank1 = reinterpret_cast<long long*>(cnt + E);     // [E] Counter insertion order (minor)
  float* lg = reinterpret_cast<float*>(rank1 + E);              // [E] logits
  float* adj = lg + E;                                          // [E] adjusted logits
  VI* scratch = reinterpret_cast<VI*>(adj + E);                 // [E] top-k work space
  int* rank0 = reinterpret_cast<int*>(scratch + E);             // [E] Counter insertion order (major), -1 absent
  unsigned char* allowed = reinterpret_cast<unsigned char*>(rank0 + E);  // [E]
  unsigned char* chosen = allowed + E;                                   // [E]

  LocState S = loc_view(state, E, c.window);
  const int raw_k = c.experts_per_token < E ? c.experts_per_token : E;
  for (int64_t t = 0; t < T; ++t) {
    const uint16_t* lrow = logits + t * E;
    for (int e = 0; e < E; ++e) {
      lg[e] = bf16_to_f32(lrow[e]);
      adj[e] = lg[e];
    }
    int raw[kLocMaxK], rt_idx[kLocMaxK];
    float rt_val[kLocMaxK];
    topk_cpu(lg, E, k, scratch, raw, nullptr);            // route(): topk(logits, k)          :271
    topk_cpu(lg, E, raw_k, scratch, rt_idx, rt_val);     // _apply_locality_bias: raw_k top    :336

    int sticky_n = 0;
    for (int e = 0; e < E; ++e) sticky_n += S.sticky_at[e] != 0;
    // sticky bonus for remembered experts within the candidate margin of the raw top-k   :337-344
    if (sticky_n > 0 && c.sticky_positive) {
      const float floor_v = __fsub_rn(rt_val[raw_k - 1], c.sticky_margin);
      for (int e = 0; e < E; ++e) {
        if (S.sticky_at[e] == 0 || !(lg[e] >= floor_v)) continue;
        float bonus = __fmul_rn(__double2float_rn(S.sticky[e]), c.sticky_strength);
        if (c.semantic_guard && c.max_bonus_positive && bonus > c.max_bonus) bonus = c.max_bonus;
        adj[e] = __fadd_rn(adj[e], bonus);
      }
    }
    // experts outside the hot set and the leading raw picks lose the exploration margin  :345-351
    if (c.max_hot > 0 && sticky_n >= c.max_hot) {
      for (int e = 0; e < E; ++e) allowed[e] = chosen[e] = 0;
      for (int h = 0; h < c.max_hot; ++h) {
        const int b = best_entry(S.sticky, S.sticky_at, E, chosen);
        if (b < 0) break;
        chosen[b] = 1;
        allowed[b] = 1;
      }
      int lead = c.experts_per_token / 2;
      if (lead < 1) lead = 1;
      if (lead > raw_k) lead = raw_k;
      for (int r = 0; r < lead; ++r) allowed[rt_idx[r]] = 1;
      for (int e = 0; e < E; ++e)
        if (!allowed[e]) adj[e] = __fsub_rn(adj[e], c.explore_margin);
    }
    // resident experts close to the best raw logit gain the cache-aware bonus           :352-357
    if (resident != nullptr && c.cache_positive) {
      const uint8_t* res = resident + t * res_stride;
      bool any = false;
      for (int e = 0; e < E; ++e) any |= res[e] != 0;
      if (any) {
        float mx = lg[0];
        for (int e = 0; e < E; ++e) {
          if (lg[e] != lg[e]) {
            mx = lg[e];
            break;
          }
          if (lg[e] > mx) mx = lg[e];
        }
        const float thr = __fsub_rn(mx, c.explore_margin);
        for (int e = 0; e < E; ++e)
          if (res[e] && lg[e] >= thr) adj[e] = __fadd_rn(adj[e], c.cache_strength);
      }
    }
    int sel[kLocMaxK];
    float sc[kLocMaxK];
    topk_cpu(adj, E, k, scratch, sel, nullptr);          // topk(adjusted, k)                  :273
    bool blocked = false;
    if (c.semantic_guard) {
      // keep at least min_raw_overlap raw experts: swap the weakest non-raw pick for the
      // first missing raw expert, then order by adjusted logit (stable)                  :376-394
      int need = c.min_raw_overlap < 0 ? 0 : c.min_raw_overlap;
      if (need > k) need = k;
      while (true) {
        int overlap = 0;
        for (int i = 0; i < k; ++i)
          for (int j = 0; j < k; ++j) overlap += sel[i] == raw[j];
        if (overlap >= need) break;
        int missing = -1;
        for (int j = 0; j < k && missing < 0; ++j) {
          bool in_sel = false;
          for (int i = 0; i < k; ++i) in_sel |= sel[i] == raw[j];
          if (!in_sel) missing = raw[j];
        }
        int evict_pos = -1;
        for (int i = 0; i < k; ++i) {
          bool in_raw = false;
          for (int j = 0; j < k; ++j) in_raw |= sel[i] == raw[j];
          if (in_raw) continue;
          if (evict_pos < 0 || adj[sel[i]] < adj[sel[evict_pos]]) evict_pos = i;
        }
        if (missing < 0 || evict_pos < 0) break;
        sel[evict_pos] = missing;
        blocked = true;
      }
      for (int i = 1; i < k; ++i) {  // stable: a pick moves ahead only past strictly smaller ones
        const int v = sel[i];
        int j = i;
        while (j > 0 && adj[sel[j - 1]] < adj[v]) {
          sel[j] = sel[j - 1];
          --j;
        }
        sel[j] = v;
      }
      for (int i = 0; i < k; ++i) sc[i] = lg[sel[i]];
    } else {
      for (int i = 0; i < k; ++i) sc[i] = adj[sel[i]];
    }
    // softmax of the selected scores, rounded once to bf16                               :281-282
    float m = sc[0];
    for (int r = 1; r < k; ++r) m = fmaxf(m, sc[r]);
    float ex[kLocMaxK];
    float sum = 0.f;
    for (int r = 0; r < k; ++r) {
      ex[r] = expf(sc[r] - m);
      sum += ex[r];
    }
    uint16_t wb[kLocMaxK];
    for (int r = 0; r < k; ++r) wb[r] = f32_to_bf16(ex[r] / sum);

    // predicted experts from the state before this token's update                       :426-440
    int npred = 0;
    if (c.predictive) {
      bool any = false;
      for (int e = 0; e < E; ++e) {
        cnt[e] = 0.0;
        rank0[e] = -1;
        rank1[e] = 0;
        if (S.workload_at[e] != 0) {
          cnt[e] = __dadd_rn(cnt[e], S.workload[e]);
          rank0[e] = 0;
          rank1[e] = S.workload_at[e];
        }
        if (S.sticky_at[e] != 0) {
          cnt[e] = __dadd_rn(cnt[e], __dmul_rn(S.sticky[e], 0.75));
          if (rank0[e] < 0) {
            rank0[e] = 1;
            rank1[e] = S.sticky_at[e];
          }
        }
      }
      for (int i = 0; i < S.h->hist_len; ++i) {
        const int e = S.hist[(S.h->hist_head + i) % c.window];
        cnt[e] = __dadd_rn(cnt[e], 0.5);
        if (rank0[e] < 0) {
          rank0[e] = 2;
          rank1[e] = i;
        }
      }
      for (int e = 0; e < E; ++e) {
        chosen[e] = 0;
        any |= rank0[e] >= 0;
      }
      if (any) {
        for (int r = 0; r < k; ++r) {  // Counter.most_common(k): value desc, insertion order
          int b = -1;
          for (int e = 0; e < E; ++e) {
            if (rank0[e] < 0 || chosen[e]) continue;
            if (b < 0 || cnt[e] > cnt[b] ||
                (cnt[e] == cnt[b] && (rank0[e] < rank0[b] || (rank0[e] == rank0[b] && rank1[e] < rank1[b]))))
              b = e;
          }
          if (b < 0) break;
          chosen[b] = 1;
          out_pred[t * k + npred++] = b;
        }
      }
    }

    // sticky scores: decay, drop the faded, add this token's weights, trim to the hot set   :396-411
    for (int e = 0; e < E; ++e) {
      if (S.sticky_at[e] == 0) continue;
      const double v = __dmul_rn(S.sticky[e], c.sticky_decay);
      if (v < 1e-4) st_remove(S.sticky, S.sticky_at, e);
      else S.sticky[e] = v;
    }
    for (int r = 0; r < k; ++r) {
      const int e = sel[r];
      const double w = double(bf16_to_f32(wb[r]));
      if (S.sticky_at[e] != 0) {
        S.sticky[e] = __dadd_rn(S.sticky[e], w);
      } else {
        S.sticky[e] = __dadd_rn(0.0, w);
        S.sticky_at[e] = ++S.h->sticky_clock;
      }
    }
    if (c.max_hot > 0) {
      int n = 0;
      for (int e = 0; e < E; ++e) n += S.sticky_at[e] != 0;
      if (n > 2 * c.max_hot) {
        for (int e = 0; e < E; ++e) chosen[e] = 0;
        for (int h = 0; h < c.max_hot; ++h) {
          const int b = best_entry(S.sticky, S.sticky_at, E, chosen);
          if (b < 0) break;
          chosen[b] = 1;
        }
        for (int e = 0; e < E; ++e)
          if (S.sticky_at[e] != 0 && !chosen[e]) st_remove(S.sticky, S.sticky_at, e);
      }
    }
    // workload scores and the recent-expert history                                       :413-424
    for (int e = 0; e < E; ++e) {
      if (S.workload_at[e] == 0) continue;
      const double v = __dmul_rn(S.workload[e], c.workload_decay);
      if (v < 1e-4) st_remove(S.workload, S.workload_at, e);
      else S.workload[e] = v;
    }
    for (int r = 0; r < k; ++r) {
      const int e = sel[r];
      const double w = double(bf16_to_f32(wb[r]));
      if (S.workload_at[e] != 0) {
        S.workload[e] = __dadd_rn(S.workload[e], w);
      } else {
        S.workload[e] = __dadd_rn(0.0, w);
        S.workload_at[e] = ++S.h->workload_clock;
      }
      if (S.h->hist_len < c.window) {
        S.hist[(S.h->hist_head + S.h->hist_len) % c.window] = e;
        ++S.h->hist_len;
      } else {
        S.hist[S.h->hist_head] = e;
        S.h->hist_head = (S.h->hist_head + 1) % c.window;
      }
    }

    bool adjusted = false;
    for (int r = 0; r < k; ++r) {
      adjusted |= sel[r] != raw[r];
      out_exp[t * k + r] = sel[r];
      out_w[t * k + r] = wb[r];
      out_raw[t * k + r] = raw[r];
    }
    out_npred[t] = npred;
    out_flags[t] = uint8_t((blocked ? 1 : 0) | (adjusted ? 2 : 0));
  }
}

size_t loc_smem_bytes(int E) { return size_t(E) * (8 + 8 + 4 + 4 + 8 + 4 + 1 + 1) + 16; }

}  // namespace
}  // namespace klc

extern "C" int klc_locality_state_bytes(int64_t experts, int prediction_window, size_t* out_bytes) {
  using namespace klc;
  KLC_CHECK_ARG(experts >= 1 && experts <= 1024 && out_bytes != nullptr, "klc_locality_state_bytes: bad arguments");
  const int window = prediction_window < 1 ? 1 : prediction_window;
  *out_bytes = loc_state_bytes(experts, window);
  return KLC_OK;
}

extern "C" int klc_locality_route(const klc_locality_config* cfg, const uint16_t* logits, int64_t tokens, int64_t experts,
                                  int k, const uint8_t* resident, int64_t resident_stride, void* state, size_t state_bytes,
                                  int32_t* out_experts, uint16_t* out_w, int32_t* out_raw, int32_t* out_pred,
                                  int32_t* out_npred, uint8_t* out_flags, void* stream) {
  using namespace klc;
  KLC_CHECK_ARG(cfg != nullptr, "klc_locality_route: null config");
  KLC_CHECK_ARG(experts >= 1 && experts <= 1024 && tokens >= 0, "klc_locality_route: need 1 <= experts <= 1024");
  KLC_CHECK_ARG(k >= 1 && k <= kLocMaxK && k <= experts, "klc_locality_route: need 1 <= k <= min(8, experts)");
  KLC_CHECK_ARG(cfg->experts_per_token >= 1 && cfg->experts_per_token <= kLocMaxK,
                "klc_locality_route: experts_per_token must be in [1, 8]");
  const int window = cfg->prediction_window < 1 ? 1 : cfg->prediction_window;
  KLC_CHECK_ARG(state != nullptr && state_bytes >= loc_state_bytes(experts, window),
                "klc_locality_route: state buffer too small (klc_locality_state_bytes)");
  KLC_CHECK_ARG((reinterpret_cast<uintptr_t>(state) & 15) == 0, "klc_locality_route: state must be 16-byte aligned");
  if (tokens == 0) return KLC_OK;
  KLC_CHECK_ARG(logits && out_experts && out_w && out_raw && out_pred && out_npred && out_flags,
                "klc_locality_route: null pointer");
  KLC_CHECK_ARG(resident == nullptr || resident_stride == 0 || resident_stride >= experts,
                "klc_locality_route: resident stride must be 0 (one mask) or >= experts");
  LocCfg c{};
  c.sticky_strength = float(cfg->sticky_strength);
  c.sticky_margin = float(std::fabs(cfg->sticky_candidate_margin));
  c.max_bonus = float(cfg->max_sticky_bonus);
  c.explore_margin = float(std::fabs(cfg->exploration_margin));
  c.cache_strength = float(cfg->cache_aware_strength);
  c.sticky_decay = cfg->sticky_decay;
  c.workload_decay = 1.0 - 1.0 / (cfg->workload_window > 1.0 ? cfg->workload_window : 1.0);
  c.semantic_guard = cfg->semantic_guard != 0;
  c.min_raw_overlap = cfg->min_raw_overlap;
  c.max_hot = cfg->max_hot_experts;
  c.window = window;
  c.predictive = cfg->predictive_prefetch != 0;
  c.experts_per_token = cfg->experts_per_token;
  c.sticky_positive = cfg->sticky_strength > 0;
  c.max_bonus_positive = cfg->max_sticky_bonus > 0;
  c.cache_positive = cfg->cache_aware_strength > 0;
  const size_t smem = loc_smem_bytes(int(experts));
  locality_route_kernel<<<1, 32, smem, as_stream(stream)>>>(c, logits, tokens, int(experts), k, resident, resident_stride,
                                                           static_cast<char*>(state), out_experts, out_w, out_raw, out_pred,
                                                           out_npred, out_flags);
  KLC_LAUNCH_CHECK("locality_route_kernel launch");
  return KLC_OK;
}
