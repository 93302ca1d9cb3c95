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

// Fast path of topk_cpu for one warp: when the row has no NaN and its k + 1 largest
// values are all different, torch.topk's result is simply the k largest in
// descending order, whatever its algorithm; returns false (the outputs may then hold
// a partial result) when a tie or a NaN makes the order depend on the algorithm.
// Lane l owns l, l + 32, ...
__device__ bool warp_topk_distinct(const float* v, int n, int k, int* out_idx, float* out_val) {
  const int lane = threadIdx.x & 31;
  bool nan = false;
  for (int e = lane; e < n; e += 32) nan |= v[e] != v[e];
  if (__any_sync(0xffffffffu, nan)) return false;
  const int rounds = k < n ? k + 1 : k;
  uint32_t taken = 0;
  float prev = 0.f;
  bool ok = true;
  for (int r = 0; r < rounds && ok; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int j = 0, e = lane; e < n; ++j, e += 32)
      if (!((taken >> j) & 1u) && (bi == 0x7fffffff || v[e] > bv || (v[e] == bv && e < bi))) {
        bv = v[e];
        bi = e;
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oi != 0x7fffffff && (bi == 0x7fffffff || ov > bv || (ov == bv && oi < bi))) {
        bv = ov;
        bi = oi;
      }
    }
    if (r > 0 && !(bv < prev)) ok = false;  // a tie (or a repeat of the k-th value just below)
    prev = bv;
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    if (r < k && lane == 0) {
      out_idx[r] = bi;
      if (out_val) out_val[r] = bv;
    }
  }
  __syncwarp();
  return ok;
}

// The warp's best entry of a stamped score table, as a stable sort of the dict by
// value descending would put it first: larger value, then earlier insertion.
// Entries with at == 0 are absent; `skip` marks entries already taken.
__device__ int warp_best_entry(const double* score, const long long* at, int E, const unsigned char* skip) {
  const int lane = threadIdx.x & 31;
  double bv = 0.0;
  long long ba = 0;
  int be = -1;
  for (int e = lane; e < E; e += 32) {
    if (at[e] == 0 || (skip != nullptr && skip[e])) continue;
    if (be < 0 || score[e] > bv || (score[e] == bv && at[e] < ba)) {
      bv = score[e];
      ba = at[e];
      be = e;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const double ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const long long oa = __shfl_xor_sync(0xffffffffu, ba, o);
    const int oe = __shfl_xor_sync(0xffffffffu, be, o);
    if (oe >= 0 && (be < 0 || ov > bv || (ov == bv && oa < ba))) {
      bv = ov;
      ba = oa;
      be = oe;
    }
  }
  return be;
}

// Python floats as the reference uses them: fp32 where they meet fp32 tensors,
// fp64 in the dict arithmetic, and the Python-side comparisons done on the host
struct LocCfg {
  float sticky_strength, sticky_margin, max_bonus, explore_margin, cache_strength;
  double sticky_decay, workload_decay;
  int semantic_guard, min_raw_overlap, max_hot, window, predictive, experts_per_token;
  int sticky_positive, max_bonus_positive, cache_positive;
};

// Shared-memory copy of one layer's state plus the per-token work arrays.
struct LocSmem {
  double *sticky, *workload, *cnt;
  long long *sticky_at, *workload_at, *rank1;
  float *lg, *adj;
  VI* scratch;
  int *hist, *rank0;
  unsigned char *allowed, *chosen;
};

__host__ __device__ inline size_t loc_smem_bytes(int E, int window) {
  return size_t(E) * (8 + 8 + 8 + 8 + 8 + 8 + 4 + 4 + 8 + 4 + 1 + 1) + size_t(window) * 4 + 64;
}

__device__ LocSmem loc_smem_view(unsigned char* p, int E, int window) {
  LocSmem m;
  m.sticky = reinterpret_cast<double*>(p);
  m.workload = m.sticky + E;
  m.cnt = m.workload + E;
  m.sticky_at = reinterpret_cast<long long*>(m.cnt + E);
  m.workload_at = m.sticky_at + E;
  m.rank1 = m.workload_at + E;
  m.lg = reinterpret_cast<float*>(m.rank1 + E);
  m.adj = m.lg + E;
  m.scratch = reinterpret_cast<VI*>(m.adj + E);
  m.hist = reinterpret_cast<int*>(m.scratch + E);
  m.rank0 = m.hist + window;
  m.allowed = reinterpret_cast<unsigned char*>(m.rank0 + E);
  m.chosen = m.allowed + E;
  return m;
}

// One warp runs the call and walks the tokens in order (each token's steps depend
// on the state the previous one left).  The state lives in shared memory for the
// call; the passes over the experts are spread over the lanes, the order-sensitive
// steps (the torch.topk restatement, the guard, insertions into the dicts) run on
// lane 0.
__global__ void __launch_bounds__(32) locality_route_kernel(LocCfg c, const uint16_t* __restrict__ logits, int64_t T, int E,
                                                            int k, const uint8_t* __restrict__ resident, int64_t res_stride,
                                                            char* state, int32_t* __restrict__ out_exp,
                                                            uint16_t* __restrict__ out_w, int32_t* __restrict__ out_raw,
                                                            int32_t* __restrict__ out_pred, int32_t* __restrict__ out_npred,
                                                            uint8_t* __restrict__ out_flags) {
  extern __shared__ __align__(16) unsigned char loc_smem[];
  __shared__ int raw_s[kLocMaxK], rt_idx_s[kLocMaxK], sel_s[kLocMaxK];
  __shared__ float rt_val_s[kLocMaxK];
  __shared__ uint16_t wb_s[kLocMaxK];
  __shared__ long long sticky_clock, workload_clock;
  __shared__ int hist_len, hist_head;
  const int lane = threadIdx.x & 31;
  const unsigned full = 0xffffffffu;
  LocState S = loc_view(state, E, c.window);
  LocSmem M = loc_smem_view(loc_smem, E, c.window);
  for (int e = lane; e < E; e += 32) {
    M.sticky[e] = S.sticky[e];
    M.workload[e] = S.workload[e];
    M.sticky_at[e] = S.sticky_at[e];
    M.workload_at[e] = S.workload_at[e];
  }
  for (int i = lane; i < c.window; i += 32) M.hist[i] = S.hist[i];
  if (lane == 0) {
    sticky_clock = S.h->sticky_clock;
    workload_clock = S.h->workload_clock;
    hist_len = S.h->hist_len;
    hist_head = S.h->hist_head;
  }
  __syncwarp();
  const int raw_k = c.experts_per_token < E ? c.experts_per_token : E;
  for (int64_t t = 0; t < T; ++t) {
    const uint16_t* lrow = logits + t * E;
    for (int e = lane; e < E; e += 32) {
      M.lg[e] = bf16_to_f32(lrow[e]);
      M.adj[e] = M.lg[e];
    }
    __syncwarp();
    // route(): topk(logits, k) :271; _apply_locality_bias: topk(logits, raw_k) :336 (the same
    // selection when k == raw_k); the restated algorithm only where ties make it matter
    const bool raw_fast = warp_topk_distinct(M.lg, E, raw_k, rt_idx_s, rt_val_s);
    if (lane == 0) {
      if (!raw_fast) topk_cpu(M.lg, E, raw_k, M.scratch, rt_idx_s, rt_val_s);
      if (raw_k == k) {
        for (int r = 0; r < k; ++r) raw_s[r] = rt_idx_s[r];
      } else {
        topk_cpu(M.lg, E, k, M.scratch, raw_s, nullptr);
      }
    }
    __syncwarp();
    int sticky_n = 0;
    for (int e = lane; e < E; e += 32) sticky_n += M.sticky_at[e] != 0;
    sticky_n = __reduce_add_sync(full, sticky_n);
    // sticky bonus for remembered experts within the candidate margin of the raw top-k   :337-344
    if (sticky_n > 0 && c.sticky_positive) {
      const float floor_v = __fsub_rn(rt_val_s[raw_k - 1], c.sticky_margin);
      for (int e = lane; e < E; e += 32) {
        if (M.sticky_at[e] == 0 || !(M.lg[e] >= floor_v)) continue;
        float bonus = __fmul_rn(__double2float_rn(M.sticky[e]), c.sticky_strength);
        if (c.semantic_guard && c.max_bonus_positive && bonus > c.max_bonus) bonus = c.max_bonus;
        M.adj[e] = __fadd_rn(M.adj[e], bonus);
      }
    }
    // experts outside the hot set and the leading raw picks lose the exploration margin  :345-351
    if (c.max_hot > 0 && sticky_n >= c.max_hot) {
      for (int e = lane; e < E; e += 32) M.allowed[e] = M.chosen[e] = 0;
      __syncwarp();
      for (int h = 0; h < c.max_hot; ++h) {
        const int b = warp_best_entry(M.sticky, M.sticky_at, E, M.chosen);
        if (b < 0) break;
        if (lane == 0) M.chosen[b] = M.allowed[b] = 1;
        __syncwarp();
      }
      if (lane == 0) {
        int lead = c.experts_per_token / 2;
        if (lead < 1) lead = 1;
        if (lead > raw_k) lead = raw_k;
        for (int r = 0; r < lead; ++r) M.allowed[rt_idx_s[r]] = 1;
      }
      __syncwarp();
      for (int e = lane; e < E; e += 32)
        if (!M.allowed[e]) M.adj[e] = __fsub_rn(M.adj[e], c.explore_margin);
    }
    // resident experts close to the best raw logit gain the cache-aware bonus           :352-357
    if (resident != nullptr && c.cache_positive) {
      const uint8_t* res = resident + t * res_stride;
      bool any = false, nan = false;
      float mx = -INFINITY;
      for (int e = lane; e < E; e += 32) {
        any |= res[e] != 0;
        const float v = M.lg[e];
        if (v != v) nan = true;
        else mx = fmaxf(mx, v);
      }
      any = __any_sync(full, any);
      nan = __any_sync(full, nan);
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(full, mx, o));
      if (any) {
        const float thr = __fsub_rn(nan ? __int_as_float(0x7fc00000) : mx, c.explore_margin);
        for (int e = lane; e < E; e += 32)
          if (res[e] && M.lg[e] >= thr) M.adj[e] = __fadd_rn(M.adj[e], c.cache_strength);
      }
    }
    __syncwarp();
    const bool adj_fast = warp_topk_distinct(M.adj, E, k, sel_s, nullptr);  // topk(adjusted, k)  :273
    bool blocked = false, adjusted = false;
    if (lane == 0) {
      int sel[kLocMaxK];
      float sc[kLocMaxK];
      if (adj_fast) {
        for (int r = 0; r < k; ++r) sel[r] = sel_s[r];
      } else {
        topk_cpu(M.adj, E, k, M.scratch, sel, nullptr);
      }
      int raw[kLocMaxK];
      for (int r = 0; r < k; ++r) raw[r] = raw_s[r];
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
            if (evict_pos < 0 || M.adj[sel[i]] < M.adj[sel[evict_pos]]) evict_pos = i;
          }
          if (missing < 0 || evict_pos < 0) break;
          sel[evict_pos] = missing;
          blocked = true;
        }
        for (int i = 1; i < k; ++i) {  // stable: a pick moves ahead only past strictly smaller ones
          const int v = sel[i];
          int j = i;
          while (j > 0 && M.adj[sel[j - 1]] < M.adj[v]) {
            sel[j] = sel[j - 1];
            --j;
          }
          sel[j] = v;
        }
        for (int i = 0; i < k; ++i) sc[i] = M.lg[sel[i]];
      } else {
        for (int i = 0; i < k; ++i) sc[i] = M.adj[sel[i]];
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
      for (int r = 0; r < k; ++r) {
        wb_s[r] = f32_to_bf16(ex[r] / sum);
        sel_s[r] = sel[r];
        adjusted |= sel[r] != raw[r];
        out_exp[t * k + r] = sel[r];
        out_w[t * k + r] = wb_s[r];
        out_raw[t * k + r] = raw[r];
      }
      out_flags[t] = uint8_t((blocked ? 1 : 0) | (adjusted ? 2 : 0));
    }
    __syncwarp();

    // predicted experts from the state before this token's update                       :426-440
    int npred = 0;
    if (c.predictive) {
      bool any = false;
      for (int e = lane; e < E; e += 32) {
        double v = 0.0;
        int r0 = -1;
        long long r1 = 0;
        if (M.workload_at[e] != 0) {
          v = __dadd_rn(v, M.workload[e]);
          r0 = 0;
          r1 = M.workload_at[e];
        }
        if (M.sticky_at[e] != 0) {
          v = __dadd_rn(v, __dmul_rn(M.sticky[e], 0.75));
          if (r0 < 0) {
            r0 = 1;
            r1 = M.sticky_at[e];
          }
        }
        for (int i = 0; i < hist_len; ++i) {
          if (M.hist[(hist_head + i) % c.window] != e) continue;
          v = __dadd_rn(v, 0.5);
          if (r0 < 0) {
            r0 = 2;
            r1 = i;
          }
        }
        M.cnt[e] = v;
        M.rank0[e] = r0;
        M.rank1[e] = r1;
        M.chosen[e] = 0;
        any |= r0 >= 0;
      }
      any = __any_sync(full, any);
      __syncwarp();
      if (any) {
        for (int r = 0; r < k; ++r) {  // Counter.most_common(k): value desc, then insertion order
          double bv = 0.0;
          int b0 = 0, be = -1;
          long long b1 = 0;
          for (int e = lane; e < E; e += 32) {
            if (M.rank0[e] < 0 || M.chosen[e]) continue;
            const double v = M.cnt[e];
            if (be < 0 || v > bv || (v == bv && (M.rank0[e] < b0 || (M.rank0[e] == b0 && M.rank1[e] < b1)))) {
              bv = v;
              b0 = M.rank0[e];
              b1 = M.rank1[e];
              be = e;
            }
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const double ov = __shfl_xor_sync(full, bv, o);
            const int o0 = __shfl_xor_sync(full, b0, o);
            const long long o1 = __shfl_xor_sync(full, b1, o);
            const int oe = __shfl_xor_sync(full, be, o);
            if (oe >= 0 && (be < 0 || ov > bv || (ov == bv && (o0 < b0 || (o0 == b0 && o1 < b1))))) {
              bv = ov;
              b0 = o0;
              b1 = o1;
              be = oe;
            }
          }
          if (be < 0) break;
          if (lane == 0) {
            M.chosen[be] = 1;
            out_pred[t * k + npred] = be;
          }
          ++npred;
          __syncwarp();
        }
      }
    }
    if (lane == 0) out_npred[t] = npred;

    // sticky scores: decay, drop the faded, add this token's weights, trim to the hot set   :396-411
    for (int e = lane; e < E; e += 32) {
      if (M.sticky_at[e] == 0) continue;
      const double v = __dmul_rn(M.sticky[e], c.sticky_decay);
      if (v < 1e-4) {
        M.sticky[e] = 0.0;
        M.sticky_at[e] = 0;
      } else {
        M.sticky[e] = v;
      }
    }
    __syncwarp();
    if (lane == 0) {
      for (int r = 0; r < k; ++r) {
        const int e = sel_s[r];
        const double w = double(bf16_to_f32(wb_s[r]));
        if (M.sticky_at[e] != 0) {
          M.sticky[e] = __dadd_rn(M.sticky[e], w);
        } else {
          M.sticky[e] = __dadd_rn(0.0, w);
          M.sticky_at[e] = ++sticky_clock;
        }
      }
    }
    __syncwarp();
    if (c.max_hot > 0) {
      int n = 0;
      for (int e = lane; e < E; e += 32) n += M.sticky_at[e] != 0;
      n = __reduce_add_sync(full, n);
      if (n > 2 * c.max_hot) {
        for (int e = lane; e < E; e += 32) M.chosen[e] = 0;
        __syncwarp();
        for (int h = 0; h < c.max_hot; ++h) {
          const int b = warp_best_entry(M.sticky, M.sticky_at, E, M.chosen);
          if (b < 0) break;
          if (lane == 0) M.chosen[b] = 1;
          __syncwarp();
        }
        for (int e = lane; e < E; e += 32)
          if (M.sticky_at[e] != 0 && !M.chosen[e]) {
            M.sticky[e] = 0.0;
            M.sticky_at[e] = 0;
          }
      }
    }
    // workload scores and the recent-expert history                                       :413-424
    for (int e = lane; e < E; e += 32) {
      if (M.workload_at[e] == 0) continue;
      const double v = __dmul_rn(M.workload[e], c.workload_decay);
      if (v < 1e-4) {
        M.workload[e] = 0.0;
        M.workload_at[e] = 0;
      } else {
        M.workload[e] = v;
      }
    }
    __syncwarp();
    if (lane == 0) {
      for (int r = 0; r < k; ++r) {
        const int e = sel_s[r];
        const double w = double(bf16_to_f32(wb_s[r]));
        if (M.workload_at[e] != 0) {
          M.workload[e] = __dadd_rn(M.workload[e], w);
        } else {
          M.workload[e] = __dadd_rn(0.0, w);
          M.workload_at[e] = ++workload_clock;
        }
        if (hist_len < c.window) {
          M.hist[(hist_head + hist_len) % c.window] = e;
          ++hist_len;
        } else {
          M.hist[hist_head] = e;
          hist_head = (hist_head + 1) % c.window;
        }
      }
    }
    __syncwarp();
  }
  // the state back to its buffer for the next call
  for (int e = lane; e < E; e += 32) {
    S.sticky[e] = M.sticky[e];
    S.workload[e] = M.workload[e];
    S.sticky_at[e] = M.sticky_at[e];
    S.workload_at[e] = M.workload_at[e];
  }
  for (int i = lane; i < c.window; i += 32) S.hist[i] = M.hist[i];
  if (lane == 0) {
    S.h->sticky_clock = sticky_clock;
    S.h->workload_clock = workload_clock;
    S.h->hist_len = hist_len;
    S.h->hist_head = hist_head;
  }
}

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
  const size_t smem = loc_smem_bytes(int(experts), window);
  if (smem > 48 * 1024)
    KLC_CUDA(cudaFuncSetAttribute(locality_route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  locality_route_kernel<<<1, 32, smem, as_stream(stream)>>>(c, logits, tokens, int(experts), k, resident, resident_stride,
                                                           static_cast<char*>(state), out_experts, out_w, out_raw, out_pred,
                                                           out_npred, out_flags);
  KLC_LAUNCH_CHECK("locality_route_kernel launch");
  return KLC_OK;
}
