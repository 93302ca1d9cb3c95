// Warp-wide top-k + softmax of one token's router scores, shared by the router
// kernels (router.cu) and the combine kernel that routes the next layer
// (combine.cu).
#pragma once

#include "klc_common.cuh"

namespace klc {

constexpr int kSelMaxK = 8;

// softmax over the k selected fp32 scores (max-subtracted, summed in selection
// order), each weight rounded once to bf16; lane 0 writes
__device__ __forceinline__ void softmax_write(const float (&sel_v)[kSelMaxK], const int (&sel_i)[kSelMaxK], int k, bool write_idx,
                                              int32_t* out_idx, uint16_t* out_w) {
  if ((threadIdx.x & 31) != 0) return;
  float m = sel_v[0];
#pragma unroll
  for (int r = 1; r < kSelMaxK; ++r)
    if (r < k) m = fmaxf(m, sel_v[r]);
  float ex[kSelMaxK];
  float sum = 0.f;
#pragma unroll
  for (int r = 0; r < kSelMaxK; ++r)
    if (r < k) {
      ex[r] = expf(sel_v[r] - m);
      sum += ex[r];
    }
#pragma unroll
  for (int r = 0; r < kSelMaxK; ++r)
    if (r < k) {
      if (write_idx) out_idx[r] = sel_i[r];
      out_w[r] = f32_to_bf16(ex[r] / sum);
    }
}

// k rounds of a warp-wide arg-max over `row` (value descending, lower index on
// ties; -inf is selectable, NaN only once nothing else is left, then the lowest
// index not taken), then the softmax.  Lane l holds experts l, l + 32, ... in
// registers (J per lane) and a bit mask of those already taken.
template <int J>
__device__ __forceinline__ void select_softmax_warp_j(const float* row, int experts, int k, int32_t* out_idx,
                                                      uint16_t* out_w) {
  const int lane = threadIdx.x & 31;
  float v[J];
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int e = lane + 32 * j;
    v[j] = e < experts ? row[e] : 0.f;
  }
  uint32_t taken = 0;
  float sel_v[kSelMaxK];
  int sel_i[kSelMaxK];
#pragma unroll
  for (int r = 0; r < kSelMaxK; ++r) {
    sel_v[r] = 0.f;
    sel_i[r] = 0;
    if (r < k) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int e = lane + 32 * j;
        if (e < experts && !((taken >> j) & 1u) && (v[j] > bv || (v[j] == bv && e < bi))) {
          bv = v[j];
          bi = e;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (bi == 0x7fffffff) {  // only NaN scores left
        int c = 0x7fffffff;
#pragma unroll
        for (int j = J - 1; j >= 0; --j) {
          const int e = lane + 32 * j;
          if (e < experts && !((taken >> j) & 1u)) c = e;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) c = min(c, __shfl_xor_sync(0xffffffffu, c, o));
        bi = c;
        bv = row[c];
      }
      if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
      sel_v[r] = bv;
      sel_i[r] = bi;
    }
  }
  softmax_write(sel_v, sel_i, k, true, out_idx, out_w);
}

// The selection of one token by one warp; with keep_order the row already
// holds exactly k scores in the wanted order (softmax only).
__device__ __forceinline__ void select_softmax_warp(const float* row, int experts, int k, bool keep_order, int32_t* out_idx,
                                    uint16_t* out_w) {
  if (keep_order) {
    float sel_v[kSelMaxK];
    int sel_i[kSelMaxK];
#pragma unroll
    for (int r = 0; r < kSelMaxK; ++r) {
      sel_v[r] = r < k ? row[r] : 0.f;
      sel_i[r] = r;
    }
    softmax_write(sel_v, sel_i, k, false, out_idx, out_w);
  } else if (experts <= 128) {
    select_softmax_warp_j<4>(row, experts, k, out_idx, out_w);
  } else if (experts <= 256) {
    select_softmax_warp_j<8>(row, experts, k, out_idx, out_w);
  } else {
    select_softmax_warp_j<32>(row, experts, k, out_idx, out_w);
  }
}

}  // namespace klc
