// Internal interfaces shared by the MoE-layer kernels of libklcmoe.
#pragma once

#include "klc_common.cuh"

namespace klc {

// ---------------------------------------------------------------------------
// permute
// ---------------------------------------------------------------------------
struct PermuteArgs {
  const int32_t* idx;  // [T, k]
  int64_t tokens;
  int k;
  int64_t experts;
  int pad;             // rows of each expert group padded to a multiple of this
  int block_n;         // max rows per row-block
  int32_t* counts;     // [E]
  int32_t* offsets;    // [E+1]
  int32_t* rows;       // [rows_cap]   padded row -> pair id (-1 = padding)
  int32_t* pair_pos;   // [T*k]        pair id -> padded row
  int32_t* chunk_hist; // [nchunks*E]  scratch
  int4* rowblocks;     // [max_rowblocks] (expert, first row, rows, 0)
  int4* pairblocks;    // null, or [max_rowblocks]: (expert, first row, rows <= 2*block_n, index of its
                       // first row-block); two consecutive row-blocks of one expert per entry
  DeviceStatus* status;
  const uint16_t* x;   // [T, H] or null (no gather)
  int64_t hidden;
  uint16_t* xp;        // [rows_cap, H] or null
  int div;             // group id = idx / div (1: group by expert; experts-per-rank: group by rank)
  int32_t* aux_out;    // optional [rows_cap]: idx % div of the pair stored at each row
  bool empty_ok;       // a negative idx marks an empty slot (skipped, pair_pos -1) instead of a fault
};

int launch_permute(const PermuteArgs& a, cudaStream_t stream);

int launch_router(const uint16_t* x, int64_t tokens, int64_t hidden, const uint16_t* w, const uint16_t* b,
                  int64_t experts, int k, const float* adjust, int32_t* out_idx, uint16_t* out_w,
                  uint16_t* out_logits, cudaStream_t stream);

// ---------------------------------------------------------------------------
// workspace layout (all offsets 256-byte aligned, status word first)
// ---------------------------------------------------------------------------
struct WorkspaceLayout {
  int64_t pairs, rows_cap, max_rowblocks, nchunks;
  int pad, block_n;
  size_t status, counts, offsets, chunk_hist, rows, pair_pos, rowblocks, normsq, xp, gated, y, idx, w;
  size_t gq, sfb1, sfb2;  // tensor-core path: hi/lo E4M3 down-pass rows and activation scale blocks
  size_t pairblocks;      // tensor-core path with 64-row blocks: the paired row-block list
  size_t total;
};

WorkspaceLayout workspace_layout(const klc_moe_dims& d, bool need_routing_buffers);

// Down-projection output rows stored into segments of other buffers instead of y
// (expert parallelism: each row goes back to its source rank's arena over
// NVLink).  Padded row r holding pair q is written to
// base[q / seg_cap] + (slot0 + q % seg_cap) * hidden * 2 bytes.
constexpr int kMaxScatterSegments = 8;
struct RowScatter {
  char* base[kMaxScatterSegments];
  int64_t seg_cap;
  int64_t slot0;
  int world;  // 0: no scatter
};

// Permute + both expert GEMMs for given routing, without the combine: the
// expert output of pair p is row pair_pos[p] of y (ws + L.pair_pos, ws + L.y;
// -1 for an empty slot when empty_ok).  `normsq` (or null) accumulates the
// per-pair squared norms.  With `scatter` the down rows go to its segments
// instead of y (weights-as-N tensor-core kernels only).
int run_expert_stage(const klc_moe_dims& d, const klc_moe_weights& wts, const uint16_t* x, const int32_t* idx, int precision,
                     float* normsq, bool empty_ok, char* ws, const WorkspaceLayout& L, cudaStream_t stream,
                     const RowScatter* scatter = nullptr);

// Argument checks shared by every layer entry point (KLC_ERR_INVALID and a
// message on failure): sizes, the expert path, and the expert weight pointers
// (non-null, blocks 16-byte aligned for the 128-bit weight loads).
int validate_dims(const klc_moe_dims* d);
int validate_weights(const klc_moe_weights* w);

// ---------------------------------------------------------------------------
// expert kernels
// ---------------------------------------------------------------------------
struct ExpertArgs {
  const klc_moe_weights* wts;
  int64_t hidden, inter, experts;
  int k;
  int precision;
  const int4* rowblocks;
  const int4* pairblocks;      // null, or the paired list (two-SM tiles; count in status->pairblocks)
  int max_rowblocks;
  const int32_t* rows;
  const DeviceStatus* status;  // rowblocks count lives here
  DeviceStatus* status_rw;
  const uint16_t* xp;          // [rows_cap, H] (SIMT)
  const uint16_t* x;           // [T, H] layer input (TC: quantized per row-block through `rows`)
  uint8_t* xq;                 // [rows_cap, 2, H] hi/lo E4M3 gate_up operand (TC)
  uint8_t* gq;                 // [rows_cap, 2, I] hi/lo E4M3 down operand (TC)
  uint8_t* sfb1;               // [max_rowblocks, H/128, nch, 512] activation scales (TC)
  uint8_t* sfb2;               // [max_rowblocks, I/128, nch, 512]
  void* gated;                 // [rows_cap, I] fp32 (SIMT) or bf16 (TC)
  uint16_t* y;                 // [rows_cap, H]
  float* normsq;               // [pairs, 2] or null
  int64_t rows_cap;
  int block_n;                 // max rows per row-block
  const RowScatter* scatter;   // null: down rows into y
};

int launch_experts_simt(const ExpertArgs& a, cudaStream_t stream);
int launch_experts_tc(const ExpertArgs& a, cudaStream_t stream);
bool tc_path_supported(int64_t hidden, int64_t inter);
bool use_tc_path(const klc_moe_dims& d);  // the dims' path choice (auto: tc_path_supported)
// true when launch_experts_tc runs these weights with the weights-as-N kernels,
// the form whose down epilogue can scatter rows (RowScatter)
bool experts_tc_can_scatter(const klc_moe_weights& w, int64_t hidden, int64_t inter, int block_n);
// 512-byte activation-scale blocks per (row-block, 128-K stage) of the tensor-core path
int mx_sfb_chunks(int block_n);
// bf16 rows -> hi/lo E4M3 rows + scale blocks for every row-block (mx_quant.cu);
// rows_map != null: source row = rows_map[row] / k (the permuted pair's token)
int launch_quantize_rows(const uint16_t* src, int64_t K, const int32_t* rows_map, int k, const int4* rowblocks,
                         const DeviceStatus* status, int max_rowblocks, int nch, uint8_t* q, uint8_t* sfb,
                         cudaStream_t stream);

// ---------------------------------------------------------------------------
// optional per-stage CUDA-event timing (klc_stage_timing / klc_stage_times)
// ---------------------------------------------------------------------------
enum Stage { kStageStart = 0, kStageRouted = 1, kStagePermuted = 2, kStageGateUp = 3, kStageDown = 4, kStageCombined = 5, kStageCount = 6 };
void stage_mark(int stage, cudaStream_t stream);

// The next layer's input RMSNorm fused into the combine (weight bf16 [H], output bf16 [T,H]).
struct PostNorm {
  const uint16_t* weight;
  float eps;
  uint16_t* normed;
  // optional: the next layer's router on the normalised rows (router_w null: none)
  const uint16_t* router_w;   // bf16 [E, H]
  const uint16_t* router_b;   // bf16 [E]
  int experts, k;
  int32_t* out_idx;           // int32 [T, k]
  uint16_t* out_w;            // bf16 [T, k]
  uint16_t* out_logits;       // bf16 [T, E] or null
};

int launch_combine(const uint16_t* y, const int32_t* pair_pos, const uint16_t* w, int64_t tokens, int k,
                   int64_t hidden, const uint16_t* residual, uint16_t* out, const float* normsq, float* norms,
                   const PostNorm* post, cudaStream_t stream);

}  // namespace klc
