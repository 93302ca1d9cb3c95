/*
 * klc_moe.h — C ABI of the B200-native KLCquant MoE block (libklcmoe.so).
 *
 * Every entry point takes plain device pointers, 64-bit sizes and a CUDA
 * stream passed as `void*` (NULL = legacy default stream), returns an `int`
 * status (KLC_OK = 0) and never aborts, throws or frees caller memory.
 * `klc_last_error()` gives a thread-local message for the last failure on the
 * calling thread.  Device tensors are row-major and contiguous unless a
 * stride argument says otherwise.  bf16 values travel as uint16_t bit
 * patterns.
 *
 * Reference interfaces replaced (KLCquant, a Python/PyTorch package):
 *   klc_mxfp4_dequant        <- dequantize_mxfp4_matrix        mxfp4_expert.py:357-379
 *   klc_router_topk          <- StreamedMoERouter.route, router part
 *                               (F.linear + topk + softmax)     streamed_moe_router.py:269-284
 *   klc_moe_permute          <- (no counterpart: the reference loops one token
 *                               and one expert at a time,       streamed_moe_router.py:499)
 *   klc_moe_experts          <- _execute_mxfp4_experts expert math (gate_up GEMM,
 *                               bias, _apply_gate, down GEMM)   streamed_moe_router.py:483-511,524-529
 *   klc_moe_combine          <- weighted bf16 combine           streamed_moe_router.py:497,512-513
 *   klc_moe_bias_only        <- execute_experts=False path      streamed_moe_router.py:317-329
 *   klc_moe_forward          <- StreamedMoERouter.route as a whole, batched over tokens
 *   klc_rms_norm             <- rms_norm                        streamed_attention.py:27-28
 *   klc_moe_combine_rmsnorm  <- combine, `hidden += moe_out` and the next layer's
 *   klc_moe_forward_rmsnorm     input rms_norm in one kernel    streamed_transformer_executor.py:235,260
 *   klc_moe_*_rmsnorm_route  <- the above plus the next layer's router (F.linear + topk + softmax,
 *                               streamed_moe_router.py:269-282) on the normalised rows
 *   klc_locality_route       <- route()'s locality steps: _apply_locality_bias :331-363,
 *                               _guarded_expert_selection :365-394, predict_experts :426-440,
 *                               _update_sticky_scores / _update_workload_scores :396-424
 *   klc_runtime_dequant      <- RuntimeDequantizer.dequantize   runtime_dequantizer.py:30-52
 *                               (unpack_lowbit adaptive_quantizer.py:183-213,
 *                                reconstruct_pruned tensor_pruner.py:62-69)
 */
#ifndef KLC_MOE_H
#define KLC_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------- */
enum klc_status {
  KLC_OK = 0,
  KLC_ERR_INVALID = 1,        /* bad pointer, shape or enum value            */
  KLC_ERR_UNSUPPORTED = 2,    /* valid request this build does not handle    */
  KLC_ERR_WORKSPACE = 3,      /* caller workspace smaller than required      */
  KLC_ERR_CUDA = 4,           /* a CUDA runtime / driver call failed         */
  KLC_ERR_DEVICE_TIMEOUT = 5, /* a bounded device-side wait gave up          */
  KLC_ERR_DEVICE_FAULT = 6,   /* a device-side check recorded a bad index    */
  KLC_ERR_NCCL = 7            /* a collective failed                         */
};

/* ---- dtype enum ------------------------------------------------------ */
enum klc_dtype { KLC_BF16 = 0, KLC_F16 = 1, KLC_F32 = 2 };

/* ---- expert math precision (the reference's matmul_precision) ----------
 * KLC_PREC_FP32: gu = x @ Wgu + b in fp32, out = gated @ Wd + b in fp32
 *                (streamed_moe_router.py:505,511).
 * KLC_PREC_BF16: both products rounded to bf16 before the fp32 bias add
 *                (streamed_moe_router.py:502-503,507-509).                 */
enum klc_precision { KLC_PREC_FP32 = 0, KLC_PREC_BF16 = 1 };

/* ---- expert kernel selection ------------------------------------------ */
enum klc_expert_path {
  KLC_PATH_AUTO = 0, /* tcgen05 grouped GEMM when available, else SIMT       */
  KLC_PATH_SIMT = 1, /* CUDA-core dequant + FMA kernels                      */
  KLC_PATH_TC = 2    /* tcgen05 block-scaled MMA on the packed E2M1 weights  */
};

int klc_version(void);
const char* klc_last_error(void);
/* Expert paths built into this library: bit 0 = KLC_PATH_SIMT,
 * bit 1 = KLC_PATH_TC (tcgen05). */
int klc_capabilities(int* flags);
/* Number of SMs of the current device (for host-side planning). */
int klc_device_sm_count(int* out_sms);
/* Kernels this library has launched in the process so far (all threads and
 * devices; a launch that failed is counted too).  No reference counterpart:
 * measurement support, e.g. launches per step.                            */
int klc_launch_count(uint64_t* out);
/* Self-test of the bounded device waits (no reference counterpart): a
 * kernel waits on an mbarrier nothing arrives on, gives up after
 * limit_cycles SM cycles and records KLC_ERR_DEVICE_TIMEOUT (site 999);
 * *code / *where receive the recorded status (synchronises `stream`).
 * Returns KLC_OK when the self-test ran; the GPU stays usable.             */
int klc_selftest_wait_timeout(int64_t limit_cycles, int* code, int* where, void* stream);
/* sizeof(klc_moe_dims) and sizeof(klc_moe_weights) as this library was
 * compiled, for bindings to check their own structure layouts against.    */
int klc_struct_sizes(size_t* dims_bytes, size_t* weights_bytes);
/* sizeof one structure of this header: 0 klc_moe_dims, 1 klc_moe_weights,
 * 2 klc_locality_config, 3 klc_next_router (KLC_ERR_INVALID for others). */
int klc_struct_size(int which, size_t* out_bytes);
/* enable != 0 (the default): the kernels of a layer call (router, permute,
 * quantize, expert GEMMs, combine) are launched with programmatic dependent
 * launch, so each launches while its predecessor finishes; 0: plain stream
 * order.  Results are identical either way; process-wide. */
int klc_set_pdl(int enable);
/* Two-SM expert tiles (tensor-core path, weights-as-N kernels, 64-row
 * blocks): a pair of SMs computes two consecutive row-blocks of one expert
 * with one 256-row block-scaled MMA, each SM loading half of the weight
 * tile.  mode 0: never; 1 (the default): when the layer averages at least
 * 192 rows per expert; 2: whenever the 64-row kernels run.  The layer
 * output is identical in every mode; process-wide. */
int klc_set_pair_tiles(int mode);
/* enable != 0 (the default): the tensor-core gate_up kernel (weights-as-N
 * forms with 64-row or two-SM tiles) writes the down GEMM's operand, the
 * hi/lo E4M3 rows and their scale blocks, straight from its SwiGLU epilogue,
 * and the separate quantize pass over the gated rows is skipped; 0: bf16
 * gated rows, then that pass (16-row decode tiles always take the pass).
 * The layer output is identical either way; process-wide. */
int klc_set_fused_quantize(int enable);

/* ---- MXFP4 dequant ---------------------------------------------------- *
 * Replaces dequantize_mxfp4_matrix(blocks, scales, dtype)
 * (mxfp4_expert.py:357-379).  blocks uint8 [out_dim, groups, 16], scales uint8
 * [out_dim, groups]; writes out [groups*32, out_dim] (the transposed [in, out]
 * matrix) in `out_dtype`.  Bit-exact: FP4[nibble] * 2^(scale-127) rounded
 * once to the target type, low nibble = even K index.                     */
int klc_mxfp4_dequant(const uint8_t* blocks, const uint8_t* scales, int64_t out_dim, int64_t groups,
                      void* out, int out_dtype, void* stream);

/* One-time re-layout of E8M0 scales [E, rows, groups] -> [E, groups, rows]
 * (the layout the expert kernels read).  No counterpart in the reference,
 * which stores scales as [E, rows, groups] (checkpoint layout).           */
int klc_mxfp4_transpose_scales(const uint8_t* scales, int64_t experts, int64_t rows, int64_t groups,
                               uint8_t* scales_t, void* stream);

/* Scales for the tensor-core (block-scaled MMA) path, once per layer: the
 * same scales re-laid as the 512-byte blocks the MMA's scale copies read,
 * one per (expert, 128-row tile, 128-K stage): byte r0*16 + r1*4 + kb is the
 * scale of row r0 + 32*r1, 32-K block kb; entries past the matrix are 0.
 * Output size (klc_mxfp4_scales_mx_bytes) = E * ceil(rows/128) *
 * ceil(groups/4) * 512 bytes.
 * No reference counterpart: layout preparation for the B200 kernel, like
 * the transpose above.                                                     */
/* Expert blocks [E, rows, groups, 16] -> [E, rows, groups_pad, 16] with
 * groups_pad = ceil(groups / 4) * 4 (each row's K padded to a multiple of 128
 * values with zero bytes), once per layer: the layout the tensor-core path
 * loads with TMA's 4-bit unpacking copy.  No reference counterpart (layout
 * preparation for the B200 kernel).  out must hold E*rows*groups_pad*16 bytes. */
int klc_mxfp4_pad_k128(const uint8_t* blocks, int64_t experts, int64_t rows, int64_t groups, uint8_t* out, void* stream);

/* Scales [E, rows, groups] in tiles of tile_rows (<= 256) rows: block
 * [e][t][stage][chunk] of 512 bytes per 128-K stage and 128-row chunk of the
 * tile, byte (m % 32)*16 + (m / 32)*4 + kb = scale of tile row chunk*128 + m,
 * 32-K block kb; zero past the matrix.  tile_rows 128 gives the
 * klc_mxfp4_scales_mx layout; 192 the tiles of the weights-as-N kernels.
 * No reference counterpart (layout preparation for the B200 kernel).     */
int klc_mxfp4_scales_tile_bytes(int64_t experts, int64_t rows, int64_t groups, int tile_rows, size_t* out_bytes);
int klc_mxfp4_scales_tile(const uint8_t* scales, int64_t experts, int64_t rows, int64_t groups, int tile_rows, uint8_t* out,
                          void* stream);

int klc_mxfp4_scales_mx_bytes(int64_t experts, int64_t rows, int64_t groups, size_t* out_bytes);
int klc_mxfp4_scales_mx(const uint8_t* scales, int64_t experts, int64_t rows, int64_t groups, uint8_t* out,
                        void* stream);

/* Activation operand of the tensor-core path: each bf16 row [K] split into
 * two E4M3 rows hi, lo with one E8M0 scale per 32 values (S = floor(log2
 * block max) - 7; hi = x with its low four mantissa bits cleared, lo = x -
 * hi, both / 2^S), so hi + lo == x exactly for |x| within 2^9 of the block
 * maximum.  x bf16 [rows, K]; q u8 [rows, 2, K] (hi row, lo row); scales u8
 * [rows, K/32].  The expert kernels run the same split on the permuted
 * rows; this entry exposes it for callers and tests.  No reference
 * counterpart (the reference multiplies bf16 activations directly).       */
int klc_mx_quantize_rows(const uint16_t* x, int64_t rows, int64_t K, uint8_t* q, uint8_t* scales, void* stream);

/* ---- router ------------------------------------------------------------ *
 * Replaces the router part of StreamedMoERouter.route
 * (streamed_moe_router.py:269-284): logits = bf16(x @ W^T + b) with fp32
 * accumulation; selection = top-k of (logits + adjust) by value, ties to the
 * lower expert index; weights = softmax over the selected fp32 scores,
 * rounded to bf16.  x bf16 [T,H], w bf16 [E,H], b bf16 [E]; adjust fp32 [E]
 * or NULL (the host-built locality bias vector); out_idx int32 [T,k];
 * out_w bf16 [T,k]; out_logits bf16 [T,E] or NULL.  Requires k <= 8, E <= 1024. */
int klc_router_topk(const uint16_t* x, int64_t tokens, int64_t hidden, const uint16_t* w, const uint16_t* b,
                    int64_t experts, int k, const float* adjust, int32_t* out_idx, uint16_t* out_w,
                    uint16_t* out_logits, void* stream);

/* Device faults of the router (a bounded wait of the tensor-core form that
 * timed out): synchronises `stream`, returns KLC_OK or the recorded status
 * (and its site) and clears it.  No reference counterpart.                */
int klc_router_status(int* code, int* where, void* stream);

/* Selection + softmax on given fp32 scores [T, E] (the locality path: the
 * host applies the reference's bias / guard policy, streamed_moe_router.py:
 * 331-394, to logits read back from klc_router_topk).  keep_order != 0:
 * the row holds exactly k scores in the wanted order (E == k) and only the
 * softmax is computed; out_idx may then be NULL.                          */
int klc_select_softmax(const float* scores, int64_t tokens, int64_t experts, int k, int keep_order, int32_t* out_idx,
                       uint16_t* out_w, void* stream);

/* ---- full layer workspace ---------------------------------------------- */
typedef struct klc_moe_dims {
  int64_t tokens;       /* T                                    */
  int64_t hidden;       /* H (multiple of 64)                   */
  int64_t intermediate; /* I (multiple of 64)                   */
  int64_t experts;      /* E experts held by this call          */
  int32_t top_k;        /* k                                    */
  int32_t path;         /* enum klc_expert_path                 */
} klc_moe_dims;

/* Bytes of device workspace klc_moe_forward / klc_moe_experts need. */
int klc_moe_workspace_size(const klc_moe_dims* dims, size_t* out_bytes);

/* Packed expert weights of one layer, all device pointers.
 * gu_blocks  uint8 [E, 2I, H/32, 16]   gate_up_proj_blocks (checkpoint layout)
 * gu_scales_t uint8 [E, H/32, 2I]      gate_up_proj_scales re-laid by klc_mxfp4_transpose_scales
 * gu_bias    bf16 [E, 2I]
 * dn_blocks  uint8 [E, H, I/32, 16]    down_proj_blocks
 * dn_scales_t uint8 [E, I/32, H]
 * dn_bias    bf16 [E, H]
 * router_w   bf16 [E, H], router_b bf16 [E]
 * gu_scales_mx / dn_scales_mx: the scales re-laid by klc_mxfp4_scales_mx;
 *            required by the tensor-core path, may be NULL for SIMT       */
typedef struct klc_moe_weights {
  const uint8_t* gu_blocks;
  const uint8_t* gu_scales_t;
  const uint16_t* gu_bias;
  const uint8_t* dn_blocks;
  const uint8_t* dn_scales_t;
  const uint16_t* dn_bias;
  const uint16_t* router_w;
  const uint16_t* router_b;
  float swiglu_limit; /* 7.0   (streamed_moe_router.py:242) */
  float alpha;        /* 1.702 (streamed_moe_router.py:248) */
  const uint8_t* gu_scales_mx; /* klc_mxfp4_scales_mx of gate_up_proj_scales (tensor-core path) */
  const uint8_t* dn_scales_mx; /* klc_mxfp4_scales_mx of down_proj_scales */
  /* gate_up / down blocks with every row's K padded to a multiple of 128
   * values (klc_mxfp4_pad_k128): the tensor-core path then loads them
   * straight into its MMA operand layout.  NULL: the blocks themselves when K
   * is already a multiple of 128, else the tensor-core path stages them
   * through its repack warps.                                               */
  const uint8_t* gu_blocks_k128;
  const uint8_t* dn_blocks_k128;
  /* gate_up / down scales in 192-row tiles (klc_mxfp4_scales_tile with
   * tile_rows 192): with the padded blocks above (and 16-byte aligned
   * biases) the tensor-core path runs its weights-as-N = 192 kernels.      */
  const uint8_t* gu_scales_t192;
  const uint8_t* dn_scales_t192;
} klc_moe_weights;

/* Expert execution + combine for given routing (idx, weights), the body of
 * _execute_mxfp4_experts (streamed_moe_router.py:483-522) batched over T
 * tokens: permute/gather, gate_up GEMM + bias + clamped SwiGLU, down GEMM +
 * bias, bf16 combine in selection order.  x bf16 [T,H]; idx int32 [T,k]
 * (values in [0,E)); w bf16 [T,k]; y bf16 [T,H].  norms fp32 [T,k,2] or NULL
 * receives (||gated||, ||out||) per pair (the expert_logs of :514-521).
 * residual: if non-NULL, y = residual + moe_out (bf16 add).               */
int klc_moe_experts(const klc_moe_dims* dims, const klc_moe_weights* wts, const uint16_t* x, const int32_t* idx,
                    const uint16_t* w, int precision, uint16_t* y, float* norms, const uint16_t* residual,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free variant of klc_moe_experts (no counterpart in the
 * reference).  For callers that cannot allocate device memory themselves --
 * e.g. a host runtime reaching this library through an FFI without a CUDA
 * allocator, or an application whose device memory belongs to another pool.
 * Same arguments and argument checks as klc_moe_experts minus the workspace;
 * the scratch is a static 16 MiB device array inside the library (held by
 * every GPU that loads it until the process exits;
 * klc_moe_noalloc_scratch_bytes reports the size).  Always runs the
 * CUDA-core expert kernels.  A batch whose scratch would exceed the array is
 * rejected with KLC_ERR_INVALID.  The first call on a device looks up the
 * array's address (cudaGetSymbolAddress): make it before any stream capture
 * on that device; the address is cached for the process, so do not call the
 * library again after cudaDeviceReset.  All calls on a device share the
 * array, so calls that overlap on the GPU race: serialise them.  Calls no
 * cudaMalloc/cudaFree or allocating library routine.
 * klc_moe_noalloc_status reads the device status word of the last call on
 * the current device (as klc_workspace_status does for a workspace): an
 * expert id outside [0, E) is reported as KLC_ERR_DEVICE_FAULT.            */
int klc_moe_experts_noalloc(const klc_moe_dims* dims, const klc_moe_weights* wts, const uint16_t* x, const int32_t* idx,
                            const uint16_t* w, int precision, uint16_t* y, float* norms, const uint16_t* residual,
                            void* stream);
int klc_moe_noalloc_scratch_bytes(size_t* out_bytes);
int klc_moe_noalloc_status(int* code, int* where, int* detail, void* stream);

/* Router + experts + combine in one call (StreamedMoERouter.route batched).
 * out_idx/out_w receive the routing (int32 [T,k], bf16 [T,k]); out_logits
 * bf16 [T,E] or NULL; adjust fp32 [E] or NULL.                            */
int klc_moe_forward(const klc_moe_dims* dims, const klc_moe_weights* wts, const uint16_t* x, const float* adjust,
                    int precision, uint16_t* y, int32_t* out_idx, uint16_t* out_w, uint16_t* out_logits,
                    float* norms, const uint16_t* residual, void* workspace, size_t workspace_bytes, void* stream);

/* Weighted combine of expert output rows back to tokens
 * (streamed_moe_router.py:497,512-513): for each token t, in slot order s,
 * out[t] = bf16(out[t] + bf16(y_rows[pair_pos[t*k+s]] * w[t,s])), starting
 * from zero (or from residual[t] added at the end when residual != NULL).
 * y_rows bf16 [*, H]; pair_pos int32 [T*k]; w bf16 [T,k]; out bf16 [T,H]. */
int klc_moe_combine(const uint16_t* y_rows, const int32_t* pair_pos, const uint16_t* w, int64_t tokens, int k,
                    int64_t hidden, const uint16_t* residual, uint16_t* out, void* stream);

/* klc_moe_combine with residual, fused with the next layer's input RMSNorm:
 * out = residual + combine (bf16, as klc_moe_combine; residual may be NULL)
 * and normed = bf16(bf16(out * bf16(rsqrt(mean(out^2) + eps))) * norm_w), the
 * executor's `hidden += moe_out` (streamed_transformer_executor.py:260)
 * followed by the next layer's rms_norm(hidden, input_layernorm.weight)
 * (:235, streamed_attention.py:27-28).  norm_w bf16 [H]; normed bf16 [T,H];
 * norm_w and normed 16-byte aligned.                                       */
int klc_moe_combine_rmsnorm(const uint16_t* y_rows, const int32_t* pair_pos, const uint16_t* w, int64_t tokens, int k,
                            int64_t hidden, const uint16_t* residual, const uint16_t* norm_w, float eps, uint16_t* out,
                            uint16_t* normed, void* stream);

/* klc_moe_forward whose combine also writes the next layer's RMSNorm input
 * (normed, as klc_moe_combine_rmsnorm): one decode layer's MoE half plus
 * the residual add and the following norm, without a separate norm launch
 * or a re-read of y.                                                       */
int klc_moe_forward_rmsnorm(const klc_moe_dims* dims, const klc_moe_weights* wts, const uint16_t* x,
                            const float* adjust, int precision, uint16_t* y, int32_t* out_idx, uint16_t* out_w,
                            uint16_t* out_logits, float* norms, const uint16_t* residual, const uint16_t* norm_w,
                            float eps, uint16_t* normed, void* workspace, size_t workspace_bytes, void* stream);

/* execute_experts=False path (streamed_moe_router.py:317-329):
 * y[t] = sum_s bf16(bias[idx[t,s]] * w[t,s]) accumulated in fp32, rounded once. */
int klc_moe_bias_only(const uint16_t* dn_bias, int64_t tokens, int64_t hidden, int k, const int32_t* idx,
                      const uint16_t* w, uint16_t* y, void* stream);

/* The next layer's router fused into the combine (decode): after the
 * residual add and the next layer's input RMSNorm (as klc_moe_forward_rmsnorm /
 * klc_moe_combine_rmsnorm), the normalised rows are routed for the next layer
 * (streamed_moe_router.py:269-282 on streamed_transformer_executor.py:247's
 * `post`): router_w bf16 [E,H], router_b bf16 [E], k <= 8, E <= 1024;
 * out_idx int32 [T,k], out_w bf16 [T,k], out_logits bf16 [T,E] or NULL.  The
 * router kernels follow the combine in the same call (logits computed inside the
 * combine, one CTA per token streaming all router rows, measured slower).  No
 * locality adjustment. */
typedef struct klc_next_router {
  const uint16_t* router_w;
  const uint16_t* router_b;
  int64_t experts;
  int k;
  int32_t* out_idx;
  uint16_t* out_w;
  uint16_t* out_logits;
} klc_next_router;
int klc_moe_forward_rmsnorm_route(const klc_moe_dims* dims, const klc_moe_weights* wts, const uint16_t* x,
                                  const float* adjust, int precision, uint16_t* y, int32_t* out_idx, uint16_t* out_w,
                                  uint16_t* out_logits, float* norms, const uint16_t* residual, const uint16_t* norm_w,
                                  float eps, uint16_t* normed, const klc_next_router* next, void* workspace,
                                  size_t workspace_bytes, void* stream);
/* Experts + combine for given routing (klc_moe_experts) + residual + RMSNorm + next router. */
int klc_moe_experts_rmsnorm_route(const klc_moe_dims* dims, const klc_moe_weights* wts, const uint16_t* x,
                                  const int32_t* idx, const uint16_t* w, int precision, uint16_t* y, float* norms,
                                  const uint16_t* residual, const uint16_t* norm_w, float eps, uint16_t* normed,
                                  const klc_next_router* next, void* workspace, size_t workspace_bytes, void* stream);
int klc_moe_combine_rmsnorm_route(const uint16_t* y_rows, const int32_t* pair_pos, const uint16_t* w, int64_t tokens,
                                  int k, int64_t hidden, const uint16_t* residual, const uint16_t* norm_w, float eps,
                                  uint16_t* out, uint16_t* normed, const klc_next_router* next, void* stream);

/* Stable counting-sort permutation of (token, slot) pairs by expert.
 * idx int32 [T,k]; writes pair_pos int32 [T*k] (padded row of each pair),
 * counts int32 [E], offsets int32 [E+1] (each group padded to `pad` rows)
 * and rows int32 [rows_cap] (pair id per padded row, -1 in padding).
 * rows_cap >= T*k + E*(pad-1).  Uses `workspace` (klc_moe_workspace_size). */
int klc_moe_permute(const int32_t* idx, int64_t tokens, int k, int64_t experts, int pad, int32_t* pair_pos,
                    int32_t* counts, int32_t* offsets, int32_t* rows, int64_t rows_cap, void* workspace,
                    size_t workspace_bytes, void* stream);

/* Per-stage timing of the layer entry points on the calling host thread.
 * klc_stage_timing(1) makes klc_moe_forward / klc_moe_experts record a CUDA
 * event on their stream at each stage boundary; klc_stage_times then
 * synchronises on those events and writes the milliseconds of the last call
 * for [router, permute+gather, gate_up GEMM, down GEMM, combine] (-1 where
 * the stage did not run), and the number of stages measured to *n_out.    */
int klc_stage_timing(int enable);
int klc_stage_times(float* ms, int max_stages, int* n_out);

/* Read back the device status word at the start of a workspace used by
 * klc_moe_experts / klc_moe_forward / klc_moe_permute (synchronises
 * `stream`).  Returns KLC_OK, or the device-side error a kernel recorded
 * (KLC_ERR_DEVICE_FAULT for an out-of-range expert index,
 * KLC_ERR_DEVICE_TIMEOUT for a bounded wait that gave up); code/where/detail
 * may be NULL.                                                             */
int klc_workspace_status(const void* workspace, int* code, int* where, int* detail, void* stream);

/* Expert-parallel dispatch packing (no counterpart in the reference, which
 * runs on one device).  Experts are sharded contiguously: rank r owns
 * experts [r*experts_per_rank, (r+1)*experts_per_rank).  Groups the (token,
 * slot) pairs of idx int32 [T,k] by destination rank (stable: token-major,
 * slot-minor) and writes send_rows bf16 [T*k, H] (x[token] of each pair in
 * that order), send_expert int32 [T*k] (the pair's expert id local to its
 * rank), send_counts int32 [nranks] and pair_pos int32 [T*k] (send row of
 * each pair, the input klc_moe_combine needs once the expert outputs come
 * back in the same order).  Workspace: klc_moe_workspace_size with dims
 * {T, 64, 64, max(nranks, k), k, KLC_PATH_SIMT}.                            */
int klc_ep_pack(const int32_t* idx, int64_t tokens, int k, int64_t experts_per_rank, int nranks, const uint16_t* x,
                int64_t hidden, uint16_t* send_rows, int32_t* send_expert, int32_t* send_counts, int32_t* pair_pos,
                void* workspace, size_t workspace_bytes, void* stream);

/* Locality-aware routing on the device (replaces the host steps of
 * StreamedMoERouter.route when RoutingLocalityConfig.enabled,
 * streamed_moe_router.py:270-302: raw top-k, _apply_locality_bias :331-363,
 * adjusted top-k, _guarded_expert_selection :365-394, softmax, predict_experts
 * :426-440, _update_sticky_scores / _update_workload_scores :396-424).  The
 * fields are RoutingLocalityConfig's (:12-35) with experts_per_token the
 * router's; Python bools as 0/1.  The policy state (sticky and workload scores,
 * recent-expert history) lives in a caller-owned device buffer of
 * klc_locality_state_bytes, zero-filled before first use, one per layer; each
 * call continues it over `tokens` rows of bf16 logits [T,E] in order.  Per
 * token t: resident (or NULL) is a 0/1 byte mask [E] of resident experts at
 * resident + t*resident_stride (stride 0: one mask for all tokens); k the
 * active expert count (the caller applies the dynamic cap).  Outputs:
 * out_experts int32 [T,k] (guarded, in the reference's order), out_w bf16
 * [T,k], out_raw int32 [T,k] (topk of the raw logits), out_pred int32 [T,k]
 * with out_npred[t] valid entries (the prediction before token t's update;
 * 0 when predictive_prefetch is off), out_flags uint8 [T] (bit 0: the guard
 * replaced an expert, bit 1: experts != raw).  Exact ties resolve as
 * torch.topk on the CPU does.  One warp walks the tokens in order (latency
 * kernel, meant for decode batches). */
typedef struct klc_locality_config {
  double sticky_strength;
  double sticky_candidate_margin;
  double max_sticky_bonus;
  double exploration_margin;
  double cache_aware_strength;
  double sticky_decay;
  double workload_window;
  int32_t semantic_guard;
  int32_t min_raw_overlap;
  int32_t max_hot_experts;
  int32_t prediction_window;
  int32_t predictive_prefetch;
  int32_t experts_per_token;
} klc_locality_config;
int klc_locality_state_bytes(int64_t experts, int prediction_window, size_t* out_bytes);
int klc_locality_route(const klc_locality_config* cfg, const uint16_t* logits, int64_t tokens, int64_t experts, int k,
                       const uint8_t* resident, int64_t resident_stride, void* state, size_t state_bytes,
                       int32_t* out_experts, uint16_t* out_w, int32_t* out_raw, int32_t* out_pred, int32_t* out_npred,
                       uint8_t* out_flags, void* stream);

/* ---- expert parallelism over NVLink peer memory ------------------------
 * No counterpart in the reference (one process, one device): the node-level
 * sharding of the MoE block, rank r owning experts [r*epr, (r+1)*epr).  One
 * handle per rank (one process per GPU).  Each handle owns an exchange arena
 * in its device's memory (cudaMalloc'd by klc_ep_create, freed by
 * klc_ep_destroy; klc_ep_arena_bytes reports the size: two row buffers of
 * world * max_tokens * top_k * hidden bf16 plus small tables) that the other
 * ranks map through CUDA IPC.  Setup: klc_ep_create on every rank ->
 * klc_ep_ipc_handle (64 bytes) -> exchange the handles between the ranks by
 * any host transport -> klc_ep_connect with all handles in rank order.
 * Per forward, on every rank, in the same order: klc_ep_dispatch ->
 * klc_ep_experts -> klc_ep_combine (or klc_ep_forward for all of it, router
 * included).  Stream-ordered; no host synchronisation; kernels of different
 * ranks signal each other through flags in the arenas with bounded waits
 * (klc_ep_set_wait_limit_ns, default 10 s; an expired wait is reported by
 * klc_ep_status as KLC_ERR_DEVICE_TIMEOUT).  A handle serves one stream of
 * one host thread at a time.  Before klc_ep_destroy every rank must have
 * finished its last forward (a host barrier): peers write into the arena.
 *
 * klc_ep_dispatch: idx int32 [T,k] (global expert ids), x bf16 [T,H]; sends
 *   every (token, slot) pair's row to its owner and writes pair_slot int32
 *   [T*k] (where its expert output will come back; input of klc_ep_combine).
 * klc_ep_experts: the local experts (klc_moe_weights of this rank's experts,
 *   dims {_, H, I, epr, _, path}) on every row received, outputs sent back.
 * klc_ep_combine: waits for the returned rows, then the weighted bf16 combine
 *   in top-k order (klc_moe_combine), optional residual, optional fused
 *   next-layer RMSNorm (norm_w/normed as klc_moe_combine_rmsnorm).
 * Workspace (caller-owned, shared by the three calls): klc_ep_workspace_size. */
typedef struct klc_ep klc_ep;
int klc_ep_create(int rank, int world, int64_t max_tokens, int top_k, int64_t hidden, int64_t experts_per_rank,
                  klc_ep** out);
int klc_ep_arena_bytes(const klc_ep* h, size_t* out_bytes);
int klc_ep_ipc_handle(const klc_ep* h, void* out_64_bytes);
int klc_ep_connect(klc_ep* h, const void* handles_world_x_64_bytes);
int klc_ep_set_wait_limit_ns(klc_ep* h, uint64_t ns);
/* enable != 0: with the weights-as-N tensor-core kernels and at most 8 ranks,
 * the down-projection epilogue of klc_ep_experts stores every expert output row
 * straight into its source rank's arena over NVLink, so the return transfer
 * overlaps the GEMM; 0: the rows go through the workspace and a separate copy
 * kernel.  Both give identical results.  Default: on for 2 ranks, off above
 * (where the epilogue's peer stores measured slower than the copy). */
int klc_ep_set_fused_return(klc_ep* h, int enable);
int klc_ep_workspace_size(const klc_ep* h, const klc_moe_dims* local_dims, size_t* out_bytes);
int klc_ep_dispatch(klc_ep* h, const int32_t* idx, int64_t tokens, const uint16_t* x, int32_t* pair_slot, void* workspace,
                    size_t workspace_bytes, void* stream);
int klc_ep_experts(klc_ep* h, const klc_moe_dims* local_dims, const klc_moe_weights* local_wts, int precision,
                   void* workspace, size_t workspace_bytes, void* stream);
int klc_ep_combine(klc_ep* h, const int32_t* pair_slot, const uint16_t* w, int64_t tokens, const uint16_t* residual,
                   const uint16_t* norm_w, float eps, uint16_t* out, uint16_t* normed, void* stream);
/* klc_ep_combine with the next layer's router on the normalised rows (see
 * klc_next_router); norm_w / normed required. */
int klc_ep_combine_route(klc_ep* h, const int32_t* pair_slot, const uint16_t* w, int64_t tokens, const uint16_t* residual,
                         const uint16_t* norm_w, float eps, uint16_t* out, uint16_t* normed, const klc_next_router* next,
                         void* stream);
/* Router (klc_router_topk over all epr*world experts) + dispatch + experts +
 * combine: one expert-parallel MoE layer forward on this rank's tokens.     */
int klc_ep_forward(klc_ep* h, const klc_moe_dims* local_dims, const klc_moe_weights* local_wts, const uint16_t* router_w,
                   const uint16_t* router_b, const uint16_t* x, int64_t tokens, int precision, const uint16_t* residual,
                   const uint16_t* norm_w, float eps, uint16_t* out, uint16_t* normed, int32_t* out_idx, uint16_t* out_w,
                   int32_t* pair_slot, void* workspace, size_t workspace_bytes, void* stream);
/* Device status of the exchange (bounded waits, counts) and of the last
 * dispatch / local-expert index checks in `workspace` (may be NULL);
 * synchronises `stream` and clears the arena's word.                       */
int klc_ep_status(klc_ep* h, const void* workspace, int* code, int* where, void* stream);
/* Rows this rank received in its last dispatch (sum over sources; synchronises). */
int klc_ep_received_rows(klc_ep* h, int64_t* out, void* stream);
int klc_ep_destroy(klc_ep* h);

/* RMSNorm (streamed_attention.py:27-28): y = bf16(bf16(x * bf16(rsqrt(mean(x^2)+eps))) * w). */
int klc_rms_norm(const uint16_t* x, const uint16_t* w, int64_t rows, int64_t hidden, float eps, uint16_t* y,
                 void* stream);

/* ---- runtime dequantizer (RuntimeDequantizer.dequantize) ---------------
 * Replaces runtime_dequantizer.py:30-52 (with unpack_lowbit,
 * adaptive_quantizer.py:183-213, and reconstruct_pruned,
 * tensor_pruner.py:62-69).  Writes `numel` elements of `out_dtype`:
 *   mode 0 ("fp16"):   out = data                  data_dtype bf16/f16/f32
 *   mode 1 (packed q1-q4, bits 1..4): out = unpack_lowbit(data) * scale[0];
 *                      data uint8, `count` bytes
 *   mode 2 (unpacked q8/q16, bits 8 or 16): out = int(data) * scale[0]
 *   mode 3 ("pruned"): out = 0, then out[index[j]] = data[j] for j < count;
 *                      data_dtype bf16/f16/f32, index int64
 * Products are formed in fp32 and rounded once to out_dtype, as the
 * reference's q.float() * scale.float() then .to(dtype).                  */
int klc_runtime_dequant(int mode, const void* data, int data_dtype, const float* scale, const int64_t* index,
                        int64_t count, int bits, int64_t numel, void* out, int out_dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KLC_MOE_H */
