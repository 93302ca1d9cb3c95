// Allocation-free variant of klc_moe_experts.
//
// Some callers cannot allocate device memory at the point where they run the
// MoE layer: a host runtime that reaches this library through a foreign
// function interface and has no CUDA allocator of its own, or an embedding
// application whose device memory is owned by another pool.  For them,
// klc_moe_experts_noalloc takes the same inputs and outputs as
// klc_moe_experts but no workspace: its scratch lives in a file-scope
// device array of fixed size (kNoAllocScratchBytes) that every GPU loading
// this library holds until the process exits.
//
// Contract:
//  * The first call on a device looks up the array's device address with
//    cudaGetSymbolAddress (with that device current) and caches it; make that
//    first call before any stream capture on that device.  The cached address
//    belongs to the device's primary context: after cudaDeviceReset (or any
//    teardown of that context) this library must not be called again in the
//    process.
//  * Device-side checks (an expert id outside [0, E)) record their status at
//    the start of the array; klc_moe_noalloc_status reads it back.
//  * The scratch is shared by every call on a device and keeps the previous
//    call's contents; the kernels clear what must start at zero.  Calls that
//    overlap on the GPU (different streams, or threads without ordering) race
//    on it: serialise them.
//  * It always runs the CUDA-core (SIMT) expert kernels with unpadded expert
//    groups, and rejects a problem whose scratch would exceed the array with
//    KLC_ERR_INVALID and a message giving the bytes it needs.
//  * It allocates nothing: no cudaMalloc, cudaFree or allocating library call.
#include <mutex>

#include "permute.cuh"

namespace klc {

int run_experts(const klc_moe_dims& d, const klc_moe_weights& wts, const uint16_t* x, const int32_t* idx,
                const uint16_t* w, int precision, uint16_t* y, float* norms, const uint16_t* residual, char* ws,
                const WorkspaceLayout& L, cudaStream_t stream);

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB per device
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once per device).
int scratch_address(char** out) {
  int dev = 0;
  KLC_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(KLC_ERR_UNSUPPORTED, "klc_moe_experts_noalloc: device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(KLC_ERR_CUDA, std::string("klc_moe_experts_noalloc: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = static_cast<char*>(g_scratch_ptr[dev]);
  return KLC_OK;
}

// Same buffers as the workspace of klc_moe_experts, with expert groups
// unpadded (pad 1) and the fp32 intermediate of the SIMT kernels.
WorkspaceLayout noalloc_layout(const klc_moe_dims& d) {
  WorkspaceLayout L{};
  L.pad = 1;
  L.block_n = 64;
  L.pairs = d.tokens * d.top_k;
  L.rows_cap = L.pairs;
  L.max_rowblocks = (L.pairs + L.block_n - 1) / L.block_n + d.experts;
  L.nchunks = (L.pairs + 1023) / 1024;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + (bytes > 0 ? bytes : 1), 256);
    return o;
  };
  L.status = take(sizeof(DeviceStatus));
  L.counts = take(size_t(d.experts) * 4);
  L.offsets = take(size_t(d.experts + 1) * 4);
  L.chunk_hist = take(size_t(L.nchunks > 0 ? L.nchunks : 1) * d.experts * 4);
  L.rows = take(size_t(L.rows_cap) * 4);
  L.pair_pos = take(size_t(L.pairs) * 4);
  L.rowblocks = take(size_t(L.max_rowblocks) * sizeof(int4));
  L.normsq = take(size_t(L.pairs) * 2 * 4);
  L.xp = take(size_t(L.rows_cap) * d.hidden * 2);
  L.gated = take(size_t(L.rows_cap) * d.intermediate * 4);
  L.y = take(size_t(L.rows_cap) * d.hidden * 2);
  L.total = off;
  return L;
}

}  // namespace

}  // namespace klc

extern "C" int klc_moe_experts_noalloc(const klc_moe_dims* dims, const klc_moe_weights* wts, const uint16_t* x,
                                       const int32_t* idx, const uint16_t* w, int precision, uint16_t* y, float* norms,
                                       const uint16_t* residual, void* stream) {
  using namespace klc;
  KLC_CHECK_ARG(dims != nullptr, "klc_moe_experts_noalloc: null dims");
  klc_moe_dims d = *dims;
  d.path = KLC_PATH_SIMT;
  // the same checks as klc_moe_experts (sizes, token bound, weight pointers
  // and their 16-byte alignment), before any size arithmetic or launch
  int st = validate_dims(&d);
  if (st != KLC_OK) return st;
  st = validate_weights(wts);
  if (st != KLC_OK) return st;
  KLC_CHECK_ARG(precision == KLC_PREC_FP32 || precision == KLC_PREC_BF16, "klc_moe_experts_noalloc: bad precision");
  if (d.tokens == 0) return KLC_OK;
  KLC_CHECK_ARG(x && idx && w && y, "klc_moe_experts_noalloc: null pointer");
  const WorkspaceLayout L = noalloc_layout(d);
  if (L.total > kNoAllocScratchBytes)
    return fail(KLC_ERR_INVALID, "klc_moe_experts_noalloc: this batch needs " + std::to_string(L.total) +
                                     " bytes of scratch, more than the " + std::to_string(kNoAllocScratchBytes) +
                                     "-byte static buffer; use klc_moe_experts with a caller workspace");
  char* scratch = nullptr;
  st = scratch_address(&scratch);
  if (st != KLC_OK) return st;
  return run_experts(d, *wts, x, idx, w, precision, y, norms, residual, scratch, L, as_stream(stream));
}

extern "C" int klc_moe_noalloc_status(int* code, int* where, int* detail, void* stream) {
  using namespace klc;
  char* scratch = nullptr;
  int st = scratch_address(&scratch);
  if (st != KLC_OK) return st;
  // the status word sits at offset 0 of the array (noalloc_layout)
  return klc_workspace_status(scratch, code, where, detail, stream);
}

extern "C" int klc_moe_noalloc_scratch_bytes(size_t* out_bytes) {
  KLC_CHECK_ARG(out_bytes != nullptr, "klc_moe_noalloc_scratch_bytes: null output");
  *out_bytes = klc::kNoAllocScratchBytes;
  return KLC_OK;
}
