// Shared helpers of libklcmoe: status plumbing, bf16/MXFP4 arithmetic,
// bounded waits.  Internal header (the public ABI is include/klc_moe.h).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "klc_moe.h"

namespace klc {

// ---------------------------------------------------------------------------
// host-side status plumbing
// ---------------------------------------------------------------------------
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_check(cudaError_t e, const char* what);
void note_launch();

#define KLC_CHECK_ARG(cond, msg)                               \
  do {                                                         \
    if (!(cond)) return ::klc::fail(KLC_ERR_INVALID, (msg));   \
  } while (0)

#define KLC_CUDA(call)                                              \
  do {                                                              \
    int _st = ::klc::cuda_check((call), #call);                     \
    if (_st != KLC_OK) return _st;                                  \
  } while (0)

// Every kernel launch of the library is followed by this check, which also
// counts the launch (klc_launch_count).
#define KLC_LAUNCH_CHECK(what)                                      \
  do {                                                              \
    ::klc::note_launch();                                           \
    int _st = ::klc::cuda_check(cudaGetLastError(), what);          \
    if (_st != KLC_OK) return _st;                                  \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

int sm_count();

// ---------------------------------------------------------------------------
// programmatic dependent launch: the kernels of a layer's chain may be launched
// while their predecessor still runs (launch latency and set-up overlap its
// tail); each of them calls pdl_wait() before it reads anything the
// predecessor wrote, and pdl_trigger() to let its own successor launch early.
// Both are no-ops for a kernel launched without the attribute.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

bool pdl_enabled();  // klc_set_pdl, default on
int pair_tiles_mode();  // klc_set_pair_tiles: 0 never, 1 by rows per expert (default), 2 always
bool fused_quantize_enabled();  // klc_set_fused_quantize, default on

// cudaLaunchKernelEx with the programmatic-serialization attribute (when enabled)
// plus, for cluster_x >= 1, a cluster of cluster_x CTAs (0: no cluster launch)
template <typename... KArgs, typename... Args>
inline cudaError_t launch_chain(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x >= 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = n > 0 ? attr : nullptr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------
// device status word (lives at the start of every workspace)
// ---------------------------------------------------------------------------
struct DeviceStatus {
  int code;      // 0 ok, else KLC_ERR_DEVICE_TIMEOUT / KLC_ERR_DEVICE_FAULT
  int where;     // kernel-defined site id
  int detail;    // e.g. the bad index
  int rowblocks; // number of row-blocks the permute produced
  int pairblocks; // number of paired row-blocks (two-SM tiles), when the permute built them
};

__device__ __forceinline__ void record_fault(DeviceStatus* st, int code, int where, int detail) {
  if (st != nullptr && atomicCAS(&st->code, 0, code) == 0) {
    st->where = where;
    st->detail = detail;
  }
}

// ---------------------------------------------------------------------------
// bf16 bit helpers (round-to-nearest-even, as torch)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16_to_f32(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

__device__ __forceinline__ float round_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }

// ---------------------------------------------------------------------------
// MXFP4 (E2M1 value x E8M0 block scale) exact arithmetic
// ---------------------------------------------------------------------------
// E2M1 nibble -> fp32, exact.  The 3 magnitude bits are placed at the top of
// the fp32 exponent/mantissa field (value = FP4 * 2^-126, possibly subnormal)
// and rescaled by an exact power of two.
__device__ __forceinline__ float fp4_to_f32(uint32_t nib) {
  float tiny = __uint_as_float(((nib & 8u) << 28) | ((nib & 7u) << 22));
  return tiny * 0x1p126f;
}

// v * 2^(s-127) with one rounding at most (exact for E2M1 inputs unless the
// result overflows, which gives +/-inf like the exact value would in fp32).
__device__ __forceinline__ float e8m0_scale(float v, uint32_t s) {
  if (s == 255u) return (v * 2.0f) * 0x1p127f;
  float m = (s >= 1u) ? __uint_as_float(s << 23) : __uint_as_float(0x00400000u);  // 2^(s-127)
  return v * m;
}

// ---------------------------------------------------------------------------
// misc device helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace klc
