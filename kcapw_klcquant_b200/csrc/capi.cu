// Status / error plumbing of the C ABI.
#include <atomic>
#include <cstdio>
#include <string>

#include "klc_common.cuh"

namespace klc {

static thread_local std::string g_last_error;
static std::atomic<unsigned long long> g_launches{0};

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return KLC_OK;
  g_last_error = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  return KLC_ERR_CUDA;
}

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return n;
}

}  // namespace klc

extern "C" int klc_version(void) { return 1; }

extern "C" const char* klc_last_error(void) { return klc::g_last_error.c_str(); }

namespace klc {
bool tc_path_supported(int64_t hidden, int64_t inter);
}

extern "C" int klc_capabilities(int* flags) {
  if (flags == nullptr) return klc::fail(KLC_ERR_INVALID, "klc_capabilities: null output");
  *flags = 1 | (klc::tc_path_supported(2880, 2880) ? 2 : 0);
  return KLC_OK;
}

extern "C" int klc_device_sm_count(int* out_sms) {
  if (out_sms == nullptr) return klc::fail(KLC_ERR_INVALID, "klc_device_sm_count: null output");
  int dev = 0;
  KLC_CUDA(cudaGetDevice(&dev));
  KLC_CUDA(cudaDeviceGetAttribute(out_sms, cudaDevAttrMultiProcessorCount, dev));
  return KLC_OK;
}

extern "C" int klc_launch_count(uint64_t* out) {
  if (out == nullptr) return klc::fail(KLC_ERR_INVALID, "klc_launch_count: null output");
  *out = klc::g_launches.load(std::memory_order_relaxed);
  return KLC_OK;
}

extern "C" int klc_struct_sizes(size_t* dims_bytes, size_t* weights_bytes) {
  if (dims_bytes == nullptr || weights_bytes == nullptr) return klc::fail(KLC_ERR_INVALID, "klc_struct_sizes: null output");
  *dims_bytes = sizeof(klc_moe_dims);
  *weights_bytes = sizeof(klc_moe_weights);
  return KLC_OK;
}

namespace klc {
namespace {
std::atomic<bool> g_pdl{true};
std::atomic<int> g_pair_tiles{1};
std::atomic<bool> g_fused_quantize{true};
}  // namespace
bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed); }
bool fused_quantize_enabled() { return g_fused_quantize.load(std::memory_order_relaxed); }
int pair_tiles_mode() { return g_pair_tiles.load(std::memory_order_relaxed); }
}  // namespace klc

extern "C" int klc_set_pdl(int enable) {
  klc::g_pdl.store(enable != 0, std::memory_order_relaxed);
  return KLC_OK;
}

extern "C" int klc_set_fused_quantize(int enable) {
  klc::g_fused_quantize.store(enable != 0, std::memory_order_relaxed);
  return KLC_OK;
}

extern "C" int klc_set_pair_tiles(int mode) {
  if (mode < 0 || mode > 2) return klc::fail(KLC_ERR_INVALID, "klc_set_pair_tiles: mode must be 0, 1 or 2");
  klc::g_pair_tiles.store(mode, std::memory_order_relaxed);
  return KLC_OK;
}

extern "C" int klc_struct_size(int which, size_t* out_bytes) {
  if (out_bytes == nullptr) return klc::fail(KLC_ERR_INVALID, "klc_struct_size: null output");
  switch (which) {
    case 0: *out_bytes = sizeof(klc_moe_dims); return KLC_OK;
    case 1: *out_bytes = sizeof(klc_moe_weights); return KLC_OK;
    case 2: *out_bytes = sizeof(klc_locality_config); return KLC_OK;
    case 3: *out_bytes = sizeof(klc_next_router); return KLC_OK;
    default: return klc::fail(KLC_ERR_INVALID, "klc_struct_size: unknown structure");
  }
}
