// Device RuntimeDequantizer (runtime_dequantizer.py:30-52).
//
// The reference unpacks q1/q2/q3/q4 artefacts on the CPU (unpack_lowbit,
// adaptive_quantizer.py:183-213) before copying to the device and scaling;
// here one pass on the GPU reads the packed bytes and writes
// round(dtype, float(q) * scale).  Pruned tensors (tensor_pruner.py:62-69)
// are a zero fill plus a scatter.  All element-wise and HBM-bound.
#include "klc_common.cuh"

namespace klc {

namespace {

template <typename T>
__device__ __forceinline__ void store_as(void* out, int64_t i, float v);
template <>
__device__ __forceinline__ void store_as<uint16_t>(void* out, int64_t i, float v) {
  static_cast<uint16_t*>(out)[i] = f32_to_bf16(v);
}
template <>
__device__ __forceinline__ void store_as<__half>(void* out, int64_t i, float v) {
  static_cast<__half*>(out)[i] = __float2half_rn(v);
}
template <>
__device__ __forceinline__ void store_as<float>(void* out, int64_t i, float v) {
  static_cast<float*>(out)[i] = v;
}

__device__ __forceinline__ float load_float(const void* data, int dtype, int64_t i) {
  switch (dtype) {
    case KLC_BF16: return bf16_to_f32(static_cast<const uint16_t*>(data)[i]);
    case KLC_F16: return __half2float(static_cast<const __half*>(data)[i]);
    default: return static_cast<const float*>(data)[i];
  }
}

// signed integer value of element i of a packed low-bit tensor
__device__ __forceinline__ int unpack_one(const uint8_t* p, int64_t nbytes, int bits, int64_t i) {
  if (bits == 3) {
    const int64_t w = i / 8;
    uint32_t b0 = 0, b1 = 0, b2 = 0;
    if (3 * w < nbytes) b0 = p[3 * w];
    if (3 * w + 1 < nbytes) b1 = p[3 * w + 1];
    if (3 * w + 2 < nbytes) b2 = p[3 * w + 2];
    const uint32_t w24 = b0 | (b1 << 8) | (b2 << 16);
    return int((w24 >> (3 * (i % 8))) & 7u) - 4;
  }
  const int per = 8 / bits;
  const int64_t byte = i / per;
  const uint32_t v = (byte < nbytes) ? p[byte] : 0u;
  const uint32_t f = (v >> (bits * (i % per))) & ((1u << bits) - 1u);
  if (bits == 1) return f ? 1 : -1;
  return int(f) - (1 << (bits - 1));
}

template <typename OutT>
__global__ void runtime_dequant_kernel(int mode, const void* __restrict__ data, int data_dtype,
                                       const float* __restrict__ scale, int64_t count, int bits, int64_t numel,
                                       void* __restrict__ out) {
  const float s = (mode == 1 || mode == 2) ? scale[0] : 1.0f;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < numel; i += int64_t(gridDim.x) * blockDim.x) {
    float v;
    if (mode == 0) {
      v = load_float(data, data_dtype, i);
    } else if (mode == 1) {
      v = float(unpack_one(static_cast<const uint8_t*>(data), count, bits, i)) * s;
    } else if (mode == 2) {
      const int q = (bits == 8) ? int(static_cast<const int8_t*>(data)[i]) : int(static_cast<const int16_t*>(data)[i]);
      v = float(q) * s;
    } else {
      v = 0.f;  // mode 3: zero fill, the scatter follows
    }
    store_as<OutT>(out, i, v);
  }
}

template <typename OutT>
__global__ void scatter_kernel(const void* __restrict__ values, int data_dtype, const int64_t* __restrict__ index,
                               int64_t count, int64_t numel, void* __restrict__ out, DeviceStatus* st) {
  for (int64_t j = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; j < count; j += int64_t(gridDim.x) * blockDim.x) {
    const int64_t i = index[j];
    if (i < 0 || i >= numel) continue;  // out-of-range indices are dropped (checked on the host as well)
    store_as<OutT>(out, i, load_float(values, data_dtype, j));
  }
}

template <typename OutT>
int launch(int mode, const void* data, int data_dtype, const float* scale, const int64_t* index, int64_t count,
           int bits, int64_t numel, void* out, cudaStream_t s) {
  const int threads = 256;
  const int64_t want = (numel + threads - 1) / threads;
  const int blocks = int(want < 4096 ? (want > 0 ? want : 1) : 4096);
  runtime_dequant_kernel<OutT><<<blocks, threads, 0, s>>>(mode, data, data_dtype, scale, count, bits, numel, out);
  KLC_LAUNCH_CHECK("klc_runtime_dequant launch");
  if (mode == 3 && count > 0) {
    const int64_t wb = (count + threads - 1) / threads;
    scatter_kernel<OutT><<<int(wb < 4096 ? wb : 4096), threads, 0, s>>>(data, data_dtype, index, count, numel, out,
                                                                         nullptr);
    KLC_LAUNCH_CHECK("klc_runtime_dequant scatter launch");
  }
  return KLC_OK;
}

}  // namespace

}  // namespace klc

extern "C" int klc_runtime_dequant(int mode, const void* data, int data_dtype, const float* scale,
                                   const int64_t* index, int64_t count, int bits, int64_t numel, void* out,
                                   int out_dtype, void* stream) {
  using namespace klc;
  KLC_CHECK_ARG(mode >= 0 && mode <= 3, "klc_runtime_dequant: mode must be 0..3");
  KLC_CHECK_ARG(numel >= 0 && count >= 0, "klc_runtime_dequant: negative size");
  if (numel == 0) return KLC_OK;
  KLC_CHECK_ARG(out != nullptr, "klc_runtime_dequant: null output");
  if (mode == 0 || mode == 3)
    KLC_CHECK_ARG(data_dtype == KLC_BF16 || data_dtype == KLC_F16 || data_dtype == KLC_F32,
                  "klc_runtime_dequant: data_dtype must be KLC_BF16, KLC_F16 or KLC_F32");
  if (mode == 1) KLC_CHECK_ARG(bits >= 1 && bits <= 4, "klc_runtime_dequant: packed bits must be 1..4");
  if (mode == 2) KLC_CHECK_ARG(bits == 8 || bits == 16, "klc_runtime_dequant: unpacked bits must be 8 or 16");
  if (mode == 1 || mode == 2) KLC_CHECK_ARG(scale != nullptr, "quantized tensor has no scale tensor");
  if (mode == 3) KLC_CHECK_ARG(count == 0 || index != nullptr, "pruned tensor has no sparse index tensor");
  if (mode != 3 || count > 0) KLC_CHECK_ARG(data != nullptr, "klc_runtime_dequant: null data");
  cudaStream_t s = as_stream(stream);
  switch (out_dtype) {
    case KLC_BF16: return launch<uint16_t>(mode, data, data_dtype, scale, index, count, bits, numel, out, s);
    case KLC_F16: return launch<__half>(mode, data, data_dtype, scale, index, count, bits, numel, out, s);
    case KLC_F32: return launch<float>(mode, data, data_dtype, scale, index, count, bits, numel, out, s);
    default: return fail(KLC_ERR_INVALID, "klc_runtime_dequant: out_dtype must be KLC_BF16, KLC_F16 or KLC_F32");
  }
}
