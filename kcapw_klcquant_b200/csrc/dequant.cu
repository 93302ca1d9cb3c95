// Standalone MXFP4 -> bf16/fp16/fp32 dequant (drop-in for the reference's
// dequantize_mxfp4_matrix, mxfp4_expert.py:357-379) and the one-time E8M0
// scale re-layout used by the expert kernels.
//
// Memory-bound: per output element 0.5 B of nibbles + 1/32 B of scale read and
// 2 B (bf16) written.  A CTA stages a 32-row x 8-group tile of nibbles
// through shared memory so both the reads (128 B per row) and the transposed
// writes (32 consecutive output columns per warp store) are coalesced.
#include "klc_common.cuh"

namespace klc {

namespace {

constexpr int kRowsPerCta = 32;
constexpr int kGroupsPerCta = 8;

template <typename OutT>
__device__ __forceinline__ OutT convert_out(float v);

template <>
__device__ __forceinline__ uint16_t convert_out<uint16_t>(float v) {
  return f32_to_bf16(v);
}
template <>
__device__ __forceinline__ __half convert_out<__half>(float v) {
  return __float2half_rn(v);
}
template <>
__device__ __forceinline__ float convert_out<float>(float v) {
  return v;
}

template <typename OutT>
__global__ void __launch_bounds__(kRowsPerCta * kGroupsPerCta)
    dequant_transpose_kernel(const uint8_t* __restrict__ blocks, const uint8_t* __restrict__ scales,
                             int64_t out_dim, int64_t groups, OutT* __restrict__ out) {
  __shared__ uint4 tile[kRowsPerCta][kGroupsPerCta];
  const int tid = threadIdx.y * kRowsPerCta + threadIdx.x;
  const int64_t row0 = int64_t(blockIdx.x) * kRowsPerCta;
  const int64_t g0 = int64_t(blockIdx.y) * kGroupsPerCta;
  // coalesced load: consecutive threads walk one row's 8 x 16 B groups
  {
    const int r = tid / kGroupsPerCta, c = tid % kGroupsPerCta;
    const int64_t row = row0 + r, g = g0 + c;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < out_dim && g < groups) v = ldg_nc_v4(blocks + (row * groups + g) * 16);
    tile[r][c] = v;
  }
  __syncthreads();
  const int64_t row = row0 + threadIdx.x;
  const int64_t g = g0 + threadIdx.y;
  if (row >= out_dim || g >= groups) return;
  const uint32_t s = scales[row * groups + g];
  const uint4 v = tile[threadIdx.x][threadIdx.y];
  const uint32_t words[4] = {v.x, v.y, v.z, v.w};
  OutT* col = out + (g * 32) * out_dim + row;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const uint32_t nib = (words[w] >> (4 * n)) & 0xFu;  // nibble n of the word = K index 8w+n
      col[int64_t(8 * w + n) * out_dim] = convert_out<OutT>(e8m0_scale(fp4_to_f32(nib), s));
    }
  }
}

__global__ void transpose_scales_kernel(const uint8_t* __restrict__ in, int64_t rows, int64_t groups,
                                        uint8_t* __restrict__ out) {
  __shared__ uint8_t tile[32][33];
  const int64_t e = blockIdx.z;
  const int64_t r0 = int64_t(blockIdx.x) * 32, g0 = int64_t(blockIdx.y) * 32;
  const uint8_t* src = in + e * rows * groups;
  uint8_t* dst = out + e * rows * groups;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t r = r0 + i, g = g0 + threadIdx.x;
    if (r < rows && g < groups) tile[i][threadIdx.x] = src[r * groups + g];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t g = g0 + i, r = r0 + threadIdx.x;
    if (r < rows && g < groups) dst[g * rows + r] = tile[threadIdx.x][i];
  }
}

}  // namespace

}  // namespace klc

extern "C" int klc_mxfp4_dequant(const uint8_t* blocks, const uint8_t* scales, int64_t out_dim, int64_t groups,
                                 void* out, int out_dtype, void* stream) {
  using namespace klc;
  KLC_CHECK_ARG(out_dim >= 0 && groups >= 0, "klc_mxfp4_dequant: negative size");
  if (out_dim == 0 || groups == 0) return KLC_OK;
  KLC_CHECK_ARG(blocks && scales && out, "klc_mxfp4_dequant: null pointer");
  KLC_CHECK_ARG((reinterpret_cast<uintptr_t>(blocks) & 15) == 0, "klc_mxfp4_dequant: blocks must be 16-byte aligned");
  dim3 block(kRowsPerCta, kGroupsPerCta);
  dim3 grid(unsigned((out_dim + kRowsPerCta - 1) / kRowsPerCta), unsigned((groups + kGroupsPerCta - 1) / kGroupsPerCta));
  KLC_CHECK_ARG(grid.y <= 65535, "klc_mxfp4_dequant: too many groups");
  cudaStream_t s = as_stream(stream);
  switch (out_dtype) {
    case KLC_BF16:
      dequant_transpose_kernel<uint16_t><<<grid, block, 0, s>>>(blocks, scales, out_dim, groups, static_cast<uint16_t*>(out));
      break;
    case KLC_F16:
      dequant_transpose_kernel<__half><<<grid, block, 0, s>>>(blocks, scales, out_dim, groups, static_cast<__half*>(out));
      break;
    case KLC_F32:
      dequant_transpose_kernel<float><<<grid, block, 0, s>>>(blocks, scales, out_dim, groups, static_cast<float*>(out));
      break;
    default:
      return fail(KLC_ERR_INVALID, "klc_mxfp4_dequant: out_dtype must be KLC_BF16, KLC_F16 or KLC_F32");
  }
  KLC_LAUNCH_CHECK("klc_mxfp4_dequant launch");
  return KLC_OK;
}

extern "C" int klc_mxfp4_transpose_scales(const uint8_t* scales, int64_t experts, int64_t rows, int64_t groups,
                                          uint8_t* scales_t, void* stream) {
  using namespace klc;
  KLC_CHECK_ARG(experts >= 0 && rows >= 0 && groups >= 0, "klc_mxfp4_transpose_scales: negative size");
  if (experts == 0 || rows == 0 || groups == 0) return KLC_OK;
  KLC_CHECK_ARG(scales && scales_t, "klc_mxfp4_transpose_scales: null pointer");
  KLC_CHECK_ARG(experts <= 65535, "klc_mxfp4_transpose_scales: too many experts");
  dim3 grid(unsigned((rows + 31) / 32), unsigned((groups + 31) / 32), unsigned(experts));
  transpose_scales_kernel<<<grid, dim3(32, 8), 0, as_stream(stream)>>>(scales, rows, groups, scales_t);
  KLC_LAUNCH_CHECK("klc_mxfp4_transpose_scales launch");
  return KLC_OK;
}
