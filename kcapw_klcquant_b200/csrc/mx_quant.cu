// Operand preparation for the block-scaled tensor-core expert GEMMs.
//
// 1. Weight scales (once per layer): the checkpoint's E8M0 scales
//    [E][rows][K/32] re-laid as the 512-byte blocks the MMA's scale copies
//    read: per (expert, 128-row m-tile, 128-K stage) one block whose byte
//    r0*16 + r1*4 + kb is the scale of row r0 + 32*r1, 32-K block kb.
//    Rows and blocks past the matrix are zero (their weights are zero-filled).
//
// 2. Activations (every forward, per row-block): each bf16 row of K values is
//    split into two E4M3 rows, hi and lo, with one shared E8M0 scale per 32-K
//    block: with S = floor(log2(block max)) - 7,
//        hi = x with the low four mantissa bits cleared, / 2^S
//        lo = (x - hi) / 2^S
//    hi keeps the top 4 significant bits of x and lo the remaining 4, so
//    hi + lo = x / 2^S exactly whenever both fit E4M3 (|x| within 2^9 of the
//    block maximum); smaller values are rounded to E4M3's smallest step,
//    2^(S-9).  Output rows: q[row][0][K] = hi, q[row][1][K] = lo; the scales
//    go to the row-block's 512-byte blocks [row-block][128-K stage][chunk]
//    with hi/lo row n2 = 2n + {0,1} of the block at chunk n2 / 128, byte
//    (n2 % 32) * 16 + ((n2 % 128) / 32) * 4 + kb.
#include "permute.cuh"

namespace klc {

namespace {

__global__ void scales_mx_kernel(const uint8_t* __restrict__ scales, int64_t rows, int64_t groups, int mtiles,
                                 int stages, uint8_t* __restrict__ out) {
  const int stage = blockIdx.x, mt = blockIdx.y;
  const int64_t e = blockIdx.z;
  const int m = threadIdx.x;  // row within the m-tile
  const int64_t row = int64_t(mt) * 128 + m;
  uint8_t* blk = out + ((e * mtiles + mt) * stages + stage) * 512;
#pragma unroll
  for (int kb = 0; kb < 4; ++kb) {
    const int64_t g = int64_t(stage) * 4 + kb;
    const uint8_t v = (row < rows && g < groups) ? scales[(e * rows + row) * groups + g] : uint8_t(0);
    blk[(m & 31) * 16 + (m >> 5) * 4 + kb] = v;
  }
}

// Weight scales in tiles of `tile` rows: block [e][t][stage][chunk] (512 bytes) holds,
// for row m = chunk*128 + mm of tile t, byte (mm % 32)*16 + (mm / 32)*4 + kb = the
// scale of 32-K block 4*stage + kb; rows past the matrix or the tile are zero.
__global__ void scales_tile_kernel(const uint8_t* __restrict__ scales, int64_t rows, int64_t groups, int tile, int ntiles,
                                   int stages, int chunks, uint8_t* __restrict__ out) {
  const int stage = blockIdx.x, t = blockIdx.y;
  const int64_t e = blockIdx.z;
  const int m = threadIdx.x;  // row within the tile, blockDim.x = chunks * 128
  const int64_t row = int64_t(t) * tile + m;
  const int chunk = m >> 7, mm = m & 127;
  uint8_t* blk = out + (((e * ntiles + t) * stages + stage) * chunks + chunk) * 512;
#pragma unroll
  for (int kb = 0; kb < 4; ++kb) {
    const int64_t g = int64_t(stage) * 4 + kb;
    const uint8_t v = (m < tile && row < rows && g < groups) ? scales[(e * rows + row) * groups + g] : uint8_t(0);
    blk[(mm & 31) * 16 + (mm >> 5) * 4 + kb] = v;
  }
}

// Rows of 16-byte groups [E*rows][groups] -> [E*rows][groups_pad], zero groups past the row.
__global__ void pad_k128_kernel(const uint4* __restrict__ src, int64_t nrows, int64_t groups, int64_t groups_pad,
                                uint4* __restrict__ dst) {
  const int64_t n = nrows * groups_pad;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / groups_pad, g = i - r * groups_pad;
    dst[i] = g < groups ? src[r * groups + g] : make_uint4(0u, 0u, 0u, 0u);
  }
}

__device__ __forceinline__ uint32_t e4m3x2(float lo_elem, float hi_elem) {
  // first operand -> upper byte, second -> lower byte
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi_elem), "f"(lo_elem));
  return r;
}

// One 32-value block: 32 bf16 at src -> 32 E4M3 hi at hi, 32 E4M3 lo at lo;
// returns the E8M0 scale byte S + 127.
__device__ __forceinline__ uint8_t quantize_block(const uint4* __restrict__ src, uint8_t* __restrict__ hi,
                                                  uint8_t* __restrict__ lo) {
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 v = src[i];
    w[4 * i] = v.x;
    w[4 * i + 1] = v.y;
    w[4 * i + 2] = v.z;
    w[4 * i + 3] = v.w;
  }
  // block maximum exponent from the bf16 bit patterns (sign dropped)
  uint32_t emax = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint32_t a = (w[i] >> 7) & 0xFFu, b = (w[i] >> 23) & 0xFFu;
    emax = max(emax, max(a, b));
  }
  // S = (emax - 127) - 7, kept where 2^S and 2^-S are normal fp32 (the E8M0
  // byte S + 127 is then in [1, 253]); all-zero blocks get S = 0
  int S = emax == 0 ? 0 : int(emax) - 134;
  S = S < -126 ? -126 : (S > 126 ? 126 : S);
  const float inv = __uint_as_float(uint32_t(127 - S) << 23);  // 2^-S
  uint32_t hi_w[8], lo_w[8];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint32_t b0 = w[i] & 0xFFFFu, b1 = w[i] >> 16;
    const float x0 = __uint_as_float(b0 << 16), x1 = __uint_as_float(b1 << 16);
    const float h0 = __uint_as_float((b0 & 0xFFF0u) << 16), h1 = __uint_as_float((b1 & 0xFFF0u) << 16);
    const uint32_t hp = e4m3x2(h0 * inv, h1 * inv);  // bytes (elem 2i, elem 2i+1)
    const uint32_t lp = e4m3x2((x0 - h0) * inv, (x1 - h1) * inv);
    if (i & 1) {
      hi_w[i >> 1] |= hp << 16;
      lo_w[i >> 1] |= lp << 16;
    } else {
      hi_w[i >> 1] = hp;
      lo_w[i >> 1] = lp;
    }
  }
  uint4* dh = reinterpret_cast<uint4*>(hi);
  uint4* dl = reinterpret_cast<uint4*>(lo);
  dh[0] = make_uint4(hi_w[0], hi_w[1], hi_w[2], hi_w[3]);
  dh[1] = make_uint4(hi_w[4], hi_w[5], hi_w[6], hi_w[7]);
  dl[0] = make_uint4(lo_w[0], lo_w[1], lo_w[2], lo_w[3]);
  dl[1] = make_uint4(lo_w[4], lo_w[5], lo_w[6], lo_w[7]);
  return uint8_t(S + 127);
}

// A quarter of a 32-value block per lane: the four lanes of a quad hold one
// block (8 bf16 each, 16 contiguous bytes), agree on its exponent by two
// shuffles and write 8 hi and 8 lo E4M3 bytes each, so a warp reads and writes
// contiguous 512- and 256-byte spans.  The values are those of quantize_block.
// All 32 lanes call it (the shuffles); `v` of a lane past the row is zero.
__device__ __forceinline__ uint8_t quantize_quarter(const uint4 v, uint2& hi, uint2& lo) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t emax = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) emax = max(emax, max((w[i] >> 7) & 0xFFu, (w[i] >> 23) & 0xFFu));
  emax = max(emax, __shfl_xor_sync(0xffffffffu, emax, 1));
  emax = max(emax, __shfl_xor_sync(0xffffffffu, emax, 2));
  int S = emax == 0 ? 0 : int(emax) - 134;
  S = S < -126 ? -126 : (S > 126 ? 126 : S);
  const float inv = __uint_as_float(uint32_t(127 - S) << 23);  // 2^-S
  uint32_t hp[4], lp[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t b0 = w[i] & 0xFFFFu, b1 = w[i] >> 16;
    const float x0 = __uint_as_float(b0 << 16), x1 = __uint_as_float(b1 << 16);
    const float h0 = __uint_as_float((b0 & 0xFFF0u) << 16), h1 = __uint_as_float((b1 & 0xFFF0u) << 16);
    hp[i] = e4m3x2(h0 * inv, h1 * inv);
    lp[i] = e4m3x2((x0 - h0) * inv, (x1 - h1) * inv);
  }
  hi = make_uint2(hp[0] | (hp[1] << 16), hp[2] | (hp[3] << 16));
  lo = make_uint2(lp[0] | (lp[1] << 16), lp[2] | (lp[3] << 16));
  return uint8_t(S + 127);
}

// One warp per row, 8 blocks of 32 K per pass (a quad per block), four passes'
// loads issued before their conversions.
__global__ void __launch_bounds__(256)
    quantize_rows_kernel(const uint16_t* __restrict__ src, int64_t K, const int32_t* __restrict__ rows_map, int k,
                         const int4* __restrict__ rowblocks, const DeviceStatus* __restrict__ st, int nch,
                         uint8_t* __restrict__ q, uint8_t* __restrict__ sfb) {
  pdl_wait();     // inputs written by the previous kernel of the chain
  pdl_trigger();  // the next kernel may launch and set up meanwhile
  const int rbi = blockIdx.x;
  if (rbi >= st->rowblocks) return;
  const int4 rb = rowblocks[rbi];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = int(K / 32);
  const int stages = (G + 3) / 4;
  const int part = lane & 3;
  constexpr int kU = 4;  // passes in flight
  for (int n = warp; n < rb.z; n += blockDim.x >> 5) {
    const int64_t row = int64_t(rb.y) + n;
    const int64_t srow = rows_map != nullptr ? int64_t(rows_map[row] / k) : row;
    const uint4* s4 = reinterpret_cast<const uint4*>(src + srow * K);
    uint8_t* qh = q + row * 2 * K;
    for (int b0 = 0; b0 < G; b0 += 8 * kU) {
      uint4 v[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int kb = b0 + 8 * u + (lane >> 2);
        v[u] = kb < G ? s4[kb * 4 + part] : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int kb = b0 + 8 * u + (lane >> 2);
        if (b0 + 8 * u >= G) break;  // uniform over the warp
        uint2 hi, lo;
        const uint8_t sb = quantize_quarter(v[u], hi, lo);
        if (kb < G) {
          *reinterpret_cast<uint2*>(qh + int64_t(kb) * 32 + part * 8) = hi;
          *reinterpret_cast<uint2*>(qh + K + int64_t(kb) * 32 + part * 8) = lo;
          if (part < 2) {  // the scale byte of the hi (part 0) and lo (part 1) row
            const int n2 = 2 * n + part;
            uint8_t* blk = sfb + ((int64_t(rbi) * stages + kb / 4) * nch + n2 / 128) * 512;
            blk[(n2 & 31) * 16 + ((n2 & 127) >> 5) * 4 + (kb & 3)] = sb;
          }
        }
      }
    }
  }
}

// Plain layout for callers: rows [R, K] -> q [R, 2, K] (hi, lo), scales [R, K/32]
__global__ void __launch_bounds__(256)
    quantize_plain_kernel(const uint16_t* __restrict__ src, int64_t rows, int64_t K, uint8_t* __restrict__ q,
                          uint8_t* __restrict__ scales) {
  const int64_t G = K / 32;
  const int64_t b = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;  // one 32-value block per thread
  if (b >= rows * G) return;
  const int64_t r = b / G, kb = b % G;
  uint8_t* qr = q + r * 2 * K;
  scales[b] = quantize_block(reinterpret_cast<const uint4*>(src + r * K) + kb * 4, qr + kb * 32, qr + K + kb * 32);
}

}  // namespace

int launch_quantize_rows(const uint16_t* src, int64_t K, const int32_t* rows_map, int k, const int4* rowblocks,
                         const DeviceStatus* status, int max_rowblocks, int nch, uint8_t* q, uint8_t* sfb,
                         cudaStream_t stream) {
  KLC_CHECK_ARG(K % 32 == 0, "quantize: K must be a multiple of 32");
  if (max_rowblocks <= 0) return KLC_OK;
  KLC_CUDA(launch_chain(quantize_rows_kernel, dim3(max_rowblocks), dim3(256), size_t(0), stream, 0u, src, K, rows_map, k, rowblocks, status, nch, q, sfb));
  KLC_LAUNCH_CHECK("activation quantize launch");
  return KLC_OK;
}

}  // namespace klc

extern "C" int klc_mx_quantize_rows(const uint16_t* x, int64_t rows, int64_t K, uint8_t* q, uint8_t* scales,
                                    void* stream) {
  using namespace klc;
  KLC_CHECK_ARG(rows >= 0 && K > 0 && K % 32 == 0, "klc_mx_quantize_rows: K must be a positive multiple of 32");
  if (rows == 0) return KLC_OK;
  KLC_CHECK_ARG(x && q && scales, "klc_mx_quantize_rows: null pointer");
  KLC_CHECK_ARG((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(q) & 15) == 0,
                "klc_mx_quantize_rows: x and q must be 16-byte aligned");
  const int64_t blocks = (rows * (K / 32) + 255) / 256;
  KLC_CHECK_ARG(blocks <= 0x7fffffff, "klc_mx_quantize_rows: too many rows");
  quantize_plain_kernel<<<unsigned(blocks), 256, 0, as_stream(stream)>>>(x, rows, K, q, scales);
  KLC_LAUNCH_CHECK("klc_mx_quantize_rows launch");
  return KLC_OK;
}

extern "C" int klc_mxfp4_scales_mx_bytes(int64_t experts, int64_t rows, int64_t groups, size_t* out_bytes) {
  using namespace klc;
  KLC_CHECK_ARG(experts >= 0 && rows >= 0 && groups >= 0, "klc_mxfp4_scales_mx_bytes: negative size");
  KLC_CHECK_ARG(out_bytes != nullptr, "klc_mxfp4_scales_mx_bytes: null output");
  *out_bytes = size_t(experts) * size_t((rows + 127) / 128) * size_t((groups + 3) / 4) * 512;
  return KLC_OK;
}

extern "C" int klc_mxfp4_scales_mx(const uint8_t* scales, int64_t experts, int64_t rows, int64_t groups,
                                   uint8_t* out, void* stream) {
  using namespace klc;
  KLC_CHECK_ARG(experts >= 0 && rows >= 0 && groups >= 0, "klc_mxfp4_scales_mx: negative size");
  if (experts == 0 || rows == 0 || groups == 0) return KLC_OK;
  KLC_CHECK_ARG(scales && out, "klc_mxfp4_scales_mx: null pointer");
  const int64_t mtiles = (rows + 127) / 128, stages = (groups + 3) / 4;
  KLC_CHECK_ARG(experts <= 65535 && mtiles <= 65535 && stages <= 0x7fffffff, "klc_mxfp4_scales_mx: too large");
  scales_mx_kernel<<<dim3(unsigned(stages), unsigned(mtiles), unsigned(experts)), 128, 0, as_stream(stream)>>>(
      scales, rows, groups, int(mtiles), int(stages), out);
  KLC_LAUNCH_CHECK("klc_mxfp4_scales_mx launch");
  return KLC_OK;
}

extern "C" int klc_mxfp4_pad_k128(const uint8_t* blocks, int64_t experts, int64_t rows, int64_t groups, uint8_t* out,
                                  void* stream) {
  using namespace klc;
  KLC_CHECK_ARG(experts >= 0 && rows >= 0 && groups >= 0, "klc_mxfp4_pad_k128: negative size");
  const int64_t nrows = experts * rows;
  if (nrows == 0 || groups == 0) return KLC_OK;
  KLC_CHECK_ARG(blocks && out, "klc_mxfp4_pad_k128: null pointer");
  KLC_CHECK_ARG((reinterpret_cast<uintptr_t>(blocks) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0,
                "klc_mxfp4_pad_k128: blocks and out must be 16-byte aligned");
  const int64_t gp = (groups + 3) / 4 * 4;
  const int64_t n = nrows * gp;
  const int64_t want = (n + 255) / 256;
  const int blocks_n = int(want < 8192 ? want : 8192);
  pad_k128_kernel<<<blocks_n, 256, 0, as_stream(stream)>>>(reinterpret_cast<const uint4*>(blocks), nrows, groups, gp,
                                                            reinterpret_cast<uint4*>(out));
  KLC_LAUNCH_CHECK("klc_mxfp4_pad_k128 launch");
  return KLC_OK;
}

extern "C" int klc_mxfp4_scales_tile_bytes(int64_t experts, int64_t rows, int64_t groups, int tile_rows, size_t* out_bytes) {
  using namespace klc;
  KLC_CHECK_ARG(experts >= 0 && rows >= 0 && groups >= 0 && tile_rows >= 1 && tile_rows <= 256,
                "klc_mxfp4_scales_tile_bytes: bad sizes");
  KLC_CHECK_ARG(out_bytes != nullptr, "klc_mxfp4_scales_tile_bytes: null output");
  *out_bytes = size_t(experts) * size_t((rows + tile_rows - 1) / tile_rows) * size_t((groups + 3) / 4) *
               size_t((tile_rows + 127) / 128) * 512;
  return KLC_OK;
}

extern "C" int klc_mxfp4_scales_tile(const uint8_t* scales, int64_t experts, int64_t rows, int64_t groups, int tile_rows,
                                     uint8_t* out, void* stream) {
  using namespace klc;
  KLC_CHECK_ARG(experts >= 0 && rows >= 0 && groups >= 0 && tile_rows >= 1 && tile_rows <= 256,
                "klc_mxfp4_scales_tile: bad sizes");
  if (experts == 0 || rows == 0 || groups == 0) return KLC_OK;
  KLC_CHECK_ARG(scales && out, "klc_mxfp4_scales_tile: null pointer");
  const int64_t ntiles = (rows + tile_rows - 1) / tile_rows, stages = (groups + 3) / 4;
  const int chunks = (tile_rows + 127) / 128;
  KLC_CHECK_ARG(experts <= 65535 && ntiles <= 65535 && stages <= 0x7fffffff, "klc_mxfp4_scales_tile: too large");
  scales_tile_kernel<<<dim3(unsigned(stages), unsigned(ntiles), unsigned(experts)), chunks * 128, 0, as_stream(stream)>>>(
      scales, rows, groups, tile_rows, int(ntiles), int(stages), chunks, out);
  KLC_LAUNCH_CHECK("klc_mxfp4_scales_tile launch");
  return KLC_OK;
}
