// quant.cu — the int4 g128 weight format on the GPU (rows a1-a3 of the path):
//   quantise      bit exact with scripts/quantize.py:32-64
//   dequantise    bit exact with qlinear.py:28-64
//   transpose     bit exact with dip_stream_predispatch.py:100-120
// fp32 division uses __fdiv_rn and rounding uses rintf (round half to even),
// the operations torch performs for `w / s`, `max / 7` and `torch.round`.
#include "dip_common.cuh"

namespace dip {

__device__ __forceinline__ int quant_one(float w, float s) {
  float q = rintf(__fdiv_rn(w, s));
  q = fminf(fmaxf(q, -8.f), 7.f);
  return (int)q;
}
__device__ __forceinline__ float scale_of(float max_abs) {
  return fmaxf(__fdiv_rn(max_abs, 7.0f), 1e-8f);
}

// One warp per (row, group of 128 columns); lane handles 4 columns.
__global__ void quantize_kernel(const uint16_t* __restrict__ w, int64_t rows, int64_t cols,
                                uint8_t* __restrict__ qw, uint16_t* __restrict__ sc) {
  const int64_t ng = cols / kGroup;
  const int64_t task = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (task >= rows * ng) return;
  const int64_t r = task / ng, g = task % ng;
  const uint2 v = *reinterpret_cast<const uint2*>(w + r * cols + g * kGroup + lane * 4);
  float f[4] = {bf16_bits_to_f32(v.x & 0xFFFF), bf16_bits_to_f32(v.x >> 16),
                bf16_bits_to_f32(v.y & 0xFFFF), bf16_bits_to_f32(v.y >> 16)};
  float m = fmaxf(fmaxf(fabsf(f[0]), fabsf(f[1])), fmaxf(fabsf(f[2]), fabsf(f[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float s = scale_of(m);
  uint32_t packed = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) packed |= (uint32_t)(quant_one(f[i], s) & 0xF) << (4 * i);
  *reinterpret_cast<uint16_t*>(qw + r * (cols / 2) + g * kGroupBytes + lane * 2) =
      (uint16_t)packed;
  if (lane == 0) sc[r * ng + g] = f32_to_bf16_bits(s);
}

// Thread per packed byte: two bf16 values bf16(q * s).
__global__ void dequantize_kernel(const uint8_t* __restrict__ qw, const uint16_t* __restrict__ sc,
                                  int64_t rows, int64_t cols, uint16_t* __restrict__ w) {
  const int64_t nbytes = rows * (cols / 2);
  for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < nbytes;
       b += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = b / (cols / 2), cb = b % (cols / 2);
    const float s = bf16_bits_to_f32(sc[r * (cols / kGroup) + (cb * 2) / kGroup]);
    const int v = qw[b];
    const int lo = ((v & 0xF) ^ 8) - 8, hi = (((v >> 4) & 0xF) ^ 8) - 8;
    const uint32_t o = (uint32_t)f32_to_bf16_bits((float)lo * s) |
                       ((uint32_t)f32_to_bf16_bits((float)hi * s) << 16);
    *reinterpret_cast<uint32_t*>(w + r * cols + cb * 2) = o;
  }
}

// Tile: 128 outputs (one output group) x 64 channels; 256 threads.
// down_qw [out_f, inter/2], down_sc [out_f, inter/128]
//   -> down_t_qw [inter, out_f/2], down_t_sc [inter, out_f/128]
__global__ void __launch_bounds__(256)
transpose_down_kernel(const uint8_t* __restrict__ dqw, const uint16_t* __restrict__ dsc,
                      int64_t out_f, int64_t inter, uint8_t* __restrict__ tqw,
                      uint16_t* __restrict__ tsc) {
  __shared__ float tile[128][65];
  __shared__ float pmax[4][64];
  const int64_t og = blockIdx.x;      // output group
  const int64_t c0 = (int64_t)blockIdx.y * 64;
  const int tid = threadIdx.x;
  // Load: 128 rows x 32 bytes.
  for (int e = tid; e < 128 * 32; e += 256) {
    const int r = e / 32, b = e % 32;
    const int64_t o = og * kGroup + r;
    const int64_t c = c0 + 2 * b;
    float w0 = 0.f, w1 = 0.f;
    if (c < inter) {
      const int v = dqw[o * (inter / 2) + c / 2];
      const float s = bf16_bits_to_f32(dsc[o * (inter / kGroup) + c / kGroup]);
      w0 = round_bf16((float)(((v & 0xF) ^ 8) - 8) * s);
      w1 = round_bf16((float)((((v >> 4) & 0xF) ^ 8) - 8) * s);
    }
    tile[r][2 * b] = w0;
    tile[r][2 * b + 1] = w1;
  }
  __syncthreads();
  const int c = tid & 63, part = tid >> 6;  // part covers outputs part*32 .. +32
  float m = 0.f;
  for (int i = 0; i < 32; ++i) m = fmaxf(m, fabsf(tile[part * 32 + i][c]));
  pmax[part][c] = m;
  __syncthreads();
  m = fmaxf(fmaxf(pmax[0][c], pmax[1][c]), fmaxf(pmax[2][c], pmax[3][c]));
  const float s = scale_of(m);
  if (c0 + c >= inter) return;
  uint32_t words[4];
#pragma unroll
  for (int wd = 0; wd < 4; ++wd) {
    uint32_t acc = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      acc |= (uint32_t)(quant_one(tile[part * 32 + wd * 8 + i][c], s) & 0xF) << (4 * i);
    words[wd] = acc;
  }
  const int64_t ch = c0 + c;
  *reinterpret_cast<uint4*>(tqw + ch * (out_f / 2) + og * kGroupBytes + part * 16) =
      make_uint4(words[0], words[1], words[2], words[3]);
  if (part == 0) tsc[ch * (out_f / kGroup) + og] = f32_to_bf16_bits(s);
}

}  // namespace dip

using namespace dip;

extern "C" int dip_quantize_int4_g128(const dip_bf16* w, int64_t rows, int64_t cols,
                                      int8_t* qweight, dip_bf16* scales, dip_stream_t stream) {
  if (rows < 0 || cols <= 0 || cols % kGroup) return DIP_ERR_ARG;
  if (rows == 0) return DIP_OK;
  if (!w || !qweight || !scales || (reinterpret_cast<uintptr_t>(w) & 7)) return DIP_ERR_ARG;
  const int64_t tasks = rows * (cols / kGroup);
  const int64_t blocks = (tasks + 7) / 8;
  if (blocks > INT32_MAX) return DIP_ERR_UNSUPPORTED;
  quantize_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      w, rows, cols, reinterpret_cast<uint8_t*>(qweight), scales);
  return launch_status(cudaGetLastError());
}

extern "C" int dip_dequantize_int4_g128(const int8_t* qweight, const dip_bf16* scales,
                                        int64_t rows, int64_t cols, dip_bf16* w,
                                        dip_stream_t stream) {
  if (rows < 0 || cols <= 0 || cols % kGroup) return DIP_ERR_ARG;
  if (rows == 0) return DIP_OK;
  if (!w || !qweight || !scales || (reinterpret_cast<uintptr_t>(w) & 3)) return DIP_ERR_ARG;
  dequantize_kernel<<<148 * 8, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const uint8_t*>(qweight), scales, rows, cols, w);
  return launch_status(cudaGetLastError());
}

extern "C" int dip_transpose_down_int4(const int8_t* down_qw, const dip_bf16* down_sc,
                                       int64_t out_f, int64_t inter, int8_t* down_t_qw,
                                       dip_bf16* down_t_sc, dip_stream_t stream) {
  if (out_f <= 0 || inter <= 0 || out_f % kGroup || inter % kGroup) return DIP_ERR_ARG;
  if (!down_qw || !down_sc || !down_t_qw || !down_t_sc ||
      (reinterpret_cast<uintptr_t>(down_t_qw) & 15))
    return DIP_ERR_ARG;
  const dim3 grid((unsigned)(out_f / kGroup), (unsigned)((inter + 63) / 64));
  transpose_down_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const uint8_t*>(down_qw), down_sc, out_f, inter,
      reinterpret_cast<uint8_t*>(down_t_qw), down_t_sc);
  return launch_status(cudaGetLastError());
}
