// stack_ops.cu — the inter-layer step of the synthetic decode stack:
//   x_next = bf16( v * rsqrt(mean(v^2) + eps) ),  v = float(y) + float(r)
// (RMSNorm with unit weight of the previous layer's output plus a bf16
// residual).  One CTA; the sum of squares is reduced in a fixed order.
#include "dip_common.cuh"

namespace dip {

__global__ void __launch_bounds__(1024)
residual_rmsnorm_kernel(const uint16_t* __restrict__ y, const uint16_t* __restrict__ r, int n,
                        float eps, uint16_t* __restrict__ out) {
  __shared__ float wsum[32];
  // one CTA per row
  y += (size_t)blockIdx.x * n;
  r += (size_t)blockIdx.x * n;
  out += (size_t)blockIdx.x * n;
  pdl_wait();
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = bf16_bits_to_f32(y[i]) + bf16_bits_to_f32(r[i]);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) wsum[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? wsum[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) wsum[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(wsum[0] / (float)n + eps);
  pdl_launch_dependents();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = bf16_bits_to_f32(y[i]) + bf16_bits_to_f32(r[i]);
    out[i] = f32_to_bf16_bits(v * inv);
  }
}

}  // namespace dip

using namespace dip;

extern "C" int dip_residual_rmsnorm(const dip_bf16* y, const dip_bf16* r, int64_t n, float eps,
                                    dip_bf16* out, dip_stream_t stream) {
  return dip_residual_rmsnorm_rows(y, r, 1, n, eps, out, stream);
}

extern "C" int dip_residual_rmsnorm_rows(const dip_bf16* y, const dip_bf16* r, int64_t rows,
                                         int64_t n, float eps, dip_bf16* out,
                                         dip_stream_t stream) {
  if (n <= 0 || n > (1 << 20) || rows <= 0 || rows > 65535 || !y || !r || !out) return DIP_ERR_ARG;
  return launch_status(launch(residual_rmsnorm_kernel, dim3((unsigned)rows), dim3(1024), 0,
                              (cudaStream_t)stream, y, r, (int)n, eps, out));
}
