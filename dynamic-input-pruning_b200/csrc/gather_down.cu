// gather_down.cu — gathered, transposed int4 down projection for sm_100a.
//
//   y[o] = bf16( sum_j h[j] * q(down_t[r_j, o]) * s(down_t[r_j, o/128]) )
//
// Reference: kernels/int4_down/int4_gather_down.cu:41-95, which runs one CTA
// per output element and reads the selected rows column-wise (adjacent
// threads 2560 B apart).  Here every selected row is read exactly once,
// fully coalesced: a "team" of out/32 threads covers one row, each thread
// owning a fixed 16-byte slice (32 outputs) and accumulating those outputs
// across all rows of its share in fp32 registers.  Several teams per CTA
// take interleaved rows; the CTA's teams are combined in shared memory in a
// fixed order and the CTA writes one fp32 partial vector.  A second kernel
// sums the partials in a fixed order and rounds to bf16 — no float atomics,
// so y is bitwise reproducible.
//
// Nibble -> fp32 uses the 2^23 magic: (bits << 4i) | 0x4B000000 is exactly
// 2^23 + u*16^i; after XOR with 8 (two's complement -> offset binary) and a
// paired subtraction, the paired FMA (sm_100 FFMA2) multiplies by
// h*s*16^-i, which is exact because h*s (bf16 x bf16) has 16 significant bits.
#include "dip_common.cuh"

namespace dip {

enum DownRowMode : int { DROW_IDENT = 0, DROW_GATHER = 1, DROW_SRCROW = 2 };

struct DownParams {
  const uint8_t* qw0; const uint16_t* sc0; int64_t n0;  // source 0
  const uint8_t* qw1; const uint16_t* sc1; int64_t n1;  // source 1 (SRCROW)
  const uint16_t* h;      // [k]
  const int32_t* idx;     // GATHER
  const int32_t* src;     // SRCROW
  const int32_t* row;     // SRCROW
  float* partial;         // [gridDim.x, out]
  const int32_t* count;   // optional device-side number of rows (<= k)
  int k;
  int out_features;
};

constexpr int kDownCtas = 148;   // partial vectors (== SMs of a B200)
constexpr int kDownUnroll = 4;   // rows in flight per thread

template <int MODE>
__device__ __forceinline__ bool down_row(const DownParams& p, int j, const uint8_t*& qw,
                                         const uint16_t*& sc) {
  const int64_t rb = p.out_features / 2, sb = p.out_features / kGroup;
  int s = 0;
  int64_t r;
  if (MODE == DROW_IDENT) r = j;
  else if (MODE == DROW_GATHER) r = p.idx[j];
  else { s = p.src[j]; r = p.row[j]; }
  const int64_t n = s == 0 ? p.n0 : p.n1;
  const bool ok = (s == 0 || s == 1) && r >= 0 && r < n;
  if (!ok) { s = 0; r = 0; }
  qw = (s == 0 ? p.qw0 : p.qw1) + r * rb;
  sc = (s == 0 ? p.sc0 : p.sc1) + r * sb;
  return ok;
}

__device__ __forceinline__ void fma_word(uint32_t w, float hs, float2& a0, float2& a1,
                                         float2& a2, float2& a3) {
  // nibbles 0..3 from bits 0..15, nibbles 4..7 from bits 16..31
  const float2 m01 = make_float2(hs, hs * 0.0625f);
  const float2 m23 = make_float2(hs * 0.00390625f, hs * 0.000244140625f);
  const float2 b01 = make_float2(8388608.f + 8.f, 8388608.f + 128.f);
  const float2 b23 = make_float2(8388608.f + 2048.f, 8388608.f + 32768.f);
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const uint32_t v = half ? (w >> 16) : w;
    float2 x01 = make_float2(__uint_as_float((v & 0x000Fu) ^ (kF32Magic | 0x0008u)),
                             __uint_as_float((v & 0x00F0u) ^ (kF32Magic | 0x0080u)));
    float2 x23 = make_float2(__uint_as_float((v & 0x0F00u) ^ (kF32Magic | 0x0800u)),
                             __uint_as_float((v & 0xF000u) ^ (kF32Magic | 0x8000u)));
    x01 = __fadd2_rn(x01, make_float2(-b01.x, -b01.y));  // (q0, 16 q1)
    x23 = __fadd2_rn(x23, make_float2(-b23.x, -b23.y));  // (256 q2, 4096 q3)
    if (half == 0) {
      a0 = __ffma2_rn(x01, m01, a0);
      a1 = __ffma2_rn(x23, m23, a1);
    } else {
      a2 = __ffma2_rn(x01, m01, a2);
      a3 = __ffma2_rn(x23, m23, a3);
    }
  }
}

// blockDim.x = teams * nch <= 640, nch = out/32 (one 16-byte slice per thread).
template <int MODE>
__global__ void __launch_bounds__(640)
gather_down_kernel(const DownParams p) {
  extern __shared__ __align__(16) float red[];  // [teams][out]
  const int nch = p.out_features / 32;
  const int teams = blockDim.x / nch;
  const int team = threadIdx.x / nch;
  const int ch = threadIdx.x - team * nch;
  float2 acc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i] = make_float2(0.f, 0.f);

  pdl_wait();
  int k = p.k;
  if (p.count) k = min(k, *p.count);
  // Rows [j0, j1) of this CTA (balanced split).
  const int j0 = (int)((int64_t)k * blockIdx.x / gridDim.x);
  const int j1 = (int)((int64_t)k * (blockIdx.x + 1) / gridDim.x);

  for (int jb = j0 + team; jb < j1; jb += teams * kDownUnroll) {
    uint4 wv[kDownUnroll];
    float hs[kDownUnroll];
#pragma unroll
    for (int u = 0; u < kDownUnroll; ++u) {
      const int j = jb + u * teams;
      hs[u] = 0.f;
      wv[u] = make_uint4(0, 0, 0, 0);
      if (j < j1) {
        const uint8_t* qw;
        const uint16_t* sc;
        const bool ok = down_row<MODE>(p, j, qw, sc);
        wv[u] = ldg_stream_u4(qw + ch * 16);
        const float s = bf16_bits_to_f32(ldg_u16(sc + (ch >> 2)));
        const float hv = bf16_bits_to_f32(ldg_u16(p.h + j));
        hs[u] = ok ? hv * s : 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < kDownUnroll; ++u) {
      fma_word(wv[u].x, hs[u], acc[0], acc[1], acc[2], acc[3]);
      fma_word(wv[u].y, hs[u], acc[4], acc[5], acc[6], acc[7]);
      fma_word(wv[u].z, hs[u], acc[8], acc[9], acc[10], acc[11]);
      fma_word(wv[u].w, hs[u], acc[12], acc[13], acc[14], acc[15]);
    }
  }
  pdl_launch_dependents();

  // acc[4w + p] holds outputs ch*32 + 8w + 2p + {0,1}.
  float4* mine = reinterpret_cast<float4*>(red + (size_t)team * p.out_features + ch * 32);
#pragma unroll
  for (int i = 0; i < 8; ++i)
    mine[i] = make_float4(acc[2 * i].x, acc[2 * i].y, acc[2 * i + 1].x, acc[2 * i + 1].y);
  __syncthreads();
  const int nvec = p.out_features / 4;
  float4* dst = reinterpret_cast<float4*>(p.partial + (size_t)blockIdx.x * p.out_features);
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    float4 v = reinterpret_cast<const float4*>(red)[i];
    for (int t = 1; t < teams; ++t) {
      const float4 o = reinterpret_cast<const float4*>(red + (size_t)t * p.out_features)[i];
      v.x += o.x; v.y += o.y; v.z += o.z; v.w += o.w;
    }
    dst[i] = v;
  }
}

// y[o] = bf16(sum_c partial[c][o]) in a fixed order; optional fp32 copy.
// grid = out/32 CTAs of 256 threads: warp w sums partials w, w+8, ...
__global__ void __launch_bounds__(256)
reduce_partials_kernel(const float* __restrict__ partial, int nparts, int out,
                       uint16_t* __restrict__ y, float* __restrict__ y_f32) {
  __shared__ float red[8][33];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int o = blockIdx.x * 32 + lane;
  pdl_wait();
  float v = 0.f;
  if (o < out) {
#pragma unroll 4
    for (int c = warp; c < nparts; c += 8) v += partial[(size_t)c * out + o];
  }
  red[warp][lane] = v;
  __syncthreads();
  pdl_launch_dependents();
  if (warp == 0 && o < out) {
    float t = red[0][lane];
#pragma unroll
    for (int w = 1; w < 8; ++w) t += red[w][lane];
    if (y) y[o] = f32_to_bf16_bits(t);
    if (y_f32) y_f32[o] = t;
  }
}

size_t down_workspace_bytes(int64_t out) { return (size_t)kDownCtas * out * sizeof(float); }

bool down_shape_ok(int64_t out) { return out > 0 && out % kGroup == 0 && out / 32 <= 640; }

template <int MODE>
int launch_down(DownParams p, uint16_t* y, float* y_f32, void* ws, size_t ws_bytes,
                cudaStream_t st) {
  const int out = p.out_features;
  if (ws_bytes < down_workspace_bytes(out) || !ws) return DIP_ERR_WORKSPACE;
  p.partial = reinterpret_cast<float*>(ws);
  const int nch = out / 32;
  int teams = 640 / nch;
  if (teams > 4) teams = 4;
  const int nparts = p.k > 0 ? (p.k < kDownCtas ? p.k : kDownCtas) : 1;
  const size_t smem = (size_t)teams * out * sizeof(float);
  auto kern = gather_down_kernel<MODE>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return launch_status(e);
  }
  int st1 = launch_status(launch(kern, dim3(nparts), dim3(teams * nch), smem, st, p));
  if (st1 != DIP_OK) return st1;
  return launch_status(launch(reduce_partials_kernel, dim3((out + 31) / 32), dim3(256), 0, st,
                              (const float*)p.partial, nparts, out, y, y_f32));
}

template int launch_down<DROW_IDENT>(DownParams, uint16_t*, float*, void*, size_t, cudaStream_t);
template int launch_down<DROW_GATHER>(DownParams, uint16_t*, float*, void*, size_t, cudaStream_t);
template int launch_down<DROW_SRCROW>(DownParams, uint16_t*, float*, void*, size_t, cudaStream_t);

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace dip

using namespace dip;

extern "C" size_t dip_gather_down_workspace_bytes(int64_t out_features) {
  return down_workspace_bytes(out_features);
}

extern "C" int dip_int4_gather_down(const int8_t* down_t, const dip_bf16* scales, int64_t n_rows,
                                    const dip_bf16* h, const int32_t* idx, int64_t k,
                                    int64_t out_features, void* workspace,
                                    size_t workspace_bytes, dip_bf16* y, dip_stream_t stream) {
  if (k < 0 || k > INT32_MAX || n_rows < 0 || !down_shape_ok(out_features)) return DIP_ERR_ARG;
  if (!y) return DIP_ERR_ARG;
  if (k > 0 && (!down_t || !scales || !h || !al16(down_t) || n_rows == 0)) return DIP_ERR_ARG;
  DownParams p = {};
  p.qw0 = reinterpret_cast<const uint8_t*>(down_t);
  p.sc0 = scales;
  p.n0 = n_rows;
  p.h = h;
  p.idx = idx;
  p.k = (int)k;
  p.out_features = (int)out_features;
  if (k == 0) {
    // y = 0: run the reduction over one zero partial.
    if (workspace_bytes < down_workspace_bytes(out_features) || !workspace)
      return DIP_ERR_WORKSPACE;
    cudaError_t e = cudaMemsetAsync(workspace, 0, (size_t)out_features * 4, (cudaStream_t)stream);
    if (e != cudaSuccess) return launch_status(e);
    return launch_status(launch(reduce_partials_kernel, dim3((out_features + 31) / 32), dim3(256),
                                0, (cudaStream_t)stream, (const float*)workspace, 1,
                                (int)out_features, y, (float*)nullptr));
  }
  if (idx) return launch_down<DROW_GATHER>(p, y, nullptr, workspace, workspace_bytes,
                                           (cudaStream_t)stream);
  return launch_down<DROW_IDENT>(p, y, nullptr, workspace, workspace_bytes, (cudaStream_t)stream);
}

extern "C" int dip_srcrow_down(const int8_t* res_dt, const dip_bf16* res_sc, int64_t n_res,
                               const int8_t* full_dt, const dip_bf16* full_sc, int64_t n_full,
                               const dip_bf16* h, const int32_t* src, const int32_t* row, int64_t k,
                               int64_t out_features, void* workspace, size_t workspace_bytes,
                               dip_bf16* y, dip_stream_t stream) {
  if (k <= 0 || k > INT32_MAX || n_res < 0 || n_full <= 0 || !down_shape_ok(out_features))
    return DIP_ERR_ARG;
  if (!full_dt || !full_sc || !h || !src || !row || !y || !al16(full_dt)) return DIP_ERR_ARG;
  if (n_res > 0 && (!res_dt || !res_sc || !al16(res_dt))) return DIP_ERR_ARG;
  DownParams p = {};
  p.qw0 = reinterpret_cast<const uint8_t*>(n_res > 0 ? res_dt : full_dt);
  p.sc0 = n_res > 0 ? res_sc : full_sc;
  p.n0 = n_res;
  p.qw1 = reinterpret_cast<const uint8_t*>(full_dt);
  p.sc1 = full_sc;
  p.n1 = n_full;
  p.h = h;
  p.src = src;
  p.row = row;
  p.k = (int)k;
  p.out_features = (int)out_features;
  return launch_down<DROW_SRCROW>(p, y, nullptr, workspace, workspace_bytes,
                                  (cudaStream_t)stream);
}

extern "C" int dip_gather_down_partial(const int8_t* down_t, const dip_bf16* scales,
                                       int64_t n_rows, const dip_bf16* h, const int32_t* idx,
                                       const int32_t* count, int64_t max_k, int64_t out_features,
                                       void* workspace, size_t workspace_bytes, float* y_f32,
                                       dip_stream_t stream) {
  if (max_k <= 0 || max_k > INT32_MAX || n_rows <= 0 || !down_shape_ok(out_features))
    return DIP_ERR_ARG;
  if (!down_t || !scales || !h || !idx || !y_f32 || !al16(down_t)) return DIP_ERR_ARG;
  DownParams p = {};
  p.qw0 = reinterpret_cast<const uint8_t*>(down_t);
  p.sc0 = scales;
  p.n0 = n_rows;
  p.h = h;
  p.idx = idx;
  p.count = count;
  p.k = (int)max_k;
  p.out_features = (int)out_features;
  return launch_down<DROW_GATHER>(p, nullptr, y_f32, workspace, workspace_bytes,
                                  (cudaStream_t)stream);
}
