// gemv_batch.cu — int4 GEMV for a batch of up to 8 tokens per weight pass
// (batched decode, config 3: the gate GEMV + SiLU and the dense up GEMV).
//
// The GEMV kernels compute a 16-row x 16-column weight tile against x on
// mma.sync m16n8k16, whose B operand has 8 columns; a single token fills one
// of them.  Here column n carries token n, so one pass over the weights
// serves 8 tokens for almost the cost of one: the dequantisation (the SM-side
// bound of the GEMV) is shared, only the MMAs and the epilogue grow.
//
// Structure as the streaming GEMV (gemv_int4.cu, gemv_ks_kernel): one CTA of
// 8 warps per SM over a contiguous range of 16-row tiles; warp w owns the
// K-slice of quantisation groups [w*GW, (w+1)*GW) and keeps the x fragments
// of its slice in registers (lane (gq, tq) holds token gq's), streaming its
// bytes of every tile through a private 4-deep cp.async ring; per-tile partial
// sums go to shared memory and are combined in a fixed order after one
// barrier.  Per output (row, token): out = bf16(sum_c q*s*x) (the fp32 sum of
// int4_gemv.cu:39-87 per token), optionally g = bf16(silu(out)).
#include "dip_common.cuh"

namespace dip {
namespace {

constexpr int kBWarps = 8;
constexpr int kBThreads = kBWarps * 32;
constexpr int kBDepth = 4;
constexpr int kBTok = 8;  // tokens per weight pass (MMA N)

struct BGeom {
  int slot, w_bytes, red_off, gsum_off, total;
};
__host__ __device__ inline BGeom b_geom(int in, int max_tiles) {
  BGeom g;
  const int G = in / kGroup;
  const int gw = G / kBWarps;
  g.w_bytes = gw * 1024;       // 16 rows x GW x 64 B
  g.slot = g.w_bytes + 16 * 32;  // + 32 bytes of each of the 16 scale rows
  g.red_off = kBWarps * kBDepth * g.slot;
  g.gsum_off = g.red_off + max_tiles * kBWarps * 16 * kBTok * 4;  // [tile][warp][16 rows][8 tok]
  g.total = g.gsum_off + kBTok * G * 4;                           // [tok][group] sums of x
  return g;
}

__device__ __forceinline__ void cpa16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cpa_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cpa_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(kBDepth - 1) : "memory");
}

template <int GW>
__global__ void __launch_bounds__(kBThreads, 1)
gemv_batch_kernel(const uint8_t* __restrict__ qw, const uint16_t* __restrict__ sc,
                  const uint16_t* __restrict__ x, int ntok, uint16_t* __restrict__ out,
                  int rows, int in, int silu, int max_tiles) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int G = in / kGroup;
  const BGeom geo = b_geom(in, max_tiles);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const int rowb = in / 2;
  float* red = reinterpret_cast<float*>(smem + geo.red_off);
  float* gsum = reinterpret_cast<float*>(smem + geo.gsum_off);
  uint8_t* ring = smem + warp * kBDepth * geo.slot;

  const int nt = (rows + 15) / 16;
  const int t0 = (int)((int64_t)nt * blockIdx.x / gridDim.x);
  const int t1 = (int)((int64_t)nt * (blockIdx.x + 1) / gridDim.x);
  const int ntile = t1 - t0;
  const int sc_lo = (2 * GW * warp) & ~15;
  const int sc_shift = 2 * GW * warp - sc_lo;  // bytes
  auto issue = [&](int i) {
    if (i < ntile) {
      uint8_t* slot = ring + (i % kBDepth) * geo.slot;
      const int ra = min((t0 + i) * 16 + gq, rows - 1), rb = min((t0 + i) * 16 + gq + 8, rows - 1);
#pragma unroll
      for (int gi = 0; gi < GW; ++gi) {
        const int off = (warp * GW + gi) * kGroupBytes + tq * 16;
        cpa16(slot + (gi * 2 + 0) * 512 + lane * 16, qw + (size_t)ra * rowb + off);
        cpa16(slot + (gi * 2 + 1) * 512 + lane * 16, qw + (size_t)rb * rowb + off);
      }
      const int rs = min((t0 + i) * 16 + (lane >> 1), rows - 1);
      const int sofs = sc_lo + (lane & 1) * 16;
      if (sofs < 2 * G)
        cpa16(slot + geo.w_bytes + lane * 16,
              reinterpret_cast<const uint8_t*>(sc + (size_t)rs * G) + sofs);
    }
    cpa_commit();
  };
#pragma unroll
  for (int i = 0; i < kBDepth - 1; ++i) issue(i);
  pdl_wait();

  // x fragments of token gq for this warp's groups, and the per-group sums of
  // x for every token (the 136 * sum(x) bias of the biased nibble decode)
  uint32_t xf[GW][16];
  const bool tok_ok = gq < ntok;
#pragma unroll
  for (int gi = 0; gi < GW; ++gi) {
    const int grp = warp * GW + gi;
    float pw[4];  // sums of the group's 16 words tq*4 + w of x (8 values each)
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const int wi = grp * 16 + tq * 4 + w;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (tok_ok) v = __ldg(reinterpret_cast<const uint4*>(x + (size_t)gq * in) + wi);
      xf[gi][4 * w + 0] = __byte_perm(v.x, v.z, 0x5410);
      xf[gi][4 * w + 1] = __byte_perm(v.x, v.z, 0x7632);
      xf[gi][4 * w + 2] = __byte_perm(v.y, v.w, 0x5410);
      xf[gi][4 * w + 3] = __byte_perm(v.y, v.w, 0x7632);
      pw[w] = bf16_bits_to_f32(v.x & 0xFFFF) + bf16_bits_to_f32(v.x >> 16) +
              bf16_bits_to_f32(v.y & 0xFFFF) + bf16_bits_to_f32(v.y >> 16) +
              bf16_bits_to_f32(v.z & 0xFFFF) + bf16_bits_to_f32(v.z >> 16) +
              bf16_bits_to_f32(v.w & 0xFFFF) + bf16_bits_to_f32(v.w >> 16);
    }
    // the single-token GEMV's butterfly over the 16 words (xor 8, 4, 2, 1 on
    // the word index), so that the bias and hence every output match it bit
    // for bit: word ^ 8 is lane tq ^ 2, word ^ 4 is tq ^ 1, word ^ 2 and ^ 1
    // are this lane's own words
    float s1[4], s2[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) s1[w] = pw[w] + __shfl_xor_sync(0xffffffffu, pw[w], 2);
#pragma unroll
    for (int w = 0; w < 4; ++w) s2[w] = s1[w] + __shfl_xor_sync(0xffffffffu, s1[w], 1);
    const float s30 = s2[0] + s2[2], s31 = s2[1] + s2[3];
    const float part = s30 + s31;
    if (tq == 0) gsum[gq * G + grp] = part;
  }
  __syncthreads();
  // this lane's outputs are tokens 2tq and 2tq + 1 (MMA C columns)
  float bias0[GW], bias1[GW];
#pragma unroll
  for (int gi = 0; gi < GW; ++gi) {
    const int grp = warp * GW + gi;
    bias0[gi] = kNibbleBias * gsum[(2 * tq) * G + grp];
    bias1[gi] = kNibbleBias * gsum[(2 * tq + 1) * G + grp];
  }

  for (int i = 0; i < ntile; ++i) {
    issue(i + kBDepth - 1);
    cpa_wait();
    __syncwarp();
    const uint8_t* slot = ring + (i % kBDepth) * geo.slot;
    const uint16_t* sca = reinterpret_cast<const uint16_t*>(slot + geo.w_bytes + gq * 32 + sc_shift);
    const uint16_t* scb = reinterpret_cast<const uint16_t*>(slot + geo.w_bytes + (gq + 8) * 32 + sc_shift);
    float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;  // (row gq | gq + 8) x (token 2tq | 2tq + 1)
#pragma unroll
    for (int gi = 0; gi < GW; ++gi) {
      const uint4 wa = *reinterpret_cast<const uint4*>(slot + (gi * 2 + 0) * 512 + lane * 16);
      const uint4 wb = *reinterpret_cast<const uint4*>(slot + (gi * 2 + 1) * 512 + lane * 16);
      const uint32_t ra[4] = {wa.x, wa.y, wa.z, wa.w};
      const uint32_t rb[4] = {wb.x, wb.y, wb.z, wb.w};
      float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        uint32_t qa4[4], qb4[4];
        nib8_biased_bf16x2(ra[w], qa4);
        nib8_biased_bf16x2(rb[w], qb4);
        const uint32_t a_even[4] = {qa4[0], qb4[0], qa4[1], qb4[1]};
        const uint32_t a_odd[4] = {qa4[2], qb4[2], qa4[3], qb4[3]};
        mma_bf16_16816(d0, a_even, xf[gi][4 * w + 0], xf[gi][4 * w + 1]);
        mma_bf16_16816(d1, a_odd, xf[gi][4 * w + 2], xf[gi][4 * w + 3]);
      }
      const float sa = bf16_bits_to_f32(sca[gi]), sb = bf16_bits_to_f32(scb[gi]);
      a0 = fmaf(sa, (d0[0] + d1[0]) - bias0[gi], a0);
      a1 = fmaf(sa, (d0[1] + d1[1]) - bias1[gi], a1);
      b0 = fmaf(sb, (d0[2] + d1[2]) - bias0[gi], b0);
      b1 = fmaf(sb, (d0[3] + d1[3]) - bias1[gi], b1);
    }
    float* rt = red + ((size_t)(i * kBWarps + warp) * 16) * kBTok;
    rt[gq * kBTok + 2 * tq] = a0;
    rt[gq * kBTok + 2 * tq + 1] = a1;
    rt[(gq + 8) * kBTok + 2 * tq] = b0;
    rt[(gq + 8) * kBTok + 2 * tq + 1] = b1;
    __syncwarp();  // the slot is refilled by a later iteration's copies
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");
  pdl_launch_dependents();
  __syncthreads();
  for (int e = tid; e < ntile * 16 * kBTok; e += kBThreads) {
    const int t = e % kBTok, r = e / kBTok;
    const int i = r >> 4, row = r & 15;
    const int j = (t0 + i) * 16 + row;
    if (j >= rows || t >= ntok) continue;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kBWarps; ++w) v += red[((size_t)(i * kBWarps + w) * 16 + row) * kBTok + t];
    out[(size_t)t * rows + j] =
        silu ? f32_to_bf16_bits(silu_f32(round_bf16(v))) : f32_to_bf16_bits(v);
  }
}

template <int GW>
int launch_batch(const uint8_t* qw, const uint16_t* sc, const uint16_t* x, int ntok, uint16_t* out,
                 int rows, int in, int silu, cudaStream_t s) {
  const int nt = (rows + 15) / 16;
  const int grid = nt < num_sms() ? nt : num_sms();
  const int max_tiles = (nt + grid - 1) / grid;
  const BGeom geo = b_geom(in, max_tiles);
  if (geo.total > 227 * 1024) return DIP_ERR_UNSUPPORTED;
  auto kern = gemv_batch_kernel<GW>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, geo.total);
  if (e != cudaSuccess) return launch_status(e);
  return launch_status(launch(kern, dim3(grid), dim3(kBThreads), (size_t)geo.total, s, qw, sc, x,
                              ntok, out, rows, in, silu, max_tiles));
}

}  // namespace
}  // namespace dip

using namespace dip;

extern "C" int dip_int4_gemv_batched(const int8_t* qweight, const dip_bf16* scales,
                                     const dip_bf16* x, dip_bf16* out, int64_t rows,
                                     int64_t in_features, int64_t ntok, int apply_silu,
                                     dip_stream_t stream) {
  if (!qweight || !scales || !x || !out || rows <= 0 || in_features <= 0 || ntok <= 0)
    return DIP_ERR_ARG;
  if (in_features % (kGroup * kBWarps) != 0 || rows > INT32_MAX / 2) return DIP_ERR_UNSUPPORTED;
  const uintptr_t al = reinterpret_cast<uintptr_t>(qweight) | reinterpret_cast<uintptr_t>(x) |
                       reinterpret_cast<uintptr_t>(scales);
  if (al & 15) return DIP_ERR_ARG;
  const int gw = (int)(in_features / kGroup / kBWarps);
  for (int64_t t0 = 0; t0 < ntok; t0 += kBTok) {
    const int nt = (int)(ntok - t0 < kBTok ? ntok - t0 : kBTok);
    const uint8_t* q = reinterpret_cast<const uint8_t*>(qweight);
    const uint16_t* xs = x + t0 * in_features;
    uint16_t* o = out + t0 * rows;
    int st;
    switch (gw) {
      case 1: st = launch_batch<1>(q, scales, xs, nt, o, (int)rows, (int)in_features, apply_silu, (cudaStream_t)stream); break;
      case 2: st = launch_batch<2>(q, scales, xs, nt, o, (int)rows, (int)in_features, apply_silu, (cudaStream_t)stream); break;
      case 3: st = launch_batch<3>(q, scales, xs, nt, o, (int)rows, (int)in_features, apply_silu, (cudaStream_t)stream); break;
      case 4: st = launch_batch<4>(q, scales, xs, nt, o, (int)rows, (int)in_features, apply_silu, (cudaStream_t)stream); break;
      case 5: st = launch_batch<5>(q, scales, xs, nt, o, (int)rows, (int)in_features, apply_silu, (cudaStream_t)stream); break;
      default: return DIP_ERR_UNSUPPORTED;
    }
    if (st != DIP_OK) return st;
  }
  return DIP_OK;
}
