// gemv_int4.cu — batch-1 int4 (g128) GEMV family for sm_100a.
//
// One kernel serves four reference operations, selected by template
// parameters:
//   * dense rows           -> int4_ops::int4_gemv (+ fused SiLU)
//                             reference: kernels/int4_gemv/int4_gemv.cu:39-108
//   * rows gathered by idx -> int4_gather_ops::int4_gather_gemv
//                             reference: kernels/int4_gather/int4_gather_gemv.cu:39-108
//   * (src,row) dual source-> ca_fused_ops::ca_fused_gemv
//                             reference: kernels/ca_fused/ca_fused_gemv.cu:44-105
//   * optional epilogue h = bf16(g[c] * bf16(u))  (dip_stream_predispatch.py:201)
//
// Design.  A CTA of 4 warps owns a tile of 16 output rows; warp w handles
// the quantisation groups w, w+4, w+8, ... of every row, so the 4 warps read
// 256 contiguous bytes of each row at a time.  Lane (g = lane/4, t = lane%4)
// loads 16 B (32 nibbles) of rows g and g+8 per group with one 128-bit
// non-allocating load each.  Nibbles become bf16 values q+136 in registers
// (magic-number conversion, 7 integer ops per 8 nibbles, no conversion
// instructions) and feed mma.sync m16n8k16 with fp32 accumulation: the tensor
// core performs the multiply-adds and the cross-lane reduction that a
// CUDA-core GEMV spends most of its issue slots on.  x is staged once per CTA
// in shared memory, permuted so that each lane's B fragment is 4 LDS.128.
// The constant bias 136 is removed per group with the group sum of x:
//   sum_k (q+136) x = sum_k q x + 136 * sum_k x.
// Each group's partial is scaled by its bf16 scale in fp32, and the 4 warps'
// partials are summed in a fixed order (deterministic).
#include "dip_common.cuh"

namespace dip {

enum RowMode : int { ROW_DENSE = 0, ROW_GATHER = 1, ROW_SRCROW = 2 };
enum Epilogue : int { EPI_PLAIN = 0, EPI_SILU = 1, EPI_H = 2 };

struct GemvParams {
  const uint8_t* qw0;  // source 0 rows [n0, in/2]
  const uint16_t* sc0; // source 0 scales [n0, in/128]
  int64_t n0;
  const uint8_t* qw1;  // source 1 (ROW_SRCROW, src == 1)
  const uint16_t* sc1;
  int64_t n1;
  const uint16_t* x;   // [in]
  const int32_t* idx;  // ROW_GATHER: row of output j
  const int32_t* src;  // ROW_SRCROW: source of output j
  const int32_t* row;  // ROW_SRCROW: row within that source
  const uint16_t* g;   // EPI_H: gate activations by channel id
  const int32_t* gid;  // EPI_H: channel id of output j
  uint16_t* out;       // [n_out]
  const int32_t* count;  // optional device-side number of outputs (<= n_out)
  unsigned* hist;        // EPI_SILU: optional 32768-bin histogram of |g| (bf16 bits)
  int n_out;
  int in_features;
};

constexpr int kGemvWarps = 4;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kGemvBatch = 5;  // groups whose loads are in flight per warp

// Counts one output's |g| (15-bit bf16 magnitude) into the top-k histogram;
// NaN is never counted, matching the top-k's exclusion of NaN.
__device__ __forceinline__ void hist_count(unsigned* hist, uint16_t o) {
  const unsigned key = o & 0x7FFFu;
  if (hist && key <= 0x7F80u) {
    atomicAdd(&hist[key], 1u);
    atomicAdd(&hist[kTopkHistBins + (key >> 7)], 1u);
  }
}

template <int MODE>
__device__ __forceinline__ bool resolve_row(const GemvParams& p, int j, const uint8_t*& qw,
                                            const uint16_t*& sc) {
  const int64_t rb = p.in_features / 2;
  const int64_t sb = p.in_features / kGroup;
  int64_t r;
  int s = 0;
  if (MODE == ROW_DENSE) {
    r = j;
  } else if (MODE == ROW_GATHER) {
    r = p.idx[j];
  } else {
    s = p.src[j];
    r = p.row[j];
  }
  const int64_t n = (s == 0) ? p.n0 : p.n1;
  const bool ok = (s == 0 || s == 1) && r >= 0 && r < n;
  if (!ok) r = 0;
  const uint8_t* q = (s == 0) ? p.qw0 : p.qw1;
  const uint16_t* c = (s == 0) ? p.sc0 : p.sc1;
  if (!ok) { q = p.qw0; c = p.sc0; }
  qw = q + r * rb;
  sc = c + r * sb;
  return ok;
}

template <int MODE, int EPI>
__global__ void __launch_bounds__(kGemvThreads)
gemv_int4_kernel(const GemvParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int in = p.in_features;
  const int G = in / kGroup;
  uint32_t* xperm = reinterpret_cast<uint32_t*>(smem_raw);              // in/2 words
  float* gsum = reinterpret_cast<float*>(smem_raw + (size_t)in * 2);    // G
  float* red = gsum + G;                                                // [4][16]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int gq = lane >> 2;  // fragment row group
  const int tq = lane & 3;   // fragment column quad
  const int tile0 = blockIdx.x * 16;

  // Row indices of gathered modes (and a device-side count) come from the
  // previous kernel.
  if (MODE != ROW_DENSE) pdl_wait();
  int n_out = p.n_out;
  if (p.count) n_out = min(n_out, *p.count);
  if (tile0 >= n_out) return;
  // Rows of this lane: tile0+gq and tile0+gq+8 (clamped for the last tile).
  const int ja = min(tile0 + gq, n_out - 1);
  const int jb = min(tile0 + gq + 8, n_out - 1);

  const uint8_t *qa, *qb;
  const uint16_t *sa_p, *sb_p;
  const bool oka = resolve_row<MODE>(p, ja, qa, sa_p);
  const bool okb = resolve_row<MODE>(p, jb, qb, sb_p);

  // First batch of weight loads is issued before waiting on the predecessor
  // (weights are never written by it).
  uint4 wa[kGemvBatch], wb[kGemvBatch];
  float sa[kGemvBatch], sbv[kGemvBatch];
  auto load_batch = [&](int base) {
#pragma unroll
    for (int u = 0; u < kGemvBatch; ++u) {
      const int grp = base + kGemvWarps * u;
      if (grp < G) {
        const int off = grp * kGroupBytes + tq * 16;
        wa[u] = ldg_stream_u4(qa + off);
        wb[u] = ldg_stream_u4(qb + off);
        sa[u] = bf16_bits_to_f32(ldg_u16(sa_p + grp));
        sbv[u] = bf16_bits_to_f32(ldg_u16(sb_p + grp));
      }
    }
  };
  load_batch(warp);
  if (MODE == ROW_DENSE) pdl_wait();

  // Stage x: each 8-column word (x0..x7) is stored as
  // [(x0,x4),(x1,x5),(x2,x6),(x3,x7)] which is the B-fragment order matching
  // the nibble pairing of nib8_biased_bf16x2; also the per-group sums of x.
  {
    const int nwords = in / 8;
    const uint4* xv = reinterpret_cast<const uint4*>(p.x);
    for (int wi = threadIdx.x; wi < ((nwords + 127) & ~127); wi += kGemvThreads) {
      float part = 0.f;
      if (wi < nwords) {
        const uint4 v = __ldg(xv + wi);
        uint4 o;
        o.x = __byte_perm(v.x, v.z, 0x5410);
        o.y = __byte_perm(v.x, v.z, 0x7632);
        o.z = __byte_perm(v.y, v.w, 0x5410);
        o.w = __byte_perm(v.y, v.w, 0x7632);
        reinterpret_cast<uint4*>(xperm)[wi] = o;
        part = bf16_bits_to_f32(v.x & 0xFFFF) + bf16_bits_to_f32(v.x >> 16) +
               bf16_bits_to_f32(v.y & 0xFFFF) + bf16_bits_to_f32(v.y >> 16) +
               bf16_bits_to_f32(v.z & 0xFFFF) + bf16_bits_to_f32(v.z >> 16) +
               bf16_bits_to_f32(v.w & 0xFFFF) + bf16_bits_to_f32(v.w >> 16);
      }
      // 16 consecutive words form one group; they sit in 16 consecutive lanes.
      part += __shfl_xor_sync(0xffffffffu, part, 8);
      part += __shfl_xor_sync(0xffffffffu, part, 4);
      part += __shfl_xor_sync(0xffffffffu, part, 2);
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      if ((lane & 15) == 0 && wi < nwords) gsum[wi >> 4] = part;
    }
  }
  __syncthreads();

  float acc_a = 0.f, acc_b = 0.f;
  for (int base = warp; base < G; base += kGemvWarps * kGemvBatch) {
    if (base != warp) load_batch(base);
#pragma unroll
    for (int u = 0; u < kGemvBatch; ++u) {
      const int grp = base + kGemvWarps * u;
      if (grp < G) {
        const uint4* bp = reinterpret_cast<const uint4*>(xperm + grp * 64 + tq * 16);
        const uint4 b01 = bp[0], b23 = bp[1], b45 = bp[2], b67 = bp[3];
        const uint32_t bw[16] = {b01.x, b01.y, b01.z, b01.w, b23.x, b23.y, b23.z, b23.w,
                                 b45.x, b45.y, b45.z, b45.w, b67.x, b67.y, b67.z, b67.w};
        const uint32_t ra[4] = {wa[u].x, wa[u].y, wa[u].z, wa[u].w};
        const uint32_t rb[4] = {wb[u].x, wb[u].y, wb[u].z, wb[u].w};
        float d0[4] = {0.f, 0.f, 0.f, 0.f};
        float d1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          uint32_t qa4[4], qb4[4];
          nib8_biased_bf16x2(ra[w], qa4);
          nib8_biased_bf16x2(rb[w], qb4);
          const uint32_t a_even[4] = {qa4[0], qb4[0], qa4[1], qb4[1]};
          const uint32_t a_odd[4] = {qa4[2], qb4[2], qa4[3], qb4[3]};
          mma_bf16_16816(d0, a_even, bw[4 * w + 0], bw[4 * w + 1]);
          mma_bf16_16816(d1, a_odd, bw[4 * w + 2], bw[4 * w + 3]);
        }
        const float bias = kNibbleBias * gsum[grp];
        acc_a = fmaf(sa[u], (d0[0] + d1[0]) - bias, acc_a);
        acc_b = fmaf(sbv[u], (d0[2] + d1[2]) - bias, acc_b);
      }
    }
  }
  pdl_launch_dependents();

  if (tq == 0) {
    red[warp * 16 + gq] = acc_a;
    red[warp * 16 + gq + 8] = acc_b;
  }
  __syncthreads();
  if (threadIdx.x < 16) {
    const int j = tile0 + threadIdx.x;
    if (j < n_out) {
      float v = red[threadIdx.x];
#pragma unroll
      for (int w = 1; w < kGemvWarps; ++w) v += red[w * 16 + threadIdx.x];
      const bool ok = (threadIdx.x < 8) ? oka : okb;
      uint16_t o;
      if (!ok) {
        o = 0;
      } else if (EPI == EPI_PLAIN) {
        o = f32_to_bf16_bits(v);
      } else if (EPI == EPI_SILU) {
        o = f32_to_bf16_bits(silu_f32(round_bf16(v)));
        hist_count(p.hist, o);
      } else {
        const float u = round_bf16(v);
        const float gv = bf16_bits_to_f32(p.g[p.gid[j]]);
        o = f32_to_bf16_bits(gv * u);
      }
      p.out[j] = o;
    }
  }
}

__device__ __forceinline__ void group_mma(const uint4& wa, const uint4& wb, const uint32_t* bw,
                                          float (&d0)[4], float (&d1)[4]) {
  const uint32_t ra[4] = {wa.x, wa.y, wa.z, wa.w};
  const uint32_t rb[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    uint32_t qa4[4], qb4[4];
    nib8_biased_bf16x2(ra[w], qa4);
    nib8_biased_bf16x2(rb[w], qb4);
    const uint32_t a_even[4] = {qa4[0], qb4[0], qa4[1], qb4[1]};
    const uint32_t a_odd[4] = {qa4[2], qb4[2], qa4[3], qb4[3]};
    mma_bf16_16816(d0, a_even, bw[4 * w + 0], bw[4 * w + 1]);
    mma_bf16_16816(d1, a_odd, bw[4 * w + 2], bw[4 * w + 3]);
  }
}

// cp.async helpers of the streaming GEMV below.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
// Waits until at most n committed groups of this thread are still pending.
__device__ __forceinline__ void cp_async_wait(int n) {
  switch (n) {
#define DIP_WAIT_CASE(N) case N: asm volatile("cp.async.wait_group " #N ";\n" ::: "memory"); break;
    DIP_WAIT_CASE(0) DIP_WAIT_CASE(1) DIP_WAIT_CASE(2) DIP_WAIT_CASE(3) DIP_WAIT_CASE(4)
    DIP_WAIT_CASE(5) DIP_WAIT_CASE(6) DIP_WAIT_CASE(7) DIP_WAIT_CASE(8) DIP_WAIT_CASE(9)
    DIP_WAIT_CASE(10) DIP_WAIT_CASE(11) DIP_WAIT_CASE(12) DIP_WAIT_CASE(13) DIP_WAIT_CASE(14)
    default: asm volatile("cp.async.wait_group 15;\n" ::: "memory"); break;
#undef DIP_WAIT_CASE
  }
}

// x staging layout: group g occupies 72 words; lane quad t's 16 words start
// at word 16 t + 4 (t >> 1), which puts the four quads in distinct banks.
__device__ __forceinline__ int xperm_word(int grp, int t) { return grp * 72 + t * 16 + (t >> 1) * 4; }

// ---------------------------------------------------------------------------
// Default variant: persistent K-slice streaming, no per-tile synchronisation.
//
// One CTA of 8 warps per SM takes a contiguous range of 16-row tiles.  Warp w
// owns the K-slice of quantisation groups [w*GW, (w+1)*GW) for EVERY tile of
// the CTA, so its x fragments and group sums live in registers for the whole
// kernel and the work of an SM is split evenly between its warps.  Each warp
// streams its slice of each tile (16 rows x GW x 64 B) plus the covering
// 32 bytes of the 16 scale rows through a private 4-deep shared-memory ring
// with 16-byte cp.async.cg copies and never waits for another warp: its
// per-tile partial sums go to shared memory, and the 8 slices of every row
// are combined, in a fixed order, once after a single barrier at the end.
// (Measured on B200: rolling per-warp cp.async pipelines stream at ~6.4 TB/s
// with ~40 KB in flight per SM; the same GEMV with a block barrier per tile
// stalled at 2.5-3 TB/s, and 8-row whole-K tiles per warp at ~2 TB/s because
// of x-fragment reloads and uneven warp loads.)
constexpr int kKsWarps = 8;
constexpr int kKsThreads = kKsWarps * 32;
constexpr int kKsDepth = 4;

struct KsGeom {
  int gw, slot, w_bytes, ring_off, ptr_off, info_off, red_off, x_off, gsum_off, total;
};
__host__ __device__ inline KsGeom ks_geom(int in, int max_tiles) {
  KsGeom g;
  const int G = in / kGroup;
  g.gw = G / kKsWarps;
  g.w_bytes = g.gw * 1024;            // 16 rows x GW x 64 B
  g.slot = g.w_bytes + 16 * 32;       // + 32 bytes of each of the 16 scale rows
  g.ring_off = 0;
  g.ptr_off = kKsWarps * kKsDepth * g.slot;
  g.info_off = g.ptr_off + max_tiles * 16 * 16;
  g.red_off = g.info_off + max_tiles * 16 * 4;
  g.x_off = g.red_off + max_tiles * kKsWarps * 16 * 4;
  g.gsum_off = g.x_off + G * 72 * 4;
  g.total = g.gsum_off + ((G * 4 + 15) & ~15);
  return g;
}

template <int MODE, int EPI, int GW>
__global__ void __launch_bounds__(kKsThreads, 1)
gemv_ks_kernel(const GemvParams p, int max_tiles) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int in = p.in_features;
  const int G = in / kGroup;
  const KsGeom geo = ks_geom(in, max_tiles);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const uint8_t** rq = reinterpret_cast<const uint8_t**>(smem + geo.ptr_off);
  const uint16_t** rs = reinterpret_cast<const uint16_t**>(smem + geo.ptr_off) + max_tiles * 16;
  float* info = reinterpret_cast<float*>(smem + geo.info_off);  // NaN marks an invalid row
  float* red = reinterpret_cast<float*>(smem + geo.red_off);    // [tile][warp][16]
  uint32_t* xs = reinterpret_cast<uint32_t*>(smem + geo.x_off);
  float* gsum = reinterpret_cast<float*>(smem + geo.gsum_off);
  uint8_t* ring = smem + geo.ring_off + warp * kKsDepth * geo.slot;

  // |g| histogram: fine bins straight to global memory (spread out), coarse
  // bins (one per exponent, a handful of them hot) aggregated per CTA first.
  __shared__ unsigned s_coarse[(EPI == EPI_SILU) ? 256 : 1];
  if (EPI == EPI_SILU)
    for (int i = threadIdx.x; i < 256; i += blockDim.x) s_coarse[i] = 0u;
  if (MODE != ROW_DENSE) pdl_wait();
  int n_out = p.n_out;
  if (p.count) n_out = min(n_out, *p.count);
  const int nt = (n_out + 15) / 16;
  const int t0 = (int)((int64_t)nt * blockIdx.x / gridDim.x);
  const int t1 = (int)((int64_t)nt * (blockIdx.x + 1) / gridDim.x);
  const int ntile = t1 - t0;
  for (int r = tid; r < ntile * 16; r += kKsThreads) {
    const int j = min(t0 * 16 + r, n_out - 1);
    const uint8_t* qw;
    const uint16_t* sc;
    const bool ok = resolve_row<MODE>(p, j, qw, sc);
    rq[r] = qw;
    rs[r] = sc;
    float v = ok ? 0.f : __int_as_float(0x7FC00000);
    if (EPI == EPI_H && ok) v = bf16_bits_to_f32(p.g[p.gid[j]]);
    info[r] = v;
  }
  __syncthreads();

  // Scale bytes of this slice: [2*GW*warp, 2*GW*(warp+1)) of each scale row,
  // covered by the 32 bytes starting at the 16-byte boundary below it.
  const int sc_lo = (2 * GW * warp) & ~15;
  const int sc_shift = 2 * GW * warp - sc_lo;  // bytes
  auto issue = [&](int i) {
    if (i < ntile) {
      uint8_t* slot = ring + (i % kKsDepth) * geo.slot;
      const uint8_t* qa = rq[i * 16 + gq];
      const uint8_t* qb = rq[i * 16 + gq + 8];
#pragma unroll
      for (int gi = 0; gi < GW; ++gi) {
        const int off = (warp * GW + gi) * kGroupBytes + tq * 16;
        cp_async16(slot + (gi * 2 + 0) * 512 + lane * 16, qa + off);
        cp_async16(slot + (gi * 2 + 1) * 512 + lane * 16, qb + off);
      }
      // lane -> scale row lane/2, 16-byte half lane%2
      const uint8_t* srow = reinterpret_cast<const uint8_t*>(rs[i * 16 + (lane >> 1)]);
      const int sofs = sc_lo + (lane & 1) * 16;
      if (sofs < 2 * G) cp_async16(slot + geo.w_bytes + lane * 16, srow + sofs);
    }
    cp_async_commit();
  };
#pragma unroll
  for (int i = 0; i < kKsDepth - 1; ++i) issue(i);

  if (MODE == ROW_DENSE) pdl_wait();
  {
    const int nwords = in / 8;
    const uint4* xv = reinterpret_cast<const uint4*>(p.x);
    for (int wi = tid; wi < ((nwords + kKsThreads - 1) / kKsThreads) * kKsThreads;
         wi += kKsThreads) {
      float part = 0.f;
      if (wi < nwords) {
        const uint4 v = __ldg(xv + wi);
        uint4 o;
        o.x = __byte_perm(v.x, v.z, 0x5410);
        o.y = __byte_perm(v.x, v.z, 0x7632);
        o.z = __byte_perm(v.y, v.w, 0x5410);
        o.w = __byte_perm(v.y, v.w, 0x7632);
        const int grp = wi >> 4, t = (wi >> 2) & 3, w = wi & 3;
        *reinterpret_cast<uint4*>(xs + xperm_word(grp, t) + 4 * w) = o;
        part = bf16_bits_to_f32(v.x & 0xFFFF) + bf16_bits_to_f32(v.x >> 16) +
               bf16_bits_to_f32(v.y & 0xFFFF) + bf16_bits_to_f32(v.y >> 16) +
               bf16_bits_to_f32(v.z & 0xFFFF) + bf16_bits_to_f32(v.z >> 16) +
               bf16_bits_to_f32(v.w & 0xFFFF) + bf16_bits_to_f32(v.w >> 16);
      }
      part += __shfl_xor_sync(0xffffffffu, part, 8);
      part += __shfl_xor_sync(0xffffffffu, part, 4);
      part += __shfl_xor_sync(0xffffffffu, part, 2);
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      if ((lane & 15) == 0 && wi < nwords) gsum[wi >> 4] = part;
    }
  }
  __syncthreads();
  uint32_t xf[GW][16];
  float bias[GW];
#pragma unroll
  for (int gi = 0; gi < GW; ++gi) {
    const int grp = warp * GW + gi;
    const uint4* bp = reinterpret_cast<const uint4*>(xs + xperm_word(grp, tq));
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 b = bp[q];
      xf[gi][4 * q + 0] = b.x; xf[gi][4 * q + 1] = b.y;
      xf[gi][4 * q + 2] = b.z; xf[gi][4 * q + 3] = b.w;
    }
    bias[gi] = kNibbleBias * gsum[grp];
  }

  for (int i = 0; i < ntile; ++i) {
    issue(i + kKsDepth - 1);
    cp_async_wait(kKsDepth - 1);
    __syncwarp();  // scale bytes were copied by other lanes of this warp
    const uint8_t* slot = ring + (i % kKsDepth) * geo.slot;
    const uint16_t* sca =
        reinterpret_cast<const uint16_t*>(slot + geo.w_bytes + gq * 32 + sc_shift);
    const uint16_t* scb =
        reinterpret_cast<const uint16_t*>(slot + geo.w_bytes + (gq + 8) * 32 + sc_shift);
    float acc_a = 0.f, acc_b = 0.f;
#pragma unroll
    for (int gi = 0; gi < GW; ++gi) {
      const uint4 wa = *reinterpret_cast<const uint4*>(slot + (gi * 2 + 0) * 512 + lane * 16);
      const uint4 wb = *reinterpret_cast<const uint4*>(slot + (gi * 2 + 1) * 512 + lane * 16);
      float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
      group_mma(wa, wb, xf[gi], d0, d1);
      acc_a = fmaf(bf16_bits_to_f32(sca[gi]), (d0[0] + d1[0]) - bias[gi], acc_a);
      acc_b = fmaf(bf16_bits_to_f32(scb[gi]), (d0[2] + d1[2]) - bias[gi], acc_b);
    }
    if (tq == 0) {
      red[(i * kKsWarps + warp) * 16 + gq] = acc_a;
      red[(i * kKsWarps + warp) * 16 + gq + 8] = acc_b;
    }
    __syncwarp();  // the slot is refilled by a later iteration's copies
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");
  pdl_launch_dependents();
  __syncthreads();
  for (int r = tid; r < ntile * 16; r += kKsThreads) {
    const int j = t0 * 16 + r;
    if (j >= n_out) continue;
    const int i = r >> 4, row = r & 15;
    float v = red[(i * kKsWarps) * 16 + row];
#pragma unroll
    for (int w = 1; w < kKsWarps; ++w) v += red[(i * kKsWarps + w) * 16 + row];
    const float inf = info[r];
    uint16_t o;
    if (inf != inf) {
      o = 0;  // invalid row index
    } else if (EPI == EPI_PLAIN) {
      o = f32_to_bf16_bits(v);
    } else if (EPI == EPI_SILU) {
      o = f32_to_bf16_bits(silu_f32(round_bf16(v)));
      const unsigned key = o & 0x7FFFu;
      if (p.hist && key <= 0x7F80u) {
        atomicAdd(&p.hist[key], 1u);
        atomicAdd(&s_coarse[key >> 7], 1u);
      }
    } else {
      o = f32_to_bf16_bits(inf * round_bf16(v));
    }
    p.out[j] = o;
  }
  if (EPI == EPI_SILU && p.hist) {
    __syncthreads();
    for (int i = tid; i < 256; i += kKsThreads)
      if (s_coarse[i]) atomicAdd(&p.hist[kTopkHistBins + i], s_coarse[i]);
  }
}

template <int MODE, int EPI, int GW>
static int launch_ks(const GemvParams& p, cudaStream_t s) {
  const int nt = (p.n_out + 15) / 16;
  const int grid = nt < num_sms() ? nt : num_sms();
  const int max_tiles = (nt + grid - 1) / grid;
  const KsGeom geo = ks_geom(p.in_features, max_tiles);
  auto kern = gemv_ks_kernel<MODE, EPI, GW>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       geo.total);
  if (e != cudaSuccess) return launch_status(e);
  return launch_status(launch(kern, dim3(grid), dim3(kKsThreads), (size_t)geo.total, s, p,
                              max_tiles));
}

// Needs whole 8-way K slices (G % 8 == 0), 16-byte aligned scale rows and a
// ring that fits in shared memory.
static bool ks_ok(const GemvParams& p) {
  const int G = p.in_features / kGroup;
  if (G % kKsWarps != 0 || G / kKsWarps > 6) return false;
  if ((reinterpret_cast<uintptr_t>(p.sc0) & 15) != 0) return false;
  if (p.qw1 && (reinterpret_cast<uintptr_t>(p.sc1) & 15) != 0) return false;
  const int nt = (p.n_out + 15) / 16;
  const int grid = nt < num_sms() ? nt : num_sms();
  return ks_geom(p.in_features, (nt + grid - 1) / grid).total <= 225 * 1024;
}

template <int MODE, int EPI>
static int launch_ks_any(const GemvParams& p, cudaStream_t s) {
  switch (p.in_features / kGroup / kKsWarps) {
    case 1: return launch_ks<MODE, EPI, 1>(p, s);
    case 2: return launch_ks<MODE, EPI, 2>(p, s);
    case 3: return launch_ks<MODE, EPI, 3>(p, s);
    case 4: return launch_ks<MODE, EPI, 4>(p, s);
    case 5: return launch_ks<MODE, EPI, 5>(p, s);
    default: return launch_ks<MODE, EPI, 6>(p, s);
  }
}

// Host launcher shared by the entry points below.
template <int MODE, int EPI>
static int launch_gemv(const GemvParams& p, cudaStream_t s) {
  if (p.n_out == 0) return DIP_OK;
  if (!force_simple_gemv() && ks_ok(p)) return launch_ks_any<MODE, EPI>(p, s);
  const int G = p.in_features / kGroup;
  const size_t smem = (size_t)p.in_features * 2 + (size_t)G * 4 + kGemvWarps * 16 * 4;
  auto kern = gemv_int4_kernel<MODE, EPI>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return launch_status(e);
  }
  const dim3 grid((p.n_out + 15) / 16);
  return launch_status(launch(kern, grid, dim3(kGemvThreads), smem, s, p));
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static bool gemv_shape_ok(int64_t in_features) {
  return in_features > 0 && in_features % kGroup == 0 && in_features <= 65536;
}

}  // namespace dip

namespace dip {
// Gate GEMV + SiLU that also fills the top-k histogram (used by the fused
// decode chain; `hist` must be zero on entry, the top-k leaves it zero).
int gemv_silu_hist(const int8_t* qweight, const uint16_t* scales, const uint16_t* x,
                   uint16_t* out, int64_t rows, int64_t in_features, unsigned* hist,
                   cudaStream_t stream) {
  if (rows <= 0 || rows > INT32_MAX || !gemv_shape_ok(in_features)) return DIP_ERR_ARG;
  if (!qweight || !scales || !x || !out || !hist || !aligned16(qweight) || !aligned16(x))
    return DIP_ERR_ARG;
  GemvParams p = {};
  p.qw0 = reinterpret_cast<const uint8_t*>(qweight);
  p.sc0 = scales;
  p.n0 = rows;
  p.x = x;
  p.out = out;
  p.hist = hist;
  p.n_out = (int)rows;
  p.in_features = (int)in_features;
  return launch_gemv<ROW_DENSE, EPI_SILU>(p, stream);
}
}  // namespace dip

using namespace dip;

extern "C" int dip_int4_gemv(const int8_t* qweight, const dip_bf16* scales, const dip_bf16* x,
                             dip_bf16* out, int64_t rows, int64_t in_features, int apply_silu,
                             dip_stream_t stream) {
  if (rows < 0 || rows > INT32_MAX || !gemv_shape_ok(in_features)) return DIP_ERR_ARG;
  if (rows == 0) return DIP_OK;
  if (!qweight || !scales || !x || !out || !aligned16(qweight) || !aligned16(x))
    return DIP_ERR_ARG;
  GemvParams p = {};
  p.qw0 = reinterpret_cast<const uint8_t*>(qweight);
  p.sc0 = scales;
  p.n0 = rows;
  p.x = x;
  p.out = out;
  p.n_out = (int)rows;
  p.in_features = (int)in_features;
  return apply_silu ? launch_gemv<ROW_DENSE, EPI_SILU>(p, (cudaStream_t)stream)
                    : launch_gemv<ROW_DENSE, EPI_PLAIN>(p, (cudaStream_t)stream);
}

extern "C" int dip_int4_gather_gemv(const int8_t* qweight, const dip_bf16* scales,
                                    int64_t n_rows, const dip_bf16* x, const int32_t* indices,
                                    int64_t k, int64_t in_features, dip_bf16* out,
                                    dip_stream_t stream) {
  if (k < 0 || k > INT32_MAX || n_rows < 0 || !gemv_shape_ok(in_features)) return DIP_ERR_ARG;
  if (k == 0) return DIP_OK;
  if (!qweight || !scales || !x || !indices || !out || n_rows == 0 || !aligned16(qweight) ||
      !aligned16(x))
    return DIP_ERR_ARG;
  GemvParams p = {};
  p.qw0 = reinterpret_cast<const uint8_t*>(qweight);
  p.sc0 = scales;
  p.n0 = n_rows;
  p.x = x;
  p.idx = indices;
  p.out = out;
  p.n_out = (int)k;
  p.in_features = (int)in_features;
  return launch_gemv<ROW_GATHER, EPI_PLAIN>(p, (cudaStream_t)stream);
}

extern "C" int dip_gather_up_h(const int8_t* up_qw, const dip_bf16* up_sc, int64_t n_rows,
                               const dip_bf16* x, const dip_bf16* g, const int32_t* idx,
                               int64_t k, int64_t in_features, dip_bf16* h,
                               dip_stream_t stream) {
  if (k < 0 || k > INT32_MAX || n_rows < 0 || !gemv_shape_ok(in_features)) return DIP_ERR_ARG;
  if (k == 0) return DIP_OK;
  if (!up_qw || !up_sc || !x || !g || !idx || !h || n_rows == 0 || !aligned16(up_qw) ||
      !aligned16(x))
    return DIP_ERR_ARG;
  GemvParams p = {};
  p.qw0 = reinterpret_cast<const uint8_t*>(up_qw);
  p.sc0 = up_sc;
  p.n0 = n_rows;
  p.x = x;
  p.idx = idx;
  p.g = g;
  p.gid = idx;
  p.out = h;
  p.n_out = (int)k;
  p.in_features = (int)in_features;
  return launch_gemv<ROW_GATHER, EPI_H>(p, (cudaStream_t)stream);
}

extern "C" int dip_ca_fused_gemv(const int8_t* res_qw, const dip_bf16* res_sc, int64_t n_res,
                                 const int8_t* str_qw, const dip_bf16* str_sc, int64_t n_str,
                                 const dip_bf16* x, const int32_t* src, const int32_t* row,
                                 int64_t k, int64_t in_features, dip_bf16* out,
                                 dip_stream_t stream) {
  if (k < 0 || k > INT32_MAX || n_res < 0 || n_str < 0 || !gemv_shape_ok(in_features))
    return DIP_ERR_ARG;
  if (k == 0) return DIP_OK;
  if (!res_qw || !res_sc || !str_qw || !str_sc || !x || !src || !row || !out ||
      !aligned16(res_qw) || !aligned16(str_qw) || !aligned16(x) || n_res + n_str == 0)
    return DIP_ERR_ARG;
  GemvParams p = {};
  p.qw0 = reinterpret_cast<const uint8_t*>(res_qw);
  p.sc0 = res_sc;
  p.n0 = n_res;
  p.qw1 = reinterpret_cast<const uint8_t*>(str_qw);
  p.sc1 = str_sc;
  p.n1 = n_str;
  p.x = x;
  p.src = src;
  p.row = row;
  p.out = out;
  p.n_out = (int)k;
  p.in_features = (int)in_features;
  return launch_gemv<ROW_SRCROW, EPI_PLAIN>(p, (cudaStream_t)stream);
}

extern "C" int dip_srcrow_up_h(const int8_t* res_qw, const dip_bf16* res_sc, int64_t n_res,
                               const int8_t* full_qw, const dip_bf16* full_sc, int64_t n_full,
                               const dip_bf16* x, const dip_bf16* g,
                               const int32_t* combined_ids, const int32_t* src,
                               const int32_t* row, int64_t k, int64_t in_features, dip_bf16* h,
                               dip_stream_t stream) {
  if (k < 0 || k > INT32_MAX || n_res < 0 || n_full <= 0 || !gemv_shape_ok(in_features))
    return DIP_ERR_ARG;
  if (k == 0) return DIP_OK;
  if (!full_qw || !full_sc || !x || !g || !combined_ids || !src || !row || !h ||
      !aligned16(full_qw) || !aligned16(x) || (n_res > 0 && (!res_qw || !res_sc)))
    return DIP_ERR_ARG;
  if (n_res > 0 && !aligned16(res_qw)) return DIP_ERR_ARG;
  GemvParams p = {};
  p.qw0 = reinterpret_cast<const uint8_t*>(n_res > 0 ? res_qw : full_qw);
  p.sc0 = n_res > 0 ? res_sc : full_sc;
  p.n0 = n_res;
  p.qw1 = reinterpret_cast<const uint8_t*>(full_qw);
  p.sc1 = full_sc;
  p.n1 = n_full;
  p.x = x;
  p.src = src;
  p.row = row;
  p.g = g;
  p.gid = combined_ids;
  p.out = h;
  p.n_out = (int)k;
  p.in_features = (int)in_features;
  return launch_gemv<ROW_SRCROW, EPI_H>(p, (cudaStream_t)stream);
}

extern "C" int dip_gather_up_h_count(const int8_t* up_qw, const dip_bf16* up_sc, int64_t n_rows,
                                     const dip_bf16* x, const dip_bf16* g, const int32_t* idx,
                                     const int32_t* count, int64_t max_k, int64_t in_features,
                                     dip_bf16* h, dip_stream_t stream) {
  if (max_k < 0 || max_k > INT32_MAX || n_rows <= 0 || !gemv_shape_ok(in_features))
    return DIP_ERR_ARG;
  if (max_k == 0) return DIP_OK;
  if (!up_qw || !up_sc || !x || !g || !idx || !count || !h || !aligned16(up_qw) || !aligned16(x))
    return DIP_ERR_ARG;
  GemvParams p = {};
  p.qw0 = reinterpret_cast<const uint8_t*>(up_qw);
  p.sc0 = up_sc;
  p.n0 = n_rows;
  p.x = x;
  p.idx = idx;
  p.g = g;
  p.gid = idx;
  p.out = h;
  p.count = count;
  p.n_out = (int)max_k;
  p.in_features = (int)in_features;
  return launch_gemv<ROW_GATHER, EPI_H>(p, (cudaStream_t)stream);
}
