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
  if (hist && key <= 0x7F80u) atomicAdd(&hist[key], 1u);
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

// ---------------------------------------------------------------------------
// Persistent ring variant (used when in_features % 1024 == 0 and the ring
// fits in shared memory).  One CTA per SM: warp 8 is the producer, streaming
// 16-row tiles (every row as one bulk copy, plus its scales) into a 4-stage
// shared-memory ring with cp.async.bulk + mbarrier completion; warps 0..7
// consume, each owning a fixed K-slice of GW groups whose x fragments stay in
// registers for the whole kernel.  Rows are stored with a 16-byte pad so the
// 128-bit shared loads of rows g and g+8 fall in different banks.  In the
// dense mode the producer issues its first copies before waiting on the
// predecessor kernel (weights are static), overlapping the previous launch.
constexpr int kRingConsumers = 8;
constexpr int kRingThreads = (kRingConsumers + 1) * 32;
constexpr int kRingStages = 4;
constexpr int kRingPad = 16;

struct RingGeom {
  int rowb, scb, row_stride, stage_bytes, x_off, gsum_off, red_off, bar_off, total;
};
__host__ __device__ inline RingGeom ring_geom(int in) {
  RingGeom g;
  const int G = in / kGroup;
  g.rowb = in / 2;
  g.scb = G * 2;
  g.row_stride = g.rowb + kRingPad;
  g.stage_bytes = 16 * g.row_stride + 16 * g.scb;
  g.stage_bytes = (g.stage_bytes + 127) & ~127;
  g.x_off = kRingStages * g.stage_bytes;
  g.gsum_off = g.x_off + in * 2;
  g.red_off = g.gsum_off + ((G * 4 + 15) & ~15);
  g.bar_off = g.red_off + 2 * kRingConsumers * 16 * 4;
  g.total = g.bar_off + 2 * kRingStages * 8;
  return g;
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

template <int MODE, int EPI, int GW>
__global__ void __launch_bounds__(kRingThreads, 1)
gemv_ring_kernel(const GemvParams p, unsigned* err) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int in = p.in_features;
  const int G = in / kGroup;
  const RingGeom geo = ring_geom(in);
  uint32_t* xstage = reinterpret_cast<uint32_t*>(smem + geo.x_off);
  float* gsum = reinterpret_cast<float*>(smem + geo.gsum_off);
  float* red = reinterpret_cast<float*>(smem + geo.red_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + geo.bar_off);
  uint64_t* empty = full + kRingStages;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kRingStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (MODE != ROW_DENSE) pdl_wait();
  int n_out = p.n_out;
  if (p.count) n_out = min(n_out, *p.count);
  const int nt = (n_out + 15) / 16;
  const int t0 = (int)((int64_t)nt * blockIdx.x / gridDim.x);
  const int t1 = (int)((int64_t)nt * (blockIdx.x + 1) / gridDim.x);
  const int ntile = t1 - t0;

  if (warp == kRingConsumers) {
    // ---------------- producer ----------------
    bool ok = true;
    for (int i = 0; i < ntile && ok; ++i) {
      const int s = i % kRingStages;
      const uint32_t par = ((i / kRingStages) & 1) ^ 1;
      if (lane == 0) ok = mbar_wait(&empty[s], par, err);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      const int r0 = (t0 + i) * 16;
      const int rows = min(16, n_out - r0);
      uint8_t* st = smem + s * geo.stage_bytes;
      if (lane == 0) mbar_arrive_expect_tx(&full[s], rows * (geo.rowb + geo.scb));
      __syncwarp();
      if (lane < rows) {
        const uint8_t* qw;
        const uint16_t* sc;
        resolve_row<MODE>(p, r0 + lane, qw, sc);
        bulk_g2s(st + lane * geo.row_stride, qw, geo.rowb, &full[s]);
        bulk_g2s(st + 16 * geo.row_stride + lane * geo.scb, sc, geo.scb, &full[s]);
      }
    }
    // Do not leave with copies in flight: wait (bounded) for the last stages.
    if (lane == 0 && ok) {
      for (int i = max(0, ntile - kRingStages); i < ntile; ++i)
        if (!mbar_wait(&full[i % kRingStages], (i / kRingStages) & 1, err)) break;
    }
    return;
  }

  // ---------------- consumers ----------------
  const int ctid = threadIdx.x;  // 0..255
  const int gq = lane >> 2, tq = lane & 3;
  if (MODE == ROW_DENSE) pdl_wait();
  {
    const int nwords = in / 8;
    const uint4* xv = reinterpret_cast<const uint4*>(p.x);
    for (int wi = ctid; wi < ((nwords + 255) & ~255); wi += kRingConsumers * 32) {
      float part = 0.f;
      if (wi < nwords) {
        const uint4 v = __ldg(xv + wi);
        uint4 o;
        o.x = __byte_perm(v.x, v.z, 0x5410);
        o.y = __byte_perm(v.x, v.z, 0x7632);
        o.z = __byte_perm(v.y, v.w, 0x5410);
        o.w = __byte_perm(v.y, v.w, 0x7632);
        reinterpret_cast<uint4*>(xstage)[wi] = o;
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
  named_bar(1, kRingConsumers * 32);
  const int g0 = warp * GW;
  uint32_t xf[GW][16];
  float bias[GW];
#pragma unroll
  for (int gi = 0; gi < GW; ++gi) {
    const int grp = min(g0 + gi, G - 1);
    const uint4* bp = reinterpret_cast<const uint4*>(xstage + grp * 64 + tq * 16);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 b = bp[q];
      xf[gi][4 * q + 0] = b.x; xf[gi][4 * q + 1] = b.y;
      xf[gi][4 * q + 2] = b.z; xf[gi][4 * q + 3] = b.w;
    }
    bias[gi] = kNibbleBias * gsum[grp];
  }

  bool ok = true;
  for (int i = 0; i < ntile; ++i) {
    const int s = i % kRingStages;
    if (ok) ok = mbar_wait(&full[s], (i / kRingStages) & 1, err);
    const uint8_t* st = smem + s * geo.stage_bytes;
    const uint8_t* rowa = st + gq * geo.row_stride;
    const uint8_t* rowbp = st + (gq + 8) * geo.row_stride;
    const uint16_t* sca = reinterpret_cast<const uint16_t*>(st + 16 * geo.row_stride + gq * geo.scb);
    const uint16_t* scbp = reinterpret_cast<const uint16_t*>(st + 16 * geo.row_stride +
                                                             (gq + 8) * geo.scb);
    float acc_a = 0.f, acc_b = 0.f;
    if (ok) {
#pragma unroll
      for (int gi = 0; gi < GW; ++gi) {
        const int grp = g0 + gi;
        if (grp < G) {
          const uint4 wa = *reinterpret_cast<const uint4*>(rowa + grp * kGroupBytes + tq * 16);
          const uint4 wb = *reinterpret_cast<const uint4*>(rowbp + grp * kGroupBytes + tq * 16);
          float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
          group_mma(wa, wb, xf[gi], d0, d1);
          acc_a = fmaf(bf16_bits_to_f32(sca[grp]), (d0[0] + d1[0]) - bias[gi], acc_a);
          acc_b = fmaf(bf16_bits_to_f32(scbp[grp]), (d0[2] + d1[2]) - bias[gi], acc_b);
        }
      }
    }
    float* rr = red + (i & 1) * kRingConsumers * 16;
    if (tq == 0) {
      rr[warp * 16 + gq] = acc_a;
      rr[warp * 16 + gq + 8] = acc_b;
    }
    named_bar(1, kRingConsumers * 32);
    if (ctid == 0) mbar_arrive(&empty[s]);
    if (warp == 0 && lane < 16) {
      const int j = (t0 + i) * 16 + lane;
      if (j < n_out && ok) {
        float v = rr[lane];
#pragma unroll
        for (int w = 1; w < kRingConsumers; ++w) v += rr[w * 16 + lane];
        const uint8_t* dq;
        const uint16_t* ds;
        const bool valid = resolve_row<MODE>(p, j, dq, ds);
        uint16_t o;
        if (!valid) o = 0;
        else if (EPI == EPI_PLAIN) o = f32_to_bf16_bits(v);
        else if (EPI == EPI_SILU) {
          o = f32_to_bf16_bits(silu_f32(round_bf16(v)));
          hist_count(p.hist, o);
        }
        else o = f32_to_bf16_bits(bf16_bits_to_f32(p.g[p.gid[j]]) * round_bf16(v));
        p.out[j] = o;
      }
    }
  }
  pdl_launch_dependents();
}

template <int MODE, int EPI, int GW>
static int launch_ring(const GemvParams& p, cudaStream_t s) {
  const RingGeom geo = ring_geom(p.in_features);
  auto kern = gemv_ring_kernel<MODE, EPI, GW>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       geo.total);
  if (e != cudaSuccess) return launch_status(e);
  const int nt = (p.n_out + 15) / 16;
  const int grid = nt < num_sms() ? nt : num_sms();
  unsigned* err = error_word_ptr();
  if (!err) return DIP_ERR_CUDA;
  return launch_status(launch(kern, dim3(grid), dim3(kRingThreads), (size_t)geo.total, s, p, err));
}

// The ring kernel needs whole 8-group K-slices (G % 8 == 0) so every row's
// scales are a 16-byte multiple, and its ring must fit in shared memory.
static bool ring_ok(const GemvParams& p) {
  const int G = p.in_features / kGroup;
  if (G % 8 != 0 || G / 8 > 8) return false;
  if (ring_geom(p.in_features).total > 220 * 1024) return false;
  if ((reinterpret_cast<uintptr_t>(p.sc0) & 15) != 0) return false;
  if (p.qw1 && (reinterpret_cast<uintptr_t>(p.sc1) & 15) != 0) return false;
  return true;
}

template <int MODE, int EPI>
static int launch_ring_any(const GemvParams& p, cudaStream_t s) {
  switch (p.in_features / kGroup / 8) {
    case 1: return launch_ring<MODE, EPI, 1>(p, s);
    case 2: return launch_ring<MODE, EPI, 2>(p, s);
    case 3: return launch_ring<MODE, EPI, 3>(p, s);
    case 4: return launch_ring<MODE, EPI, 4>(p, s);
    case 5: return launch_ring<MODE, EPI, 5>(p, s);
    case 6: return launch_ring<MODE, EPI, 6>(p, s);
    case 7: return launch_ring<MODE, EPI, 7>(p, s);
    default: return launch_ring<MODE, EPI, 8>(p, s);
  }
}

// Host launcher shared by the entry points below.
template <int MODE, int EPI>
static int launch_gemv(const GemvParams& p, cudaStream_t s) {
  if (p.n_out == 0) return DIP_OK;
  if (ring_ok(p) && !force_simple_gemv()) return launch_ring_any<MODE, EPI>(p, s);
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
