// layer_fused.cu — one decode DIP MLP layer as ONE persistent kernel.
//
//   phase A  gate GEMV + SiLU over this CTA's rows of W_gate; |g| histogram
//   --- grid barrier ---
//   phase B  exact top-k thresholds from the histograms (every CTA,
//            redundantly, ~2 KB of reads); each CTA lists ITS OWN selected
//            rows: tier A (> hi) is local, tier B (ties) needs the B count
//            of the rows before its own, read straight from g
//   phases C+D, one cp.async stream: gathered up GEMV of the listed channels,
//            h = bf16(g * u) kept in shared memory, then the gathered down
//            projection of the SAME channels over all outputs (tensor cores),
//            one fp32 partial vector per CTA
//   --- grid barrier ---
//   phase E  fixed-order sum of the partials -> y
//
// Semantics are those of StreamingDIPMlp.forward (dip_stream_predispatch.py:
// 176-204) with topk_select.cu's selection; the kernels of gemv_int4.cu,
// topk.cu and gather_down.cu compute the same steps as separate launches.
//
// Why one kernel: at batch 1 every step is short (10-12 us of HBM traffic for
// the GEMVs, a few us for the top-k) and separate launches each pay a ramp-up
// and a tail; here the CTAs stay resident (one per SM, cooperative launch),
// the x fragments of the CTA's K-slice are loaded once and used by both GEMVs,
// and the up and down rows of a channel are read by the same CTA.  Each warp
// streams its bytes through a private 4-deep cp.async ring and never waits for
// another warp inside a phase.  The gate phase's first tiles are requested
// before waiting on the previous kernel (weights are static), so consecutive
// layers overlap.
#include "dip_block.cuh"
#include "dip_common.cuh"

namespace dip {

// Phase tracing (compile with -DDIP_TRACE): CTA 0's thread 0 records the
// global timer at each phase boundary into dip_lf_trace[].
#ifdef DIP_TRACE
__device__ unsigned long long dip_lf_trace[16];
__device__ unsigned long long dip_lf_cta[160][16];
}  // namespace dip
extern "C" void dip_lf_trace_read(unsigned long long* out) {
  cudaMemcpyFromSymbol(out, dip::dip_lf_trace, 16 * sizeof(unsigned long long));
}
extern "C" void dip_lf_cta_read(unsigned long long* out) {
  cudaMemcpyFromSymbol(out, dip::dip_lf_cta, 160 * 16 * sizeof(unsigned long long));
}
namespace dip {
#define LF_TRACE(n) \
  do { if (threadIdx.x == 0 && blockIdx.x == 0) { unsigned long long t; \
       asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t)); dip_lf_trace[n] = t; } } while (0)
#define LF_CTA(n) \
  do { if (threadIdx.x == 0) { dip_lf_cta[blockIdx.x][n] = clock64(); } } while (0)
#else
#define LF_TRACE(n) do { } while (0)
#define LF_CTA(n) do { } while (0)
#endif

constexpr int kLfWarps = 20;
constexpr int kLfThreads = kLfWarps * 32;
constexpr int kLfDepth = 4;
constexpr int kLfTilesA = 12;   // max gate tiles (16 rows) per CTA
constexpr int kLfDnPitch = 144;  // bytes per channel row of a down slot (128 + pad)

struct LfArgs {
  const uint8_t* gate_qw; const uint16_t* gate_sc;
  const uint8_t* up_qw; const uint16_t* up_sc;
  const uint8_t* dn_qw; const uint16_t* dn_sc;   // transposed down [inter, hidden/2]
  int hidden, inter, k;
  const uint16_t* x;        // layer input, or the previous y when resid != nullptr
  const uint16_t* resid;    // optional: input = RMSNorm(x + resid), unit weight
  float eps;
  uint16_t* x_used;         // optional: the (normalised) input actually used
  uint16_t* g;              // [inter]
  int32_t* idx;             // [k]
  unsigned* scratch;        // top-k scratch (zero on entry, left zero)
  float* partial;           // [gridDim.x][hidden]
  uint16_t* y;              // [hidden]
  float* y_f32;             // optional
  GridBar* bar;
  unsigned* err;
};

// Byte offsets of the dynamic shared memory.
template <int GW>
struct LfGeom {
  // GEMV phases: 16 rows x GW x 64 B + scale words; down phase: 16 rows at a
  // 144-byte pitch + scale words.
  static constexpr int slot = (GW * 1024 + 64 > 16 * kLfDnPitch + 64) ? GW * 1024 + 64
                                                                       : 16 * kLfDnPitch + 64;
  static constexpr int ring = kLfWarps * kLfDepth * slot;
  static constexpr int xs = ring;                      // x staging (G*72 words)
  static constexpr int G = kLfWarps * GW;
  static constexpr int gsum = xs + G * 72 * 4;
  static constexpr int red = gsum + ((G * 4 + 15) & ~15);  // [tiles][warps][16]
  static constexpr int red_words = kLfTilesA * kLfWarps * 16;
  static constexpr int rowp = red + red_words * 4;         // C/D: channel of each list entry
  static constexpr int hv = rowp + kLfTilesA * 16 * 4;     // C/D: g value, then h (fp32)
  static constexpr int gloc = hv + kLfTilesA * 16 * 4;     // this CTA's g values (bf16)
  static constexpr int misc = gloc + kLfTilesA * 16 * 2;   // small scalars
  static constexpr int total = misc + 1024;
};

__device__ __forceinline__ uint16_t ld_cg_u16(const uint16_t* p) {
  unsigned short v;
  asm volatile("ld.global.cg.u16 %0, [%1];\n" : "=h"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ int ld_cg_i32(const int32_t* p) {
  int v;
  asm volatile("ld.global.cg.s32 %0, [%1];\n" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ void cp_async16_lf(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async4_lf(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_commit_lf() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_wait_lf() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(kLfDepth - 1) : "memory");
}

// grid_sync (dip_common.cuh) split in two so that a CTA can do independent
// work between its arrival and the release.  Thread 0 keeps the generation it
// saw before arriving; the wait is bounded like grid_sync's.
__device__ __forceinline__ unsigned lf_bar_arrive(GridBar* b) {
  __syncthreads();
  unsigned g0 = 0;
  if (threadIdx.x == 0) {
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(g0) : "l"(&b->gen) : "memory");
    __threadfence();
    if (atomicAdd(&b->count, 1u) == gridDim.x - 1) {
      atomicExch(&b->count, 0u);
      __threadfence();
      atomicAdd(&b->gen, 1u);
    }
  }
  return g0;
}
__device__ __forceinline__ void lf_bar_wait(GridBar* b, unsigned g0, unsigned* err) {
  if (threadIdx.x == 0) {
    bool done = false;
    for (uint32_t it = 0; it < kSpinLimit && !done; ++it) {
      unsigned g;
      asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];\n" : "=r"(g) : "l"(&b->gen) : "memory");
      done = (g != g0);
    }
    if (!done) atomicOr(err, kErrTimeout);
    asm volatile("fence.acq_rel.gpu;\n" ::: "memory");
  }
  __syncthreads();
}

// K-slice GEMV step shared by phases A and C: this warp's GW groups of 16
// rows (rows gq and gq+8 of the tile) -> two partial dot products.
template <int GW>
__device__ __forceinline__ void lf_tile_dot(const uint8_t* slot, const uint32_t (&xf)[GW][16],
                                            const float (&bias)[GW], int lane, int sofs,
                                            float& acc_a, float& acc_b) {
  const int gq = lane >> 2;
  const uint16_t* sca = reinterpret_cast<const uint16_t*>(slot + GW * 1024 + gq * 4);
  const uint16_t* scb = reinterpret_cast<const uint16_t*>(slot + GW * 1024 + (gq + 8) * 4);
  acc_a = 0.f;
  acc_b = 0.f;
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
    acc_a = fmaf(bf16_bits_to_f32(sca[gi + sofs]), (d0[0] + d1[0]) - bias[gi], acc_a);
    acc_b = fmaf(bf16_bits_to_f32(scb[gi + sofs]), (d0[2] + d1[2]) - bias[gi], acc_b);
  }
}

// Issue one GEMV tile slice into this warp's ring slot: rows r_a (=gq) and
// r_b (=gq+8) of the tile, groups [warp*GW, (warp+1)*GW), plus the 4-byte
// scale pairs of the tile's 16 rows (lanes 0..15).
template <int GW>
__device__ __forceinline__ void lf_issue_gemv(uint8_t* slot, const uint8_t* qa, const uint8_t* qb,
                                              const uint16_t* srow_lane, int warp, int lane) {
  const int tq = lane & 3;
#pragma unroll
  for (int gi = 0; gi < GW; ++gi) {
    const int off = (warp * GW + gi) * kGroupBytes + tq * 16;
    cp_async16_lf(slot + (gi * 2 + 0) * 512 + lane * 16, qa + off);
    cp_async16_lf(slot + (gi * 2 + 1) * 512 + lane * 16, qb + off);
  }
  if (lane < 16) {
    // GW == 2: the 4 bytes [4 warp, 4 warp + 4); GW == 1: 2 bytes, copy the
    // aligned 4-byte word containing them.
    const uint16_t* p = srow_lane + ((warp * GW) & ~1);
    cp_async4_lf(slot + GW * 1024 + lane * 4, p);
  }
}

template <int GW>
__global__ void __launch_bounds__(kLfThreads, 1) layer_fused_kernel(const LfArgs a) {
  using Geo = LfGeom<GW>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const int H = a.hidden, I = a.inter, K = a.k;
  const int rowb = H / 2, scw = H / kGroup;  // bytes per packed row, scales per row
  uint8_t* ring = smem + warp * kLfDepth * Geo::slot;
  uint32_t* xs = reinterpret_cast<uint32_t*>(smem + Geo::xs);
  float* gsum = reinterpret_cast<float*>(smem + Geo::gsum);
  float* red = reinterpret_cast<float*>(smem + Geo::red);
  int* rowp = reinterpret_cast<int*>(smem + Geo::rowp);
  float* hv = reinterpret_cast<float*>(smem + Geo::hv);
  float* misc = reinterpret_cast<float*>(smem + Geo::misc);
  const int nb = gridDim.x, b = blockIdx.x;
  // GW == 1 reads the scale of group `warp` from the 4-byte word copied at
  // (warp & ~1); GW == 2 reads both halves.
  const int sc_sel = (GW == 1) ? (warp & 1) : 0;

  // ------------------------------------------------------------ phase A
  const int ra0 = (int)((int64_t)I * b / nb), ra1 = (int)((int64_t)I * (b + 1) / nb);
  const int na = ra1 - ra0, nta = (na + 15) / 16;
  auto issue_a = [&](int i) {
    if (i < nta) {
      const int ra = min(ra0 + i * 16 + gq, ra1 - 1), rb = min(ra0 + i * 16 + gq + 8, ra1 - 1);
      const int rs = min(ra0 + i * 16 + (lane & 15), ra1 - 1);
      lf_issue_gemv<GW>(ring + (i % kLfDepth) * Geo::slot, a.gate_qw + (size_t)ra * rowb,
                        a.gate_qw + (size_t)rb * rowb, a.gate_sc + (size_t)rs * scw, warp, lane);
    }
    cp_commit_lf();
  };
#pragma unroll
  for (int i = 0; i < kLfDepth - 1; ++i) issue_a(i);
  LF_TRACE(0);
  LF_CTA(0);
  pdl_wait();
  LF_TRACE(1);

  // Layer input: x, or RMSNorm(x + resid); staged in the B-fragment order.
  {
    float ssq = 0.f;
    if (a.resid) {
      for (int e = tid; e < H; e += kLfThreads) {
        const float v = bf16_bits_to_f32(ld_cg_u16(a.x + e)) + bf16_bits_to_f32(ld_cg_u16(a.resid + e));
        ssq = fmaf(v, v, ssq);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ssq += __shfl_xor_sync(0xffffffffu, ssq, o);
      if (lane == 0) misc[warp] = ssq;
      __syncthreads();
      if (tid == 0) {
        float t = 0.f;
        for (int w = 0; w < kLfWarps; ++w) t += misc[w];
        misc[32] = rsqrtf(t / (float)H + a.eps);
      }
      __syncthreads();
    }
    const float inv = a.resid ? misc[32] : 1.f;
    const int nwords = H / 8;
    for (int wi = tid; wi < ((nwords + kLfThreads - 1) / kLfThreads) * kLfThreads;
         wi += kLfThreads) {
      float part = 0.f;
      if (wi < nwords) {
        uint32_t v4[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t lo = ld_cg_u16(a.x + wi * 8 + 2 * q), hi = ld_cg_u16(a.x + wi * 8 + 2 * q + 1);
          uint32_t pr = lo | (hi << 16);
          if (a.resid) {
            const uint32_t rl = ld_cg_u16(a.resid + wi * 8 + 2 * q);
            const uint32_t rh = ld_cg_u16(a.resid + wi * 8 + 2 * q + 1);
            const float fl = (bf16_bits_to_f32(lo) + bf16_bits_to_f32(rl)) * inv;
            const float fh = (bf16_bits_to_f32(hi) + bf16_bits_to_f32(rh)) * inv;
            pr = (uint32_t)f32_to_bf16_bits(fl) | ((uint32_t)f32_to_bf16_bits(fh) << 16);
          }
          v4[q] = pr;
        }
        if (a.x_used && b == 0)
          *reinterpret_cast<uint4*>(a.x_used + wi * 8) = make_uint4(v4[0], v4[1], v4[2], v4[3]);
        uint4 o;
        o.x = __byte_perm(v4[0], v4[2], 0x5410);
        o.y = __byte_perm(v4[0], v4[2], 0x7632);
        o.z = __byte_perm(v4[1], v4[3], 0x5410);
        o.w = __byte_perm(v4[1], v4[3], 0x7632);
        const int grp = wi >> 4, t = (wi >> 2) & 3, w = wi & 3;
        *reinterpret_cast<uint4*>(xs + grp * 72 + t * 16 + (t >> 1) * 4 + 4 * w) = o;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          part += bf16_bits_to_f32(v4[q] & 0xFFFF) + bf16_bits_to_f32(v4[q] >> 16);
      }
      part += __shfl_xor_sync(0xffffffffu, part, 8);
      part += __shfl_xor_sync(0xffffffffu, part, 4);
      part += __shfl_xor_sync(0xffffffffu, part, 2);
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      if ((lane & 15) == 0 && wi < nwords) gsum[wi >> 4] = part;
    }
  }
  __syncthreads();
  LF_TRACE(2);
  uint32_t xf[GW][16];
  float bias[GW];
#pragma unroll
  for (int gi = 0; gi < GW; ++gi) {
    const int grp = warp * GW + gi;
    const uint4* bp = reinterpret_cast<const uint4*>(xs + grp * 72 + tq * 16 + (tq >> 1) * 4);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 v = bp[q];
      xf[gi][4 * q] = v.x; xf[gi][4 * q + 1] = v.y; xf[gi][4 * q + 2] = v.z; xf[gi][4 * q + 3] = v.w;
    }
    bias[gi] = kNibbleBias * gsum[grp];
  }

  for (int i = 0; i < nta; ++i) {
    issue_a(i + kLfDepth - 1);
    cp_wait_lf();
    __syncwarp();
    float pa, pb;
    lf_tile_dot<GW>(ring + (i % kLfDepth) * Geo::slot, xf, bias, lane, sc_sel, pa, pb);
    if (tq == 0) {
      red[(i * kLfWarps + warp) * 16 + gq] = pa;
      red[(i * kLfWarps + warp) * 16 + gq + 8] = pb;
    }
    __syncwarp();
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");
  LF_TRACE(3);
  LF_CTA(1);
  __syncthreads();
  uint16_t* gloc = reinterpret_cast<uint16_t*>(smem + Geo::gloc);
  for (int r = tid; r < na; r += kLfThreads) {
    const int i = r >> 4, row = r & 15;
    float v = 0.f;
    for (int w = 0; w < kLfWarps; ++w) v += red[(i * kLfWarps + w) * 16 + row];
    const uint16_t o = f32_to_bf16_bits(silu_f32(round_bf16(v)));
    a.g[ra0 + r] = o;
    gloc[r] = o;
  }
  __syncthreads();
  // Histogram counts aggregated over the CTA first (SiLU's minimum piles ~1/8
  // of all values into two or three fine bins, and per-row global atomics on
  // those serialise): a shared-memory copy of the bins, in the ring (idle
  // now); the first row to reach a bin later adds the bin's total.
  {
    unsigned* sfine = reinterpret_cast<unsigned*>(smem);            // [kTopkHistBins]
    unsigned* scoarse = sfine + kTopkHistBins;                       // [256]
    const unsigned kk = tid < na ? (gloc[tid] & 0x7FFFu) : 0xFFFFu;
    const bool valid = kk <= 0x7F80u;
    if (valid) sfine[kk] = 0u;
    for (int i = tid; i < 256; i += kLfThreads) scoarse[i] = 0u;
    __syncthreads();
    bool lead_f = false, lead_c = false;
    if (valid) {
      lead_f = atomicAdd(&sfine[kk], 1u) == 0u;
      lead_c = atomicAdd(&scoarse[kk >> 7], 1u) == 0u;
    }
    __syncthreads();
    if (lead_f) atomicAdd(&a.scratch[kk], sfine[kk]);
    if (lead_c) atomicAdd(&a.scratch[kTopkHistBins + (kk >> 7)], scoarse[kk >> 7]);
  }
  LF_TRACE(4);
  LF_CTA(2);
  const unsigned gen1 = lf_bar_arrive(a.bar);
  lf_bar_wait(a.bar, gen1, a.err);
  LF_TRACE(5);
  LF_CTA(8);

  // ------------------------------------------------------------ phase B
  __shared__ int coarse_suffix[257];
  __shared__ int2 warp_tot[33];
  __shared__ int2 s_off;
  __shared__ int s_tot[2];
  __shared__ float s_lohi[2];
  if (warp == 0) {
    const unsigned* coarse = a.scratch + kTopkHistBins;
    int cnt[8], loc = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      int v;
      asm volatile("ld.global.cg.s32 %0, [%1];\n" : "=r"(v) : "l"(coarse + 255 - (lane * 8 + q)));
      cnt[q] = v;
      loc += v;
    }
    int incl = loc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    int run = incl - loc;
#pragma unroll
    for (int q = 0; q < 8; ++q) { run += cnt[q]; coarse_suffix[255 - (lane * 8 + q)] = run; }
    if (lane == 0) coarse_suffix[256] = 0;
    __syncwarp();
    LF_CTA(13);
    const int nvalid = coarse_suffix[0];
    const bool has_w = nvalid >= K + 1;
    // highest non-empty coarse bin, and the coarse bin b1 holding the
    // (K+1)-th largest key
    int topb = -1, b1 = -1;
    for (int bb = lane; bb < 256; bb += 32) {
      if (coarse_suffix[bb] - coarse_suffix[bb + 1] > 0) topb = max(topb, bb);
      if (coarse_suffix[bb + 1] < K + 1 && K + 1 <= coarse_suffix[bb]) b1 = bb;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      topb = max(topb, __shfl_xor_sync(0xffffffffu, topb, o));
      b1 = max(b1, __shfl_xor_sync(0xffffffffu, b1, o));
    }
    // One round of fine-bin reads: the top bin, and bins b1-1, b1, b1+1 (the
    // final lo and hi lie within a key of the (K+1)-th key, so their counts
    // come from these bins; other bins are read on demand below).
    const int32_t* fine = reinterpret_cast<const int32_t*>(a.scratch);
    int ft[4], fb[3][4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int f = lane * 4 + q;
      ft[q] = topb >= 0 ? ld_cg_i32(fine + ((topb << 7) | f)) : 0;
#pragma unroll
      for (int d = 0; d < 3; ++d) {
        const int cb = b1 - 1 + d;
        fb[d][q] = (has_w && cb >= 0 && cb < 256) ? ld_cg_i32(fine + ((cb << 7) | f)) : 0;
      }
    }
    LF_CTA(14);
    int maxkey = 0;
    if (topb >= 0) {
      int mk = -1;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (ft[q] != 0) mk = (topb << 7) | (lane * 4 + q);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mk = max(mk, __shfl_xor_sync(0xffffffffu, mk, o));
      maxkey = max(mk, 0);
    }
    float wv = 0.f;
    if (has_w) {
      // the rank-th largest key of bin b1: suffix sums over the fine bins
      const int rank = K + 1 - coarse_suffix[b1 + 1];
      const int ls = fb[1][0] + fb[1][1] + fb[1][2] + fb[1][3];
      int suf = ls;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_down_sync(0xffffffffu, suf, o);
        if (lane + o < 32) suf += t;
      }
      int runf = suf - ls, found = -1;
#pragma unroll
      for (int q = 3; q >= 0; --q) {
        runf += fb[1][q];
        if (found < 0 && runf >= rank && runf - fb[1][q] < rank) found = lane * 4 + q;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) found = max(found, __shfl_xor_sync(0xffffffffu, found, o));
      wv = bf16_bits_to_f32((unsigned)((b1 << 7) | found));
    }
    // the reference's 25-step fp32 bisection, run on the exact (K+1)-th key
    float hi = bf16_bits_to_f32((unsigned)maxkey), lo = 0.0f;
    float t = __fmul_rn(0.5f, __fadd_rn(lo, hi));
    for (int step = 0; step < 25; ++step) {
      if (has_w && wv > t) lo = t; else hi = t;
      t = __fmul_rn(0.5f, __fadd_rn(lo, hi));
    }
    // #keys > tt = #keys >= kmin, kmin = bf16 key just above tt
    auto count_above = [&](float tt) -> int {
      const int kmin = (int)(__float_as_uint(tt) >> 16) + 1;
      if (kmin > 0x7F80) return 0;
      const int cb = kmin >> 7, f0 = kmin & 127, d = cb - (b1 - 1);
      const bool held = has_w && d >= 0 && d < 3;
      int part = 0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int f = lane * 4 + q;
        if (f >= f0) {
          const int v = held ? (d == 0 ? fb[0][q] : d == 1 ? fb[1][q] : fb[2][q])
                             : ld_cg_i32(fine + ((cb << 7) | f));
          part += v;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      return part + (cb < 255 ? coarse_suffix[cb + 1] : 0);
    };
    const int c0n = count_above(hi), c1n = count_above(lo);
    if (lane == 0) { s_lohi[0] = lo; s_lohi[1] = hi; s_tot[0] = c0n; s_tot[1] = c1n; }
  }
  __syncthreads();
  LF_CTA(9);
  // Selection (topk_select.cu): every key > hi ("tier A", all of them fit),
  // then keys in (lo, hi] ("tier B") in index order while positions remain,
  // then zero indices up to K.  Tier A of this CTA's rows is known locally;
  // tier B needs the B counts of the rows before this CTA's, counted below
  // straight from g (complete since the barrier).
  const float lo = s_lohi[0], hi = s_lohi[1];
  const int totA = s_tot[0], filled = min(K, s_tot[1]), selB = filled - totA;
  const uint16_t key = tid < na ? (gloc[tid] & 0x7FFF) : 0x7FFF;  // NaN: never selected
  const float kv = bf16_bits_to_f32(key);
  const bool isA = kv > hi;
  const bool isB = kv > lo && kv <= hi;
  int2 tot;
  const int2 off = block_excl_scan2(isA, isB, warp_tot, tot);
  // local channel list: this CTA's tier A rows, then its selected tier B rows
  if (isA) {
    rowp[off.x] = ra0 + tid;
    hv[off.x] = bf16_bits_to_f32(gloc[tid]);
  }
  __syncthreads();
  auto issue_c = [&](int i) {
    const int ra = rowp[i * 16 + gq], rb = rowp[i * 16 + gq + 8];
    const int rs = rowp[i * 16 + (lane & 15)];
    lf_issue_gemv<GW>(ring + (i % kLfDepth) * Geo::slot, a.up_qw + (size_t)ra * rowb,
                      a.up_qw + (size_t)rb * rowb, a.up_sc + (size_t)rs * scw, warp, lane);
  };
  LF_CTA(15);
  // full tiles of tier A rows do not depend on the other CTAs: start them now
  const int n_early = min(kLfDepth - 1, tot.x / 16);
  for (int i = 0; i < n_early; ++i) {
    issue_c(i);
    cp_commit_lf();
  }
  LF_CTA(6);
  {
    // tier A and tier B counts of rows [0, ra0), 8 keys per 16-byte load
    int pa = 0, pb = 0;
    const int nv = ra0 >> 3;
    auto tally = [&](uint32_t w2) {
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const float v = bf16_bits_to_f32((h2 ? (w2 >> 16) : w2) & 0x7FFFu);
        pa += v > hi;
        pb += v > lo && v <= hi;
      }
    };
    for (int i2 = tid; i2 < nv; i2 += kLfThreads) {
      uint32_t w0, w1, w2, w3;
      asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                   : "=r"(w0), "=r"(w1), "=r"(w2), "=r"(w3)
                   : "l"(a.g + (size_t)i2 * 8));
      tally(w0); tally(w1); tally(w2); tally(w3);
    }
    for (int e = nv * 8 + tid; e < ra0; e += kLfThreads) {
      const float v = bf16_bits_to_f32(ld_cg_u16(a.g + e) & 0x7FFFu);
      pa += v > hi;
      pb += v > lo && v <= hi;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      pa += __shfl_xor_sync(0xffffffffu, pa, o);
      pb += __shfl_xor_sync(0xffffffffu, pb, o);
    }
    if (lane == 0) warp_tot[warp] = make_int2(pa, pb);
    __syncthreads();
    if (tid == 0) {
      int sa = 0, sb = 0;
      for (int w = 0; w < kLfWarps; ++w) { sa += warp_tot[w].x; sb += warp_tot[w].y; }
      s_off = make_int2(sa, sb);
    }
    __syncthreads();
  }
  LF_CTA(7);
  const int preA = s_off.x, preB = s_off.y;
  const int nB = max(0, min(tot.y, selB - preB));  // this CTA's selected tier B rows
  if (isB && off.y < nB) {
    rowp[tot.x + off.y] = ra0 + tid;
    hv[tot.x + off.y] = bf16_bits_to_f32(gloc[tid]);
    a.idx[totA + preB + off.y] = ra0 + tid;
  }
  if (isA && preA + off.x < K) a.idx[preA + off.x] = ra0 + tid;
  {
    const int per = (K - filled + nb - 1) / nb;
    const int z0 = filled + b * per, z1 = min(K, z0 + per);
    for (int i2 = z0 + tid; i2 < z1; i2 += kLfThreads) a.idx[i2] = 0;
  }
  // The K - filled zero indices select channel 0 that many times: CTA 0
  // (owner of row 0) adds one list entry for it, its h scaled by the count.
  int nloc = tot.x + nB;
  const int pad_row = (b == 0 && filled < K) ? nloc : -1;
  if (pad_row >= 0) {
    if (tid == 0) {
      rowp[nloc] = 0;
      hv[nloc] = bf16_bits_to_f32(gloc[0]);
    }
    ++nloc;
  }
  const int ntc = (nloc + 15) / 16;
  __syncthreads();
  // pad the last tile with a valid row and h = 0
  for (int r = nloc + tid; r < ntc * 16; r += kLfThreads) {
    rowp[r] = rowp[nloc - 1];
    hv[r] = 0.f;
  }
  __syncthreads();
  LF_TRACE(6);
  LF_CTA(3);

  // ------------------------------------------------------------ phases C + D
  // One cp.async stream per warp: the ntc up tiles, then the ntc down tiles
  // of the same channels (the first down tiles are in flight while h is formed).
  const int seg = warp * GW * kGroupBytes;
  auto issue_d = [&](int i) {
    uint8_t* slot = ring + ((ntc + i) % kLfDepth) * Geo::slot;
    // 16 rows x GW*64 bytes = 16*GW*4 chunks of 16 B
#pragma unroll
    for (int q = 0; q < (16 * GW * 4) / 32; ++q) {
      const int chk = lane + 32 * q;
      const int r = chk / (GW * 4), part = chk % (GW * 4);
      const int ch = rowp[i * 16 + r];
      cp_async16_lf(slot + r * kLfDnPitch + part * 16, a.dn_qw + (size_t)ch * rowb + seg + part * 16);
    }
    if (lane < 16) {
      const int ch = rowp[i * 16 + lane];
      cp_async4_lf(slot + 16 * kLfDnPitch + lane * 4, a.dn_sc + (size_t)ch * scw + ((warp * GW) & ~1));
    }
  };
  auto issue = [&](int j) {
    if (j < ntc) issue_c(j);
    else if (j < 2 * ntc) issue_d(j - ntc);
    cp_commit_lf();
  };
  for (int j = n_early; j < kLfDepth - 1; ++j) issue(j);
  float acc[GW][8][4];
#pragma unroll
  for (int u = 0; u < GW; ++u)
#pragma unroll
    for (int m = 0; m < 8; ++m) acc[u][m][0] = acc[u][m][1] = acc[u][m][2] = acc[u][m][3] = 0.f;
  float colsum[GW];
#pragma unroll
  for (int u = 0; u < GW; ++u) colsum[u] = 0.f;
  const int tpair = lane & 7, twhich = (lane >> 3) & 1;
  for (int j = 0; j < ntc; ++j) {
    issue(j + kLfDepth - 1);
    cp_wait_lf();
    __syncwarp();
    float pa, pb;
    lf_tile_dot<GW>(ring + (j % kLfDepth) * Geo::slot, xf, bias, lane, sc_sel, pa, pb);
    if (tq == 0) {
      red[(j * kLfWarps + warp) * 16 + gq] = pa;
      red[(j * kLfWarps + warp) * 16 + gq + 8] = pb;
    }
    __syncwarp();
  }
  // h = bf16(g * bf16(u)) for the whole list (padding rows give 0) while the
  // first down tiles are in flight
  __syncthreads();
  for (int r = tid; r < ntc * 16; r += kLfThreads) {
    const int ti = r >> 4, row = r & 15;
    float v = 0.f;
    for (int w = 0; w < kLfWarps; ++w) v += red[(ti * kLfWarps + w) * 16 + row];
    float h = r < nloc ? round_bf16(hv[r] * round_bf16(v)) : 0.f;
    if (r == pad_row) h *= (float)(K - filled);
    hv[r] = h;
  }
  __syncthreads();
  LF_TRACE(7);
  LF_CTA(10);
  for (int j = ntc; j < 2 * ntc; ++j) {
    issue(j + kLfDepth - 1);
    cp_wait_lf();
    __syncwarp();
    const uint8_t* slot = ring + (j % kLfDepth) * Geo::slot;
    const int i = j - ntc;
#pragma unroll
    for (int u = 0; u < GW; ++u) {
      uint32_t bval = 0;
      if (lane < 16) {
        float v2[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int c = 2 * tpair + e;
          const uint16_t* sp = reinterpret_cast<const uint16_t*>(slot + 16 * kLfDnPitch + c * 4);
          const int sidx = (GW == 1) ? (warp & 1) : u;
          const float hs = hv[i * 16 + c] * bf16_bits_to_f32(sp[sidx]);
          const float h1 = round_bf16(hs);
          v2[e] = twhich ? round_bf16(hs - h1) : h1;
        }
        colsum[u] += v2[0] + v2[1];
        bval = (uint32_t)f32_to_bf16_bits(v2[0]) | ((uint32_t)f32_to_bf16_bits(v2[1]) << 16);
      }
      const int src = (gq & 1) * 8;
      const uint32_t b0 = __shfl_sync(0xffffffffu, bval, src + tq);
      const uint32_t b1 = __shfl_sync(0xffffffffu, bval, src + tq + 4);
      const uint8_t* base = slot + u * 64 + gq * 8;
      const uint2 r0 = *reinterpret_cast<const uint2*>(base + (2 * tq) * kLfDnPitch);
      const uint2 r1 = *reinterpret_cast<const uint2*>(base + (2 * tq + 1) * kLfDnPitch);
      const uint2 r2 = *reinterpret_cast<const uint2*>(base + (2 * tq + 8) * kLfDnPitch);
      const uint2 r3 = *reinterpret_cast<const uint2*>(base + (2 * tq + 9) * kLfDnPitch);
      const uint32_t pab[4] = {__byte_perm(r0.x, r1.x, 0x5410), __byte_perm(r0.x, r1.x, 0x7632),
                               __byte_perm(r0.y, r1.y, 0x5410), __byte_perm(r0.y, r1.y, 0x7632)};
      const uint32_t pcd[4] = {__byte_perm(r2.x, r3.x, 0x5410), __byte_perm(r2.x, r3.x, 0x7632),
                               __byte_perm(r2.y, r3.y, 0x5410), __byte_perm(r2.y, r3.y, 0x7632)};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t xa[4], xc[4];
        nib8_biased_bf16x2(pab[q], xa);
        nib8_biased_bf16x2(pcd[q], xc);
        const uint32_t a0[4] = {xa[0], xa[1], xc[0], xc[1]};
        const uint32_t a1[4] = {xa[2], xa[3], xc[2], xc[3]};
        mma_bf16_16816(acc[u][2 * q], a0, b0, b1);
        mma_bf16_16816(acc[u][2 * q + 1], a1, b0, b1);
      }
    }
    __syncwarp();
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");
  LF_TRACE(9);
  LF_CTA(4);
  pdl_launch_dependents();
#pragma unroll
  for (int u = 0; u < GW; ++u) {
    float cs = colsum[u];
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) cs += __shfl_xor_sync(0xffffffffu, cs, o);
    const float bias_d = kNibbleBias * __shfl_sync(0xffffffffu, cs, 0);
    if (tq == 0) {
      float* dst = a.partial + (size_t)b * H + (warp * GW + u) * kGroup + gq * 16;
      float v[16];
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        v[2 * m] = acc[u][m][0] + acc[u][m][1] - bias_d;
        v[2 * m + 1] = acc[u][m][2] + acc[u][m][3] - bias_d;
      }
#pragma unroll
      for (int q = 0; q < 4; ++q)
        reinterpret_cast<float4*>(dst)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
  }
  LF_TRACE(10);
  LF_CTA(5);
  grid_sync(a.bar, a.err);
  LF_TRACE(11);
  LF_CTA(11);

  // ------------------------------------------------------------ phase E
  // The histograms have no readers left: clear it
  // for the next call, spread over the CTAs.
  {
    const int nwords = kTopkHistBins + 256;
    const int per = (nwords + nb - 1) / nb;
    for (int i2 = b * per + tid; i2 < min(nwords, (b + 1) * per); i2 += kLfThreads) a.scratch[i2] = 0u;
  }
  // y[4q .. 4q+3] for this CTA's quads: R row-lanes per quad each sum every
  // R-th partial vector, then a fixed-shape tree over the R lanes.
  {
    const int n4 = H >> 2;
    const int q0 = (int)((int64_t)n4 * b / nb), q1 = (int)((int64_t)n4 * (b + 1) / nb);
    const int nq = q1 - q0;
    if (nq > 0) {
      int R = 64;
      while (R > 1 && R * nq > kLfThreads) R >>= 1;
      float4* e4 = reinterpret_cast<float4*>(red);
      const int q = tid % nq, rr = tid / nq;
      if (rr < R) {
        float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int c = rr; c < nb; c += R) {
          float4 v;
          asm volatile("ld.global.cg.v4.f32 {%0,%1,%2,%3}, [%4];\n"
                       : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                       : "l"(a.partial + (size_t)c * H + 4 * (q0 + q)));
          s4.x += v.x; s4.y += v.y; s4.z += v.z; s4.w += v.w;
        }
        e4[rr * nq + q] = s4;
      }
      __syncthreads();
      for (int st = R >> 1; st > 0; st >>= 1) {
        if (rr < st) {
          const float4 o = e4[(rr + st) * nq + q];
          float4& m = e4[rr * nq + q];
          m.x += o.x; m.y += o.y; m.z += o.z; m.w += o.w;
        }
        __syncthreads();
      }
      if (rr == 0) {
        const float4 s4 = e4[q];
        const int o = 4 * (q0 + q);
        if (a.y) {
          a.y[o] = f32_to_bf16_bits(s4.x); a.y[o + 1] = f32_to_bf16_bits(s4.y);
          a.y[o + 2] = f32_to_bf16_bits(s4.z); a.y[o + 3] = f32_to_bf16_bits(s4.w);
        }
        if (a.y_f32) *reinterpret_cast<float4*>(a.y_f32 + o) = s4;
      }
    }
  }
  LF_TRACE(12);
  LF_CTA(12);
}

size_t layer_fused_workspace_bytes(int64_t hidden, int64_t inter, int64_t k) {
  const size_t s = ((topk_scratch_bytes() + 255) & ~size_t(255)) + 256 +
                   (((size_t)inter * 2 + 255) & ~size_t(255)) + (((size_t)k * 4 + 255) & ~size_t(255)) +
                   (size_t)num_sms() * hidden * 4;
  return s;
}

}  // namespace dip

using namespace dip;

extern "C" size_t dip_mlp_fused_workspace_bytes(int64_t hidden, int64_t inter, int64_t k) {
  if (hidden <= 0 || inter <= 0 || k <= 0) return 0;
  // device independent upper bound (up to 160 SMs)
  return ((topk_scratch_bytes() + 255) & ~size_t(255)) + 256 +
         (((size_t)inter * 2 + 255) & ~size_t(255)) + (((size_t)k * 4 + 255) & ~size_t(255)) +
         (size_t)160 * hidden * 4;
}

extern "C" int dip_mlp_decode_fused(const dip_layer_t* L, const dip_bf16* x, const dip_bf16* resid,
                                    float eps, int64_t k, void* workspace, size_t workspace_bytes,
                                    dip_bf16* y, dip_bf16* g_out, int32_t* idx_out,
                                    dip_bf16* x_used, dip_stream_t stream) {
  if (!L || !x || !y || !workspace) return DIP_ERR_ARG;
  const int64_t H = L->hidden, I = L->inter;
  if (k < 1 || k > I || H <= 0 || I <= 0) return DIP_ERR_ARG;
  const int nb = num_sms();
  if (nb > 160) return DIP_ERR_UNSUPPORTED;
  const int G = (int)(H / kGroup);
  int gw = 0;
  if (H % kGroup == 0 && G == kLfWarps * 1) gw = 1;
  if (H % kGroup == 0 && G == kLfWarps * 2) gw = 2;
  if (!gw) return DIP_ERR_UNSUPPORTED;
  // per-CTA limits: gate rows (= candidate channels) plus one padding entry
  // <= 16*kLfTilesA, and at most one row per thread
  if ((I + nb - 1) / nb > 16 * kLfTilesA - 1 || (I + nb - 1) / nb > kLfThreads)
    return DIP_ERR_UNSUPPORTED;
  if (workspace_bytes < dip_mlp_fused_workspace_bytes(H, I, k)) return DIP_ERR_WORKSPACE;
  const uintptr_t al = reinterpret_cast<uintptr_t>(L->gate_qw) | reinterpret_cast<uintptr_t>(L->up_qw) |
                       reinterpret_cast<uintptr_t>(L->down_t_qw) | reinterpret_cast<uintptr_t>(x) |
                       reinterpret_cast<uintptr_t>(g_out) | reinterpret_cast<uintptr_t>(workspace);
  if (al & 15) return DIP_ERR_ARG;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  LfArgs a = {};
  a.scratch = reinterpret_cast<unsigned*>(ws);
  ws += (topk_scratch_bytes() + 255) & ~size_t(255);
  a.bar = reinterpret_cast<GridBar*>(ws);
  ws += 256;
  a.g = g_out ? g_out : reinterpret_cast<uint16_t*>(ws);
  ws += ((size_t)I * 2 + 255) & ~size_t(255);
  a.idx = idx_out ? idx_out : reinterpret_cast<int32_t*>(ws);
  ws += ((size_t)k * 4 + 255) & ~size_t(255);
  a.partial = reinterpret_cast<float*>(ws);
  a.gate_qw = reinterpret_cast<const uint8_t*>(L->gate_qw);
  a.gate_sc = L->gate_sc;
  a.up_qw = reinterpret_cast<const uint8_t*>(L->up_qw);
  a.up_sc = L->up_sc;
  a.dn_qw = reinterpret_cast<const uint8_t*>(L->down_t_qw);
  a.dn_sc = L->down_t_sc;
  a.hidden = (int)H;
  a.inter = (int)I;
  a.k = (int)k;
  a.x = x;
  a.resid = resid;
  a.eps = eps;
  a.x_used = x_used;
  a.y = y;
  a.err = error_word_ptr();
  if (!a.err) return DIP_ERR_CUDA;
  cudaError_t e;
  if (gw == 1) {
    e = cudaFuncSetAttribute(layer_fused_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             LfGeom<1>::total);
    if (e != cudaSuccess) return launch_status(e);
    return launch_status(launch_coop(layer_fused_kernel<1>, dim3(nb), dim3(kLfThreads),
                                     (size_t)LfGeom<1>::total, (cudaStream_t)stream, a));
  }
  e = cudaFuncSetAttribute(layer_fused_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           LfGeom<2>::total);
  if (e != cudaSuccess) return launch_status(e);
  return launch_status(launch_coop(layer_fused_kernel<2>, dim3(nb), dim3(kLfThreads),
                                   (size_t)LfGeom<2>::total, (cudaStream_t)stream, a));
}
