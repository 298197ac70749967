// layer_fused.cu — one decode DIP MLP layer as ONE persistent kernel.
//
// CTA 0 coordinates; CTAs 1..n-1 ("workers") each own a contiguous range of
// gate rows (= candidate channels):
//
//   workers    phase A  gate GEMV + SiLU over the owned rows -> g; coarse |g|
//                       histogram (no arrival flag: the coordinator checks the
//                       histogram totals)
//              spec C   up GEMV of the owned rows with the largest |g| (about
//                       their expected share of k, nearly always selected),
//                       started while the selection is computed
//   CTA 0      waits until the histograms hold every key, computes the exact selection
//              (topk_select.cu semantics) over all of g, publishes thresholds
//              and each worker's tier counts, releases
//   workers    take the thresholds, list the owned selected rows, write their
//              part of idx, up GEMV of the selected rows not yet done, then
//              the gathered down projection of the selected rows (tensor
//              cores) into one fp32 partial vector per worker
//   --- grid barrier ---
//   all        phase E  fixed-order sum of the partials -> y
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
// streams its bytes through a private 3-deep cp.async ring and never waits for
// another warp inside a phase.  The gate phase's first tiles are requested
// before waiting on the previous kernel (weights are static), so consecutive
// layers overlap.
#include "dip_block.cuh"
#include "dip_common.cuh"

namespace dip {

constexpr int kLfWarps = 20;
constexpr int kLfThreads = kLfWarps * 32;
#ifndef DIP_LF_DEPTH
#define DIP_LF_DEPTH 3
#endif
constexpr int kLfDepth = DIP_LF_DEPTH;  // cp.async ring slots per warp
constexpr int kLfTilesA = 12;   // max gate tiles (16 rows) per CTA
constexpr int kLfDnPitch = 144;  // bytes per channel row of a down slot (128 + pad)
constexpr int kLfMaxCtas = 160;  // CTAs per grid (SMs per GPU) supported
constexpr int kLfMaxRanks = 8;   // tensor-parallel ranks supported
constexpr int kLfPfTiles = 3;    // next-layer gate tiles per worker moved into L2

struct LfSel;
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
  unsigned* scratch;        // selection block (LfSel; zero on entry, left zero)
  float* partial;           // [gridDim.x][hidden]
  uint16_t* y;              // [hidden]
  float* y_f32;             // optional
  uint16_t* h_out;          // optional [inter_total]: h of each selected channel, by channel id
  // optional: the next layer's gate weights (same shape); each worker moves
  // the first rows of its range into L2 once its own work is done
  const uint8_t* pf_qw; const uint16_t* pf_sc;
  GridBar* bar;
  unsigned* err;
  // cache-aware DIP (dip_ca.py:127-188), optional: channel c's up and down
  // rows come from the resident cache row id2slot[c] when that is >= 0
  const int64_t* id2slot;
  const uint8_t* res_up_qw; const uint16_t* res_up_sc;
  const uint8_t* res_dn_qw; const uint16_t* res_dn_sc;
  // tensor parallel along I (template TP): this rank's rows are the channels
  // [c0, c0 + inter) of inter_total.  psel / pysl / pyflag[q]: rank q's
  // selection block, y slots [world][hidden] fp32 and y flags [world][160],
  // as this rank maps them (q == rank: its own).  Single GPU: inter_total =
  // inter, rank 0, world 1, c0 0.
  int inter_total, rank, world, c0;
  LfSel* psel[kLfMaxRanks];
  float* pysl[kLfMaxRanks];
  unsigned long long* pyflag[kLfMaxRanks];
};

// Byte offsets of the dynamic shared memory.
constexpr int kLfListMax = (kLfTilesA + 1) * 16;  // entries of the C / D lists
template <int GW>
struct LfGeom {
  // GEMV phases: 16 rows x GW x 64 B + scale words; down phase: 16 rows at a
  // 144-byte pitch + scale words.
  static constexpr int slot = (GW * 1024 + 64 > 16 * kLfDnPitch + 64) ? GW * 1024 + 64
                                                                       : 16 * kLfDnPitch + 64;
  static constexpr int ring = kLfWarps * kLfDepth * slot;
  static constexpr int xs = ring;                      // x staging (G*72 words), phase A start
  static constexpr int G = kLfWarps * GW;
  static constexpr int lists = xs;                     // after phase A: rank / C / D lists
  static constexpr int lists_bytes = 6 * kLfListMax * 4;
  static constexpr int xs_bytes = (G * 72 * 4 > lists_bytes) ? G * 72 * 4 : lists_bytes;
  static constexpr int gsum = xs + xs_bytes;
  // gsum: per group the sums of the even- and odd-indexed x values
  static constexpr int red = gsum + ((G * 8 + 15) & ~15);  // [tiles][warps][16]
  static constexpr int red_words = (kLfTilesA + 1) * kLfWarps * 16;
  static constexpr int gloc = red + red_words * 4;         // this CTA's g values (bf16)
  static constexpr int lslot = gloc + kLfListMax * 2;      // this CTA's cache slots (CA-DIP)
  static constexpr int misc = lslot + kLfListMax * 4;      // small scalars
  static constexpr int hist = misc + 256;                  // CTA histogram: hash keys,
  static constexpr int slot64 = hist + 3 * 256 * 4;        // counts, coarse bins; CA: id2slot
  static constexpr int total = slot64 + kLfListMax * 8;    // of this CTA's rows (int64)
  static_assert(total <= 227 * 1024, "shared memory per CTA");
};

__device__ __forceinline__ uint16_t ld_cg_u16(const uint16_t* p) {
  unsigned short v;
  asm volatile("ld.global.cg.u16 %0, [%1];\n" : "=h"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ld_cg_v4u(const uint16_t* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
// Polled words are read with relaxed loads: a weak load (ld.cg) of an
// unchanged address may be hoisted out of the polling loop.
__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint4 ld_relaxed_v4(const unsigned* p) {  // 16-byte aligned
  uint4 v;
  asm volatile("ld.relaxed.gpu.global.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_cg_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.global.cg.u32 %0, [%1];\n" : "=r"(v) : "l"(p));
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
// As cp_async16_lf / cp_async4_lf, but an invalid source writes zeros and
// reads nothing (src-size 0): the padding rows of a partial tile cost no
// memory request.  The address must still be a valid one (a real row).
__device__ __forceinline__ void cp_async16_zf(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async4_zf(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(valid ? 4 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_commit_lf() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_wait_lf() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(kLfDepth - 1) : "memory");
}
__device__ __forceinline__ void cp_wait_lf2() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(kLfDepth - 2) : "memory");
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
      // fp16 operands: the k-high registers (out[1], out[3]) carry 16 x
      // the weight, and their x fragments 1/16 of x (see the prologue)
      uint32_t qa4[4], qb4[4];
      nib8_biased_f16x2(ra[w], qa4);
      nib8_biased_f16x2(rb[w], qb4);
      const uint32_t a_even[4] = {qa4[0], qb4[0], qa4[1], qb4[1]};
      const uint32_t a_odd[4] = {qa4[2], qb4[2], qa4[3], qb4[3]};
      mma_f16_16816(d0, a_even, xf[gi][4 * w + 0], xf[gi][4 * w + 1]);
      mma_f16_16816(d1, a_odd, xf[gi][4 * w + 2], xf[gi][4 * w + 3]);
    }
    acc_a = fmaf(bf16_bits_to_f32(sca[gi + sofs]), (d0[0] + d1[0]) - bias[gi], acc_a);
    acc_b = fmaf(bf16_bits_to_f32(scb[gi + sofs]), (d0[2] + d1[2]) - bias[gi], acc_b);
  }
}

// Issue one GEMV tile slice into this warp's ring slot: groups [warp*GW,
// (warp+1)*GW) of the tile's 16 rows (qrow(r) / srow(r) give tile row r's
// packed row and scale row), plus the 4-byte scale words of the 16 rows
// (lanes 0..15).  Slot layout
// (read by lf_tile_dot): [group gi][rows 0-7 | rows 8-15][lane (row&7)*4 + tq]
// x 16 bytes.  With GW == 2 a warp's slice of a row is one aligned 128-byte
// line, so each instruction fetches 4 whole lines (8 lanes per row); with
// GW == 1 it is 64 bytes (4 lanes per row, 8 rows per instruction).
// Rows r >= nvalid are tile padding: zero-filled, not read.
template <int GW, class QRow, class SRow>
__device__ __forceinline__ void lf_issue_gemv(uint8_t* slot, QRow qrow, SRow srow, int nvalid,
                                              int warp, int lane) {
  if (GW == 2) {
    const int rsub = lane >> 3, c = lane & 7, gi = c >> 2, tq = c & 3;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = 4 * j + rsub;
      cp_async16_zf(slot + (gi * 2 + (r >> 3)) * 512 + ((r & 7) * 4 + tq) * 16,
                    qrow(r) + warp * 128 + c * 16, r < nvalid);
    }
  } else {
    const int gq = lane >> 2, tq = lane & 3;
    const int off = warp * kGroupBytes + tq * 16;
    cp_async16_zf(slot + lane * 16, qrow(gq) + off, gq < nvalid);
    cp_async16_zf(slot + 512 + lane * 16, qrow(gq + 8) + off, gq + 8 < nvalid);
  }
  if (lane < 16) {
    // GW == 2: the 4 bytes [4 warp, 4 warp + 4); GW == 1: 2 bytes, copy the
    // aligned 4-byte word containing them.
    cp_async4_zf(slot + GW * 1024 + lane * 4, srow(lane) + ((warp * GW) & ~1), lane < nvalid);
  }
}

// Selection parameters of one call, written by the coordinating CTA (CTA 0)
// once every worker has arrived, read by the workers.
// Words written once per call carry the call's tag (bit 31 set, never 0) in
// their upper half, so a reader polls the word itself and needs no separate
// flag: 64-bit stores and loads are single-copy atomic.
struct LfSel {
  unsigned long long done;  // final barrier: arrivals of all calls so far (grows by gridDim.x per call)
  unsigned pad_done[30];
  unsigned coarse[256];  // coarse |g| histogram (one bin per bf16 exponent); zero between calls
  unsigned nan_count;    // NaN keys (in no bin): the bins plus this add up to inter once
                         // every worker's keys are in; zero between calls
  unsigned pad0[31];
  unsigned long long par[4];             // tagged: lo bits, hi bits, totA, filled
  unsigned long long pre[kLfMaxCtas][2];  // tagged, per worker: tier A, tier B counts before it
  // tagged, per rank and worker: tier A << 16 | tier B (single GPU: rank 0)
  unsigned long long cnt[kLfMaxRanks][kLfMaxCtas];
  // fine |g| histogram (one bin per key).  Single GPU: set 0 only, zero
  // between calls.  Tensor parallel: set (call index & 1); a call clears the
  // other set, which the previous call used (see layer_fused_kernel).
  unsigned fine[2][kTopkHistBins];
};
static_assert(offsetof(LfSel, coarse) % 16 == 0 && offsetof(LfSel, fine) % 16 == 0,
              "histograms are read in 16-byte pieces");
__device__ __forceinline__ unsigned lf_tag(unsigned long long done0) {
  return (unsigned)(done0 + 1u) | 0x80000000u;
}
__device__ __forceinline__ unsigned long long ld_cg_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.global.cg.u64 %0, [%1];\n" : "=l"(v) : "l"(p));
  return v;
}
// Final grid barrier: one release-add per CTA on a counter that only grows,
// each CTA polls the counter itself until the call's last arrival (the next
// multiple of the grid size).  Bounded like grid_sync.
__device__ __forceinline__ void lf_final_barrier(unsigned long long* done, unsigned* err) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned long long nb = gridDim.x;
    unsigned long long old;
    asm volatile("atom.add.release.gpu.global.u64 %0, [%1], 1;\n" : "=l"(old) : "l"(done) : "memory");
    const unsigned long long target = old - old % nb + nb;
    bool ok = old + 1 == target;
    for (uint32_t it = 0, lim = spin_limit(err); it < lim && !ok; ++it) {
      unsigned long long v;
      asm volatile("ld.acquire.gpu.global.u64 %0, [%1];\n" : "=l"(v) : "l"(done) : "memory");
      ok = v >= target;
    }
    if (!ok) atomicOr(err, kErrTimeout);
    asm volatile("fence.acq_rel.gpu;\n" ::: "memory");
  }
  __syncthreads();
}
__device__ __forceinline__ unsigned long long lf_tagged(unsigned tag, unsigned v) {
  return ((unsigned long long)tag << 32) | v;
}
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// System-scope forms for words that other GPUs write over NVLink (TP).
__device__ __forceinline__ unsigned ld_relaxed_sys_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint4 ld_relaxed_sys_v4(const unsigned* p) {  // 16-byte aligned
  uint4 v;
  asm volatile("ld.relaxed.sys.global.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_add_sys(unsigned* p, unsigned v) {
  asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;\n" ::"l"(p), "l"(v) : "memory");
}
template <bool TP>
__device__ __forceinline__ unsigned lf_ld_u32(const unsigned* p) {
  return TP ? ld_relaxed_sys_u32(p) : ld_relaxed_u32(p);
}
template <bool TP>
__device__ __forceinline__ uint4 lf_ld_v4(const unsigned* p) {
  return TP ? ld_relaxed_sys_v4(p) : ld_relaxed_v4(p);
}

// Gate rows of worker CTA b (1..nb-1); CTA 0 only coordinates.
__device__ __forceinline__ int lf_row_start(int I, int nwk, int w) {
  return I * w / nwk;  // I * w < 2^31 (checked on the host)
}

// CTA 0 coordinates one call in two releases (tagged words of LfSel):
//   1. once the histograms hold every key: the (K+1)-th largest key w from the
//      coarse and fine histograms, topk_select.cu's 25-step fp32 bisection run
//      on w, the tier totals -> lo, hi, totA, filled; release 1
//   2. once every worker has published its tier A / tier B counts: their
//      exclusive prefix -> pre[]; release 2
// The workers add their keys with relaxed atomics and no fence or arrival
// flag: the coarse bins are complete once they and the NaN count add up to I
// (every count only grows towards its final value), and a coarse bin's fine
// bins once they add up to its coarse count.  It clears the coarse histogram
// and the NaN count; the workers clear the fine bins.
//
// Tensor parallel (TP): every rank's workers add their keys to every rank's
// histograms (remote reductions over NVLink), so each rank's coordinator sees
// the histogram of all I channels and computes the same selection.  The
// prefix of release 2 runs over the workers of all ranks in rank order:
// worker counts of lower ranks arrive as tagged words in cnt[q][*].
template <bool TP>
__device__ __noinline__ void lf_coordinate(unsigned* err, LfSel* sel, int K, int I, int nb,
                                           unsigned tag, int rank, int par) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwk = nb - 1;
  const unsigned* fine = sel->fine[par];
  __shared__ int s_cnt[2 * kLfMaxCtas];
  if (warp == 0) {
    int c8[8], loc = 0;
    bool ok = false;
    for (uint32_t it = 0, lim = spin_limit(err); it < lim && !ok; ++it) {
      // bins 255 - 8 lane - q, q = 0..7: the 8 words from 248 - 8 lane, reversed
      const uint4 hi4 = lf_ld_v4<TP>(sel->coarse + 252 - 8 * lane);
      const uint4 lo4 = lf_ld_v4<TP>(sel->coarse + 248 - 8 * lane);
      c8[0] = (int)hi4.w; c8[1] = (int)hi4.z; c8[2] = (int)hi4.y; c8[3] = (int)hi4.x;
      c8[4] = (int)lo4.w; c8[5] = (int)lo4.z; c8[6] = (int)lo4.y; c8[7] = (int)lo4.x;
      loc = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) loc += c8[q];
      const int nan = lane == 0 ? (int)lf_ld_u32<TP>(&sel->nan_count) : 0;
      ok = __reduce_add_sync(0xffffffffu, loc + nan) == I;
    }
    if (!ok && lane == 0) atomicOr(err, kErrTimeout);
    int incl = loc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    int suf8[8], run = incl - loc;
#pragma unroll
    for (int q = 0; q < 8; ++q) { run += c8[q]; suf8[q] = run; }
    auto suffix_at = [&](int bin) -> int {  // #keys in coarse bins >= bin (warp-uniform bin)
      if (bin >= 256) return 0;
      const int src = (255 - bin) >> 3, q = (255 - bin) & 7;
      int v = 0;
#pragma unroll
      for (int qq = 0; qq < 8; ++qq) v = (qq == q) ? suf8[qq] : v;
      return __shfl_sync(0xffffffffu, v, src);
    };
    auto coarse_at = [&](int bin) -> int {
      return (bin < 0 || bin >= 256) ? 0 : suffix_at(bin) - suffix_at(bin + 1);
    };
    const int nvalid = __shfl_sync(0xffffffffu, run, 31);
    const bool has_w = nvalid >= K + 1;
    int b1 = -1, btop = -1;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      if (suf8[q] - c8[q] < K + 1 && K + 1 <= suf8[q]) b1 = 255 - (lane * 8 + q);
      if (c8[q] > 0) btop = max(btop, 255 - (lane * 8 + q));
    }
    b1 = __reduce_max_sync(0xffffffffu, b1 + 1) - 1;
    btop = __reduce_max_sync(0xffffffffu, btop + 1) - 1;
    // fine bins of b1 - 1, b1, b1 + 1 (lo and hi end within a key of w, so
    // the tier totals come from these too) and of the top coarse bin (the
    // largest key), loaded together until each adds up to its coarse count
    int fb[4][4];
    const int fbin[4] = {b1 - 1, b1, b1 + 1, btop};
    ok = false;
    for (uint32_t it = 0, lim = spin_limit(err); it < lim && !ok; ++it) {
#pragma unroll
      for (int d = 0; d < 4; ++d) {
        const int cb = fbin[d];
        const bool use = cb >= 0 && cb < 256 && (d == 3 || has_w);
        const uint4 v = use ? lf_ld_v4<TP>(fine + ((cb << 7) | (lane * 4)))
                            : make_uint4(0u, 0u, 0u, 0u);
        fb[d][0] = (int)v.x; fb[d][1] = (int)v.y; fb[d][2] = (int)v.z; fb[d][3] = (int)v.w;
      }
      ok = true;
#pragma unroll
      for (int d = 0; d < 4; ++d) {
        const int cb = fbin[d];
        const bool use = cb >= 0 && cb < 256 && (d == 3 || has_w);
        const int sum = __reduce_add_sync(0xffffffffu, fb[d][0] + fb[d][1] + fb[d][2] + fb[d][3]);
        ok = ok && (!use || sum == coarse_at(cb));
      }
    }
    if (!ok && lane == 0) atomicOr(err, kErrTimeout);
    int kmax = -1;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (btop >= 0 && fb[3][q] > 0) kmax = (btop << 7) | (lane * 4 + q);
    kmax = __reduce_max_sync(0xffffffffu, kmax + 1) - 1;
    const unsigned maxkey = kmax < 0 ? 0u : (unsigned)kmax;
    float wv = 0.f;
    if (has_w) {
      const int rank = K + 1 - suffix_at(b1 + 1);
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
      found = __reduce_max_sync(0xffffffffu, found + 1) - 1;
      wv = bf16_bits_to_f32((unsigned)((b1 << 7) | found));
    }
    // topk_select.cu's bisection: hi from the fp32 max of |g|, 25 halvings,
    // "count(> t) > k" decided exactly by "w > t"
    float hi = bf16_bits_to_f32(maxkey), lo = 0.0f;
    float t = __fmul_rn(0.5f, __fadd_rn(lo, hi));
#pragma unroll
    for (int step = 0; step < 25; ++step) {
      const bool up = has_w && wv > t;
      lo = up ? t : lo;
      hi = up ? hi : t;
      t = __fmul_rn(0.5f, __fadd_rn(lo, hi));
    }
    // #keys > tt = #keys >= kmin, kmin the bf16 key just above tt
    auto count_above = [&](float tt) -> int {
      const int kmin = (int)(__float_as_uint(tt) >> 16) + 1;
      if (kmin > 0x7F80) return 0;
      const int cb = kmin >> 7, f0 = kmin & 127, d = cb - (b1 - 1);
      int fv[4];
      if (has_w && d >= 0 && d < 3) {
#pragma unroll
        for (int q = 0; q < 4; ++q) fv[q] = d == 0 ? fb[0][q] : d == 1 ? fb[1][q] : fb[2][q];
      } else if (cb == btop) {
#pragma unroll
        for (int q = 0; q < 4; ++q) fv[q] = fb[3][q];
      } else {  // rare: a bin not loaded above, read until complete
        const int want = coarse_at(cb);
        bool okb = false;
        for (uint32_t it = 0, lim = spin_limit(err); it < lim && !okb; ++it) {
          const uint4 v = lf_ld_v4<TP>(fine + ((cb << 7) | (lane * 4)));
          fv[0] = (int)v.x; fv[1] = (int)v.y; fv[2] = (int)v.z; fv[3] = (int)v.w;
          okb = __reduce_add_sync(0xffffffffu, fv[0] + fv[1] + fv[2] + fv[3]) == want;
        }
        if (!okb && lane == 0) atomicOr(err, kErrTimeout);
      }
      int part = 0;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (lane * 4 + q >= f0) part += fv[q];
      return __reduce_add_sync(0xffffffffu, part) + suffix_at(cb + 1);
    };
    const int totA = count_above(hi);
    const int above_lo = count_above(lo);
    // all keys are in: clear the coarse bins for the next call
    *reinterpret_cast<uint4*>(sel->coarse + 4 * lane) = make_uint4(0u, 0u, 0u, 0u);
    *reinterpret_cast<uint4*>(sel->coarse + 128 + 4 * lane) = make_uint4(0u, 0u, 0u, 0u);
    if (lane == 0) sel->nan_count = 0u;
    if (lane < 4) {  // release 1
      const unsigned v = lane == 0 ? __float_as_uint(lo) : lane == 1 ? __float_as_uint(hi)
                       : lane == 2 ? (unsigned)totA : (unsigned)min(K, above_lo);
      sel->par[lane] = lf_tagged(tag, v);
    }
  }
  // round 2: every worker's (tier A, tier B) count word (TP: of this rank
  // and the lower ranks), prefix, release 2
  __shared__ int s_low[2];
  for (int i = tid; i < 2 * kLfMaxCtas; i += kLfThreads) s_cnt[i] = 0;
  if (tid < 2) s_low[tid] = 0;
  __syncthreads();
  {
    int la = 0, lb = 0;
    const int nent = (TP ? rank + 1 : 1) * nwk;
    for (int e = tid; e < nent; e += kLfThreads) {
      const int q = e / nwk, w = 1 + e - q * nwk;
      const unsigned long long* p = &sel->cnt[q][w];
      unsigned long long v = 0;
      bool ok = false;
      for (uint32_t it = 0, lim = spin_limit(err); it < lim && !ok; ++it) {
        if (TP) v = ld_acquire_sys_u64(p);
        else asm volatile("ld.acquire.gpu.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
        ok = (unsigned)(v >> 32) == tag;
      }
      if (!ok) { atomicOr(err, kErrTimeout); v = 0; }
      const int ca = (int)((v >> 16) & 0xFFFFu), cb = (int)(v & 0xFFFFu);
      if (TP && q < rank) {
        la += ca;
        lb += cb;
      } else {
        s_cnt[2 * (w - 1)] = ca;
        s_cnt[2 * (w - 1) + 1] = cb;
      }
    }
    if (TP && rank > 0) {
      la = __reduce_add_sync(0xffffffffu, la);
      lb = __reduce_add_sync(0xffffffffu, lb);
      if (lane == 0 && (la | lb)) { atomicAdd(&s_low[0], la); atomicAdd(&s_low[1], lb); }
    }
  }
  __syncthreads();
  if (warp == 0) {
    int va[5], vb[5], la = 0, lb = 0;
#pragma unroll
    for (int q = 0; q < 5; ++q) {
      const int c = lane * 5 + q;
      va[q] = c < nwk ? s_cnt[2 * c] : 0;
      vb[q] = c < nwk ? s_cnt[2 * c + 1] : 0;
      la += va[q];
      lb += vb[q];
    }
    int ia = la, ib = lb;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int ta = __shfl_up_sync(0xffffffffu, ia, o), tb = __shfl_up_sync(0xffffffffu, ib, o);
      if (lane >= o) { ia += ta; ib += tb; }
    }
    int pa = ia - la + s_low[0], pb = ib - lb + s_low[1];
#pragma unroll
    for (int q = 0; q < 5; ++q) {  // release 2
      const int c = lane * 5 + q;
      if (c < nwk) {
        sel->pre[c + 1][0] = lf_tagged(tag, (unsigned)pa);
        sel->pre[c + 1][1] = lf_tagged(tag, (unsigned)pb);
      }
      pa += va[q];
      pb += vb[q];
    }
  }
}

template <int GW, bool CA, bool TP>
__global__ void __launch_bounds__(kLfThreads, 1) layer_fused_kernel(const LfArgs a) {
  using Geo = LfGeom<GW>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;
  // I: this GPU's rows; IT: all channels (equal unless TP)
  const int H = a.hidden, I = a.inter, K = a.k, IT = TP ? a.inter_total : a.inter;
  const int rowb = H / 2, scw = H / kGroup;  // bytes per packed row, scales per row
  const int nb = gridDim.x, b = blockIdx.x, nwk = nb - 1;
  const int rank = TP ? a.rank : 0;
  LfSel* sel = reinterpret_cast<LfSel*>(a.scratch);
  // this call's tag (from the final barrier's counter, which grows by the
  // grid size once per call) and, TP, the parity of the call index (which
  // fine histogram set the call uses)
  __shared__ unsigned s_tag;
  __shared__ int s_cpar;
  auto read_tag = [&]() {
    if (tid == 0) {
      const unsigned long long d0 = ld_cg_u64(&sel->done);
      s_tag = lf_tag(d0);
      s_cpar = TP ? (int)((d0 / (unsigned long long)nb) & 1ull) : 0;
    }
  };

  if (b == 0) {
    pdl_wait();
    read_tag();
    __syncthreads();
    lf_coordinate<TP>(a.err, sel, K, IT, nb, s_tag, rank, s_cpar);
  } else {
  uint8_t* ring = smem + warp * kLfDepth * Geo::slot;
  uint32_t* xs = reinterpret_cast<uint32_t*>(smem + Geo::xs);
  float* gsum = reinterpret_cast<float*>(smem + Geo::gsum);
  float* red = reinterpret_cast<float*>(smem + Geo::red);
  uint16_t* gloc = reinterpret_cast<uint16_t*>(smem + Geo::gloc);
  float* misc = reinterpret_cast<float*>(smem + Geo::misc);
  // GW == 1 reads the scale of group `warp` from the 4-byte word copied at
  // (warp & ~1); GW == 2 reads both halves.
  const int sc_sel = (GW == 1) ? (warp & 1) : 0;

  // ------------------------------------------------------------ phase A
  const int ra0 = lf_row_start(I, nwk, b - 1), ra1 = lf_row_start(I, nwk, b);
  const int na = ra1 - ra0, nta = (na + 15) / 16;
  auto issue_a = [&](int i) {
    if (i < nta) {
      const int rbase = ra0 + i * 16, rlast = ra1 - 1;
      lf_issue_gemv<GW>(ring + (i % kLfDepth) * Geo::slot,
                        [&](int r) { return a.gate_qw + (size_t)min(rbase + r, rlast) * rowb; },
                        [&](int r) { return a.gate_sc + (size_t)min(rbase + r, rlast) * scw; },
                        ra1 - rbase, warp, lane);
    }
    cp_commit_lf();
  };
  // Only the first tile goes out ahead of the layer input: the input loads
  // queue behind every line this SM has requested, so the other tiles are
  // requested right after them.
  // CA-DIP: the cache slots of this CTA's rows travel with the first gate
  // tile (they are static like the weights); loaded after the gate they held
  // the whole CTA for a DRAM round trip at the next barrier.
  if (CA && tid < na)
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(smem_u32(smem + Geo::slot64 + tid * 8)),
                 "l"(a.id2slot + ra0 + tid)
                 : "memory");
  issue_a(0);
  pdl_wait();
  read_tag();

  // Layer input: x, or RMSNorm(x + resid); one 16-byte word (8 values) per
  // thread (H / 8 <= kLfThreads, checked on the host), staged in the
  // B-fragment order.
  {
    const int nwords = H / 8;
    const bool mine = tid < nwords;
    uint4 xw = make_uint4(0u, 0u, 0u, 0u), rw = make_uint4(0u, 0u, 0u, 0u);
    if (mine) {
      xw = ld_cg_v4u(a.x + tid * 8);
      if (a.resid) rw = ld_cg_v4u(a.resid + tid * 8);
    }
#pragma unroll
    for (int i = 1; i < kLfDepth - 1; ++i) issue_a(i);
    const uint32_t xa[4] = {xw.x, xw.y, xw.z, xw.w}, ra[4] = {rw.x, rw.y, rw.z, rw.w};
    float v[8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      v[2 * q] = bf16_bits_to_f32(xa[q] & 0xFFFFu);
      v[2 * q + 1] = bf16_bits_to_f32(xa[q] >> 16);
    }
    // One block reduction gives both the RMSNorm sum of squares and max |v|.
    // The GEMV phases run on fp16 operands: x is scaled by 2^m (exact for a
    // bf16 value above fp16's normal range floor) so that max|x| lands near
    // [2^13, 2^14) (taken from max|v| * the norm factor; the bf16 rounding of
    // the normalised values can only move it by one part in 256), far inside
    // fp16's range whatever the input; the results are scaled back by 2^-m.
    // The odd-indexed values of each 8-value word go to the k-high fragment
    // registers, whose weights carry a factor 16 (nib8_biased_f16x2), so they
    // are scaled by 2^(m-4).
    float ssq = 0.f, amax = 0.f;
    if (a.resid) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        v[2 * q] += bf16_bits_to_f32(ra[q] & 0xFFFFu);
        v[2 * q + 1] += bf16_bits_to_f32(ra[q] >> 16);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ssq = fmaf(v[e], v[e], ssq);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ssq += __shfl_xor_sync(0xffffffffu, ssq, o);
    }
    if (mine) {
#pragma unroll
      for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(v[e]));
    }
    // |v| >= 0: its bit pattern orders like the value
    amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(amax)));
    if (lane == 0) {
      misc[warp] = ssq;
      misc[40 + warp] = amax;
    }
    __syncthreads();
    // every thread combines the per-warp values itself (same order, same
    // result everywhere): no second barrier
    float sc_m, sc_minv, inv;
    {
      float t = 0.f, mx = 0.f;
      for (int w = 0; w < kLfWarps; ++w) {
        t += misc[w];
        mx = fmaxf(mx, misc[40 + w]);
      }
      inv = a.resid ? rsqrtf(t / (float)H + a.eps) : 1.f;
      mx *= inv;
      // 2^m with 2^13 <= mx 2^m < 2^14 (m = 0 for zero / non-finite input)
      int m = 0;
      if (mx > 0.f && mx <= 3.0e38f) {
        int e;
        frexpf(mx, &e);  // mx = f 2^e, f in [0.5, 1)
        m = max(-100, min(100, 14 - e));
      }
      sc_m = ldexpf(1.f, m);
      sc_minv = ldexpf(1.f, -m);
    }
    uint32_t v4[4] = {0u, 0u, 0u, 0u};
    float vv[8];
    if (mine) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        v4[q] = a.resid ? ((uint32_t)f32_to_bf16_bits(v[2 * q] * inv) |
                           ((uint32_t)f32_to_bf16_bits(v[2 * q + 1] * inv) << 16))
                        : xa[q];
        vv[2 * q] = bf16_bits_to_f32(v4[q] & 0xFFFF);
        vv[2 * q + 1] = bf16_bits_to_f32(v4[q] >> 16);
      }
      if (a.x_used && b == 1)
        *reinterpret_cast<uint4*>(a.x_used + tid * 8) = make_uint4(v4[0], v4[1], v4[2], v4[3]);
    }
    const float sc_lo = sc_m, sc_hi = sc_m * 0.0625f;
    if (tid == 0) {
      misc[33] = sc_m;
      misc[34] = sc_minv;
    }
    float part_e = 0.f, part_o = 0.f;
    if (mine) {
#pragma unroll
      for (int q = 0; q < 4; ++q) { part_e += vv[2 * q]; part_o += vv[2 * q + 1]; }
      auto h2 = [](float lo, float hi) {
        const __half2 p = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<const uint32_t*>(&p);
      };
      uint4 o;  // values (0,4), (1,5), (2,6), (3,7) of the word
      o.x = h2(vv[0] * sc_lo, vv[4] * sc_lo);
      o.y = h2(vv[1] * sc_hi, vv[5] * sc_hi);
      o.z = h2(vv[2] * sc_lo, vv[6] * sc_lo);
      o.w = h2(vv[3] * sc_hi, vv[7] * sc_hi);
      const int grp = tid >> 4, t = (tid >> 2) & 3, w = tid & 3;
      *reinterpret_cast<uint4*>(xs + grp * 72 + t * 16 + (t >> 1) * 4 + 4 * w) = o;
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
      part_e += __shfl_xor_sync(0xffffffffu, part_e, o);
      part_o += __shfl_xor_sync(0xffffffffu, part_o, o);
    }
    if ((lane & 15) == 0 && mine) {
      gsum[2 * (tid >> 4)] = part_e;
      gsum[2 * (tid >> 4) + 1] = part_o;
    }
  }
  __syncthreads();
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
    // in the 2^m units of the products: sum_even q x + sum_odd (q + 72) x
    bias[gi] = misc[33] * kNibbleBias16Hi * gsum[2 * grp + 1];
  }
  const float xinv = misc[34];  // 2^-m: the GEMV sums back in x's units

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
  __syncthreads();
  for (int r = tid; r < na; r += kLfThreads) {
    const int i = r >> 4, row = r & 15;
    float v = 0.f;
    for (int w = 0; w < kLfWarps; ++w) v += red[(i * kLfWarps + w) * 16 + row];
    v *= xinv;
    const uint16_t o = f32_to_bf16_bits(silu_f32(round_bf16(v)));
    a.g[ra0 + r] = o;
    gloc[r] = o;
  }
  {
    // cache slots of this CTA's rows (-1: no cache), narrowed from the
    // staged int64 values by the threads the loop above leaves idle
    int* lslot_w = reinterpret_cast<int*>(smem + Geo::lslot);
    const int t = tid - (kLfThreads - 16 * kLfTilesA);
    if (CA && t >= 0 && t < na)
      lslot_w[t] = (int)reinterpret_cast<const int64_t*>(smem + Geo::slot64)[t];
  }
  unsigned* hkey = reinterpret_cast<unsigned*>(smem + Geo::hist);  // [256] hash slots: key
  unsigned* hcnt = hkey + 256;                                      // [256] its count
  unsigned* hcrs = hcnt + 256;                                      // [256] coarse bins
  __shared__ unsigned s_nnan;
  for (int i = tid; i < 256; i += kLfThreads) { hkey[i] = 0xFFFFFFFFu; hcnt[i] = 0u; hcrs[i] = 0u; }
  if (tid == 0) s_nnan = 0u;
  __syncthreads();
  // ------------------------------------------------------------ speculation
  // This CTA's nts*16 rows with the largest |g| (about its expected share of
  // k, so nearly all of them end up selected): their up projection starts now,
  // while the coordinator computes the exact selection.  T, the (nts*16)-th
  // largest key, comes from the CTA's coarse histogram (built with the hash
  // table below) and a 128-bin histogram of the one coarse bin holding it;
  // warp 0 then lists the rows (keys > T, then keys == T while places
  // remain, each in row order).
  int* crow = reinterpret_cast<int*>(smem + Geo::lists);  // C list: spec rows, then rest rows
  int* drow = crow + kLfListMax;         // D list: selected channels
  int* dsrc = drow + kLfListMax;         // D entry -> C list position
  float* dh = reinterpret_cast<float*>(dsrc + kLfListMax);  // D entry: g, then h
  int* cpos = reinterpret_cast<int*>(dh + kLfListMax);      // local row -> C position or -1
  __shared__ int2 warp_tot[33];
  __shared__ int s_nts, s_b1, s_rank;
  __shared__ unsigned s_fine[128];
  const unsigned my_key = tid < na ? (gloc[tid] & 0x7FFFu) : 0xFFFFu;
  const bool my_valid = my_key <= 0x7F80u;
  if (warp == 0) {
    for (int r = lane; r < na; r += 32) cpos[r] = -1;
    for (int i = lane; i < 128; i += 32) s_fine[i] = 0u;
  } else if ((warp - 1) * 32 < na) {
    // |g| histograms of this CTA's keys: equal keys are merged in a shared
    // memory hash table first (SiLU's minimum piles ~1/8 of all values onto
    // two or three keys; per-row global atomics on them would serialise).
    const int r = (warp - 1) * 32 + lane;
    if (r < na) {
      const unsigned kk = gloc[r] & 0x7FFFu;
      if (kk <= 0x7F80u) {
        unsigned h = (kk * 0x9E3779B1u) >> 24;
        for (int p = 0; p < 256; ++p, h = (h + 1) & 255u) {
          const unsigned old = atomicCAS(&hkey[h], 0xFFFFFFFFu, kk);
          if (old == 0xFFFFFFFFu || old == kk) { atomicAdd(&hcnt[h], 1u); break; }
        }
        atomicAdd(&hcrs[kk >> 7], 1u);
      } else {
        atomicAdd(&s_nnan, 1u);
      }
    }
  }
  __syncthreads();
  if (warp == 0) {
    // coarse bins 255 - (8 lane + q), q = 0..7, in descending order
    int c8[8], loc = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) { c8[q] = (int)hcrs[255 - (8 * lane + q)]; loc += c8[q]; }
    int incl = loc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    const int nv = __shfl_sync(0xffffffffu, incl, 31);  // valid (non-NaN) keys
    const int nts_w = min(na * K / IT / 16, nv / 16);     // na * K < 2^31 (host check)
    const int nspec = nts_w * 16;
    int b1 = -1, above = 0, run = incl - loc;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      if (nspec > 0 && run < nspec && run + c8[q] >= nspec) { b1 = 255 - (8 * lane + q); above = run; }
      run += c8[q];
    }
    const int bl = __reduce_max_sync(0xffffffffu, b1 + 1) - 1;
    const int ab = __reduce_max_sync(0xffffffffu, b1 == bl ? above : 0);
    if (lane == 0) {
      s_nts = max(nts_w, 0);
      s_b1 = nts_w > 0 ? bl : -1;
      s_rank = nspec - ab;  // 1-based rank of T from the top inside bin b1
    }
  }
  __syncthreads();
  const int nts = s_nts;
  if (s_b1 >= 0 && my_valid && (int)(my_key >> 7) == s_b1) atomicAdd(&s_fine[my_key & 127], 1u);
  __syncthreads();
  if (warp == 0 && nts > 0) {
    const int b1 = s_b1, rank = s_rank, nspec = nts * 16;
    // fine bins 127 - (4 lane + q), descending
    int f4[4], loc = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) { f4[q] = (int)s_fine[127 - (4 * lane + q)]; loc += f4[q]; }
    int incl = loc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    int f = -1, run = incl - loc;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (run < rank && run + f4[q] >= rank) f = 127 - (4 * lane + q);
      run += f4[q];
    }
    f = __reduce_max_sync(0xffffffffu, f + 1) - 1;
    const unsigned T = ((unsigned)b1 << 7) | (unsigned)max(f, 0);
    constexpr int kPer = (16 * kLfTilesA + 31) / 32;  // rows per lane
    const unsigned lt = (1u << lane) - 1u;
    unsigned key[kPer];
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int r = q * 32 + lane;
      key[q] = r < na ? (gloc[r] & 0x7FFFu) : 0xFFFFu;
      if (key[q] > 0x7F80u) key[q] = 0xFFFFu;  // NaN: never speculated
    }
    int pos = 0;
#pragma unroll
    for (int q = 0; q < kPer; ++q) {  // keys > T
      const bool gt = key[q] != 0xFFFFu && key[q] > T;
      const unsigned m = __ballot_sync(0xffffffffu, gt);
      if (gt) { crow[pos + __popc(m & lt)] = ra0 + q * 32 + lane; cpos[q * 32 + lane] = pos + __popc(m & lt); }
      pos += __popc(m);
    }
#pragma unroll
    for (int q = 0; q < kPer; ++q) {  // keys == T while places remain
      const bool eq = key[q] == T;
      const unsigned m = __ballot_sync(0xffffffffu, eq);
      const int p = pos + __popc(m & lt);
      if (eq && p < nspec) { crow[p] = ra0 + q * 32 + lane; cpos[q * 32 + lane] = p; }
      pos += __popc(m);
    }
  }
  __syncthreads();

  // ------------------------------------------------------------ phases C + D
  // One cp.async stream per warp: spec up tiles, rest up tiles (this CTA's
  // tier A rows and tie candidates outside the speculation), then the down
  // tiles of the selected rows.
  __shared__ float s_lohi[2];
  __shared__ int s_par[4];
  __shared__ int s_n[2];
  int nC = nts, nD = 0, nDA = 0;
  int nCvalid = nts * 16;  // real rows of the C list (the rest is tile padding)
  bool have1 = false, have2 = false, c_done = false;
  // h = bf16(g * bf16(u)) for down list entries [r0, r1) once their up sums
  // are complete (entries hold g until then)
  auto make_h = [&](int r0, int r1) {
    const int pad_row = s_n[0];
    const float mult = (float)s_n[1];
    for (int r = r0 + tid; r < r1; r += kLfThreads) {
      const int src = dsrc[r];
      float h = 0.f;
      if (src >= 0) {
        const int ti = src >> 4, row = src & 15;
        float v = 0.f;
        for (int w = 0; w < kLfWarps; ++w) v += red[(ti * kLfWarps + w) * 16 + row];
        v *= xinv;
        h = round_bf16(dh[r] * round_bf16(v));
        if (a.h_out) a.h_out[(TP ? a.c0 : 0) + drow[r]] = f32_to_bf16_bits(h);
        if (r == pad_row) h *= mult;
      }
      dh[r] = h;
    }
    __syncthreads();
  };
  // Row sources: channel ch (one of this CTA's rows) reads its up / down row
  // from the resident cache when it has a slot there, else from the full
  // matrices.
  const int* lslot = reinterpret_cast<const int*>(smem + Geo::lslot);
  auto slot_of = [&](int ch) { return CA ? lslot[ch - ra0] : -1; };
  auto up_q = [&](int ch) {
    const int sl = slot_of(ch);
    return sl >= 0 ? a.res_up_qw + (size_t)sl * rowb : a.up_qw + (size_t)ch * rowb;
  };
  auto up_s = [&](int ch) {
    const int sl = slot_of(ch);
    return sl >= 0 ? a.res_up_sc + (size_t)sl * scw : a.up_sc + (size_t)ch * scw;
  };
  auto issue_c = [&](int i) {
    const int* rp = crow + i * 16;
    lf_issue_gemv<GW>(ring + (i % kLfDepth) * Geo::slot, [&](int r) { return up_q(rp[r]); },
                      [&](int r) { return up_s(rp[r]); }, nCvalid - i * 16, warp, lane);
  };
  const int seg = warp * GW * kGroupBytes;
  auto issue_d = [&](int j) {  // j: stream index; D tile j - nC
    const int i = j - nC;
    uint8_t* slot = ring + (j % kLfDepth) * Geo::slot;
#pragma unroll
    for (int q = 0; q < (16 * GW * 4) / 32; ++q) {
      const int chk = lane + 32 * q;
      const int r = chk / (GW * 4), part = chk % (GW * 4);
      const int ch = drow[i * 16 + r];
      const int sl = slot_of(ch);
      const uint8_t* row = sl >= 0 ? a.res_dn_qw + (size_t)sl * rowb : a.dn_qw + (size_t)ch * rowb;
      // padding entries (dsrc < 0) carry h = 0: zero-fill, no read
      cp_async16_zf(slot + r * kLfDnPitch + part * 16, row + seg + part * 16, dsrc[i * 16 + r] >= 0);
    }
    if (lane < 16) {
      const int ch = drow[i * 16 + lane];
      const int sl = slot_of(ch);
      const uint16_t* srow = sl >= 0 ? a.res_dn_sc + (size_t)sl * scw : a.dn_sc + (size_t)ch * scw;
      cp_async4_zf(slot + 16 * kLfDnPitch + lane * 4, srow + ((warp * GW) & ~1),
                   dsrc[i * 16 + lane] >= 0);
    }
  };
  auto issue = [&](int j) {
    if (j < nC) issue_c(j);
    else if (j < nC + nD) issue_d(j);
    cp_commit_lf();
  };
  // Tier A ("> hi") and tier B ("in (lo, hi]") of topk_select.cu; NaN for rows past na.
  const float kv = bf16_bits_to_f32(my_key);
  bool isA = false, isB = false;
  int2 offAB = make_int2(0, 0), totAB = make_int2(0, 0);
  // Release 1: the thresholds.  Publish this CTA's tier counts, clear the fine
  // bins it filled, queue the up rows of its tier A rows and tie candidates
  // not speculated on, and list its tier A rows for the down projection.
  auto poll1 = [&]() {
    if (tid == 0) {
      const unsigned tag = s_tag;
      unsigned long long p[4];
      bool done = false;
      for (uint32_t it = 0, lim = spin_limit(a.err); it < lim && !done; ++it) {
#pragma unroll
        for (int q = 0; q < 4; ++q) p[q] = ld_relaxed_u64(sel->par + q);
        done = (unsigned)(p[0] >> 32) == tag && (unsigned)(p[1] >> 32) == tag &&
               (unsigned)(p[2] >> 32) == tag && (unsigned)(p[3] >> 32) == tag;
      }
      if (!done) atomicOr(a.err, kErrTimeout);
      s_lohi[0] = __uint_as_float((unsigned)p[0]);
      s_lohi[1] = __uint_as_float((unsigned)p[1]);
      s_par[0] = (int)(unsigned)p[2];
      s_par[1] = (int)(unsigned)p[3];
    }
    __syncthreads();
  };
  auto apply1 = [&]() {
    const float lo = s_lohi[0], hi = s_lohi[1];
    isA = kv > hi;
    isB = kv > lo && kv <= hi;
    offAB = block_excl_scan2(isA, isB, warp_tot, totAB);
    if (!TP) {
      if (my_valid) sel->fine[0][my_key] = 0u;  // the coordinator has read the fine bins
    } else {
      // Keys of every rank land in every rank's histogram, and a remote fine
      // bin increment may still be in flight after the coordinator has read
      // the bins it needs.  So a call clears the other set, which the
      // previous call used: every increment of the previous call was issued
      // before its rank sent its y slots of that call, which this rank
      // received before this call.  The next call, which uses that set,
      // starts its increments only after receiving this rank's y slots of
      // this call, sent after this clear.
      uint4* f4 = reinterpret_cast<uint4*>(sel->fine[s_cpar ^ 1]);
      const int n4 = kTopkHistBins / 4;
      for (int i = n4 * (b - 1) / nwk + tid; i < n4 * b / nwk; i += kLfThreads)
        f4[i] = make_uint4(0u, 0u, 0u, 0u);
    }
    if (tid == 0) {
      // tagged word, its own payload: a relaxed store suffices.  TP: to this
      // rank and every higher rank (their prefixes count this rank's rows).
      const unsigned long long word = ((unsigned long long)s_tag << 32) |
                                      ((unsigned)totAB.x << 16) | (unsigned)totAB.y;
      if (TP) {
        for (int q = rank; q < a.world; ++q) st_relaxed_sys_u64(&a.psel[q]->cnt[rank][b], word);
      } else {
        asm volatile("st.relaxed.gpu.global.u64 [%0], %1;\n" ::"l"(&sel->cnt[0][b]), "l"(word)
                     : "memory");
      }
    }
    // the owner of channel 0 may need it for the index padding
    const bool pad_maybe = b == 1 && rank == 0 && s_par[1] < K;
    const bool restr = tid < na && (isA || isB || (pad_maybe && tid == 0)) && cpos[tid] < 0;
    int2 t2;
    const int2 o2 = block_excl_scan2(restr, false, warp_tot, t2);
    if (restr) {
      crow[nts * 16 + o2.x] = ra0 + tid;
      cpos[tid] = nts * 16 + o2.x;
    }
    __syncthreads();
    const int nrest = t2.x, ntr = (nrest + 15) / 16;
    for (int r = nrest + tid; r < ntr * 16; r += kLfThreads) crow[nts * 16 + r] = crow[nts * 16 + nrest - 1];
    if (isA) {  // down list: tier A rows first
      drow[offAB.x] = ra0 + tid;
      dsrc[offAB.x] = cpos[tid];
      dh[offAB.x] = bf16_bits_to_f32(gloc[tid]);
    }
    nC = nts + ntr;
    nCvalid = nts * 16 + nrest;
    nDA = totAB.x;
    nD = nDA / 16;  // the full tier A tiles need no release 2
    if (tid == 0) s_n[0] = -1;
    __syncthreads();
  };
  // Release 2: this CTA's prefix counts.  Write its part of idx, append the
  // selected tie rows and the padding entry to the down list.
  auto poll2 = [&]() {
    if (tid == 0) {
      const unsigned tag = s_tag;
      unsigned long long p0 = 0, p1 = 0;
      bool done = false;
      for (uint32_t it = 0, lim = spin_limit(a.err); it < lim && !done; ++it) {
        p0 = ld_relaxed_u64(&sel->pre[b][0]);
        p1 = ld_relaxed_u64(&sel->pre[b][1]);
        done = (unsigned)(p0 >> 32) == tag && (unsigned)(p1 >> 32) == tag;
      }
      if (!done) atomicOr(a.err, kErrTimeout);
      s_par[2] = (int)(unsigned)p0;
      s_par[3] = (int)(unsigned)p1;
    }
    __syncthreads();
  };
  auto apply2 = [&]() {
    const int totA = s_par[0], filled = s_par[1], selB = filled - totA;
    const int preA = s_par[2], preB = s_par[3];
    const int nB = max(0, min(totAB.y, selB - preB));
    const int c0 = TP ? a.c0 : 0;  // channel id of this GPU's row 0
    if (isA && preA + offAB.x < K && a.idx) a.idx[preA + offAB.x] = c0 + ra0 + tid;
    if (isB && offAB.y < nB) {
      if (a.idx) a.idx[totA + preB + offAB.y] = c0 + ra0 + tid;
      drow[nDA + offAB.y] = ra0 + tid;
      dsrc[nDA + offAB.y] = cpos[tid];
      dh[nDA + offAB.y] = bf16_bits_to_f32(gloc[tid]);
    }
    {
      const int per = (K - filled + nwk - 1) / nwk;
      const int z0 = filled + (b - 1) * per, z1 = min(K, z0 + per);
      if (rank == 0 && a.idx)
        for (int i2 = z0 + tid; i2 < z1; i2 += kLfThreads) a.idx[i2] = 0;
    }
    // The K - filled zero indices select channel 0 that many times: the
    // owner of row 0 adds one down entry for it, h scaled by the count.
    const bool pad = b == 1 && rank == 0 && filled < K;
    const int nd = nDA + nB + (pad ? 1 : 0);
    if (tid == 0) {
      if (pad) {
        drow[nDA + nB] = 0;
        dsrc[nDA + nB] = cpos[0];
        dh[nDA + nB] = bf16_bits_to_f32(gloc[0]);
      }
      s_n[0] = pad ? nDA + nB : -1;
      s_n[1] = K - filled;
    }
    __syncthreads();
    const int ntd = (nd + 15) / 16;
    for (int r = nd + tid; r < ntd * 16; r += kLfThreads) {
      drow[r] = drow[nd - 1];
      dsrc[r] = -1;
    }
    nD = ntd;
    __syncthreads();
    if (c_done) make_h(nDA, nD * 16);
  };
  // Release 1 before the first rest up tile; release 2 before the first down
  // tile that is not a full tile of tier A rows.
  // (blocking poll only when the stream reaches that point first)
  auto need = [&](int j) {  // before issuing stream index j
    if (!have1 && j >= nts) { poll1(); apply1(); have1 = true; }
    if (have1 && !have2 && j >= nC + nD) { poll2(); apply2(); have2 = true; }
  };
  // Per stream index j: wait for tile j, issue tile j + kLfDepth - 1 (into
  // the slot tile j - 1 used), compute tile j.
  // The first speculative up tiles are requested before the histogram
  // atomics below: requests queued behind ~500 same-address atomics per SM
  // landed ~6 us after the gate instead of ~2 us.
  const int npre = min(nts, kLfDepth - 1);
#pragma unroll 1
  for (int j = 0; j < npre; ++j) issue(j);  // j < nts: no release needed
  // This CTA's part of the global histograms: one relaxed atomic per distinct
  // key and coarse bin, no fence and no arrival flag (the coordinator checks
  // the totals), then the stream goes on at once.
  // TP: the same increments go to every rank's histograms over NVLink.
  if (tid < 256) {
    const unsigned kk = hkey[tid];
    if (kk != 0xFFFFFFFFu) {
      if (TP) {
        for (int q = 0; q < a.world; ++q) red_add_sys(&a.psel[q]->fine[s_cpar][kk], hcnt[tid]);
      } else {
        atomicAdd(&sel->fine[0][kk], hcnt[tid]);
      }
    }
  } else if (tid < 512) {
    const unsigned c = hcrs[tid - 256];
    if (c) {
      if (TP) {
        for (int q = 0; q < a.world; ++q) red_add_sys(&a.psel[q]->coarse[tid - 256], c);
      } else {
        atomicAdd(&sel->coarse[tid - 256], c);
      }
    }
  } else if (tid == 512 && s_nnan) {
    if (TP) {
      for (int q = 0; q < a.world; ++q) red_add_sys(&a.psel[q]->nan_count, s_nnan);
    } else {
      atomicAdd(&sel->nan_count, s_nnan);
    }
  }
#pragma unroll 1
  for (int j = npre; j < kLfDepth - 1; ++j) { need(j); issue(j); }
  for (int j = 0; j < nC; ++j) {
    cp_wait_lf2();
    __syncwarp();
    need(j + kLfDepth - 1);
    issue(j + kLfDepth - 1);
    float pa, pb;
    lf_tile_dot<GW>(ring + (j % kLfDepth) * Geo::slot, xf, bias, lane, sc_sel, pa, pb);
    if (tq == 0) {
      red[(j * kLfWarps + warp) * 16 + gq] = pa;
      red[(j * kLfWarps + warp) * 16 + gq + 8] = pb;
    }
    __syncwarp();
  }
  // h for the down list known so far, while its first tiles are in flight
  __syncthreads();
  make_h(0, have2 ? nD * 16 : nDA);
  c_done = true;
  float acc[GW][8][4];
#pragma unroll
  for (int u = 0; u < GW; ++u)
#pragma unroll
    for (int m = 0; m < 8; ++m) acc[u][m][0] = acc[u][m][1] = acc[u][m][2] = acc[u][m][3] = 0.f;
  // B values: lane l computes group ub = l / 16 (GW == 2; lanes 0-15 when
  // GW == 1), channel pair l & 7, hi or lo part (l / 8) & 1, so both groups'
  // values come from one pass of the whole warp
  float colsum = 0.f;
  // The down operands B = h s 2^p run in fp16 hi + lo parts (22 bits).  2^p
  // is this warp's: set from the first tile's max |h s| so that it lands in
  // [2^13, 2^14); a later tile that would pass 2^15 lowers it, and the
  // accumulators and column sums are rescaled by the same exact power of two.
  float dsc = 0.f;  // 2^p; 0 = not set yet
  const int tpair = lane & 7, twhich = (lane >> 3) & 1, ub = (GW == 2) ? (lane >> 4) : 0;
  for (int j = nC; j < nC + nD; ++j) {
    cp_wait_lf2();
    __syncwarp();
    need(j + kLfDepth - 1);
    issue(j + kLfDepth - 1);
    const uint8_t* slot = ring + (j % kLfDepth) * Geo::slot;
    const int i = j - nC;
    uint32_t bval = 0;
    float hs2[2] = {0.f, 0.f}, hmx = 0.f;
    if (GW == 2 || lane < 16) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int c = 2 * tpair + e;
        const uint16_t* sp = reinterpret_cast<const uint16_t*>(slot + 16 * kLfDnPitch + c * 4);
        const int sidx = (GW == 1) ? (warp & 1) : ub;
        hs2[e] = dh[i * 16 + c] * bf16_bits_to_f32(sp[sidx]);
      }
      hmx = fmaxf(fabsf(hs2[0]), fabsf(hs2[1]));
    }
    // this tile's max |h s| (warp-uniform) and the scale decision
    hmx = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(hmx)));
    if (hmx > 0.f && hmx <= 3.0e38f && (dsc == 0.f || hmx * dsc >= 32768.f)) {
      int e;
      frexpf(hmx, &e);
      const float nsc = ldexpf(1.f, max(-120, min(120, 14 - e)));
      if (dsc != 0.f) {  // lower the scale: rescale what is accumulated
        const float d = nsc / dsc;
#pragma unroll
        for (int u = 0; u < GW; ++u)
#pragma unroll
          for (int m = 0; m < 8; ++m)
#pragma unroll
            for (int t = 0; t < 4; ++t) acc[u][m][t] *= d;
        colsum *= d;
      }
      dsc = nsc;
    }
    if (GW == 2 || lane < 16) {
      // B = h s 2^p as fp16 hi + lo
      float v2[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float hs = hs2[e] * dsc;
        const float h1 = __half2float(__float2half_rn(hs));
        v2[e] = twhich ? __half2float(__float2half_rn(hs - h1)) : h1;
      }
      colsum += v2[0] + v2[1];
      const __half2 p2 = __floats2half2_rn(v2[0], v2[1]);
      bval = *reinterpret_cast<const uint32_t*>(&p2);
    }
#pragma unroll
    for (int u = 0; u < GW; ++u) {
      const int src = (gq & 1) * 8 + 16 * u;
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
        // rows gq (a[0], a[2]): exact q; rows gq + 8 (a[1], a[3]): 16 (q + 72)
        uint32_t xa[4], xc[4];
        nib8_biased_f16x2(pab[q], xa);
        nib8_biased_f16x2(pcd[q], xc);
        const uint32_t a0[4] = {xa[0], xa[1], xc[0], xc[1]};
        const uint32_t a1[4] = {xa[2], xa[3], xc[2], xc[3]};
        mma_f16_16816(acc[u][2 * q], a0, b0, b1);
        mma_f16_16816(acc[u][2 * q + 1], a1, b0, b1);
      }
    }
    __syncwarp();
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");
  const float dsc_inv = dsc != 0.f ? 1.f / dsc : 1.f;  // exact: a power of two
#pragma unroll
  for (int u = 0; u < GW; ++u) {
    float cs = colsum;
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) cs += __shfl_xor_sync(0xffffffffu, cs, o);
    const float bias_d = kNibbleBias16Hi * __shfl_sync(0xffffffffu, cs, 16 * u);
    if (tq == 0) {
      float* dst = a.partial + (size_t)b * H + (warp * GW + u) * kGroup + gq * 16;
      float v[16];
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        v[2 * m] = (acc[u][m][0] + acc[u][m][1]) * dsc_inv;
        v[2 * m + 1] = ((acc[u][m][2] + acc[u][m][3]) * 0.0625f - bias_d) * dsc_inv;
      }
#pragma unroll
      for (int q = 0; q < 4; ++q)
        reinterpret_cast<float4*>(dst)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
  }
  // The next layer's first gate tiles of this worker's rows go to L2 now:
  // DRAM is mostly idle while the slowest workers finish and during the
  // final barrier and reduction, and the next launch's first tiles then
  // come from L2 (one bulk prefetch per range, issued by one thread).
  // A bulk prefetch needs a 16-byte aligned start and a multiple of 16
  // bytes: packed rows are (hidden / 2 is a multiple of 64), but a scale
  // row is hidden / 64 bytes (40 at hidden 2560), so the scale range is
  // widened to 16-byte boundaries and clamped to the scale tensor, whose
  // size (inter * hidden / 64, inter a multiple of 8) is a multiple of 16.
  if (a.pf_qw && tid == 0) {
    const int nr = min(na, 16 * kLfPfTiles);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(a.pf_qw + (size_t)ra0 * rowb),
                 "r"(nr * rowb) : "memory");
    const size_t s_end = (size_t)I * scw * 2;
    const size_t s0 = ((size_t)ra0 * scw * 2) & ~size_t(15);
    const size_t s1 = min(s_end, ((size_t)(ra0 + nr) * scw * 2 + 15) & ~size_t(15));
    if (s1 > s0)
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n"
                   ::"l"(reinterpret_cast<const uint8_t*>(a.pf_sc) + s0), "r"((unsigned)(s1 - s0))
                   : "memory");
  }
  }  // worker
  pdl_launch_dependents();
  lf_final_barrier(&sel->done, a.err);

  // ------------------------------------------------------------ phase E
  // y[4q .. 4q+3] for this CTA's quads (at most 10): two warps per quad, lane
  // l of the pair sums workers 1 + l, 1 + l + 64, ...; then a fixed shuffle
  // tree and the pair's sum.
  {
    float* red = reinterpret_cast<float*>(smem + Geo::red);
    const int n4 = H >> 2;
    const int q0 = n4 * b / nb, q1 = n4 * (b + 1) / nb;
    const int nq = q1 - q0;  // <= 10 (checked on the host)
    const int q = warp >> 1, l64 = (warp & 1) * 32 + lane;
    float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (q < nq) {
      float4 v[3];  // nb <= 160: at most 3 partial rows per lane, loaded together
#pragma unroll
      for (int u = 0; u < 3; ++u) {
        const int c = 1 + l64 + 64 * u;
        v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (c < nb)
          asm volatile("ld.global.cg.v4.f32 {%0,%1,%2,%3}, [%4];\n"
                       : "=f"(v[u].x), "=f"(v[u].y), "=f"(v[u].z), "=f"(v[u].w)
                       : "l"(a.partial + (size_t)c * H + 4 * (q0 + q)));
      }
#pragma unroll
      for (int u = 0; u < 3; ++u) { s4.x += v[u].x; s4.y += v[u].y; s4.z += v[u].z; s4.w += v[u].w; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s4.x += __shfl_xor_sync(0xffffffffu, s4.x, o);
      s4.y += __shfl_xor_sync(0xffffffffu, s4.y, o);
      s4.z += __shfl_xor_sync(0xffffffffu, s4.z, o);
      s4.w += __shfl_xor_sync(0xffffffffu, s4.w, o);
    }
    float4* e4 = reinterpret_cast<float4*>(red);
    if (lane == 0 && (warp & 1)) e4[q] = s4;
    __syncthreads();
    const bool owner = lane == 0 && !(warp & 1) && q < nq;
    if (owner) {
      const float4 o4 = e4[q];
      s4.x += o4.x; s4.y += o4.y; s4.z += o4.z; s4.w += o4.w;
    }
    if (TP) {
      // This rank's partial sums of the CTA's quads go to slot `rank` of
      // every rank's y slots (plain 16-byte stores over NVLink), then one
      // tagged flag per rank; CTA b of every rank owns the same quads, so it
      // waits for the flags of CTA b of every rank and sums the slots in rank
      // order: y is identical on every rank.
      const int o = 4 * (q0 + q);
      if (owner)
        for (int r = 0; r < a.world; ++r)
          *reinterpret_cast<float4*>(a.pysl[r] + (size_t)rank * H + o) = s4;
      __syncthreads();
      if (tid == 0) {
        const unsigned long long tag = s_tag;
        asm volatile("fence.acq_rel.sys;\n" ::: "memory");
        for (int r = 0; r < a.world; ++r)
          st_relaxed_sys_u64(a.pyflag[r] + (size_t)rank * kLfMaxCtas + b, tag);
        const unsigned long long* mine = a.pyflag[rank];
        bool ok = true;
        for (int r = 0; r < a.world && ok; ++r) {
          ok = false;
          for (uint32_t it = 0, lim = spin_limit(a.err); it < lim && !ok; ++it)
            ok = ld_acquire_sys_u64(mine + (size_t)r * kLfMaxCtas + b) == tag;
        }
        if (!ok) atomicOr(a.err, kErrTimeout);
      }
      __syncthreads();
      if (owner) {
        const float* ys = a.pysl[rank];
        s4 = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < a.world; ++r) {
          float4 v;
          asm volatile("ld.relaxed.sys.global.v4.f32 {%0,%1,%2,%3}, [%4];\n"
                       : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                       : "l"(ys + (size_t)r * H + o) : "memory");
          s4.x += v.x; s4.y += v.y; s4.z += v.z; s4.w += v.w;
        }
      }
    }
    if (owner) {
      const int o = 4 * (q0 + q);
      if (a.y) {
        a.y[o] = f32_to_bf16_bits(s4.x); a.y[o + 1] = f32_to_bf16_bits(s4.y);
        a.y[o + 2] = f32_to_bf16_bits(s4.z); a.y[o + 3] = f32_to_bf16_bits(s4.w);
      }
      if (a.y_f32) *reinterpret_cast<float4*>(a.y_f32 + o) = s4;
    }
  }
}

constexpr size_t kLfSelBytes = (sizeof(LfSel) + 255) & ~size_t(255);

// Workspace layout (byte offsets).  The single-GPU workspace is the prefix up
// to `ysl`; the tensor-parallel one adds the y slots and y flags that the
// peers write into.
struct LfLayout {
  size_t bar, g, idx, part, ysl, yflag, single_total, tp_total;
};
static size_t lf_al(size_t v) { return (v + 255) & ~size_t(255); }
static LfLayout lf_layout(int64_t hidden, int64_t inter, int64_t k) {
  LfLayout L;
  L.bar = kLfSelBytes;
  L.g = L.bar + 256;
  L.idx = L.g + lf_al((size_t)inter * 2);
  L.part = L.idx + lf_al((size_t)k * 4);
  L.ysl = L.part + (size_t)kLfMaxCtas * hidden * 4;  // device independent: up to 160 SMs
  L.single_total = L.ysl;
  L.yflag = L.ysl + lf_al((size_t)kLfMaxRanks * hidden * 4);
  L.tp_total = L.yflag + lf_al((size_t)kLfMaxRanks * kLfMaxCtas * 8);
  return L;
}

}  // namespace dip

namespace dip {
template <int GW, bool CA, bool TP>
static int lf_launch(const LfArgs& a, int nb, dip_stream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(layer_fused_kernel<GW, CA, TP>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       LfGeom<GW>::total);
  if (e != cudaSuccess) return launch_status(e);
  return launch_status(launch_coop(layer_fused_kernel<GW, CA, TP>, dim3(nb), dim3(kLfThreads),
                                   (size_t)LfGeom<GW>::total, (cudaStream_t)stream, a));
}

// Shape checks shared by the entry points; returns 0 and the K-slice width
// (GW) or a status.  I: rows on this GPU, IT: all channels.
static int lf_check_shape(int64_t H, int64_t I, int64_t IT, int64_t k, int nb, int* gw_out) {
  if (k < 1 || k > IT || H <= 0 || I <= 0) return DIP_ERR_ARG;
  if (nb > kLfMaxCtas) return DIP_ERR_UNSUPPORTED;
  const int G = (int)(H / kGroup);
  int gw = 0;
  if (H % kGroup == 0 && G == kLfWarps * 1) gw = 1;
  if (H % kGroup == 0 && G == kLfWarps * 2) gw = 2;
  if (!gw || I % 8 != 0) return DIP_ERR_UNSUPPORTED;
  // per-worker limits (CTA 0 coordinates): gate rows <= 16*kLfTilesA - 1
  // (C list: rows plus one padding entry, in at most kLfTilesA + 1 tiles)
  if (nb < 2 || (I + nb - 2) / (nb - 1) > 16 * kLfTilesA - 1 || IT * (int64_t)nb >= (int64_t(1) << 31) ||
      (H / 4 + nb - 1) / nb > kLfWarps / 2 ||
      (int64_t)16 * kLfTilesA * k >= (int64_t(1) << 31))
    return DIP_ERR_UNSUPPORTED;
  *gw_out = gw;
  return DIP_OK;
}

// Optional extras of a call; false if they are malformed.
static bool lf_apply_opts(LfArgs& a, const dip_fused_opts_t* o) {
  if (!o) return true;
  a.h_out = o->h_out;
  if ((o->prefetch_gate_qw == nullptr) != (o->prefetch_gate_sc == nullptr)) return false;
  if ((reinterpret_cast<uintptr_t>(o->prefetch_gate_qw) |
       reinterpret_cast<uintptr_t>(o->prefetch_gate_sc)) & 15)
    return false;
  a.pf_qw = reinterpret_cast<const uint8_t*>(o->prefetch_gate_qw);
  a.pf_sc = o->prefetch_gate_sc;
  return true;
}

static void lf_fill_common(LfArgs& a, const dip_layer_t* L, uint8_t* ws, const LfLayout& lay,
                           const dip_bf16* x, const dip_bf16* resid, float eps, int64_t k,
                           dip_bf16* y, dip_bf16* g_out, int32_t* idx_out, dip_bf16* x_used) {
  a.scratch = reinterpret_cast<unsigned*>(ws);
  a.bar = reinterpret_cast<GridBar*>(ws + lay.bar);
  a.g = g_out ? g_out : reinterpret_cast<uint16_t*>(ws + lay.g);
  a.idx = idx_out ? idx_out : reinterpret_cast<int32_t*>(ws + lay.idx);
  a.partial = reinterpret_cast<float*>(ws + lay.part);
  a.gate_qw = reinterpret_cast<const uint8_t*>(L->gate_qw);
  a.gate_sc = L->gate_sc;
  a.up_qw = reinterpret_cast<const uint8_t*>(L->up_qw);
  a.up_sc = L->up_sc;
  a.dn_qw = reinterpret_cast<const uint8_t*>(L->down_t_qw);
  a.dn_sc = L->down_t_sc;
  a.hidden = (int)L->hidden;
  a.inter = (int)L->inter;
  a.inter_total = (int)L->inter;
  a.world = 1;
  a.k = (int)k;
  a.x = x;
  a.resid = resid;
  a.eps = eps;
  a.x_used = x_used;
  a.y = y;
}
}  // namespace dip

using namespace dip;

extern "C" size_t dip_mlp_fused_workspace_bytes(int64_t hidden, int64_t inter, int64_t k) {
  if (hidden <= 0 || inter <= 0 || k <= 0) return 0;
  return lf_layout(hidden, inter, k).single_total;
}

extern "C" size_t dip_mlp_fused_tp_workspace_bytes(int64_t hidden, int64_t inter_total, int64_t k) {
  if (hidden <= 0 || inter_total <= 0 || k <= 0) return 0;
  return lf_layout(hidden, inter_total, k).tp_total;
}

extern "C" int dip_mlp_decode_fused(const dip_layer_t* L, const dip_bf16* x, const dip_bf16* resid,
                                    float eps, int64_t k, void* workspace, size_t workspace_bytes,
                                    dip_bf16* y, dip_bf16* g_out, int32_t* idx_out,
                                    dip_bf16* x_used, dip_stream_t stream) {
  return dip_mlp_decode_fused_ca(L, nullptr, x, resid, eps, k, workspace, workspace_bytes, y, g_out,
                                 idx_out, x_used, stream);
}

extern "C" int dip_mlp_decode_fused_tp(const dip_layer_t* shard, int64_t inter_total, int rank,
                                       int world, void* const* workspaces, size_t workspace_bytes,
                                       const dip_bf16* x, const dip_bf16* resid, float eps,
                                       int64_t k, dip_bf16* y, dip_bf16* g_out, int32_t* idx_out,
                                       dip_bf16* x_used, const dip_fused_opts_t* opts,
                                       dip_stream_t stream) {
  if (!shard || !x || !y || !workspaces) return DIP_ERR_ARG;
  if (world < 1 || world > kLfMaxRanks || rank < 0 || rank >= world) return DIP_ERR_ARG;
  const int64_t H = shard->hidden, I = shard->inter;
  if (I <= 0 || inter_total != I * world) return DIP_ERR_ARG;
  const int nb = num_sms();
  int gw = 0;
  const int st = lf_check_shape(H, I, inter_total, k, nb, &gw);
  if (st) return st;
  const LfLayout lay = lf_layout(H, inter_total, k);
  if (workspace_bytes < lay.tp_total) return DIP_ERR_WORKSPACE;
  for (int q = 0; q < world; ++q) {
    if (!workspaces[q] || (reinterpret_cast<uintptr_t>(workspaces[q]) & 255)) return DIP_ERR_ARG;
    // a peer's workspace is another GPU's memory: it must be a mapping this
    // library opened (dip_ipc_open) or allocated, of at least the layout's
    // size, or the peer stores below would land outside it
    if (q != rank && p2p_registered_bytes(workspaces[q]) < lay.tp_total) return DIP_ERR_ARG;
  }
  const uintptr_t al = reinterpret_cast<uintptr_t>(shard->gate_qw) |
                       reinterpret_cast<uintptr_t>(shard->up_qw) |
                       reinterpret_cast<uintptr_t>(shard->down_t_qw) | reinterpret_cast<uintptr_t>(x) |
                       reinterpret_cast<uintptr_t>(resid) | reinterpret_cast<uintptr_t>(x_used) |
                       reinterpret_cast<uintptr_t>(g_out);
  if (al & 15) return DIP_ERR_ARG;
  LfArgs a = {};
  uint8_t* ws = static_cast<uint8_t*>(workspaces[rank]);
  lf_fill_common(a, shard, ws, lay, x, resid, eps, k, y, g_out, idx_out, x_used);
  a.idx = idx_out;  // optional: only this rank's entries are written
  if (!lf_apply_opts(a, opts)) return DIP_ERR_ARG;
  a.inter_total = (int)inter_total;
  a.rank = rank;
  a.world = world;
  a.c0 = (int)(I * rank);
  for (int q = 0; q < world; ++q) {
    uint8_t* wq = static_cast<uint8_t*>(workspaces[q]);
    a.psel[q] = reinterpret_cast<LfSel*>(wq);
    a.pysl[q] = reinterpret_cast<float*>(wq + lay.ysl);
    a.pyflag[q] = reinterpret_cast<unsigned long long*>(wq + lay.yflag);
  }
  a.err = error_word_ptr();
  if (!a.err) return DIP_ERR_CUDA;
  return gw == 1 ? lf_launch<1, false, true>(a, nb, stream) : lf_launch<2, false, true>(a, nb, stream);
}

extern "C" int dip_mlp_decode_fused_ca(const dip_layer_t* L, const dip_ca_cache_t* cache,
                                       const dip_bf16* x, const dip_bf16* resid, float eps,
                                       int64_t k, void* workspace, size_t workspace_bytes,
                                       dip_bf16* y, dip_bf16* g_out, int32_t* idx_out,
                                       dip_bf16* x_used, dip_stream_t stream) {
  return dip_mlp_decode_fused_ex(L, cache, x, resid, eps, k, workspace, workspace_bytes, y, g_out,
                                 idx_out, x_used, nullptr, stream);
}

extern "C" int dip_mlp_decode_fused_ex(const dip_layer_t* L, const dip_ca_cache_t* cache,
                                       const dip_bf16* x, const dip_bf16* resid, float eps,
                                       int64_t k, void* workspace, size_t workspace_bytes,
                                       dip_bf16* y, dip_bf16* g_out, int32_t* idx_out,
                                       dip_bf16* x_used, const dip_fused_opts_t* opts,
                                       dip_stream_t stream) {
  if (!L || !x || !y || !workspace) return DIP_ERR_ARG;
  if (cache && (!cache->id2slot || !cache->res_up_qw || !cache->res_up_sc || !cache->res_dn_qw ||
                !cache->res_dn_sc))
    return DIP_ERR_ARG;
  if (cache && ((reinterpret_cast<uintptr_t>(cache->res_up_qw) |
                 reinterpret_cast<uintptr_t>(cache->res_dn_qw)) & 15))
    return DIP_ERR_ARG;
  const int64_t H = L->hidden, I = L->inter;
  const int nb = num_sms();
  int gw = 0;
  const int st = lf_check_shape(H, I, I, k, nb, &gw);
  if (st) return st;
  const LfLayout lay = lf_layout(H, I, k);
  if (workspace_bytes < lay.single_total) return DIP_ERR_WORKSPACE;
  const uintptr_t al = reinterpret_cast<uintptr_t>(L->gate_qw) | reinterpret_cast<uintptr_t>(L->up_qw) |
                       reinterpret_cast<uintptr_t>(L->down_t_qw) | reinterpret_cast<uintptr_t>(x) |
                       reinterpret_cast<uintptr_t>(resid) | reinterpret_cast<uintptr_t>(x_used) |
                       reinterpret_cast<uintptr_t>(g_out) | reinterpret_cast<uintptr_t>(workspace);
  if (al & 15) return DIP_ERR_ARG;
  LfArgs a = {};
  lf_fill_common(a, L, static_cast<uint8_t*>(workspace), lay, x, resid, eps, k, y, g_out, idx_out,
                 x_used);
  if (!lf_apply_opts(a, opts)) return DIP_ERR_ARG;
  a.err = error_word_ptr();
  if (!a.err) return DIP_ERR_CUDA;
  if (cache) {
    a.id2slot = cache->id2slot;
    a.res_up_qw = reinterpret_cast<const uint8_t*>(cache->res_up_qw);
    a.res_up_sc = cache->res_up_sc;
    a.res_dn_qw = reinterpret_cast<const uint8_t*>(cache->res_dn_qw);
    a.res_dn_sc = cache->res_dn_sc;
  }
  const bool ca = cache != nullptr;
  if (gw == 1)
    return ca ? lf_launch<1, true, false>(a, nb, stream) : lf_launch<1, false, false>(a, nb, stream);
  return ca ? lf_launch<2, true, false>(a, nb, stream) : lf_launch<2, false, false>(a, nb, stream);
}
