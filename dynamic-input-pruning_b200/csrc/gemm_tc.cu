// gemm_tc.cu — int4 (g128) weight x bf16 activation GEMMs on the 5th-generation
// tensor cores (tcgen05, accumulators in TMEM), for the batched decode layer
// (B independent tokens per step) and the dense QuantLinear forward.
//
// Per token the math is the reference's pure-PyTorch DIP path
// (dip_stream_predispatch.py:176-204 with qlinear.py:28-64's dequantise):
// every weight is dequantised to bf16(q * s) exactly as dequantize() does, the
// products are accumulated in fp32 on the tensor cores, and the epilogues
// round where the reference's bf16 tensors round:
//   gate   g = bf16(silu(bf16(W_gate x)))
//   up     h = bf16(g * bf16(W_up x)) for the token's selected channels, 0 elsewhere
//   down   y = bf16(sum_c h_c W_down_t[c])      (split over channels, fixed-order sum)
//
// Kernel structure (one CTA per SM, persistent over work units):
//   warps 0-7  producers: each thread streams 16 bytes of packed int4 per
//              K-step through a private cp.async ring (12 steps deep), turns
//              them into bf16(q * s) and stores them into the A operand stage
//              in the 128-byte-swizzled layout the MMA reads; then the
//              epilogue (tcgen05.ld of the fp32 accumulator).
//   warp 8     lane 0 issues tcgen05.mma (M = 128 weight rows, N = the padded
//              token count, K = 16) four per K-step, and tcgen05.commit to the
//              stage's "empty" barrier and, at the end of a unit, to the
//              accumulator's "full" barrier.
//   warp 9     copies the activation tile (B operand, bf16 [N][64] per step,
//              rows past the batch zero-filled) into the stage.
// Stages are handed over with mbarriers (full: one arrival per producer warp
// and one from the loader, after each lane's proxy fence;
// empty: the MMA commit).  Every wait is bounded: on timeout the kernel flags
// the library's error word, skips ahead and still frees its TMEM.
//
// Two A layouts:
//   rows   (gate, up, QuantLinear): W [R, K/2] as scripts/quantize.py packs it,
//          one scale per row and 128 K; A tile K-major.
//   trans  (down): W_down_t [K = inter, R = hidden / 2] (the transposed down of
//          _transpose_down_to_int4), one scale per K row and 128 outputs; A
//          tile MN-major, so each thread dequantises 32 consecutive outputs of
//          one channel row and no transposition is needed.
#include "dip_common.cuh"

namespace dip {


constexpr int kTcM = 128;        // weight rows (outputs) per tile = MMA M
constexpr int kTcK = 64;         // K per pipeline step (4 MMAs of K = 16)
constexpr int kTcStages = 4;     // A / B operand stages
constexpr int kTcRaw = 12;       // trans: raw int4 ring depth per producer thread (steps)
constexpr int kTcChunkK = 256;   // rows: K per raw chunk (one 128-byte line per row)
constexpr int kTcRawC = 5;       // rows: raw chunk ring depth per producer warp
constexpr int kTcProd = 256;     // producer threads (warps 0-7)
constexpr int kTcThreads = 320;  // + MMA warp + activation loader warp
constexpr int kTcMaxN = 128;     // padded tokens per launch

enum TcEpi : int { kTcEpiBf16 = 0, kTcEpiSilu = 1, kTcEpiH = 2, kTcEpiF32 = 3 };

struct TcArgs {
  const uint8_t* w;   // rows: [R, K/2]; trans: [K, R/2]
  const uint16_t* s;  // rows: [R, K/128]; trans: [K, R/128]
  const uint16_t* x;  // [B, K] activations (B operand), row stride K
  int R, K, B;
  int ksplit;         // K ranges per tile (their fp32 partials are summed by tc_reduce_kernel)
  int kgran;          // K steps a range is a multiple of (rows: one raw chunk)
  uint16_t* out;      // [B, R] bf16 (kTcEpiBf16 / Silu / H)
  float* out_f32;     // kTcEpiF32: [ksplit][B][R] partial sums
  const uint16_t* g;  // kTcEpiH: [B, R] gate activations
  const uint32_t* cnt;  // kTcEpiH: [B, R] times each channel is selected (0 = not)
  unsigned* err;
};

// Shared memory map (dynamic, 1024-byte aligned base).
template <int NT>
struct TcSmem {
  static constexpr int a_stage = kTcM * kTcK * 2;           // 16 KB bf16
  static constexpr int b_stage = NT * kTcK * 2;             // NT x 128 B
  static constexpr int a = 0;
  static constexpr int b = a + kTcStages * a_stage;
  static constexpr int raw = b + kTcStages * b_stage;
  // trans: [kTcRaw][kTcProd] x (16 B of weights), then x 4 B of scale words
  static constexpr int raw_t = kTcRaw * kTcProd * 20;
  // rows: per producer warp [kTcRawC] x (16 rows x 128 B + 16 x 4 B of scale words)
  static constexpr int wslot = 16 * 128 + 16 * 4;
  static constexpr int raw_r = 8 * kTcRawC * wslot;
  static constexpr int rsc = raw + kTcRaw * kTcProd * 16;   // trans scale words
  static constexpr int bars = raw + (raw_t > raw_r ? raw_t : raw_r);  // full[S], empty[S], accf, acce
  static constexpr int tmem_slot = bars + (2 * kTcStages + 2) * 8;
  static constexpr int total = tmem_slot + 16 + 1024;       // + alignment slack
  static_assert(b_stage % 1024 == 0, "B stages keep the 1024-byte swizzle alignment");
};

__device__ __forceinline__ void cp_async16_zfill(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async4_tc(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_commit_tc() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait_tc() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}

// Shared memory matrix descriptor, 128-byte swizzle (sm_100 format: start >> 4
// in bits 0-13, leading byte offset >> 4 in 16-29, stride byte offset >> 4 in
// 32-45, version 1 in 46-47, layout type 2 = SWIZZLE_128B in 61-63).
__device__ __forceinline__ uint64_t tc_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor, kind::f16: fp32 accumulator, bf16 A and B, B K-major,
// A K-major (a_mn = false) or MN-major, N = n, M = 128.
__host__ __device__ constexpr uint32_t tc_idesc(int n, bool a_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kTcM >> 4) << 24);
}
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// 32 lanes x 16 consecutive fp32 columns of the accumulator (this warp's lane quadrant).
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Eight packed nibbles (low nibble = lower K index) -> four bf16x2 words
// holding bf16(q * s) for K positions (0,1) (2,3) (4,5) (6,7): q + 136 by the
// magic-number LOP3, - 136 exactly, then one bf16 multiply (the single
// rounding of dequantize()'s q * s -> bf16).
__device__ __forceinline__ uint4 tc_dequant8(uint32_t w, __nv_bfloat162 s2) {
  uint32_t o[4];
  nib8_biased_bf16x2(w, o);  // o[j] = (k_j, k_{j+4}) biased by 136
  const uint32_t p0 = __byte_perm(o[0], o[1], 0x5410), p1 = __byte_perm(o[2], o[3], 0x5410);
  const uint32_t p2 = __byte_perm(o[0], o[1], 0x7632), p3 = __byte_perm(o[2], o[3], 0x7632);
  const __nv_bfloat162 bias = __float2bfloat162_rn(136.f);
  uint32_t q[4] = {p0, p1, p2, p3};
  uint4 r;
  uint32_t* rr = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&q[i]);
    v = __hmul2(__hsub2(v, bias), s2);
    rr[i] = *reinterpret_cast<uint32_t*>(&v);
  }
  return r;
}

// As tc_dequant8 but leaving the eight K positions in the order the nibble
// extraction yields them, (0,4) (1,5) (2,6) (3,7): the activations are given
// to the MMA with the same order inside every 8-element group (a permutation
// of the summation index), which saves the four byte permutes.
__device__ __forceinline__ uint4 tc_dequant8_k8perm(uint32_t w, __nv_bfloat162 s2) {
  uint32_t o[4];
  nib8_biased_bf16x2(w, o);
  const __nv_bfloat162 bias = __float2bfloat162_rn(136.f);
  uint4 r;
  uint32_t* rr = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&o[i]);
    v = __hmul2(__hsub2(v, bias), s2);
    rr[i] = *reinterpret_cast<uint32_t*>(&v);
  }
  return r;
}

// x [B, K] -> the same values with each 8-element group in the order
// (0,4,1,5,2,6,3,7), the order tc_dequant8_k8perm leaves the weights in.
__global__ void tc_permute_k8_kernel(const uint4* __restrict__ x, int64_t n16, uint4* __restrict__ xp) {
  pdl_wait();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n16;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 v = x[i];
    xp[i] = make_uint4(__byte_perm(v.x, v.z, 0x5410), __byte_perm(v.x, v.z, 0x7632),
                       __byte_perm(v.y, v.w, 0x5410), __byte_perm(v.y, v.w, 0x7632));
  }
}

// Work unit u of this launch -> (tile, k range); steps of kTcK.
struct TcUnit {
  int tile, k0, nsteps;
};
__device__ __forceinline__ TcUnit tc_unit(const TcArgs& a, int u) {
  const int kunits = a.K / (kTcK * a.kgran);
  const int tile = u / a.ksplit, part = u % a.ksplit;
  const int s0 = (int)((int64_t)kunits * part / a.ksplit) * a.kgran;
  const int s1 = (int)((int64_t)kunits * (part + 1) / a.ksplit) * a.kgran;
  return {tile, s0 * kTcK, s1 - s0};
}

template <int NT, int EPI, bool TRANS>
__global__ void __launch_bounds__(kTcThreads, 1) gemm_tc_kernel(const TcArgs a) {
  using Sm = TcSmem<NT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Sm::bars);
  uint64_t* empty = full + kTcStages;
  uint64_t* accf = empty + kTcStages;
  uint64_t* acce = accf + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Sm::tmem_slot);
  constexpr uint32_t kCols = NT < 32 ? 32 : NT;  // power of two >= 32

  const int ntile = (a.R + kTcM - 1) / kTcM;
  const int nunits = ntile * a.ksplit;
  // this CTA's units: u = blockIdx.x + j * gridDim.x; its steps run back to back
  int nsteps_total = 0;
  for (int u = blockIdx.x; u < nunits; u += gridDim.x) nsteps_total += tc_unit(a, u).nsteps;

  if (tid == 0) {
    for (int i = 0; i < kTcStages; ++i) {
      mbar_init(&full[i], 8 + 1);  // one arrival per producer warp + the loader warp
      mbar_init(&empty[i], 1);
    }
    mbar_init(accf, 1);
    mbar_init(acce, 8);
    mbar_fence_init();
  }
  if (warp == 8) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // After one wait times out (error word flagged) this thread skips every
  // later wait, so a broken pipeline ends in bounded time.
  bool dead = false;
  auto wait = [&](uint64_t* bar, uint32_t parity) {
    if (dead) return;
    for (uint32_t i = 0; i < (1u << 20); ++i)
      if (mbar_try_wait(bar, parity)) return;
    atomicOr(a.err, kErrTimeout);
    dead = true;
  };

  if (warp < 8 && !TRANS) {
    // ------------------------------------------------------------ producers (rows)
    // Warp w streams rows [16w, 16w + 16) of the tile in raw chunks of 256 K
    // (one whole 128-byte line per row: lane l copies row l/2's 64-byte half
    // l&1, lanes 0-15 the rows' scale words) through a kTcRawC-deep ring; per
    // K step (64) lane l dequantises 16 bytes of row l/2 (K half l&1).
    uint8_t* wring = smem + Sm::raw + warp * kTcRawC * Sm::wslot;
    constexpr int kStepsPerChunk = kTcChunkK / kTcK;
    const int nchunks_total = nsteps_total / kStepsPerChunk;
    int iu = blockIdx.x, ic = 0;
    TcUnit iun = iu < nunits ? tc_unit(a, iu) : TcUnit{0, 0, 0};
    auto issue_chunk = [&](int gc) {
      if (gc < nchunks_total) {
        while (ic >= iun.nsteps / kStepsPerChunk) { iu += gridDim.x; iun = tc_unit(a, iu); ic = 0; }
        const int cidx = iun.k0 / kTcChunkK + ic;  // chunk of the row
        const int row = min(iun.tile * kTcM + warp * 16 + (lane >> 1), a.R - 1);
        uint8_t* slot = wring + (gc % kTcRawC) * Sm::wslot;
        const uint8_t* src = a.w + (size_t)row * (a.K / 2) + (size_t)cidx * 128 + (lane & 1) * 64;
#pragma unroll
        for (int i = 0; i < 4; ++i)
          cp_async16_zfill(slot + (lane >> 1) * 128 + (lane & 1) * 64 + i * 16, src + i * 16, true);
        if (lane < 16) {
          const int srow = min(iun.tile * kTcM + warp * 16 + lane, a.R - 1);
          cp_async4_tc(slot + 16 * 128 + lane * 4, a.s + (size_t)srow * (a.K / 128) + cidx * 2);
        }
        ++ic;
      }
      cp_commit_tc();
    };
#pragma unroll 1
    for (int gc = 0; gc < kTcRawC - 1; ++gc) issue_chunk(gc);  // weights: static, before the PDL wait
    pdl_wait();

    int cu = blockIdx.x, cs = 0, unit_idx = 0;
    TcUnit cun = cu < nunits ? tc_unit(a, cu) : TcUnit{0, 0, 0};
#pragma unroll 1
    for (int q = 0; q < nsteps_total; ++q) {
      while (cs >= cun.nsteps) { cu += gridDim.x; cun = tc_unit(a, cu); cs = 0; ++unit_idx; }
      const int gc = q / (kTcChunkK / kTcK), s4 = q % (kTcChunkK / kTcK);
      if (s4 == 0) {
        __syncwarp();  // every lane is done with the slot the next chunk reuses
        issue_chunk(gc + kTcRawC - 1);
        cp_wait_tc<kTcRawC - 1>();
        __syncwarp();
      }
      const uint8_t* slot = wring + (gc % kTcRawC) * Sm::wslot;
      const uint4 raw = *reinterpret_cast<const uint4*>(slot + (lane >> 1) * 128 + s4 * 32 + (lane & 1) * 16);
      const uint32_t sw = *reinterpret_cast<const uint32_t*>(slot + 16 * 128 + (lane >> 1) * 4);
      const uint16_t sbits = (uint16_t)((s4 >> 1) ? (sw >> 16) : (sw & 0xFFFFu));
      const __nv_bfloat162 s2 = __halves2bfloat162(__ushort_as_bfloat16(sbits), __ushort_as_bfloat16(sbits));
      const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
      const int st = q % kTcStages;
      if (q >= kTcStages) wait(&empty[st], (uint32_t)((q / kTcStages) - 1) & 1u);
      uint8_t* A = smem + Sm::a + st * Sm::a_stage;
      const int r = warp * 16 + (lane >> 1);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 v = tc_dequant8_k8perm(wv[i], s2);
        // K-major SW128: row r, 16-byte chunk j (8 K) -> (r/8)*1024 + (r%8)*128 + (j ^ r%8)*16
        const int j = (lane & 1) * 4 + i;
        *reinterpret_cast<uint4*>(A + (r >> 3) * 1024 + (r & 7) * 128 + ((j ^ (r & 7)) << 4)) = v;
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[st]);
      ++cs;
      if (cs == cun.nsteps) {
        // ------------------------------------------------ epilogue of this unit
        wait(accf, (uint32_t)unit_idx & 1u);
        tc_fence_after();
        const int quad = warp & 3, half = warp >> 2;
        const int row = cun.tile * kTcM + quad * 32 + lane;
        constexpr int kHalfN = NT / 2;
        const uint32_t tbase = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(half * kHalfN);
#pragma unroll
        for (int c0 = 0; c0 < kHalfN; c0 += 16) {
          float v[16];
          if (kHalfN - c0 >= 16) {
            tc_ld16(tbase + c0, v);
          } else {
            // NT == 16: 8 columns per half; load 16 and use the first 8
            // (columns past NT are allocated, kCols >= 32)
            tc_ld16(tbase + c0, v);
          }
          // EPI_H: the block's g and selection counts, loaded together
          uint16_t gv[16];
          uint32_t cv[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int n = half * kHalfN + c0 + i;
            const bool ok = EPI == kTcEpiH && c0 + i < kHalfN && n < a.B && row < a.R;
            gv[i] = ok ? a.g[(size_t)n * a.R + row] : (uint16_t)0;
            cv[i] = ok ? a.cnt[(size_t)n * a.R + row] : 0u;
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int n = half * kHalfN + c0 + i;
            if (c0 + i >= kHalfN || n >= a.B || row >= a.R) continue;
            const size_t o = (size_t)n * a.R + row;
            if (EPI == kTcEpiF32) {
              a.out_f32[((size_t)(cu % a.ksplit) * a.B + n) * a.R + row] = v[i];
            } else if (EPI == kTcEpiSilu) {
              a.out[o] = f32_to_bf16_bits(silu_f32(round_bf16(v[i])));
            } else if (EPI == kTcEpiH) {
              const uint32_t c = cv[i];
              float h = 0.f;
              if (c) h = round_bf16(bf16_bits_to_f32(gv[i]) * round_bf16(v[i])) * (float)c;
              a.out[o] = f32_to_bf16_bits(h);
            } else {
              a.out[o] = f32_to_bf16_bits(v[i]);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acce);
      }
    }
    cp_wait_tc<0>();
  } else if (warp < 8 && TRANS) {
    // ------------------------------------------------------------ producers
    // Thread -> its 16 bytes of a step.  rows: row t/2, K half t&1 (32 K).
    // trans: K row t/4 (of 64), output quarter t&3 (32 outputs).
    const int t = tid;
    auto src_of = [&](int step_unit_tile, int kpos, const uint8_t*& q, const uint16_t*& sc) {
      if (!TRANS) {
        const int row = min(step_unit_tile * kTcM + (t >> 1), a.R - 1);
        q = a.w + (size_t)row * (a.K / 2) + kpos / 2 + (t & 1) * 16;
        sc = a.s + (size_t)row * (a.K / 128) + ((kpos / 128) & ~1);
      } else {
        const int krow = kpos + (t >> 2);
        const int col = step_unit_tile * kTcM + (t & 3) * 32;
        q = a.w + (size_t)krow * (a.R / 2) + col / 2;
        sc = a.s + (size_t)krow * (a.R / 128) + (((step_unit_tile * kTcM) / 128) & ~1);
      }
    };
    // step iterator for the issue side (runs kTcRaw - 1 steps ahead)
    int iu = blockIdx.x, is = 0;
    TcUnit iun = iu < nunits ? tc_unit(a, iu) : TcUnit{0, 0, 0};
    auto issue_next = [&](int q) {
      if (q < nsteps_total) {
        while (is >= iun.nsteps) { iu += gridDim.x; iun = tc_unit(a, iu); is = 0; }
        const uint8_t* qp;
        const uint16_t* sp;
        src_of(iun.tile, iun.k0 + is * kTcK, qp, sp);
        const int slot = q % kTcRaw;
        cp_async16_zfill(smem + Sm::raw + (slot * kTcProd + t) * 16, qp, true);
        cp_async4_tc(smem + Sm::rsc + (slot * kTcProd + t) * 4, sp);
        ++is;
      }
      cp_commit_tc();
    };
#pragma unroll 1
    for (int q = 0; q < kTcRaw - 1; ++q) issue_next(q);  // weights: static, before the PDL wait
    pdl_wait();

    int cu = blockIdx.x, cs = 0, unit_idx = 0;
    TcUnit cun = cu < nunits ? tc_unit(a, cu) : TcUnit{0, 0, 0};
#pragma unroll 1
    for (int q = 0; q < nsteps_total; ++q) {
      while (cs >= cun.nsteps) { cu += gridDim.x; cun = tc_unit(a, cu); cs = 0; ++unit_idx; }
      issue_next(q + kTcRaw - 1);
      cp_wait_tc<kTcRaw - 1>();
      const int slot = q % kTcRaw;
      const uint4 raw = *reinterpret_cast<const uint4*>(smem + Sm::raw + (slot * kTcProd + t) * 16);
      const uint32_t sw = *reinterpret_cast<const uint32_t*>(smem + Sm::rsc + (slot * kTcProd + t) * 4);
      const int kpos = cun.k0 + cs * kTcK;
      uint16_t sbits;
      if (!TRANS) sbits = (uint16_t)(((kpos / 128) & 1) ? (sw >> 16) : (sw & 0xFFFFu));
      else sbits = (uint16_t)((((cun.tile * kTcM) / 128) & 1) ? (sw >> 16) : (sw & 0xFFFFu));
      const __nv_bfloat162 s2 = __halves2bfloat162(__ushort_as_bfloat16(sbits), __ushort_as_bfloat16(sbits));
      const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
      const int st = q % kTcStages;
      if (q >= kTcStages) wait(&empty[st], (uint32_t)((q / kTcStages) - 1) & 1u);
      uint8_t* A = smem + Sm::a + st * Sm::a_stage;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 v = tc_dequant8(wv[i], s2);
        uint32_t off;
        if (!TRANS) {
          // K-major SW128: row r, 16-byte chunk j (8 K) -> (r/8)*1024 + (r%8)*128 + (j ^ r%8)*16
          const int r = t >> 1, j = (t & 1) * 4 + i;
          off = (r >> 3) * 1024 + (r & 7) * 128 + ((j ^ (r & 7)) << 4);
        } else {
          // MN-major SW128: K row kr, 16-byte chunk of 8 outputs m8 (0..15):
          // K block kr/8 (stride 2048), M block m8/8 (stride 1024), row kr%8
          // (128 B), chunk (m8%8) ^ (kr%8)
          const int kr = t >> 2, m8 = (t & 3) * 4 + i;
          off = (kr >> 3) * 2048 + (m8 >> 3) * 1024 + (kr & 7) * 128 + (((m8 & 7) ^ (kr & 7)) << 4);
        }
        *reinterpret_cast<uint4*>(A + off) = v;
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[st]);
      ++cs;
      if (cs == cun.nsteps) {
        // ------------------------------------------------ epilogue of this unit
        wait(accf, (uint32_t)unit_idx & 1u);
        tc_fence_after();
        const int quad = warp & 3, half = warp >> 2;
        const int row = cun.tile * kTcM + quad * 32 + lane;
        constexpr int kHalfN = NT / 2;
        const uint32_t tbase = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(half * kHalfN);
#pragma unroll
        for (int c0 = 0; c0 < kHalfN; c0 += 16) {
          float v[16];
          if (kHalfN - c0 >= 16) {
            tc_ld16(tbase + c0, v);
          } else {
            // NT == 16: 8 columns per half; load 16 and use the first 8
            // (columns past NT are allocated, kCols >= 32)
            tc_ld16(tbase + c0, v);
          }
          // EPI_H: the block's g and selection counts, loaded together
          uint16_t gv[16];
          uint32_t cv[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int n = half * kHalfN + c0 + i;
            const bool ok = EPI == kTcEpiH && c0 + i < kHalfN && n < a.B && row < a.R;
            gv[i] = ok ? a.g[(size_t)n * a.R + row] : (uint16_t)0;
            cv[i] = ok ? a.cnt[(size_t)n * a.R + row] : 0u;
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int n = half * kHalfN + c0 + i;
            if (c0 + i >= kHalfN || n >= a.B || row >= a.R) continue;
            const size_t o = (size_t)n * a.R + row;
            if (EPI == kTcEpiF32) {
              a.out_f32[((size_t)(cu % a.ksplit) * a.B + n) * a.R + row] = v[i];
            } else if (EPI == kTcEpiSilu) {
              a.out[o] = f32_to_bf16_bits(silu_f32(round_bf16(v[i])));
            } else if (EPI == kTcEpiH) {
              const uint32_t c = cv[i];
              float h = 0.f;
              if (c) h = round_bf16(bf16_bits_to_f32(gv[i]) * round_bf16(v[i])) * (float)c;
              a.out[o] = f32_to_bf16_bits(h);
            } else {
              a.out[o] = f32_to_bf16_bits(v[i]);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acce);
      }
    }
    cp_wait_tc<0>();
  } else if (warp == 8) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = tc_idesc(NT, TRANS);
      const uint32_t a0 = smem_u32(smem + Sm::a), b0 = smem_u32(smem + Sm::b);
      int unit_idx = 0, cs = 0;
      int u = blockIdx.x;
      TcUnit un = u < nunits ? tc_unit(a, u) : TcUnit{0, 0, 0};
#pragma unroll 1
      for (int q = 0; q < nsteps_total; ++q) {
        while (cs >= un.nsteps) { u += gridDim.x; un = tc_unit(a, u); cs = 0; ++unit_idx; }
        if (cs == 0 && unit_idx > 0) wait(acce, (uint32_t)(unit_idx - 1) & 1u);
        const int st = q % kTcStages;
        wait(&full[st], (uint32_t)(q / kTcStages) & 1u);
        tc_fence_after();
        const uint32_t as = a0 + st * Sm::a_stage, bs = b0 + st * Sm::b_stage;
#pragma unroll
        for (int k = 0; k < kTcK / 16; ++k) {
          // K-major: the next 16 K are 32 bytes further along the swizzled rows;
          // MN-major: two K blocks (2 x 2048 bytes) further
          const uint64_t ad = TRANS ? tc_desc_sw128(as + k * 4096, 1024, 2048)
                                    : tc_desc_sw128(as + k * 32, 16, 1024);
          const uint64_t bd = tc_desc_sw128(bs + k * 32, 16, 1024);
          tc_mma(tmem, ad, bd, idesc, (cs > 0 || k > 0) ? 1u : 0u);
        }
        tc_commit(&empty[st]);
        ++cs;
        if (cs == un.nsteps) tc_commit(accf);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ activation loader
    pdl_wait();
    int u = blockIdx.x, cs = 0;
    TcUnit un = u < nunits ? tc_unit(a, u) : TcUnit{0, 0, 0};
    auto load = [&](int q) {
      while (cs >= un.nsteps) { u += gridDim.x; un = tc_unit(a, u); cs = 0; }
      const int kpos = un.k0 + cs * kTcK;
      const int st = q % kTcStages;
      uint8_t* B = smem + Sm::b + st * Sm::b_stage;
      // NT rows x 8 chunks of 16 bytes; K-major SW128 like the A rows
#pragma unroll
      for (int c = lane; c < NT * 8; c += 32) {
        const int n = c >> 3, j = c & 7;
        const bool valid = n < a.B;
        const uint16_t* src = a.x + (size_t)(valid ? n : 0) * a.K + kpos + j * 8;
        cp_async16_zfill(B + (n >> 3) * 1024 + (n & 7) * 128 + ((j ^ (n & 7)) << 4), src, valid);
      }
      cp_commit_tc();
      ++cs;
    };
    // Up to kLag steps in flight (the tile comes from L2; one step at a time
    // would pace the whole pipeline at one L2 round trip per step).
    constexpr int kLag = kTcStages - 1;
    auto publish = [&](int q) {
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[q % kTcStages]);
    };
#pragma unroll 1
    for (int q = 0; q < nsteps_total; ++q) {
      const int st = q % kTcStages;
      if (q >= kTcStages) wait(&empty[st], (uint32_t)((q / kTcStages) - 1) & 1u);
      load(q);
      if (q >= kLag) {
        cp_wait_tc<kLag>();
        publish(q - kLag);
      }
    }
    cp_wait_tc<0>();
    for (int q = nsteps_total - kLag < 0 ? 0 : nsteps_total - kLag; q < nsteps_total; ++q) publish(q);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kCols)
                 : "memory");
  }
}

// Fixed-order sum of the split-K partials, then the epilogue:
// y[i] = epi(sum_p part[p][i]) (kTcEpiBf16 / Silu / H as in the GEMM).
__global__ void tc_reduce_kernel(const float* __restrict__ part, int ksplit, int64_t n, int epi,
                                 const uint16_t* __restrict__ g, const uint32_t* __restrict__ cnt,
                                 uint16_t* __restrict__ y) {
  pdl_wait();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int p = 0; p < ksplit; ++p) s += part[p * n + i];
    float o = s;
    if (epi == kTcEpiSilu) {
      o = silu_f32(round_bf16(s));
    } else if (epi == kTcEpiH) {
      const uint32_t c = cnt[i];
      o = c ? round_bf16(bf16_bits_to_f32(g[i]) * round_bf16(s)) * (float)c : 0.f;
    }
    y[i] = f32_to_bf16_bits(o);
  }
}

template <int NT, int EPI, bool TRANS>
static int tc_launch_nt(const TcArgs& a, cudaStream_t st) {
  auto k = gemm_tc_kernel<NT, EPI, TRANS>;
  const int smem = TcSmem<NT>::total;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return launch_status(e);
  const int nunits = ((a.R + kTcM - 1) / kTcM) * a.ksplit;
  const int grid = nunits < num_sms() ? nunits : num_sms();
  return launch_status(launch(k, dim3(grid), dim3(kTcThreads), (size_t)smem, st, a));
}

template <int EPI, bool TRANS>
static int tc_launch(const TcArgs& a, cudaStream_t st) {
  if (a.B <= 16) return tc_launch_nt<16, EPI, TRANS>(a, st);
  if (a.B <= 32) return tc_launch_nt<32, EPI, TRANS>(a, st);
  if (a.B <= 64) return tc_launch_nt<64, EPI, TRANS>(a, st);
  return tc_launch_nt<128, EPI, TRANS>(a, st);
}

}  // namespace dip

using namespace dip;

static int tc_check_rows(const void* w, const void* s, const void* x, int64_t R, int64_t K,
                         int64_t B) {
  if (!w || !s || !x || R <= 0 || K <= 0 || B <= 0 || B > kTcMaxN) return DIP_ERR_ARG;
  // scale words are fetched 4 bytes at a time: an even number of groups per row
  if (K % 256 != 0 || R > (1 << 24) || K > (1 << 20)) return DIP_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x)) & 15) return DIP_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(s) & 3) return DIP_ERR_ARG;
  return DIP_OK;
}

constexpr int kTcMaxSplitRows = 4;

// Split K so that tiles x splits fill the SMs most evenly (a wave of 148 SMs
// over 200 tiles leaves 96 SMs idle for half the time).
static int tc_pick_split(int ntile, int kunits, int maxs) {
  const int sms = num_sms();
  int ks = 1;
  double best = 0.0;
  for (int c = 1; c <= maxs && c <= kunits; ++c) {
    const int units = ntile * c, waves = (units + sms - 1) / sms;
    const double eff = (double)units / ((double)waves * sms);
    if (eff > best + 1e-9) { best = eff; ks = c; }
  }
  return ks;
}

extern "C" size_t dip_int4_gemm_tc_workspace_bytes(int64_t rows, int64_t in_features, int64_t batch) {
  if (rows <= 0 || in_features <= 0 || batch <= 0) return 0;
  return (((size_t)batch * in_features * 2 + 255) & ~size_t(255)) +
         (size_t)kTcMaxSplitRows * batch * rows * sizeof(float);
}

extern "C" int dip_int4_gemm_tc_auto_split(int64_t rows, int64_t in_features) {
  if (rows <= 0 || in_features <= 0 || in_features % kTcChunkK) return 0;
  return tc_pick_split((int)((rows + kTcM - 1) / kTcM), (int)(in_features / kTcChunkK),
                       kTcMaxSplitRows);
}

extern "C" int dip_int4_gemm_tc(const int8_t* qweight, const dip_bf16* scales, const dip_bf16* x,
                                int64_t rows, int64_t in_features, int64_t batch, int epilogue,
                                const dip_bf16* g, const uint32_t* sel_count, void* workspace,
                                size_t workspace_bytes, dip_bf16* out, dip_stream_t stream) {
  return dip_int4_gemm_tc_split(qweight, scales, x, rows, in_features, batch, epilogue, g,
                                sel_count, 0, workspace, workspace_bytes, out, stream);
}

extern "C" int dip_int4_gemm_tc_split(const int8_t* qweight, const dip_bf16* scales,
                                      const dip_bf16* x, int64_t rows, int64_t in_features,
                                      int64_t batch, int epilogue, const dip_bf16* g,
                                      const uint32_t* sel_count, int ksplit, void* workspace,
                                      size_t workspace_bytes, dip_bf16* out, dip_stream_t stream) {
  if (ksplit < 0 || ksplit > kTcMaxSplitRows) return DIP_ERR_ARG;
  int rc = tc_check_rows(qweight, scales, x, rows, in_features, batch);
  if (rc) return rc;
  if (!out || !workspace) return DIP_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(workspace) & 15) return DIP_ERR_ARG;
  if (workspace_bytes < dip_int4_gemm_tc_workspace_bytes(rows, in_features, batch)) return DIP_ERR_WORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  // the activations with each 8-element group in the weights' dequantised order
  const int64_t n16 = batch * in_features / 8;
  rc = launch_status(launch(tc_permute_k8_kernel, dim3((unsigned)((n16 + 255) / 256 < 2048 ? (n16 + 255) / 256 : 2048)),
                            dim3(256), 0, st, reinterpret_cast<const uint4*>(x), n16,
                            static_cast<uint4*>(workspace)));
  if (rc) return rc;
  TcArgs a = {};
  a.w = reinterpret_cast<const uint8_t*>(qweight);
  a.s = scales;
  a.x = static_cast<const uint16_t*>(workspace);
  a.R = (int)rows;
  a.K = (int)in_features;
  a.B = (int)batch;
  a.kgran = kTcChunkK / kTcK;
  a.ksplit = ksplit ? ksplit
                   : tc_pick_split((int)((rows + kTcM - 1) / kTcM), (int)(in_features / kTcChunkK),
                                   kTcMaxSplitRows);
  if (a.ksplit > (int)(in_features / kTcChunkK)) return DIP_ERR_ARG;
  a.out = out;
  a.g = g;
  a.cnt = sel_count;
  a.err = error_word_ptr();
  if (!a.err) return DIP_ERR_CUDA;
  if (epilogue < 0 || epilogue > 2) return DIP_ERR_ARG;
  if (epilogue == 2 && (!g || !sel_count)) return DIP_ERR_ARG;
  if (a.ksplit > 1) {
    // fp32 partials of the K ranges, then one fixed-order sum with the epilogue
    a.out_f32 = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                         (((size_t)batch * in_features * 2 + 255) & ~size_t(255)));
    rc = tc_launch<kTcEpiF32, false>(a, st);
    if (rc) return rc;
    const int64_t n = batch * rows;
    return launch_status(launch(tc_reduce_kernel, dim3((unsigned)((n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184)),
                                dim3(256), 0, st, (const float*)a.out_f32, a.ksplit, n, epilogue,
                                (const uint16_t*)g, sel_count, (uint16_t*)out));
  }
  switch (epilogue) {
    case 0: return tc_launch<kTcEpiBf16, false>(a, st);
    case 1: return tc_launch<kTcEpiSilu, false>(a, st);
    case 2: return tc_launch<kTcEpiH, false>(a, st);
    default: return DIP_ERR_ARG;
  }
}

extern "C" size_t dip_int4_down_tc_workspace_bytes(int64_t out_features, int64_t batch) {
  if (out_features <= 0 || batch <= 0) return 0;
  return (size_t)8 * batch * out_features * sizeof(float);
}

namespace dip {
static int down_tc_impl(const int8_t* down_t, const dip_bf16* scales, const dip_bf16* h,
                        int64_t inter, int64_t out_features, int64_t batch, void* workspace,
                        size_t workspace_bytes, dip_bf16* y, float* y_f32, dip_stream_t stream);
}

extern "C" int dip_int4_down_tc(const int8_t* down_t, const dip_bf16* scales, const dip_bf16* h,
                                int64_t inter, int64_t out_features, int64_t batch,
                                void* workspace, size_t workspace_bytes, dip_bf16* y,
                                dip_stream_t stream) {
  if (!y) return DIP_ERR_ARG;
  return down_tc_impl(down_t, scales, h, inter, out_features, batch, workspace, workspace_bytes, y,
                      nullptr, stream);
}

extern "C" int dip_int4_down_tc_f32(const int8_t* down_t, const dip_bf16* scales,
                                    const dip_bf16* h, int64_t inter, int64_t out_features,
                                    int64_t batch, void* workspace, size_t workspace_bytes,
                                    float* y_f32, dip_stream_t stream) {
  if (!y_f32) return DIP_ERR_ARG;
  return down_tc_impl(down_t, scales, h, inter, out_features, batch, workspace, workspace_bytes,
                      nullptr, y_f32, stream);
}

namespace dip {
__global__ void tc_reduce_f32_kernel(const float* __restrict__ part, int ksplit, int64_t n,
                                     float* __restrict__ y) {
  pdl_wait();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int p = 0; p < ksplit; ++p) s += part[p * n + i];
    y[i] = s;
  }
}

static int down_tc_impl(const int8_t* down_t, const dip_bf16* scales, const dip_bf16* h,
                        int64_t inter, int64_t out_features, int64_t batch, void* workspace,
                        size_t workspace_bytes, dip_bf16* y, float* y_f32, dip_stream_t stream) {
  if (!down_t || !scales || !h || !workspace || inter <= 0 || out_features <= 0 ||
      batch <= 0 || batch > kTcMaxN)
    return DIP_ERR_ARG;
  if (inter % kTcK != 0 || out_features % 256 != 0 || inter > (1 << 24)) return DIP_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(down_t) | reinterpret_cast<uintptr_t>(h) |
       reinterpret_cast<uintptr_t>(workspace)) & 15)
    return DIP_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(scales) & 3) return DIP_ERR_ARG;
  if (workspace_bytes < dip_int4_down_tc_workspace_bytes(out_features, batch)) return DIP_ERR_WORKSPACE;
  TcArgs a = {};
  a.w = reinterpret_cast<const uint8_t*>(down_t);
  a.s = scales;
  a.x = h;
  a.R = (int)out_features;
  a.K = (int)inter;
  a.B = (int)batch;
  // split the channels so that tiles x splits fill the SMs most evenly (at most 8 splits)
  const int ks = tc_pick_split((int)(out_features / kTcM), (int)(inter / kTcK), 8);
  a.ksplit = ks;
  a.kgran = 1;
  a.out_f32 = static_cast<float*>(workspace);
  a.err = error_word_ptr();
  if (!a.err) return DIP_ERR_CUDA;
  cudaStream_t st = (cudaStream_t)stream;
  int rc = tc_launch<kTcEpiF32, true>(a, st);
  if (rc) return rc;
  const int64_t n = batch * out_features;
  const dim3 grid((unsigned)((n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184));
  if (y_f32)
    return launch_status(launch(tc_reduce_f32_kernel, grid, dim3(256), 0, st,
                                (const float*)a.out_f32, ks, n, y_f32));
  return launch_status(launch(tc_reduce_kernel, grid, dim3(256), 0, st, (const float*)a.out_f32, ks,
                              n, (int)kTcEpiBf16, (const uint16_t*)nullptr,
                              (const uint32_t*)nullptr, y));
}
}  // namespace dip

namespace dip {
// cnt[b][c] = number of times channel c appears in idx[b] (zeroed first by the host).
__global__ void select_count_kernel(const int32_t* __restrict__ idx, int64_t batch, int64_t k,
                                    int64_t inter, uint32_t* __restrict__ cnt) {
  pdl_wait();
  const int64_t n = batch * k;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / k;
    const int32_t c = idx[i];
    if (c >= 0 && c < inter) atomicAdd(&cnt[b * inter + c], 1u);
  }
}
}  // namespace dip

extern "C" int dip_select_count(const int32_t* idx, int64_t batch, int64_t k, int64_t inter,
                                uint32_t* cnt, dip_stream_t stream) {
  if (!idx || !cnt || batch <= 0 || k < 0 || inter <= 0) return DIP_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(cnt, 0, (size_t)batch * inter * sizeof(uint32_t), st);
  if (e != cudaSuccess) return launch_status(e);
  if (k == 0) return DIP_OK;
  const int64_t n = batch * k;
  const unsigned grid = (unsigned)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
  return launch_status(launch(select_count_kernel, dim3(grid), dim3(256), 0, st, idx, batch, k,
                              inter, cnt));
}
