// topk.cu — exact, deterministic top-k of |s| in ONE launch, and the
// cache-aware hit/miss split.
//
// Reference semantics (kernels/topk_select/topk_select.cu:134-164):
//   hi = max|s|, lo = 0, t = (lo+hi)/2; 25 times: if #{|s| > t} > k then
//   lo = t else hi = t; t = (lo+hi)/2.  Output: {|s| > hi} in ascending
//   index, then {lo < |s| <= hi} in ascending index, truncated to k, the rest
//   of idx zero.  The reference runs 25 count kernels with a host sync each.
//
// Here the bisection is emulated exactly without any counting pass:
//   #{|s| > t} > k  <=>  w > t,   w = the (k+1)-th largest |s|
// so the fp32 bisection only needs the single value w, found with a two-level
// radix select on the 15-bit magnitude of the bf16 (exponent byte, then the 7
// mantissa bits).  One CTA of 1024 threads: histogram, select, 25 scalar fp32
// steps (no FMA contraction, identical rounding to the reference's host
// loop), then a block-wide scan compaction of the two tiers.  NaN never
// compares greater than a threshold in the reference, so NaNs are excluded
// from the ranking and never selected.
#include "dip_common.cuh"
#include "dip_block.cuh"

namespace dip {

constexpr int kTopkThreads = 1024;

constexpr int kTopkMaxN = 98304;  // keys kept in shared memory (2 B each)
constexpr uint16_t kNanKey = 0xFFFF;  // as a float pattern (<<16) this is a NaN

// Find, scanning bins from the top, the bin holding the element of 1-based
// rank `rank`; returns the bin and writes the count above it.  One warp.
__device__ __forceinline__ int warp_find_rank_bin(const int* hist, int nbins, int rank,
                                                  int* above_out) {
  const int lane = threadIdx.x & 31;
  const int per = nbins / 32;  // bins per lane, counted from the top
  int local = 0;
  for (int i = 0; i < per; ++i) local += hist[nbins - 1 - (lane * per + i)];
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  const int excl = incl - local;
  const unsigned m = __ballot_sync(0xffffffffu, excl < rank && rank <= incl);
  const int owner = __ffs(m) - 1;
  int bin = -1, above = 0;
  if (lane == owner) {
    int run = excl;
    for (int i = 0; i < per; ++i) {
      const int b = nbins - 1 - (lane * per + i);
      if (run + hist[b] >= rank) { bin = b; above = run; break; }
      run += hist[b];
    }
  }
  bin = __shfl_sync(0xffffffffu, bin, owner);
  above = __shfl_sync(0xffffffffu, above, owner);
  *above_out = above;
  return bin;
}

// Adds one key's bin to this warp's private histogram; lanes of the warp
// holding the same bin are combined first, so each bin sees one atomic per
// warp instruction instead of a serialised run of same-address atomics.
__device__ __forceinline__ void warp_hist_add(int* whist, int bin, bool active) {
  const unsigned act = __ballot_sync(0xffffffffu, active);
  if (!active) return;
  const unsigned peers = __match_any_sync(act, bin);
  if ((int)(threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&whist[bin], __popc(peers));
}

constexpr int kWarps = kTopkThreads / 32;

__global__ void __launch_bounds__(kTopkThreads)
topk_select_kernel(const uint16_t* __restrict__ s_all, int n, int k, int32_t* __restrict__ idx_all,
                   int64_t s_stride, int64_t idx_stride) {
  extern __shared__ __align__(16) uint16_t keys[];
  __shared__ int whist[kWarps][256];  // per-warp histograms (level 1, then level 2)
  __shared__ int hist[256];
  __shared__ int2 warp_tot[33];
  __shared__ unsigned s_max;
  __shared__ int s_nvalid;
  __shared__ int s_sel[2];  // level-1 bin, count above it
  __shared__ float s_lohi[2];

  const uint16_t* s = s_all + blockIdx.x * s_stride;
  int32_t* idx = idx_all + blockIdx.x * idx_stride;
  const int tid = threadIdx.x, warp = tid >> 5;
  int* mine = whist[warp];
  for (int i = tid; i < kWarps * 256; i += kTopkThreads) (&whist[0][0])[i] = 0;
  if (tid == 0) { s_max = 0; s_nvalid = 0; }
  __syncthreads();

  pdl_wait();
  // Pass 1: magnitudes into shared memory, exponent histogram, max, count.
  // Eight keys per thread per step (16-byte loads when s is 16-byte aligned).
  unsigned lmax = 0;
  int lvalid = 0;
  const bool vec = ((reinterpret_cast<uintptr_t>(s) & 15) == 0);
  const int nvec = vec ? n / 8 : 0;
  const int steps = (nvec + kTopkThreads - 1) / kTopkThreads;
  for (int st = 0; st < steps; ++st) {
    const int v = st * kTopkThreads + tid;
    uint4 raw = make_uint4(0, 0, 0, 0);
    if (v < nvec) raw = __ldg(reinterpret_cast<const uint4*>(s) + v);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    uint16_t kk[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      uint16_t key = (uint16_t)((w[e >> 1] >> (16 * (e & 1))) & 0x7FFF);
      if (key > 0x7F80) key = kNanKey;
      kk[e] = key;
      const bool ok = v < nvec && key != kNanKey;
      if (ok) { lmax = max(lmax, (unsigned)key); ++lvalid; }
      warp_hist_add(mine, key >> 7, ok);
    }
    if (v < nvec) {
      uint4 o;
      o.x = kk[0] | ((uint32_t)kk[1] << 16);
      o.y = kk[2] | ((uint32_t)kk[3] << 16);
      o.z = kk[4] | ((uint32_t)kk[5] << 16);
      o.w = kk[6] | ((uint32_t)kk[7] << 16);
      reinterpret_cast<uint4*>(keys)[v] = o;
    }
  }
  for (int base = nvec * 8; base < n; base += kTopkThreads) {  // scalar tail
    const int i = base + tid;
    uint16_t key = kNanKey;
    if (i < n) {
      key = s[i] & 0x7FFF;
      if (key > 0x7F80) key = kNanKey;
      keys[i] = key;
    }
    const bool ok = i < n && key != kNanKey;
    if (ok) { lmax = max(lmax, (unsigned)key); ++lvalid; }
    warp_hist_add(mine, key >> 7, ok);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lmax = max(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
    lvalid += __shfl_xor_sync(0xffffffffu, lvalid, o);
  }
  if ((tid & 31) == 0) {
    atomicMax(&s_max, lmax);
    atomicAdd(&s_nvalid, lvalid);
  }
  __syncthreads();
  if (tid < 256) {
    int t = 0;
#pragma unroll 8
    for (int w = 0; w < kWarps; ++w) t += whist[w][tid];
    hist[tid] = t;
  }
  __syncthreads();
  const int nvalid = s_nvalid;
  const bool has_w = nvalid >= k + 1;

  // Level 1 select: exponent byte of the (k+1)-th largest magnitude.
  if (has_w && tid < 32) {
    int above;
    const int b = warp_find_rank_bin(hist, 256, k + 1, &above);
    if (tid == 0) { s_sel[0] = b; s_sel[1] = above; }
  }
  for (int i = tid; i < kWarps * 128; i += kTopkThreads) whist[i >> 7][i & 127] = 0;
  __syncthreads();
  if (has_w) {
    const int b1 = s_sel[0];
    for (int base = 0; base < n; base += kTopkThreads) {
      const int i = base + tid;
      const uint16_t key = i < n ? keys[i] : kNanKey;
      const bool ok = key != kNanKey && (key >> 7) == b1;
      warp_hist_add(mine, key & 0x7F, ok);
    }
  }
  __syncthreads();
  if (tid < 128) {
    int t = 0;
#pragma unroll 8
    for (int w = 0; w < kWarps; ++w) t += whist[w][tid];
    hist[tid] = t;
  }
  __syncthreads();
  if (tid < 32) {
    float wv = 0.f;
    if (has_w) {
      int above2;
      const int m = warp_find_rank_bin(hist, 128, k + 1 - s_sel[1], &above2);
      wv = bf16_bits_to_f32((unsigned)((s_sel[0] << 7) | m));
    }
    if (tid == 0) {
      // The reference's host loop, step for step, in fp32 round-to-nearest.
      float hi = bf16_bits_to_f32(s_max);
      float lo = 0.0f;
      float t = __fmul_rn(0.5f, __fadd_rn(lo, hi));
      for (int step = 0; step < 25; ++step) {
        if (has_w && wv > t) lo = t; else hi = t;
        t = __fmul_rn(0.5f, __fadd_rn(lo, hi));
      }
      s_lohi[0] = lo;
      s_lohi[1] = hi;
    }
  }
  __syncthreads();
  const float lo = s_lohi[0], hi = s_lohi[1];

  // Compaction of the two tiers (ascending index within each).
  int2 tot;
  block_compact2(
      n, [&](int i) { return bf16_bits_to_f32(keys[i]) > hi; },
      [&](int i) { const float v = bf16_bits_to_f32(keys[i]); return v > lo && v <= hi; },
      [&](int pos, int i) { if (pos < k) idx[pos] = i; }, warp_tot, tot);
  pdl_launch_dependents();
  const int filled = min(k, tot.x + tot.y);
  for (int i = filled + tid; i < k; i += kTopkThreads) idx[i] = 0;
}

// Shard selection for tensor parallelism along the intermediate dimension:
// the entries of idx owned by this rank ([lo, hi)), in idx order, as local
// row ids, and their number.
__global__ void __launch_bounds__(kTopkThreads)
shard_select_kernel(const int32_t* __restrict__ idx, int k, int lo, int hi,
                    int32_t* __restrict__ local, int32_t* __restrict__ count) {
  __shared__ int2 warp_tot[33];
  pdl_wait();
  int2 tot;
  block_compact2(
      k, [&](int j) { return idx[j] >= lo && idx[j] < hi; }, [&](int) { return false; },
      [&](int pos, int j) { local[pos] = idx[j] - lo; }, warp_tot, tot);
  pdl_launch_dependents();
  if (threadIdx.x == 0) count[0] = tot.x;
}

// Cache hit/miss split (dip_ca.py:137-142 with the src/row tables of
// :164-171, misses pointing at the full resident rows).
__global__ void __launch_bounds__(kTopkThreads)
ca_split_kernel(const int32_t* __restrict__ idx, int k, const int64_t* __restrict__ id2slot,
                int64_t n_channels, int32_t* __restrict__ combined, int32_t* __restrict__ src,
                int32_t* __restrict__ row, int32_t* __restrict__ n_hit) {
  __shared__ int2 warp_tot[33];
  pdl_wait();
  auto slot_of = [&](int j) -> int64_t {
    const int c = idx[j];
    return (c >= 0 && c < n_channels) ? id2slot[c] : -1;
  };
  int2 tot;
  block_compact2(
      k, [&](int j) { return slot_of(j) >= 0; }, [&](int j) { return slot_of(j) < 0; },
      [&](int pos, int j) {
        const int c = idx[j];
        const int64_t sl = slot_of(j);
        combined[pos] = c;
        src[pos] = sl >= 0 ? 0 : 1;
        row[pos] = sl >= 0 ? (int32_t)sl : c;
      },
      warp_tot, tot);
  pdl_launch_dependents();
  if (threadIdx.x == 0) n_hit[0] = tot.x;
}

// ---------------------------------------------------------------------------
// Histogram-based top-k (the fast path).  The exact bisection emulation needs
// only w, the (k+1)-th largest |s|, and max|s|; both come from a 32768-bin
// histogram of the 15-bit magnitudes.  In the decode chain the gate kernel
// fills the histogram in its epilogue, so the select step only reads a few
// slices of it and compacts; it leaves the histogram zero for the next call.
constexpr int kHistBins = 32768;

// ---------------------------------------------------------------------------
// Top-k v3: select from a two-level histogram, compact on many SMs.
//
// Scratch (dip_topk_hist_bytes): fine[32768] counts of the 15-bit |s| key,
// coarse[256] counts of its exponent byte, status[256] look-back words.  It
// must be zero on entry.  The selection reads only the coarse histogram and
// three 128-bin slices of the fine one, so no SM moves more than a few
// hundred bytes of it.  Each CTA then compacts its own 2048-element chunk:
// the two tier counts of earlier chunks come from a bounded decoupled
// look-back on status[], and the total of tier A (needed to place tier B)
// comes from the histogram, so no CTA waits on a later one.
constexpr int kCoarseOff = kHistBins;                 // in u32 words
constexpr int kStatusOffBytes = (kHistBins + 256) * 4;
constexpr int kCompactChunk = 2048;                   // elements per CTA
constexpr int kMaxCompactCtas = 256;
constexpr size_t kTopkScratchBytes = kStatusOffBytes + kMaxCompactCtas * 8;

// #{keys > t} from the histograms (t >= 0, fp32): keys above bf16 bin b0 =
// (bits(t) >> 16) are all keys with key >= b0 + 1.  One warp.
__device__ __forceinline__ int warp_count_above(const unsigned* hist, const int* coarse_suffix,
                                                float t) {
  const int lane = threadIdx.x & 31;
  const int kmin = (int)(__float_as_uint(t) >> 16) + 1;  // smallest key counted
  if (kmin > 0x7F80) return 0;
  const int cb = kmin >> 7;
  int part = 0;
  for (int f = lane; f < 128; f += 32) {
    const int key = (cb << 7) | f;
    if (key >= kmin) part += hist[key];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  return part + (cb < 255 ? coarse_suffix[cb + 1] : 0);
}

__global__ void __launch_bounds__(kTopkThreads)
topk_compact_kernel(const uint16_t* __restrict__ s, int n, int k, int32_t* __restrict__ idx,
                    unsigned* __restrict__ scratch, unsigned* err) {
  __shared__ int coarse_suffix[257];   // coarse_suffix[b] = #keys with exponent byte >= b
  __shared__ uint16_t keys[kCompactChunk];
  __shared__ int2 warp_tot[33];
  __shared__ float s_lohi[2];
  __shared__ int s_tot[2];              // #(> hi), #(> lo)
  __shared__ int2 s_off;                // tier A / B counts of earlier chunks
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c0 = blockIdx.x * kCompactChunk;
  const int cn = min(kCompactChunk, n - c0);
  unsigned long long* status =
      reinterpret_cast<unsigned long long*>(reinterpret_cast<uint8_t*>(scratch) + kStatusOffBytes);
  pdl_wait();
  // Keys of this chunk (two per thread).
  for (int e = tid; e < cn; e += kTopkThreads) keys[e] = s[c0 + e] & 0x7FFF;
  if (warp == 0) {
    // Coarse histogram: suffix sums, total, the bins of w and of max.
    const unsigned* coarse = scratch + kCoarseOff;
    int cnt[8], loc = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) { cnt[q] = coarse[255 - (lane * 8 + q)]; loc += cnt[q]; }
    int incl = loc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    int run = incl - loc;  // count in bins above this lane's
#pragma unroll
    for (int q = 0; q < 8; ++q) { run += cnt[q]; coarse_suffix[255 - (lane * 8 + q)] = run; }
    if (lane == 0) coarse_suffix[256] = 0;
  }
  __syncthreads();
  if (warp == 0) {
    const int nvalid = coarse_suffix[0];
    const bool has_w = nvalid >= k + 1;
    // highest non-empty coarse bin, then the highest non-empty key in it
    int topb = -1;
    for (int b = lane; b < 256; b += 32)
      if (coarse_suffix[b] - coarse_suffix[b + 1] > 0) topb = max(topb, b);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) topb = max(topb, __shfl_xor_sync(0xffffffffu, topb, o));
    int maxkey = 0;
    if (topb >= 0) {
      int mk = -1;
      for (int f = lane; f < 128; f += 32)
        if (scratch[(topb << 7) | f] != 0) mk = max(mk, (topb << 7) | f);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mk = max(mk, __shfl_xor_sync(0xffffffffu, mk, o));
      maxkey = max(mk, 0);
    }
    float wv = 0.f;
    if (has_w) {
      // coarse bin b1 holding rank k+1 from the top: suffix[b1+1] < k+1 <= suffix[b1]
      int b1 = -1;
      for (int b = lane; b < 256; b += 32)
        if (coarse_suffix[b + 1] < k + 1 && k + 1 <= coarse_suffix[b]) b1 = b;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) b1 = max(b1, __shfl_xor_sync(0xffffffffu, b1, o));
      const int rank = k + 1 - coarse_suffix[b1 + 1];
      // fine bins of b1 from the top: lane owns 4 consecutive bins
      int f4[4], loc = 0;
#pragma unroll
      for (int q = 0; q < 4; ++q) { f4[q] = scratch[(b1 << 7) | (127 - (lane * 4 + q))]; loc += f4[q]; }
      int incl = loc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      int runf = incl - loc, found = -1;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        runf += f4[q];
        if (found < 0 && runf >= rank && runf - f4[q] < rank) found = 127 - (lane * 4 + q);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) found = max(found, __shfl_xor_sync(0xffffffffu, found, o));
      wv = bf16_bits_to_f32((unsigned)((b1 << 7) | found));
    }
    // The reference's host loop, step for step, in fp32 round-to-nearest.
    float hi = bf16_bits_to_f32((unsigned)maxkey), lo = 0.0f;
    float t = __fmul_rn(0.5f, __fadd_rn(lo, hi));
    for (int step = 0; step < 25; ++step) {
      if (has_w && wv > t) lo = t; else hi = t;
      t = __fmul_rn(0.5f, __fadd_rn(lo, hi));
    }
    const int n_hi = warp_count_above(scratch, coarse_suffix, hi);
    const int n_lo = warp_count_above(scratch, coarse_suffix, lo);
    if (lane == 0) { s_lohi[0] = lo; s_lohi[1] = hi; s_tot[0] = n_hi; s_tot[1] = n_lo; }
  }
  __syncthreads();
  const float lo = s_lohi[0], hi = s_lohi[1];
  auto isA = [&](int e) { return bf16_bits_to_f32(keys[e]) > hi; };
  auto isB = [&](int e) { const float v = bf16_bits_to_f32(keys[e]); return v > lo && v <= hi; };
  // Chunk counts -> publish -> look back over earlier chunks.
  int ca = 0, cb = 0;
  for (int e = tid; e < cn; e += kTopkThreads) { ca += isA(e); cb += isB(e); }
  int2 tot;
  block_excl_scan2(ca, cb, warp_tot, tot);
  if (tid == 0) {
    const unsigned long long word = (1ull << 63) | ((unsigned long long)tot.x << 32) | (unsigned)tot.y;
    asm volatile("st.release.gpu.global.u64 [%0], %1;\n" ::"l"(status + blockIdx.x), "l"(word)
                 : "memory");
  }
  if (warp == 0) {
    int pa = 0, pb = 0;
    for (int c = lane; c < (int)blockIdx.x; c += 32) {
      unsigned long long v = 0;
      for (uint32_t it = 0, lim = spin_limit(err); it < lim; ++it) {
        asm volatile("ld.acquire.gpu.global.u64 %0, [%1];\n" : "=l"(v) : "l"(status + c) : "memory");
        if (v >> 63) break;
      }
      if (!(v >> 63)) { atomicOr(err, kErrTimeout); v = 0; }
      pa += (int)((v >> 32) & 0x7FFFFFFF);
      pb += (int)(v & 0xFFFFFFFFu);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      pa += __shfl_xor_sync(0xffffffffu, pa, o);
      pb += __shfl_xor_sync(0xffffffffu, pb, o);
    }
    if (lane == 0) s_off = make_int2(pa, pb);
  }
  __syncthreads();
  const int baseA = s_off.x, baseB = s_tot[0] + s_off.y;
  int2 tot2;
  block_compact2(
      cn, isA, isB,
      [&](int pos, int e) {
        const int p = pos < tot.x ? baseA + pos : baseB + (pos - tot.x);
        if (p < k) idx[p] = c0 + e;
      },
      warp_tot, tot2);
  pdl_launch_dependents();
  // Unfilled tail (only when fewer than k keys qualify): zeros, as the reference.
  const int filled = min(k, s_tot[1]);
  const int per = (k - filled + gridDim.x - 1) / gridDim.x;
  const int z0 = filled + blockIdx.x * per, z1 = min(k, z0 + per);
  for (int i = z0 + tid; i < z1; i += kTopkThreads) idx[i] = 0;
}

// Clears the top-k scratch (histograms and look-back words); grid-stride.
__global__ void zero_words_kernel(uint4* __restrict__ p, int n16) {
  pdl_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += gridDim.x * blockDim.x)
    p[i] = make_uint4(0, 0, 0, 0);
  pdl_launch_dependents();
}

__global__ void __launch_bounds__(256)
topk_hist2_kernel(const uint16_t* __restrict__ s, int n, unsigned* __restrict__ scratch) {
  pdl_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const unsigned key = s[i] & 0x7FFFu;
    if (key <= 0x7F80u) {
      atomicAdd(&scratch[key], 1u);
      atomicAdd(&scratch[kCoarseOff + (key >> 7)], 1u);
    }
  }
  pdl_launch_dependents();
}

int topk_compact_launch(const uint16_t* s, int64_t n, int64_t k, int32_t* idx, unsigned* scratch,
                        cudaStream_t st) {
  if (n < 1 || n > kMaxCompactCtas * kCompactChunk || k < 1 || k > INT32_MAX || !s || !idx ||
      !scratch)
    return DIP_ERR_ARG;
  unsigned* err = error_word_ptr();
  if (!err) return DIP_ERR_CUDA;
  const int grid = (int)((n + kCompactChunk - 1) / kCompactChunk);
  return launch_status(launch(topk_compact_kernel, dim3(grid), dim3(kTopkThreads), 0, st, s,
                              (int)n, (int)k, idx, scratch, err));
}

size_t topk_scratch_bytes() { return kTopkScratchBytes; }

int topk_launch(const uint16_t* s, int64_t n, int64_t k, int32_t* idx, int batch,
                int64_t s_stride, int64_t idx_stride, cudaStream_t st) {
  if (n < 1 || n > kTopkMaxN || k < 0 || k > INT32_MAX || batch < 1) return DIP_ERR_ARG;
  if (!s || (k > 0 && !idx)) return DIP_ERR_ARG;
  if (k == 0) return DIP_OK;
  const size_t smem = (size_t)n * 2;
  {  // static (~34 KB) + dynamic shared memory exceeds the 48 KB default
    cudaError_t e = cudaFuncSetAttribute(topk_select_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return launch_status(e);
  }
  return launch_status(launch(topk_select_kernel, dim3(batch), dim3(kTopkThreads), smem, st, s,
                              (int)n, (int)k, idx, s_stride, idx_stride));
}

}  // namespace dip

using namespace dip;

extern "C" int dip_topk_select(const dip_bf16* s, int64_t n, int64_t k, int32_t* idx,
                               dip_stream_t stream) {
  return topk_launch(s, n, k, idx, 1, 0, 0, (cudaStream_t)stream);
}

extern "C" int dip_topk_select_batched(const dip_bf16* s, int64_t batch, int64_t n,
                                       int64_t s_stride, int64_t k, int32_t* idx,
                                       int64_t idx_stride, dip_stream_t stream) {
  if (batch < 1 || batch > 65535 || s_stride < n || idx_stride < k) return DIP_ERR_ARG;
  return topk_launch(s, n, k, idx, (int)batch, s_stride, idx_stride, (cudaStream_t)stream);
}

extern "C" int dip_ca_split(const int32_t* idx, int64_t k, const int64_t* id2slot,
                            int64_t n_channels, int32_t* combined_ids, int32_t* src,
                            int32_t* row, int32_t* n_hit, dip_stream_t stream) {
  if (k < 0 || k > INT32_MAX || n_channels < 0) return DIP_ERR_ARG;
  if (!n_hit) return DIP_ERR_ARG;
  if (k > 0 && (!idx || !id2slot || !combined_ids || !src || !row)) return DIP_ERR_ARG;
  return launch_status(launch(ca_split_kernel, dim3(1), dim3(kTopkThreads), 0,
                              (cudaStream_t)stream, idx, (int)k, id2slot, n_channels,
                              combined_ids, src, row, n_hit));
}

extern "C" int dip_shard_select(const int32_t* idx, int64_t k, int64_t lo, int64_t hi,
                                int32_t* local_idx, int32_t* count, dip_stream_t stream) {
  if (k < 0 || k > INT32_MAX || lo < 0 || hi < lo || hi > INT32_MAX || !count) return DIP_ERR_ARG;
  if (k > 0 && (!idx || !local_idx)) return DIP_ERR_ARG;
  return launch_status(launch(shard_select_kernel, dim3(1), dim3(kTopkThreads), 0,
                              (cudaStream_t)stream, idx, (int)k, (int)lo, (int)hi, local_idx,
                              count));
}

extern "C" size_t dip_topk_hist_bytes(void) { return kTopkScratchBytes; }

extern "C" int dip_topk_select_ws(const dip_bf16* s, int64_t n, int64_t k, int32_t* idx,
                                  void* hist, dip_stream_t stream) {
  if (n < 1 || n > kMaxCompactCtas * kCompactChunk || k < 0 || k > INT32_MAX || !s || !hist)
    return DIP_ERR_ARG;
  if (k == 0) return DIP_OK;
  if (!idx || (reinterpret_cast<uintptr_t>(hist) & 15)) return DIP_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  unsigned* sc = static_cast<unsigned*>(hist);
  const int grid = (int)((n + 255) / 256 < 148 ? (n + 255) / 256 : 148);
  int r = launch_status(launch(topk_hist2_kernel, dim3(grid), dim3(256), 0, st, s, (int)n, sc));
  if (r) return r;
  r = topk_compact_launch(s, n, k, idx, sc, st);
  if (r) return r;
  return launch_status(launch(zero_words_kernel, dim3(33), dim3(256), 0, st,
                              reinterpret_cast<uint4*>(hist), (int)(kTopkScratchBytes / 16)));
}
