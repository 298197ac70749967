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

namespace dip {

constexpr int kTopkThreads = 1024;
constexpr int kTopkMaxN = 98304;  // keys kept in shared memory (2 B each)
constexpr uint16_t kNanKey = 0xFFFF;  // as a float pattern (<<16) this is a NaN

// Block-wide exclusive scan of two counters; returns totals through tot.
__device__ __forceinline__ int2 block_excl_scan2(int a, int b, int2* warp_tot, int2& tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int ia = a, ib = b;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int ta = __shfl_up_sync(0xffffffffu, ia, o);
    const int tb = __shfl_up_sync(0xffffffffu, ib, o);
    if (lane >= o) { ia += ta; ib += tb; }
  }
  if (lane == 31) warp_tot[warp] = make_int2(ia, ib);
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    int2 v = lane < nw ? warp_tot[lane] : make_int2(0, 0);
    int sa = v.x, sb = v.y;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int ta = __shfl_up_sync(0xffffffffu, sa, o);
      const int tb = __shfl_up_sync(0xffffffffu, sb, o);
      if (lane >= o) { sa += ta; sb += tb; }
    }
    if (lane < nw) warp_tot[lane] = make_int2(sa - v.x, sb - v.y);  // exclusive
    if (lane == nw - 1) warp_tot[32] = make_int2(sa, sb);
  }
  __syncthreads();
  const int2 wbase = warp_tot[warp];
  tot = warp_tot[32];
  return make_int2(wbase.x + ia - a, wbase.y + ib - b);
}

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

  // Compaction: thread tid owns the contiguous range [beg, end).
  const int per = (n + kTopkThreads - 1) / kTopkThreads;
  const int beg = min(n, tid * per), end = min(n, beg + per);
  int ca = 0, cb = 0;
  for (int i = beg; i < end; ++i) {
    const float v = bf16_bits_to_f32(keys[i]);
    ca += (v > hi);
    cb += (v > lo && v <= hi);
  }
  int2 tot;
  const int2 off = block_excl_scan2(ca, cb, warp_tot, tot);
  int pa = off.x, pb = tot.x + off.y;
  for (int i = beg; i < end; ++i) {
    const float v = bf16_bits_to_f32(keys[i]);
    if (v > hi) { if (pa < k) idx[pa] = i; ++pa; }
    else if (v > lo && v <= hi) { if (pb < k) idx[pb] = i; ++pb; }
  }
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
  const int tid = threadIdx.x;
  const int per = (k + kTopkThreads - 1) / kTopkThreads;
  const int beg = min(k, tid * per), end = min(k, beg + per);
  int c = 0;
  for (int j = beg; j < end; ++j) c += (idx[j] >= lo && idx[j] < hi);
  int2 tot;
  const int2 off = block_excl_scan2(c, 0, warp_tot, tot);
  int pos = off.x;
  for (int j = beg; j < end; ++j) {
    const int v = idx[j];
    if (v >= lo && v < hi) local[pos++] = v - lo;
  }
  pdl_launch_dependents();
  if (tid == 0) count[0] = tot.x;
}

// Cache hit/miss split (dip_ca.py:137-142 with the src/row tables of
// :164-171, misses pointing at the full resident rows).
__global__ void __launch_bounds__(kTopkThreads)
ca_split_kernel(const int32_t* __restrict__ idx, int k, const int64_t* __restrict__ id2slot,
                int64_t n_channels, int32_t* __restrict__ combined, int32_t* __restrict__ src,
                int32_t* __restrict__ row, int32_t* __restrict__ n_hit) {
  __shared__ int2 warp_tot[33];
  pdl_wait();
  const int tid = threadIdx.x;
  const int per = (k + kTopkThreads - 1) / kTopkThreads;
  const int beg = min(k, tid * per), end = min(k, beg + per);
  int ch = 0, cm = 0;
  for (int j = beg; j < end; ++j) {
    const int c = idx[j];
    const int64_t sl = (c >= 0 && c < n_channels) ? id2slot[c] : -1;
    if (sl >= 0) ++ch; else ++cm;
  }
  int2 tot;
  const int2 off = block_excl_scan2(ch, cm, warp_tot, tot);
  int ph = off.x, pm = tot.x + off.y;
  for (int j = beg; j < end; ++j) {
    const int c = idx[j];
    const int64_t sl = (c >= 0 && c < n_channels) ? id2slot[c] : -1;
    if (sl >= 0) { combined[ph] = c; src[ph] = 0; row[ph] = (int32_t)sl; ++ph; }
    else { combined[pm] = c; src[pm] = 1; row[pm] = c; ++pm; }
  }
  pdl_launch_dependents();
  if (tid == 0) n_hit[0] = tot.x;
}

// ---------------------------------------------------------------------------
// Histogram-based top-k (the fast path).  The exact bisection emulation needs
// only w, the (k+1)-th largest |s|, and max|s|; both come from a 32768-bin
// histogram of the 15-bit magnitudes.  In the fused decode chain the gate
// kernel fills the histogram in its epilogue (one global atomic per channel),
// so the select kernel below only scans 128 KB and compacts.  It leaves the
// histogram zero for the next call.
constexpr int kHistBins = 32768;

__global__ void __launch_bounds__(256)
topk_hist_kernel(const uint16_t* __restrict__ s, int n, unsigned* __restrict__ hist) {
  pdl_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const unsigned key = s[i] & 0x7FFFu;
    if (key <= 0x7F80u) atomicAdd(&hist[key], 1u);
  }
  pdl_launch_dependents();
}

__global__ void __launch_bounds__(kTopkThreads)
topk_from_hist_kernel(const uint16_t* __restrict__ s, int n, int k, int32_t* __restrict__ idx,
                      unsigned* __restrict__ hist) {
  extern __shared__ __align__(16) uint16_t keys[];
  __shared__ int2 warp_tot[33];
  __shared__ unsigned s_max;
  __shared__ unsigned s_w;
  __shared__ float s_lohi[2];
  const int tid = threadIdx.x;
  if (tid == 0) { s_max = 0; s_w = 0; }
  pdl_wait();
  // Thread tid owns bins [32 tid, 32 tid + 32): counts, then zero them.
  uint4* hv = reinterpret_cast<uint4*>(hist) + tid * 8;
  unsigned c[32];
  int tot_mine = 0;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const uint4 v = hv[q];
    c[4 * q] = v.x; c[4 * q + 1] = v.y; c[4 * q + 2] = v.z; c[4 * q + 3] = v.w;
    tot_mine += v.x + v.y + v.z + v.w;
  }
#pragma unroll
  for (int q = 0; q < 8; ++q) hv[q] = make_uint4(0, 0, 0, 0);
  // Stage |s| for the compaction meanwhile.
  const bool vec = ((reinterpret_cast<uintptr_t>(s) & 15) == 0);
  const int nvec = vec ? n / 8 : 0;
  for (int v = tid; v < nvec; v += kTopkThreads) {
    uint4 r = __ldg(reinterpret_cast<const uint4*>(s) + v);
    r.x &= 0x7FFF7FFFu; r.y &= 0x7FFF7FFFu; r.z &= 0x7FFF7FFFu; r.w &= 0x7FFF7FFFu;
    reinterpret_cast<uint4*>(keys)[v] = r;
  }
  for (int i = nvec * 8 + tid; i < n; i += kTopkThreads) keys[i] = s[i] & 0x7FFF;
  int2 tot;
  const int2 pre = block_excl_scan2(tot_mine, 0, warp_tot, tot);  // also a barrier
  const int nvalid = tot.x;
  const int above = nvalid - pre.x - tot_mine;  // count in bins above my range
  if (tot_mine > 0) {
    int top = 31;
    while (c[top] == 0) --top;
    atomicMax(&s_max, (unsigned)(tid * 32 + top));
  }
  const bool has_w = nvalid >= k + 1;
  if (has_w && above < k + 1 && k + 1 <= above + tot_mine) {
    int run = above;
    for (int b = 31; b >= 0; --b) {
      run += c[b];
      if (run >= k + 1) { s_w = (unsigned)(tid * 32 + b); break; }
    }
  }
  __syncthreads();
  if (tid == 0) {
    const float wv = bf16_bits_to_f32(s_w);
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
  __syncthreads();
  const float lo = s_lohi[0], hi = s_lohi[1];
  const int per = (n + kTopkThreads - 1) / kTopkThreads;
  const int beg = min(n, tid * per), end = min(n, beg + per);
  int ca = 0, cb = 0;
  for (int i = beg; i < end; ++i) {
    const float v = bf16_bits_to_f32(keys[i]);
    ca += (v > hi);
    cb += (v > lo && v <= hi);
  }
  const int2 off = block_excl_scan2(ca, cb, warp_tot, tot);
  int pa = off.x, pb = tot.x + off.y;
  for (int i = beg; i < end; ++i) {
    const float v = bf16_bits_to_f32(keys[i]);
    if (v > hi) { if (pa < k) idx[pa] = i; ++pa; }
    else if (v > lo && v <= hi) { if (pb < k) idx[pb] = i; ++pb; }
  }
  pdl_launch_dependents();
  const int filled = min(k, tot.x + tot.y);
  for (int i = filled + tid; i < k; i += kTopkThreads) idx[i] = 0;
}

int topk_from_hist_launch(const uint16_t* s, int64_t n, int64_t k, int32_t* idx,
                          unsigned* hist, cudaStream_t st) {
  if (n < 1 || n > kTopkMaxN || k < 1 || k > INT32_MAX || !s || !idx || !hist) return DIP_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(hist) & 15) != 0) return DIP_ERR_ARG;
  const size_t smem = (size_t)n * 2;
  cudaError_t e = cudaFuncSetAttribute(topk_from_hist_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return launch_status(e);
  return launch_status(launch(topk_from_hist_kernel, dim3(1), dim3(kTopkThreads), smem, st, s,
                              (int)n, (int)k, idx, hist));
}

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

extern "C" size_t dip_topk_hist_bytes(void) { return kHistBins * sizeof(unsigned); }

extern "C" int dip_topk_select_ws(const dip_bf16* s, int64_t n, int64_t k, int32_t* idx,
                                  void* hist, dip_stream_t stream) {
  if (n < 1 || n > kTopkMaxN || k < 0 || k > INT32_MAX || !s || !hist) return DIP_ERR_ARG;
  if (k == 0) return DIP_OK;
  if (!idx) return DIP_ERR_ARG;
  const int grid = (int)((n + 255) / 256 < 148 ? (n + 255) / 256 : 148);
  int st = launch_status(launch(topk_hist_kernel, dim3(grid), dim3(256), 0, (cudaStream_t)stream,
                                s, (int)n, static_cast<unsigned*>(hist)));
  if (st) return st;
  return topk_from_hist_launch(s, n, k, idx, static_cast<unsigned*>(hist), (cudaStream_t)stream);
}
