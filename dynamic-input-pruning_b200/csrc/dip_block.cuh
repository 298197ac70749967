// dip_block.cuh — block-wide scan and stable compaction helpers.
#pragma once
#include "dip_common.cuh"

namespace dip {

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


// Stable two-tier compaction of the index range [0, n): elements with
// isA(i) go, in index order, to positions [0, nA); elements with isB(i) to
// [nA, nA + nB) (the tiers are disjoint).  Each warp owns one contiguous
// chunk and walks it 32 elements per round, so the positions written by one
// store instruction are consecutive (coalesced), unlike a per-thread run.
// emit(pos, i) is called once per selected element; tot = (nA, nB).
template <class FA, class FB, class EMIT>
__device__ __forceinline__ void block_compact2(int n, FA isA, FB isB, EMIT emit, int2* warp_tot,
                                               int2& tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int chunk = (((n + nw - 1) / nw) + 31) & ~31;
  const int beg = min(n, warp * chunk), end = min(n, beg + chunk);
  int ca = 0, cb = 0;
  for (int base = beg; base < end; base += 32) {
    const int i = base + lane;
    const bool a = i < end && isA(i);
    const bool b = i < end && !a && isB(i);
    ca += __popc(__ballot_sync(0xffffffffu, a));
    cb += __popc(__ballot_sync(0xffffffffu, b));
  }
  const int2 off = block_excl_scan2(lane == 0 ? ca : 0, lane == 0 ? cb : 0, warp_tot, tot);
  int pa = __shfl_sync(0xffffffffu, off.x, 0);
  int pb = tot.x + __shfl_sync(0xffffffffu, off.y, 0);
  const unsigned lt = (1u << lane) - 1u;
  for (int base = beg; base < end; base += 32) {
    const int i = base + lane;
    const bool a = i < end && isA(i);
    const bool b = i < end && !a && isB(i);
    const unsigned ma = __ballot_sync(0xffffffffu, a);
    const unsigned mb = __ballot_sync(0xffffffffu, b);
    if (a) emit(pa + __popc(ma & lt), i);
    if (b) emit(pb + __popc(mb & lt), i);
    pa += __popc(ma);
    pb += __popc(mb);
  }
}


}  // namespace dip
