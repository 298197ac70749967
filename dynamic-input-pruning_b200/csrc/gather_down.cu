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
#include <atomic>

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
  uint4* clear;           // optional: zeroed by the reduction kernel
  int clear_n16;
  GridBar* bar;           // fused reduction: grid barrier words (zero on first use)
  unsigned* err;
  uint16_t* y;            // fused reduction outputs
  float* y_f32;
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
                       uint16_t* __restrict__ y, float* __restrict__ y_f32,
                       uint4* __restrict__ clear, int clear_n16) {
  __shared__ float red[8][33];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int o = blockIdx.x * 32 + lane;
  pdl_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < clear_n16; i += gridDim.x * blockDim.x)
    clear[i] = make_uint4(0, 0, 0, 0);
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

// ---------------------------------------------------------------------------
// Tensor-core variant (used when out % 1024 == 0 and out <= 5120).
//
//   y[o] = sum_c q[c,o] * (h_c * s[c, o/128])
//
// is computed as D[o][n] = sum_c A[o][c] * B[c][n] with mma.sync m16n8k16:
// A = the int4 weights (outputs on M, channels on K) converted in registers
// to bf16 q+136 (magic number, see nib8_biased_bf16x2); two channel rows are
// interleaved byte-wise with one PRMT so each 32-bit register holds the same
// output of two channels.  B holds hs = h*s split exactly into bf16 hi + lo:
// even columns carry hi, odd columns lo, so D[o][2t] + D[o][2t+1] is the sum
// over channels of q*hs (+136 * sum hs, removed with the column sums at the
// end).  The tensor core therefore does both the multiply-adds and the
// channel reduction; a lane spends ~1.2 instructions per weight nibble.
//
// Grid: 2 output halves x S channel slices.  A CTA has out/256 warps; warp w
// owns output group w of its half (64 bytes of every selected row, 8
// accumulator m-tiles = 32 fp32 registers) and streams its own bytes with
// asynchronous 16-byte copies (cp.async.cg; the warp's 64 bytes of 16 rows
// are 64 chunks, two per lane) plus the 4-byte scale pairs through a private
// 6-tile shared-memory pipeline, so no block-level synchronisation is needed
// after the prologue.  (16-byte .cg copies measured 6.7 TB/s on B200 in this
// access pattern; .ca copies 4.2 TB/s.)
constexpr int kDmChan = 16;       // channels per tile (one MMA K step)
constexpr int kDmSlices = 74;     // channel slices; 2 x 74 = 148 CTAs
constexpr int kDmDepth = 6;       // tiles in flight per warp
constexpr int kDmRowPitch = 80;   // 64 bytes of a row + pad (conflict-free 8-byte reads)
constexpr int kDmSlotW = kDmChan * kDmRowPitch;
constexpr int kDmSlotBytes = kDmSlotW + kDmChan * 4;  // weights + scale pairs

__device__ __forceinline__ void cp_async16g(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit_d() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_depth() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(kDmDepth - 1) : "memory");
}

struct DmGeom {
  int ring_off, rows_off, h_off, total;
};
__host__ __device__ inline DmGeom dm_geom(int nwarps, int max_slice) {
  DmGeom g;
  g.ring_off = 0;
  g.rows_off = nwarps * kDmDepth * kDmSlotBytes;
  g.h_off = g.rows_off + max_slice * 16;  // two pointers per channel
  g.total = g.h_off + max_slice * 4;
  return g;
}

template <int MODE, bool FUSED>
__global__ void __launch_bounds__(640, 1)
down_mma_kernel(const DownParams p, int max_slice) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int out = p.out_features;
  const int nwarps = out / 256;
  const DmGeom geo = dm_geom(nwarps, max_slice);
  const uint8_t** rowq = reinterpret_cast<const uint8_t**>(smem + geo.rows_off);
  const uint16_t** rows_sc = reinterpret_cast<const uint16_t**>(smem + geo.rows_off) + max_slice;
  float* hsm = reinterpret_cast<float*>(smem + geo.h_off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = blockIdx.x & 1, slice = blockIdx.x >> 1, nslices = gridDim.x >> 1;

  pdl_wait();
  int k = p.k;
  if (p.count) k = min(k, *p.count);
  const int j0 = (int)((int64_t)k * slice / nslices);
  const int j1 = (int)((int64_t)k * (slice + 1) / nslices);
  const int nrow = j1 - j0;
  for (int j = threadIdx.x; j < nrow; j += blockDim.x) {
    const uint8_t* qw;
    const uint16_t* sc;
    const bool okr = down_row<MODE>(p, j0 + j, qw, sc);
    rowq[j] = qw;
    rows_sc[j] = sc;
    hsm[j] = okr ? bf16_bits_to_f32(p.h[j0 + j]) : 0.f;
  }
  __syncthreads();

  const int gq = lane >> 2, tq = lane & 3;
  const int og = half * nwarps + warp;  // global output group of this warp
  const int seg_off = half * (out / 4) + warp * 64;  // this warp's 64 bytes of a row
  uint8_t* ring = smem + geo.ring_off + warp * kDmDepth * kDmSlotBytes;
  const int ntile = (nrow + kDmChan - 1) / kDmChan;

  auto issue = [&](int i) {
    if (i < ntile) {
      uint8_t* slot = ring + (i % kDmDepth) * kDmSlotBytes;
      const int c0 = i * kDmChan;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int ch = lane + 32 * h2;  // 64 chunks: row ch/4, 16-byte part ch%4
        const int r = ch >> 2, part = ch & 3;
        const int c = min(c0 + r, nrow - 1);
        cp_async16g(slot + r * kDmRowPitch + part * 16, rowq[c] + seg_off + part * 16);
      }
      if (lane < kDmChan) {
        const int c = min(c0 + lane, nrow - 1);
        cp_async4(slot + kDmSlotW + lane * 4, rows_sc[c] + (og & ~1));
      }
    }
    cp_async_commit_d();
  };
#pragma unroll
  for (int i = 0; i < kDmDepth - 1; ++i) issue(i);

  const int tpair = lane & 7, twhich = (lane >> 3) & 1;
  float acc[8][4];
#pragma unroll
  for (int m = 0; m < 8; ++m) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.f;
  float colsum = 0.f;
  for (int i = 0; i < ntile; ++i) {
    issue(i + kDmDepth - 1);
    cp_async_wait_depth();
    __syncwarp();
    const uint8_t* slot = ring + (i % kDmDepth) * kDmSlotBytes;
    const int c0 = i * kDmChan;
    // B values: lane (pair, which) packs channels 2*pair, 2*pair+1 as bf16x2
    // of hi (which 0) or lo (which 1) of h*s.
    uint32_t bval = 0;
    if (lane < 16) {
      float v2[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int c = 2 * tpair + e;
        float hs = 0.f;
        if (c0 + c < nrow) {
          const uint16_t* scp = reinterpret_cast<const uint16_t*>(slot + kDmSlotW + c * 4);
          hs = hsm[c0 + c] * bf16_bits_to_f32(scp[og & 1]);
        }
        const float hi = round_bf16(hs);
        v2[e] = twhich ? round_bf16(hs - hi) : hi;
      }
      colsum += v2[0] + v2[1];
      bval = (uint32_t)f32_to_bf16_bits(v2[0]) | ((uint32_t)f32_to_bf16_bits(v2[1]) << 16);
    }
    const int src = (gq & 1) * 8;
    const uint32_t b0 = __shfl_sync(0xffffffffu, bval, src + tq);
    const uint32_t b1 = __shfl_sync(0xffffffffu, bval, src + tq + 4);
    // rows 2t, 2t+1, 2t+8, 2t+9 of the tile, bytes [8g, 8g+8) of the segment
    const uint2 ra = *reinterpret_cast<const uint2*>(slot + (2 * tq) * kDmRowPitch + gq * 8);
    const uint2 rb = *reinterpret_cast<const uint2*>(slot + (2 * tq + 1) * kDmRowPitch + gq * 8);
    const uint2 rc = *reinterpret_cast<const uint2*>(slot + (2 * tq + 8) * kDmRowPitch + gq * 8);
    const uint2 rd = *reinterpret_cast<const uint2*>(slot + (2 * tq + 9) * kDmRowPitch + gq * 8);
    const uint32_t pab[4] = {__byte_perm(ra.x, rb.x, 0x5410), __byte_perm(ra.x, rb.x, 0x7632),
                             __byte_perm(ra.y, rb.y, 0x5410), __byte_perm(ra.y, rb.y, 0x7632)};
    const uint32_t pcd[4] = {__byte_perm(rc.x, rd.x, 0x5410), __byte_perm(rc.x, rd.x, 0x7632),
                             __byte_perm(rc.y, rd.y, 0x5410), __byte_perm(rc.y, rd.y, 0x7632)};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t xa[4], xc[4];
      nib8_biased_bf16x2(pab[q], xa);
      nib8_biased_bf16x2(pcd[q], xc);
      // m-tile 2q+e: byte 2q+e of the lane's 8 (low nibble -> row g, high -> g+8)
      const uint32_t a0[4] = {xa[0], xa[1], xc[0], xc[1]};
      const uint32_t a1[4] = {xa[2], xa[3], xc[2], xc[3]};
      mma_bf16_16816(acc[2 * q], a0, b0, b1);
      mma_bf16_16816(acc[2 * q + 1], a1, b0, b1);
    }
    __syncwarp();  // the slot is refilled by the next iteration's copies
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");
  pdl_launch_dependents();
  // Column sums of hi (lanes 0..7) and lo (lanes 8..15) -> their total.
#pragma unroll
  for (int o = 1; o < 16; o <<= 1) colsum += __shfl_xor_sync(0xffffffffu, colsum, o);
  const float bias = kNibbleBias * __shfl_sync(0xffffffffu, colsum, 0);
  if (tq == 0) {
    // lane g holds outputs 16g .. 16g+15 of the group: m-tile m -> byte m,
    // row g -> low nibble (even output), row g+8 -> high nibble (odd).
    float* dst = p.partial + (size_t)slice * out + og * kGroup + gq * 16;
    float v[16];
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      v[2 * m] = acc[m][0] + acc[m][1] - bias;
      v[2 * m + 1] = acc[m][2] + acc[m][3] - bias;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q)
      reinterpret_cast<float4*>(dst)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2],
                                                      v[4 * q + 3]);
  }
  if (FUSED) {
    // All partial vectors written -> every CTA sums a slice of the outputs
    // over the slices in a fixed order (8 threads per output, fixed tree).
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.clear_n16;
         i += gridDim.x * blockDim.x)
      p.clear[i] = make_uint4(0, 0, 0, 0);
    grid_sync(p.bar, p.err);
    const int per = (out + gridDim.x - 1) / gridDim.x;
    const int o0 = blockIdx.x * per;
    const int oi = threadIdx.x >> 3, part = threadIdx.x & 7;
    for (int ob = 0; ob < per; ob += blockDim.x >> 3) {
      const int o = o0 + ob + oi;
      float acc = 0.f;
      if (ob + oi < per && o < out)
        for (int c = part; c < nslices; c += 8) acc += p.partial[(size_t)c * out + o];
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      acc += __shfl_xor_sync(0xffffffffu, acc, 4);
      if (part == 0 && ob + oi < per && o < out) {
        if (p.y) p.y[o] = f32_to_bf16_bits(acc);
        if (p.y_f32) p.y_f32[o] = acc;
      }
    }
  }
}

static bool dm_ok(const DownParams& p) {
  const int out = p.out_features;
  if (out % 1024 != 0 || out / 256 > 20) return false;
  if ((reinterpret_cast<uintptr_t>(p.sc0) & 15) != 0) return false;
  if (p.qw1 && (reinterpret_cast<uintptr_t>(p.sc1) & 15) != 0) return false;
  return true;
}

size_t down_workspace_bytes(int64_t out) { return (size_t)kDownCtas * out * sizeof(float); }

bool down_shape_ok(int64_t out) { return out > 0 && out % kGroup == 0 && out / 32 <= 640; }

template <int MODE>
int launch_down(DownParams p, uint16_t* y, float* y_f32, void* ws, size_t ws_bytes,
                cudaStream_t st) {
  const int out = p.out_features;
  if (ws_bytes < down_workspace_bytes(out) || !ws) return DIP_ERR_WORKSPACE;
  p.partial = reinterpret_cast<float*>(ws);
  if (dm_ok(p) && !force_simple_gemv() && p.k > 0) {
    const int nsl = p.k < kDmSlices ? p.k : kDmSlices;
    const int max_slice = (p.k + nsl - 1) / nsl + 1;
    const DmGeom geo = dm_geom(out / 256, max_slice);
    if (geo.total <= 220 * 1024) {
      if (p.bar && 2 * nsl <= num_sms()) {
        auto kf = down_mma_kernel<MODE, true>;
        cudaError_t e = cudaFuncSetAttribute(kf, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             geo.total);
        if (e != cudaSuccess) return launch_status(e);
        p.y = y;
        p.y_f32 = y_f32;
        return launch_status(launch_coop(kf, dim3(2 * nsl), dim3(out / 256 * 32),
                                         (size_t)geo.total, st, p, max_slice));
      }
      auto kern = down_mma_kernel<MODE, false>;
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           geo.total);
      if (e != cudaSuccess) return launch_status(e);
      int st1 = launch_status(launch(kern, dim3(2 * nsl), dim3(out / 256 * 32), (size_t)geo.total,
                                     st, p, max_slice));
      if (st1 != DIP_OK) return st1;
      return launch_status(launch(reduce_partials_kernel, dim3((out + 31) / 32), dim3(256), 0,
                                  st, (const float*)p.partial, nsl, out, y, y_f32, p.clear,
                                  p.clear_n16));
    }
  }
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
                              (const float*)p.partial, nparts, out, y, y_f32, p.clear,
                              p.clear_n16));
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
                                (int)out_features, y, (float*)nullptr, (uint4*)nullptr, 0));
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

// ---------------------------------------------------------------------------
// Allocation-free down projection.
//
// Some callers cannot allocate device memory at call time: code running
// inside another framework's memory pool or under a fixed memory budget,
// plugins that are handed only input and output buffers, and C / FFI callers
// without a CUDA allocator of their own.  For them this entry point keeps the
// per-CTA partial sums in a library-owned static device array instead of a
// caller workspace.  The array lives in every GPU that loads the library
// until the process exits.
constexpr int64_t kNoAllocMaxOut = 8192;  // largest supported out_features
static __device__ __align__(256) float g_noalloc_partials[kDownCtas * kNoAllocMaxOut];

// Device address of g_noalloc_partials on the current device.  In host code
// the array's name is only a host-side stand-in, so the real address is
// looked up once per device (with that device current) and cached in an
// atomic slot (concurrent first calls from several host threads store the
// same value).  The cached address is valid while the device's primary
// context lives; after cudaDeviceReset the library must be reloaded.
static float* noalloc_partials_ptr() {
  static std::atomic<float*> cache[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  float* p = cache[dev].load(std::memory_order_acquire);
  if (!p) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_partials) != cudaSuccess) return nullptr;
    p = static_cast<float*>(ptr);
    cache[dev].store(p, std::memory_order_release);
  }
  return p;
}

extern "C" int dip_int4_gather_down_noalloc(const int8_t* down_t, const dip_bf16* scales,
                                            int64_t n_rows, const dip_bf16* h,
                                            const int32_t* idx, int64_t k, int64_t out_features,
                                            dip_bf16* y, dip_stream_t stream) {
  if (out_features > kNoAllocMaxOut) return DIP_ERR_UNSUPPORTED;
  float* scratch = noalloc_partials_ptr();
  if (!scratch) {
    launch_status(cudaGetLastError());  // records the CUDA error text
    return DIP_ERR_CUDA;
  }
  return dip_int4_gather_down(down_t, scales, n_rows, h, idx, k, out_features, scratch,
                              sizeof(g_noalloc_partials), y, stream);
}

namespace dip {
int gather_down_clear(const int8_t* down_t, const uint16_t* scales, int64_t n_rows,
                      const uint16_t* h, const int32_t* idx, int64_t k, int64_t out_features,
                      void* workspace, size_t workspace_bytes, uint16_t* y, void* clear,
                      size_t clear_bytes, GridBar* bar, cudaStream_t stream) {
  if (k <= 0 || k > INT32_MAX || n_rows <= 0 || !down_shape_ok(out_features) || !y || !down_t ||
      !scales || !h || !idx || !al16(down_t) || (clear_bytes % 16) != 0)
    return DIP_ERR_ARG;
  DownParams p = {};
  p.qw0 = reinterpret_cast<const uint8_t*>(down_t);
  p.sc0 = scales;
  p.n0 = n_rows;
  p.h = h;
  p.idx = idx;
  p.clear = static_cast<uint4*>(clear);
  p.clear_n16 = (int)(clear_bytes / 16);
  p.bar = bar;
  p.err = error_word_ptr();
  if (bar && !p.err) return DIP_ERR_CUDA;
  p.k = (int)k;
  p.out_features = (int)out_features;
  return launch_down<DROW_GATHER>(p, y, nullptr, workspace, workspace_bytes, stream);
}
}  // namespace dip
