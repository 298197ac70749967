// dip_common.cuh — shared device helpers for the sm_100a DIP kernels.
//
// Weight format (identical to the reference's, scripts/quantize.py:32-64 and
// qlinear.py:28-64): a row of `in` int4 values is `in/2` bytes, two signed
// (two's complement) nibbles per byte, low nibble = even column; one bf16
// scale per 128 consecutive columns.  w = q * s.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "../../include/dip_b200.h"

namespace dip {

constexpr int kGroup = 128;          // quantisation group (columns per scale)
constexpr int kGroupBytes = kGroup / 2;

// ---------------------------------------------------------------------------
// bf16 <-> float on raw 16-bit patterns (the C-ABI passes bf16 as uint16_t).
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) {
  return __uint_as_float(b << 16);
}
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  __nv_bfloat16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}
__device__ __forceinline__ float round_bf16(float f) {
  return bf16_bits_to_f32(f32_to_bf16_bits(f));
}

// ---------------------------------------------------------------------------
// int4 -> bf16 in-register conversion (the "magic number" technique: place
// an integer in the low mantissa bits of a float whose exponent makes the
// mantissa step exactly 1, here bf16 128.0 = 0x4300).  The nibble is stored
// in two's complement; XOR with 8 turns it into offset binary, so each
// 16-bit lane below holds exactly  128 + (q + 8) = q + 136  with q in [-8,7].
// Lane pairing: out[p] = (nibble p, nibble p+4) for p = 0..3.
constexpr float kNibbleBias = 136.0f;
// (a & 0x000F000F) ^ 0x43084308 as a single LOP3 (lookup table 0x6a).
__device__ __forceinline__ uint32_t nib_lop3(uint32_t a) {
  uint32_t d;
  asm("lop3.b32 %0, %1, 0x000F000F, 0x43084308, 0x6a;\n" : "=r"(d) : "r"(a));
  return d;
}
__device__ __forceinline__ void nib8_biased_bf16x2(uint32_t w, uint32_t (&o)[4]) {
  o[0] = nib_lop3(w);
  o[1] = nib_lop3(w >> 4);
  o[2] = nib_lop3(w >> 8);
  o[3] = nib_lop3(w >> 12);
}

// fp16 variant for the GEMV phases: fp16 has 10 mantissa bits, so the
// nibbles at bits 4-7 fit without a shift: 0x6400 = 1024.0 (step 1), so
//   (w & 0x000F000F) ^ 0x64086408 = 1024 + (q + 8)        = q + 1032
//   (w & 0x00F000F0) ^ 0x64806480 = 1024 + 16 (q + 8)     = 16 (q + 72)
// and one shift by 8 serves nibbles 2, 3, 6, 7: 5 ALU instructions per 8
// weights instead of 7 (plus two sub.f16x2 on the FMA pipe, below).  Pairing as nib8_biased_bf16x2: out[p] = (nibble p,
// nibble p + 4); out[1] and out[3] carry the factor 16.
constexpr float kNibbleBias16Hi = 72.0f;
__device__ __forceinline__ uint32_t nib_lop3_f16lo(uint32_t a) {
  uint32_t d;
  asm("lop3.b32 %0, %1, 0x000F000F, 0x64086408, 0x6a;\n" : "=r"(d) : "r"(a));
  return d;
}
__device__ __forceinline__ uint32_t nib_lop3_f16hi(uint32_t a) {
  uint32_t d;
  asm("lop3.b32 %0, %1, 0x00F000F0, 0x64806480, 0x6a;\n" : "=r"(d) : "r"(a));
  return d;
}
// The low-nibble outputs then have 1032 subtracted exactly (one sub.f16x2
// each, on the FMA pipe): out[0] and out[2] hold q itself, so no large bias
// has to cancel after the tensor core's fp32 accumulation; out[1] and out[3]
// keep 16 (q + 72).
__device__ __forceinline__ uint32_t sub_f16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;\n" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ void nib8_biased_f16x2(uint32_t w, uint32_t (&o)[4]) {
  const uint32_t t = w >> 8;
  const uint32_t k1032 = 0x64086408u;  // (1032.0, 1032.0) in fp16
  o[0] = sub_f16x2(nib_lop3_f16lo(w), k1032);
  o[1] = nib_lop3_f16hi(w);
  o[2] = sub_f16x2(nib_lop3_f16lo(t), k1032);
  o[3] = nib_lop3_f16hi(t);
}
// Warp-level MMA m16n8k16, fp16 x fp16 -> fp32.
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                              uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Same idea in fp32: 2^23 = 0x4B000000 has a mantissa step of 1, so
// (nibble bits << 4j) | 0x4B000000 == 2^23 + u*16^j exactly for bit
// positions below 23.
constexpr uint32_t kF32Magic = 0x4B000000u;

// Warp-level MMA m16n8k16, bf16 x bf16 -> fp32 (legacy tensor path; used as
// the multiply-accumulate engine of the batch-1 GEMVs).
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Streaming 128-bit load that bypasses L1 allocation (weights are read once).
__device__ __forceinline__ uint4 ldg_stream_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint16_t ldg_u16(const uint16_t* p) {
  return __ldg(reinterpret_cast<const unsigned short*>(p));
}

// Programmatic dependent launch (PDL).  A kernel launched with the
// programmatic-serialisation attribute may start before its predecessor
// finishes; it must call pdl_wait() before touching the predecessor's
// outputs.  pdl_launch_dependents() lets the successor start early.  Both are
// no-ops when the kernel was launched without the attribute.
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
}
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

__device__ __forceinline__ float silu_f32(float v) {
  return v / (1.0f + expf(-v));
}

// ---------------------------------------------------------------------------
// Host side helpers.
int launch_status(cudaError_t e);

// Whether kernels launched through the C-ABI use programmatic dependent
// launch (set with dip_set_pdl; default on).
bool pdl_enabled();

template <typename Kernel, typename... Args>
cudaError_t launch(Kernel k, dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                   Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

// As launch(), additionally asking for a cooperative launch (all CTAs
// resident at once; the launch fails instead of running otherwise).
template <typename Kernel, typename... Args>
cudaError_t launch_coop(Kernel k, dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                        Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

int num_sms();

// Words of a grid-wide barrier (see grid_sync).
// The arrival counter and the generation word sit on separate 128-byte lines
// so that the CTAs polling the generation do not contend with the arrivals.
struct GridBar {
  unsigned count;
  unsigned pad0[31];
  unsigned gen;
  unsigned pad1[31];
};
static_assert(sizeof(GridBar) == 256, "grid barrier words occupy 256 bytes of workspace");

// Test switch: route the GEMV family through the simple (non-ring) kernel.
bool force_simple_gemv();

// Bytes from `p` to the end of a device allocation this library made with
// dip_p2p_alloc or mapped with dip_ipc_open (0 when `p` lies in neither):
// the bound every peer-memory store of an exchange is checked against.
size_t p2p_registered_bytes(const void* p);

// Device address of the library's error word on the current device (looked
// up once per device with cudaGetSymbolAddress); nullptr on failure.
unsigned* error_word_ptr();

int gemv_silu_hist(const int8_t* qweight, const uint16_t* scales, const uint16_t* x,
                   uint16_t* out, int64_t rows, int64_t in_features, unsigned* hist,
                   cudaStream_t stream);
// Top-k scratch: fine histogram [32768], coarse histogram [256], look-back words.
constexpr int kTopkHistBins = 32768;
size_t topk_scratch_bytes();
int topk_compact_launch(const uint16_t* s, int64_t n, int64_t k, int32_t* idx, unsigned* scratch,
                        cudaStream_t st);
// Gathered down projection that also clears `clear_bytes` of `clear` (16-byte
// multiple) in its reduction kernel.
int gather_down_clear(const int8_t* down_t, const uint16_t* scales, int64_t n_rows,
                      const uint16_t* h, const int32_t* idx, int64_t k, int64_t out_features,
                      void* workspace, size_t workspace_bytes, uint16_t* y, void* clear,
                      size_t clear_bytes, GridBar* bar, cudaStream_t stream);

}  // namespace dip

namespace dip {
// ---------------------------------------------------------------------------
// mbarrier + bulk-copy (TMA, non-tensor, copies into this CTA only) helpers.  Every wait
// is bounded: after kSpinLimit polls it ORs an error code into the device
// error word (a kernel argument, see error_word_ptr) and reports failure
// instead of hanging.
#ifndef DIP_SPIN_LIMIT
#define DIP_SPIN_LIMIT (1u << 24)
#endif
constexpr uint32_t kSpinLimit = DIP_SPIN_LIMIT;
constexpr unsigned kErrTimeout = 1u;
// `err` points at the library's device control block (error_word_ptr):
// word 0 holds the error bits, word 1 the poll limit of the bounded waits
// (0: kSpinLimit; set with dip_set_spin_limit).
__device__ __forceinline__ uint32_t spin_limit(const unsigned* err) {
  const unsigned v = err ? *reinterpret_cast<const volatile unsigned*>(err + 1) : 0u;
  return v ? v : kSpinLimit;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait; returns false (and flags the error) on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned* err) {
  for (uint32_t i = 0, lim = spin_limit(err); i < lim; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  atomicOr(err, kErrTimeout);
  return false;
}
// Global -> shared bulk copy completing on an mbarrier (size % 16 == 0,
// both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Grid-wide barrier (declared above) for a grid whose CTAs are all resident at once (one CTA
// per SM, grid <= SM count, launched cooperatively).  Sense-reversing: the
// last CTA to arrive resets the count and advances the generation, so the two
// words can be reused by any later launch, whatever its grid size; they must
// be zero before the first use.  The wait is bounded: on timeout the error
// word is flagged and the CTA continues (its results are then invalid).
__device__ __forceinline__ void grid_sync(GridBar* b, unsigned* err) {
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned g0;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(g0) : "l"(&b->gen) : "memory");
    __threadfence();
    const unsigned nb = gridDim.x * gridDim.y * gridDim.z;
    if (atomicAdd(&b->count, 1u) == nb - 1) {
      atomicExch(&b->count, 0u);
      __threadfence();
      atomicAdd(&b->gen, 1u);
    } else {
      bool done = false;
      for (uint32_t it = 0, lim = spin_limit(err); it < lim && !done; ++it) {
        unsigned g;
        asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];\n" : "=r"(g) : "l"(&b->gen) : "memory");
        done = (g != g0);
      }
      asm volatile("fence.acq_rel.gpu;\n" ::: "memory");
      if (!done) atomicOr(err, kErrTimeout);
    }
    __threadfence();
  }
  __syncthreads();
}

// Named barrier for a subset of warps (id 1..15).
__device__ __forceinline__ void named_bar(int id, int threads) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(threads) : "memory");
}
}  // namespace dip
