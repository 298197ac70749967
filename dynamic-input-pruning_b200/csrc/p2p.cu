// p2p.cu — the two exchanges of the tensor-parallel DIP layer (rank r of P
// owns channels [r I/P, (r+1) I/P)) over peer memory instead of NCCL:
//
//   gather:  every rank stores its g slice into every rank's full g buffer,
//            then publishes a flag; each rank waits for all P flags.
//   reduce:  every rank stores its fp32 down partial [H] into slot r of every
//            rank's [P][H] buffer, publishes a flag, waits for all P flags and
//            sums the P slots in rank order (identical on every rank, and
//            deterministic).
//
// Each rank owns a mailbox allocated once (dip_p2p_alloc; its IPC handle is
// shared with the peers, which map it with dip_ipc_open over NVLink):
//   [0, 256)           flags: gather[8], reduce[8] (u64, the writer's epoch + 1)
//   [256, 512)         epochs: this rank's gather / reduce call counts (u64)
//   [512, ...)         g buffer [I] bf16, then the partials [P][H] fp32
// The flag written is the writer's epoch + 1, so the same mailbox serves every
// call without resets and the exchange replays correctly from a CUDA graph
// (the epochs live in device memory).  A rank cannot overwrite a peer's g
// buffer before the peer has used it: its next gather follows its reduce, which
// waits for that peer's partial, written after the peer's top-k.  Likewise for
// the partial slots.  Waits are bounded: on timeout the library's error word
// is flagged and the kernel returns.
#include <cstring>
#include <map>
#include <mutex>

#include "dip_common.cuh"

namespace dip {

// Host-side record of the device ranges this library allocated for peer
// exchange or mapped from a peer: base -> size.
static std::mutex g_reg_mu;
static std::map<uintptr_t, size_t> g_reg;

static void reg_add(const void* base, size_t bytes) {
  std::lock_guard<std::mutex> lk(g_reg_mu);
  g_reg[reinterpret_cast<uintptr_t>(base)] = bytes;
}
static void reg_del(const void* base) {
  std::lock_guard<std::mutex> lk(g_reg_mu);
  g_reg.erase(reinterpret_cast<uintptr_t>(base));
}
size_t p2p_registered_bytes(const void* p) {
  const uintptr_t v = reinterpret_cast<uintptr_t>(p);
  std::lock_guard<std::mutex> lk(g_reg_mu);
  auto it = g_reg.upper_bound(v);
  if (it == g_reg.begin()) return 0;
  --it;
  const uintptr_t end = it->first + it->second;
  return v < end ? (size_t)(end - v) : 0;
}

// Size of the allocation an IPC mapping covers, from the driver
// (cuMemGetAddressRange, fetched through the runtime's entry-point query so
// the library needs no link against libcuda).
static size_t mapped_range_bytes(void* ptr) {
  using Fn = int (*)(unsigned long long*, size_t*, unsigned long long);
  static Fn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<Fn>(f);
  });
  if (!fn) return 0;
  unsigned long long base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<unsigned long long>(ptr)) != 0) return 0;
  const unsigned long long v = reinterpret_cast<unsigned long long>(ptr);
  return v >= base && v < base + size ? (size_t)(base + size - v) : 0;
}

constexpr int kP2PMaxRanks = 8;
constexpr size_t kP2PHeader = 512;

struct P2PArgs {
  int rank, world;
  uint8_t* mb[kP2PMaxRanks];  // per rank q: its mailbox, as this rank maps it
  int64_t n_local;            // gather: values per rank
  int64_t inter;              // g buffer length
  int64_t hidden;             // reduce: partial length
  const uint16_t* g_local;
  const float* partial;
  uint16_t* y;
  unsigned* err;
};

__device__ __forceinline__ unsigned long long* p2p_flags(uint8_t* mb) {
  return reinterpret_cast<unsigned long long*>(mb);
}
__device__ __forceinline__ unsigned long long* p2p_epochs(uint8_t* mb) {
  return reinterpret_cast<unsigned long long*>(mb + 256);
}
__device__ __forceinline__ uint16_t* p2p_g(uint8_t* mb) {
  return reinterpret_cast<uint16_t*>(mb + kP2PHeader);
}
__device__ __forceinline__ float* p2p_part(uint8_t* mb, int64_t inter) {
  return reinterpret_cast<float*>(mb + kP2PHeader + ((inter * 2 + 255) & ~int64_t(255)));
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;\n" ::"l"(p), "l"(v) : "memory");
}

// which = 0: gather, 1: reduce.  One CTA: 16-byte stores to every rank's
// mailbox, a CTA barrier, then thread q < P publishes to rank q and waits for
// rank q's flag.
__global__ void __launch_bounds__(1024) p2p_exchange_kernel(const P2PArgs a, int which) {
  pdl_wait();
  const int tid = threadIdx.x, nt = blockDim.x;
  uint8_t* mine = a.mb[a.rank];
  const unsigned long long epoch = p2p_epochs(mine)[which];
  if (which == 0) {
    const int64_t n16 = a.n_local / 8;  // n_local % 8 == 0 (host check)
    const uint4* src = reinterpret_cast<const uint4*>(a.g_local);
    for (int64_t i = tid; i < n16 * a.world; i += nt) {
      const int q = (int)(i / n16);
      const int64_t e = i % n16;
      uint4* dst = reinterpret_cast<uint4*>(p2p_g(a.mb[q]) + (int64_t)a.rank * a.n_local);
      dst[e] = src[e];
    }
  } else {
    const int64_t n4 = a.hidden / 4;
    const float4* src = reinterpret_cast<const float4*>(a.partial);
    for (int64_t i = tid; i < n4 * a.world; i += nt) {
      const int q = (int)(i / n4);
      const int64_t e = i % n4;
      float4* dst = reinterpret_cast<float4*>(p2p_part(a.mb[q], a.inter) + (int64_t)a.rank * a.hidden);
      dst[e] = src[e];
    }
  }
  __syncthreads();
  if (tid < a.world) {
    // every thread's stores (ordered by the barrier) before this release
    __threadfence_system();
    st_release_sys(p2p_flags(a.mb[tid]) + which * kP2PMaxRanks + a.rank, epoch + 1);
    const unsigned long long* f = p2p_flags(mine) + which * kP2PMaxRanks + tid;
    bool ok = false;
    for (uint32_t it = 0, lim = spin_limit(a.err); it < lim && !ok; ++it) ok = ld_acquire_sys(f) >= epoch + 1;
    if (!ok) atomicOr(a.err, kErrTimeout);
  }
  __syncthreads();
  if (which == 1) {
    // fixed-order sum of the P partials -> y
    const float* part = p2p_part(mine, a.inter);
    for (int64_t i = tid; i < a.hidden; i += nt) {
      float s = 0.f;
      for (int q = 0; q < a.world; ++q) s += part[(int64_t)q * a.hidden + i];
      a.y[i] = f32_to_bf16_bits(s);
    }
  }
  if (tid == 0) p2p_epochs(mine)[which] = epoch + 1;
}

}  // namespace dip

using namespace dip;

extern "C" size_t dip_p2p_mailbox_bytes(int64_t inter, int64_t hidden, int64_t world) {
  if (inter <= 0 || hidden <= 0 || world <= 0 || world > kP2PMaxRanks) return 0;
  return kP2PHeader + (((size_t)inter * 2 + 255) & ~size_t(255)) + (size_t)world * hidden * 4;
}

extern "C" int dip_p2p_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return DIP_ERR_ARG;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return launch_status(e);
  e = cudaMemset(*ptr, 0, bytes);
  if (e != cudaSuccess) return launch_status(e);
  reg_add(*ptr, bytes);
  return DIP_OK;
}

extern "C" int dip_p2p_free(void* ptr) {
  reg_del(ptr);
  return launch_status(cudaFree(ptr));
}

extern "C" int dip_ipc_handle(const void* ptr, void* handle64) {
  if (!ptr || !handle64) return DIP_ERR_ARG;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess) return launch_status(e);
  static_assert(sizeof(h) == 64, "IPC handles are 64 bytes");
  memcpy(handle64, &h, sizeof(h));
  return DIP_OK;
}

extern "C" int dip_ipc_open(const void* handle64, void** ptr) {
  if (!handle64 || !ptr) return DIP_ERR_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  const int st = launch_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  if (st != DIP_OK) return st;
  const size_t n = mapped_range_bytes(*ptr);
  if (n == 0) {
    cudaIpcCloseMemHandle(*ptr);
    *ptr = nullptr;
    return DIP_ERR_CUDA;
  }
  reg_add(*ptr, n);
  return DIP_OK;
}

extern "C" int dip_ipc_close(void* ptr) {
  reg_del(ptr);
  return launch_status(cudaIpcCloseMemHandle(ptr));
}

static int p2p_launch(int which, int rank, int world, void* const* mailboxes, int64_t n_local,
                      int64_t inter, int64_t hidden, const dip_bf16* g_local, const float* partial,
                      dip_bf16* y, dip_stream_t stream) {
  if (world < 1 || world > kP2PMaxRanks || rank < 0 || rank >= world || !mailboxes) return DIP_ERR_ARG;
  if (inter <= 0 || hidden <= 0 || inter % world || n_local != inter / world) return DIP_ERR_ARG;
  const size_t need = dip_p2p_mailbox_bytes(inter, hidden, world);
  P2PArgs a = {};
  a.rank = rank;
  a.world = world;
  for (int q = 0; q < world; ++q) {
    if (!mailboxes[q] || (reinterpret_cast<uintptr_t>(mailboxes[q]) & 255)) return DIP_ERR_ARG;
    // every mailbox receives stores from this kernel: each must be a range
    // this library allocated or mapped, large enough for this shape
    if (p2p_registered_bytes(mailboxes[q]) < need) return DIP_ERR_ARG;
    a.mb[q] = static_cast<uint8_t*>(mailboxes[q]);
  }
  a.n_local = n_local;
  a.inter = inter;
  a.hidden = hidden;
  a.g_local = g_local;
  a.partial = partial;
  a.y = y;
  a.err = error_word_ptr();
  if (!a.err) return DIP_ERR_CUDA;
  return launch_status(launch(p2p_exchange_kernel, dim3(1), dim3(1024), 0, (cudaStream_t)stream, a, which));
}

extern "C" int dip_p2p_gather(int rank, int world, void* const* mailboxes, const dip_bf16* g_local,
                              int64_t n_local, int64_t hidden, dip_stream_t stream) {
  if (!g_local || n_local <= 0 || n_local % 8 || (reinterpret_cast<uintptr_t>(g_local) & 15))
    return DIP_ERR_ARG;
  return p2p_launch(0, rank, world, mailboxes, n_local, n_local * world, hidden, g_local, nullptr,
                    nullptr, stream);
}

extern "C" int dip_p2p_reduce(int rank, int world, void* const* mailboxes, const float* partial,
                              int64_t inter, int64_t hidden, dip_bf16* y, dip_stream_t stream) {
  if (!partial || !y || hidden <= 0 || hidden % 4 || (reinterpret_cast<uintptr_t>(partial) & 15))
    return DIP_ERR_ARG;
  return p2p_launch(1, rank, world, mailboxes, inter / world, inter, hidden, nullptr, partial, y,
                    stream);
}
