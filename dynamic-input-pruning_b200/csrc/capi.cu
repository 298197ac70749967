// capi.cu — library-wide entry points: status handling, PDL switch and the
// whole-layer decode chain (StreamingDIPMlp.forward,
// dip_stream_predispatch.py:176-204, with the PCIe staging removed because
// every weight is resident in HBM).
#include <atomic>
#include <cstring>

#include "dip_common.cuh"

namespace dip {

// Device control block: word 0 = error bits (kErrTimeout, ...), word 1 =
// poll limit of the bounded waits (0 = the compiled default).
__device__ unsigned int dip_device_ctl[2] = {0u, 0u};

static std::atomic<int> g_pdl{1};
static std::atomic<int> g_simple_gemv{0};
static thread_local char g_last_err[256] = "";

bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed) != 0; }
bool force_simple_gemv() { return g_simple_gemv.load(std::memory_order_relaxed) != 0; }

// The address is looked up once per device (host threads may race on the
// first call: every racer stores the same value).  It stays valid while the
// device's primary context lives; after cudaDeviceReset the library must be
// reloaded.
unsigned* error_word_ptr() {
  static std::atomic<unsigned*> cache[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  unsigned* p = cache[dev].load(std::memory_order_acquire);
  if (!p) {
    void* q = nullptr;
    if (cudaGetSymbolAddress(&q, dip_device_ctl) != cudaSuccess) return nullptr;
    p = static_cast<unsigned*>(q);
    cache[dev].store(p, std::memory_order_release);
  }
  return p;
}

int launch_status(cudaError_t e) {
  if (e == cudaSuccess) return DIP_OK;
  std::strncpy(g_last_err, cudaGetErrorString(e), sizeof(g_last_err) - 1);
  return DIP_ERR_CUDA;
}

int num_sms() {
  static int cache[64] = {};
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev]) return cache[dev];
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  cache[dev] = n;
  return n;
}

size_t down_workspace_bytes(int64_t out);
static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }


}  // namespace dip

using namespace dip;

extern "C" int dip_version(void) { return 100; }

extern "C" const char* dip_status_string(int status) {
  switch (status) {
    case DIP_OK: return "ok";
    case DIP_ERR_ARG: return "invalid argument (null pointer, size or alignment)";
    case DIP_ERR_CUDA: return "CUDA error";
    case DIP_ERR_WORKSPACE: return "workspace too small";
    case DIP_ERR_UNSUPPORTED: return "unsupported shape";
    default: return "unknown status";
  }
}

extern "C" const char* dip_last_cuda_error(void) { return g_last_err; }

extern "C" int dip_set_pdl(int enable) { return g_pdl.exchange(enable ? 1 : 0); }

extern "C" int dip_set_gemv_variant(int simple) { return g_simple_gemv.exchange(simple ? 1 : 0); }

extern "C" int dip_take_device_error(unsigned int* out) {
  if (!out) return DIP_ERR_ARG;
  unsigned int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, dip_device_ctl, sizeof(unsigned int));
  if (e != cudaSuccess) return launch_status(e);
  return launch_status(cudaMemcpyToSymbol(dip_device_ctl, &zero, sizeof(unsigned int)));
}

extern "C" int dip_set_spin_limit(unsigned int polls) {
  return launch_status(cudaMemcpyToSymbol(dip_device_ctl, &polls, sizeof(unsigned int),
                                          sizeof(unsigned int)));
}

extern "C" size_t dip_mlp_workspace_bytes(int64_t hidden, int64_t inter, int64_t k) {
  if (hidden <= 0 || inter <= 0 || k < 0) return 0;
  return align256(topk_scratch_bytes()) + 256 + align256((size_t)inter * 2) + align256((size_t)k * 4) +
         align256((size_t)k * 2) + align256(down_workspace_bytes(hidden));
}

extern "C" int dip_mlp_decode(const dip_layer_t* L, const dip_bf16* x, int64_t k, void* workspace,
                              size_t workspace_bytes, dip_bf16* y, dip_bf16* g_out,
                              int32_t* idx_out, dip_stream_t stream) {
  if (!L || !x || !y || !workspace) return DIP_ERR_ARG;
  if (k < 1 || k > L->inter) return DIP_ERR_ARG;
  const size_t need = dip_mlp_workspace_bytes(L->hidden, L->inter, k);
  if (need == 0) return DIP_ERR_ARG;
  if (workspace_bytes < need) return DIP_ERR_WORKSPACE;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  unsigned* hist = reinterpret_cast<unsigned*>(ws);
  ws += align256(topk_scratch_bytes());
  GridBar* bars = reinterpret_cast<GridBar*>(ws);  // stays valid across calls
  ws += 256;
  dip_bf16* g = reinterpret_cast<dip_bf16*>(ws);
  ws += align256((size_t)L->inter * 2);
  int32_t* idx = reinterpret_cast<int32_t*>(ws);
  ws += align256((size_t)k * 4);
  dip_bf16* h = reinterpret_cast<dip_bf16*>(ws);
  ws += align256((size_t)k * 2);
  void* part = ws;
  const size_t part_bytes = workspace_bytes - (size_t)(ws - static_cast<uint8_t*>(workspace));
  if (g_out) g = g_out;
  if (idx_out) idx = idx_out;

  int st = gemv_silu_hist(L->gate_qw, L->gate_sc, x, g, L->inter, L->hidden, hist,
                          (cudaStream_t)stream);
  if (st) return st;
  st = topk_compact_launch(g, L->inter, k, idx, hist, (cudaStream_t)stream);
  if (st) return st;
  st = dip_gather_up_h(L->up_qw, L->up_sc, L->inter, x, g, idx, k, L->hidden, h, stream);
  if (st) return st;
  return gather_down_clear(L->down_t_qw, L->down_t_sc, L->inter, h, idx, k, L->hidden, part,
                           part_bytes, y, hist, topk_scratch_bytes(), &bars[0],
                           (cudaStream_t)stream);
}
