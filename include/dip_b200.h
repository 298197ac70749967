/*
 * dip_b200.h — C ABI of the B200 (sm_100a) Dynamic Input Pruning MLP kernels.
 *
 * Every entry point takes raw DEVICE pointers, element counts and a CUDA
 * stream, launches asynchronously on that stream and returns a status code
 * (DIP_OK = 0).  Nothing here allocates device memory: outputs and scratch
 * ("workspace") are provided by the caller, sized with the *_workspace_bytes
 * helpers.  bf16 tensors are passed as arrays of 16-bit patterns (dip_bf16).
 *
 * Weight format (unchanged from the reference, scripts/quantize.py:32-64):
 *   qweight int8 [rows, in/2], two's complement nibbles, low nibble = even col
 *   scales  bf16 [rows, in/128], w = q * s
 * down_proj is used in the transposed layout produced by
 * dip_stream_predispatch.py:100-120 (_transpose_down_to_int4):
 *   down_t  int8 [inter, hidden/2], scales bf16 [inter, hidden/128].
 *
 * Each declaration names the reference interface it replaces (file:line in
 * the reference project).
 */
#ifndef DIP_B200_H_
#define DIP_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define DIP_API __attribute__((visibility("default")))
#else
#define DIP_API
#endif

typedef struct CUstream_st* dip_stream_t; /* == cudaStream_t */
typedef uint16_t dip_bf16;                /* raw bfloat16 bits */

#define DIP_OK 0
#define DIP_ERR_ARG 1         /* null pointer, bad size or misaligned pointer */
#define DIP_ERR_CUDA 2        /* a CUDA launch / runtime error */
#define DIP_ERR_WORKSPACE 3   /* caller workspace smaller than required */
#define DIP_ERR_UNSUPPORTED 4 /* shape outside what the kernels handle */

/* Library version (major*10000 + minor*100 + patch). */
DIP_API int dip_version(void);
/* Human readable text of a status code; never NULL. */
DIP_API const char* dip_status_string(int status);
/* Last CUDA error text seen by the library on this thread (or ""). */
DIP_API const char* dip_last_cuda_error(void);
/* Enable (1) / disable (0) programmatic dependent launch between the kernels
 * of one call chain.  Default 1.  Returns the previous setting. */
DIP_API int dip_set_pdl(int enable);
/* Reads and clears the device error word of the current device: bit 0 set
 * means a kernel gave up a bounded wait (a pipeline barrier that never
 * completed) and returned early; its outputs are then invalid.  Synchronous
 * (a device-to-host copy).  0 = no error recorded. */
DIP_API int dip_take_device_error(unsigned int* out);
/* Sets the poll limit of every bounded device wait (grid barriers, the fused
 * layer's selection hand-offs, the peer-memory exchanges) on the current
 * device; 0 restores the compiled default (2^24 polls).  A wait that runs out
 * sets bit 0 of the device error word and the kernel returns; its outputs and
 * the workspace's selection state are then invalid (zero the workspace
 * before reusing it).  No counterpart in the reference (it has no device
 * waits); exists so that callers and tests can bound how long a missing peer
 * can hold a kernel.  Synchronous. */
DIP_API int dip_set_spin_limit(unsigned int polls);
/* Selects the kernel implementations: 0 (default) = the streaming kernels
 * (K-slice cp.async GEMV family and tensor-core down projection) where the
 * shape allows them, 1 = the simple kernels (one tile per CTA GEMV, CUDA-core
 * down).
 * Both give the same values up to fp32 summation order; the switch exists
 * for testing and comparison.  Returns the previous setting. */
DIP_API int dip_set_gemv_variant(int simple);

/* ---- a5/a6: int4 GEMV, optionally fused with SiLU --------------------------
 * out[r] = bf16(sum_c q[r,c]*s[r,c/128]*x[c]); with apply_silu != 0 the result
 * is then g = bf16(silu(out)).  Replaces int4_ops::int4_gemv
 * (kernels/int4_gemv/int4_gemv.cu:89-115) and the separate F.silu of
 * dip_stream_predispatch.py:182.  in_features % 128 == 0. */
DIP_API int dip_int4_gemv(const int8_t* qweight, const dip_bf16* scales, const dip_bf16* x,
                  dip_bf16* out, int64_t rows, int64_t in_features, int apply_silu,
                  dip_stream_t stream);

/* ---- config 3: the same GEMV for a batch of tokens -------------------------
 * out[t, r] = bf16(sum_c q[r,c]*s[r,c/128]*x[t,c]) for t < ntok (x [ntok, in],
 * out [ntok, rows], both row-major); with apply_silu != 0 then bf16(silu(.)).
 * Each token's result equals dip_int4_gemv's bit for bit.  One pass over the
 * weights serves 8 tokens (the 8 columns of the tensor-core tile); larger
 * batches take ceil(ntok / 8) passes.  Replaces the per-token gate GEMV of
 * the batch loop (dip_stream_predispatch.py:166-174 per token).  in_features
 * must be a multiple of 1024; 16-byte aligned pointers. */
DIP_API int dip_int4_gemv_batched(const int8_t* qweight, const dip_bf16* scales, const dip_bf16* x,
                                  dip_bf16* out, int64_t rows, int64_t in_features, int64_t ntok,
                                  int apply_silu, dip_stream_t stream);

/* ---- a7: top-k of |s| -------------------------------------------------------
 * Exactly the selection of topk_ops::topk_select
 * (kernels/topk_select/topk_select.cu:134-164): 25-step fp32 bisection on
 * [0, max|s|], then indices with |s| > hi in ascending order followed by
 * lo < |s| <= hi in ascending order, truncated to k; unfilled slots are 0.
 * One launch, no host synchronisation.  1 <= n <= 98304, 0 <= k. */
DIP_API int dip_topk_select(const dip_bf16* s, int64_t n, int64_t k, int32_t* idx,
                    dip_stream_t stream);
/* Per-token variant for batched decode (one CTA per row of s): row b of s
 * starts at s + b*s_stride, its k indices at idx + b*idx_stride.  The
 * reference decode path is batch-1 only (dip_stream_predispatch.py:170,182);
 * each row gets exactly the selection of dip_topk_select. */
DIP_API int dip_topk_select_batched(const dip_bf16* s, int64_t batch, int64_t n, int64_t s_stride,
                            int64_t k, int32_t* idx, int64_t idx_stride, dip_stream_t stream);

/* Faster form of dip_topk_select (same indices): a histogram pass plus a
 * select/compaction pass over a caller-provided histogram of
 * dip_topk_hist_bytes() bytes (16-byte aligned) that must be ZERO on entry;
 * the call leaves it zero again, so one buffer serves any number of calls on
 * one stream. */
DIP_API size_t dip_topk_hist_bytes(void);
DIP_API int dip_topk_select_ws(const dip_bf16* s, int64_t n, int64_t k, int32_t* idx, void* hist,
                               dip_stream_t stream);

/* ---- a8: gathered int4 GEMV --------------------------------------------------
 * out[j] = bf16(dot(dequant(W[indices[j]]), x)), j < k.  Replaces
 * int4_gather_ops::int4_gather_gemv (kernels/int4_gather/int4_gather_gemv.cu:
 * 87-115).  n_rows bounds the index range (out-of-range indices read row 0
 * and set the result to 0). */
DIP_API int dip_int4_gather_gemv(const int8_t* qweight, const dip_bf16* scales, int64_t n_rows,
                         const dip_bf16* x, const int32_t* indices, int64_t k,
                         int64_t in_features, dip_bf16* out, dip_stream_t stream);

/* ---- a8+a9: gathered up GEMV with the g*u product folded in --------------------
 * h[j] = bf16(g[idx[j]] * bf16(dot(W_up[idx[j]], x))).  Replaces the up call
 * and the `h_sel = (g[idx] * up_sel).to(bf16)` line of
 * dip_stream_predispatch.py:199-201. */
DIP_API int dip_gather_up_h(const int8_t* up_qw, const dip_bf16* up_sc, int64_t n_rows,
                    const dip_bf16* x, const dip_bf16* g, const int32_t* idx, int64_t k,
                    int64_t in_features, dip_bf16* h, dip_stream_t stream);

/* ---- a10: gathered transposed down projection -------------------------------
 * y[o] = bf16(sum_j h[j] * q(down_t[r_j, o]) * s(down_t[r_j, o/128])) with
 * r_j = idx[j] (or r_j = j when idx == NULL, the reference's staging-buffer
 * layout).  Replaces int4_down_ops::int4_gather_down
 * (kernels/int4_down/int4_gather_down.cu:77-102).  The cross-CTA sum is
 * deterministic (fixed order, no float atomics). */
DIP_API size_t dip_gather_down_workspace_bytes(int64_t out_features);
DIP_API int dip_int4_gather_down(const int8_t* down_t, const dip_bf16* scales, int64_t n_rows,
                         const dip_bf16* h, const int32_t* idx, int64_t k,
                         int64_t out_features, void* workspace, size_t workspace_bytes,
                         dip_bf16* y, dip_stream_t stream);

/* ---- allocation-free variant of dip_int4_gather_down ------------------------
 * No counterpart in the reference.  For callers that cannot allocate device
 * memory when they call in (a host framework owns the memory pool, a fixed
 * memory budget, or an FFI caller with no CUDA allocator): the same
 * computation and arguments as dip_int4_gather_down, minus the workspace.
 * The partial sums go to a static device array of the library, sized for
 * out_features <= 8192 (148 * 8192 fp32 = 4.6 MiB, held on every GPU that
 * loads the library until the process exits); larger out_features returns
 * DIP_ERR_UNSUPPORTED.  Nothing is allocated: no cudaMalloc, no cudaFree.
 * The first call on a device looks up the array's device address (with that
 * device current); make that first call before any stream capture.  All calls
 * share the array and it keeps the last call's contents (every call rewrites
 * what it reads, so nothing has to start at zero); calls that overlap on the
 * GPU, on any streams, race on it and must be serialised by the caller. */
DIP_API int dip_int4_gather_down_noalloc(const int8_t* down_t, const dip_bf16* scales,
                                         int64_t n_rows, const dip_bf16* h, const int32_t* idx,
                                         int64_t k, int64_t out_features, dip_bf16* y,
                                         dip_stream_t stream);

/* ---- a13: dual-source gathered GEMV (cache-aware up) ---------------------------
 * out[j] = dot(dequant(src[j]==0 ? res[row[j]] : str[row[j]]), x).  Replaces
 * ca_fused_ops::ca_fused_gemv (kernels/ca_fused/ca_fused_gemv.cu:87-112);
 * in_features is the length of x, as in the reference wrapper. */
DIP_API int dip_ca_fused_gemv(const int8_t* res_qw, const dip_bf16* res_sc, int64_t n_res,
                      const int8_t* str_qw, const dip_bf16* str_sc, int64_t n_str,
                      const dip_bf16* x, const int32_t* src, const int32_t* row, int64_t k,
                      int64_t in_features, dip_bf16* out, dip_stream_t stream);

/* ---- a12: cache hit/miss split -------------------------------------------------
 * For slots = id2slot[idx]: hits (slot >= 0) in idx order, then misses in idx
 * order, as dip_ca.py:137-142 and :164-171.  Writes combined_ids[k], src[k]
 * (0 = resident cache, 1 = full weights), row[k] (cache slot for a hit, the
 * channel id for a miss) and n_hit[0].  One launch, no host synchronisation. */
DIP_API int dip_ca_split(const int32_t* idx, int64_t k, const int64_t* id2slot, int64_t n_channels,
                 int32_t* combined_ids, int32_t* src, int32_t* row, int32_t* n_hit,
                 dip_stream_t stream);

/* ---- a12/a13 fused: cache-aware up with h, and down, over (src,row) tables ----
 * Source 0 = resident cache rows, source 1 = full resident rows. */
DIP_API int dip_srcrow_up_h(const int8_t* res_qw, const dip_bf16* res_sc, int64_t n_res,
                    const int8_t* full_qw, const dip_bf16* full_sc, int64_t n_full,
                    const dip_bf16* x, const dip_bf16* g, const int32_t* combined_ids,
                    const int32_t* src, const int32_t* row, int64_t k, int64_t in_features,
                    dip_bf16* h, dip_stream_t stream);
DIP_API int dip_srcrow_down(const int8_t* res_dt, const dip_bf16* res_sc, int64_t n_res,
                    const int8_t* full_dt, const dip_bf16* full_sc, int64_t n_full,
                    const dip_bf16* h, const int32_t* src, const int32_t* row, int64_t k,
                    int64_t out_features, void* workspace, size_t workspace_bytes,
                    dip_bf16* y, dip_stream_t stream);

/* ---- a11: one whole decode DIP MLP layer, batch 1 --------------------------------
 * gate GEMV + SiLU -> top-k -> gathered up (h) -> gathered down, four launches
 * chained with programmatic dependent launch, no host synchronisation.
 * Replaces StreamingDIPMlp.forward (dip_stream_predispatch.py:176-204). */
typedef struct dip_layer {
  const int8_t* gate_qw;   /* [inter, hidden/2]   */
  const dip_bf16* gate_sc; /* [inter, hidden/128] */
  const int8_t* up_qw;     /* [inter, hidden/2]   */
  const dip_bf16* up_sc;   /* [inter, hidden/128] */
  const int8_t* down_t_qw; /* [inter, hidden/2]   */
  const dip_bf16* down_t_sc; /* [inter, hidden/128] */
  int64_t hidden;
  int64_t inter;
} dip_layer_t;

DIP_API size_t dip_mlp_workspace_bytes(int64_t hidden, int64_t inter, int64_t k);
/* The workspace must be ZERO before its first use (its first 130 KB hold the
 * top-k histograms, which the gate kernel fills and the last kernel clears); every
 * call leaves that region zero, so a workspace can be reused call after call
 * on one stream. */
/* g_out (bf16[inter]) and idx_out (int32[k]) may be NULL; when given they
 * receive the layer's gate activations and selected channels. */
DIP_API int dip_mlp_decode(const dip_layer_t* layer, const dip_bf16* x, int64_t k, void* workspace,
                   size_t workspace_bytes, dip_bf16* y, dip_bf16* g_out, int32_t* idx_out,
                   dip_stream_t stream);

/* ---- a11, one launch: the whole decode layer as one persistent kernel ---------
 * Same result as dip_mlp_decode (same selection; y within rounding), computed
 * by one cooperative launch of one CTA per SM: gate GEMV + SiLU + histogram,
 * grid barrier, top-k thresholds, gathered up and down for the channels each
 * CTA selected among its own gate rows, grid barrier, fixed-order reduction.
 * With resid != NULL the layer input is RMSNorm(x + resid) (unit weight, eps),
 * the inter-layer step of the synthetic stack; x_used (optional) receives the
 * input used.  The workspace (dip_mlp_fused_workspace_bytes) must be ZERO
 * before its first use and is left reusable.  Weights, x, g_out and the
 * workspace, and resid / x_used when given, must be 16-byte aligned
 * (DIP_ERR_ARG otherwise).  Requires
 * hidden = 2560 or 5120 (20 warps x 1 or 2 quantisation groups), inter a multiple of 8 and at most
 * 16*12-1 gate rows per SM; otherwise DIP_ERR_UNSUPPORTED. */
DIP_API size_t dip_mlp_fused_workspace_bytes(int64_t hidden, int64_t inter, int64_t k);
DIP_API int dip_mlp_decode_fused(const dip_layer_t* layer, const dip_bf16* x,
                                 const dip_bf16* resid, float eps, int64_t k, void* workspace,
                                 size_t workspace_bytes, dip_bf16* y, dip_bf16* g_out,
                                 int32_t* idx_out, dip_bf16* x_used, dip_stream_t stream);

/* ---- a11 + a12/a13, one launch: the cache-aware layer --------------------------
 * dip_mlp_decode_fused with the cache-aware DIP split of dip_ca.py:127-188
 * folded into the row reads: selected channel c reads its up and down rows
 * from row id2slot[c] of the resident cache when id2slot[c] >= 0 (a hit),
 * else from the full matrices (a miss).  Every channel's rows are the same
 * bytes either way, so y, g and idx equal dip_mlp_decode_fused's; the split
 * itself (hits then misses, dip_ca_split) is not materialised.  The cache
 * arrays have the layer's row formats (up [n_res, hidden/2] + scales, down_t
 * [n_res, hidden/2] + scales); 16-byte aligned. */
typedef struct dip_ca_cache {
  const int64_t* id2slot;     /* [inter], -1 = not cached */
  const int8_t* res_up_qw;    /* [n_res, hidden/2] */
  const dip_bf16* res_up_sc;  /* [n_res, hidden/128] */
  const int8_t* res_dn_qw;    /* [n_res, hidden/2] (transposed down rows) */
  const dip_bf16* res_dn_sc;  /* [n_res, hidden/128] */
  int64_t n_res;
} dip_ca_cache_t;
DIP_API int dip_mlp_decode_fused_ca(const dip_layer_t* layer, const dip_ca_cache_t* cache,
                                    const dip_bf16* x, const dip_bf16* resid, float eps, int64_t k,
                                    void* workspace, size_t workspace_bytes, dip_bf16* y,
                                    dip_bf16* g_out, int32_t* idx_out, dip_bf16* x_used,
                                    dip_stream_t stream);
/* Optional extras of a fused-layer call (any field may be NULL).
 *   h_out [inter] bf16: for every selected channel c, h_out[c] =
 *     bf16(g[c] * bf16(u[c])), the h_sel of dip_stream_predispatch.py:201
 *     that the down projection consumes (other entries untouched); lets a
 *     caller check the up stage and the down stage separately.
 *   prefetch_gate_qw / prefetch_gate_sc: the NEXT layer's gate weights (same
 *     shape as this layer's, 16-byte aligned, both or neither).  Once a worker
 *     SM has finished its own rows it moves the first rows of the same range
 *     of those weights into L2, so the next call's first tiles come from L2.
 *     A hint only: results do not depend on it. */
typedef struct {
  dip_bf16* h_out;
  const int8_t* prefetch_gate_qw;
  const dip_bf16* prefetch_gate_sc;
} dip_fused_opts_t;
/* As dip_mlp_decode_fused_ca, with the extras of `opts` (may be NULL). */
DIP_API int dip_mlp_decode_fused_ex(const dip_layer_t* layer, const dip_ca_cache_t* cache,
                                    const dip_bf16* x, const dip_bf16* resid, float eps, int64_t k,
                                    void* workspace, size_t workspace_bytes, dip_bf16* y,
                                    dip_bf16* g_out, int32_t* idx_out, dip_bf16* x_used,
                                    const dip_fused_opts_t* opts, dip_stream_t stream);

/* ---- batched decode and dense forward on tcgen05 tensor cores ------------------
 * The reference decode path is batch-1 (dip_stream_predispatch.py:170, :182); a
 * batch of B tokens is B independent DIP decodes.  These entry points compute
 * them with dense int4 x bf16 GEMMs on the 5th-generation tensor cores
 * (M = 128 weight rows per tile, N = B padded to 16/32/64/128, fp32
 * accumulators in TMEM), every weight dequantised to bf16(q * s) as
 * dequantize() (qlinear.py:28-64) does.
 *
 * dip_int4_gemm_tc: out[b][r] = epi(sum_k W[r][k] x[b][k]), W in the layout of
 * QuantLinear (qweight [rows, in/2], scales [rows, in/128]; replaces
 * QuantLinear.forward's F.linear(x, dequantize(...)), qlinear.py:86-88, for
 * 1 <= batch <= 128).  epilogue 0: bf16(acc); 1: bf16(silu(bf16(acc))) (the
 * gate, dip_stream_predispatch.py:182); 2: the DIP up product
 * h = bf16(g * bf16(acc)) * sel_count (dip_stream_predispatch.py:199-201 with
 * the token's selected channels, sel_count[b][r] = times r is in its index
 * list; 0 = not selected, h = 0), g and sel_count [batch, rows].  in_features
 * a multiple of 256; qweight, x and the workspace (a reordered copy of x and
 * the fp32 partial sums when K is split over the SMs,
 * dip_int4_gemm_tc_workspace_bytes) 16-byte aligned, scales 4-byte aligned. */
DIP_API size_t dip_int4_gemm_tc_workspace_bytes(int64_t rows, int64_t in_features, int64_t batch);
DIP_API int dip_int4_gemm_tc(const int8_t* qweight, const dip_bf16* scales, const dip_bf16* x,
                             int64_t rows, int64_t in_features, int64_t batch, int epilogue,
                             const dip_bf16* g, const uint32_t* sel_count, void* workspace,
                             size_t workspace_bytes, dip_bf16* out, dip_stream_t stream);
/* Dense down projection of a batch over the transposed down weights
 * (down_t [inter, out/2] + scales [inter, out/128] of _transpose_down_to_int4,
 * dip_stream_predispatch.py:100-120): y[b] = bf16(sum_c h[b][c] W_down_t[c]),
 * h [batch, inter] (zero for unselected channels; replaces the per-token
 * int4_gather_down, int4_gather_down.cu:41-95).  Channels are split over the
 * SMs; the fp32 partials (workspace, dip_int4_down_tc_workspace_bytes) are
 * summed in a fixed order.  out a multiple of 256, inter of 64. */
/* As dip_int4_gemm_tc with the number of K ranges fixed (ksplit 1..4; 0 =
 * automatic).  Each K range's partial is summed in a fixed order, so two
 * calls with the same ksplit compute every output row with the same
 * summation order whatever the number of rows: a tensor-parallel shard of
 * the gate passes the full layer's automatic choice
 * (dip_int4_gemm_tc_auto_split(full rows, in_features)) and gets rows
 * bit-identical to the unsharded GEMM.  No counterpart in the reference. */
DIP_API int dip_int4_gemm_tc_auto_split(int64_t rows, int64_t in_features);
DIP_API int dip_int4_gemm_tc_split(const int8_t* qweight, const dip_bf16* scales,
                                   const dip_bf16* x, int64_t rows, int64_t in_features,
                                   int64_t batch, int epilogue, const dip_bf16* g,
                                   const uint32_t* sel_count, int ksplit, void* workspace,
                                   size_t workspace_bytes, dip_bf16* out, dip_stream_t stream);
DIP_API size_t dip_int4_down_tc_workspace_bytes(int64_t out_features, int64_t batch);
DIP_API int dip_int4_down_tc(const int8_t* down_t, const dip_bf16* scales, const dip_bf16* h,
                             int64_t inter, int64_t out_features, int64_t batch, void* workspace,
                             size_t workspace_bytes, dip_bf16* y, dip_stream_t stream);
/* As dip_int4_down_tc with the fp32 sums as output (y_f32 [batch, out]):
 * a tensor-parallel shard's partial, summed over the ranks before the one
 * bf16 rounding.  No counterpart in the reference. */
DIP_API int dip_int4_down_tc_f32(const int8_t* down_t, const dip_bf16* scales, const dip_bf16* h,
                                 int64_t inter, int64_t out_features, int64_t batch,
                                 void* workspace, size_t workspace_bytes, float* y_f32,
                                 dip_stream_t stream);
/* cnt[b][c] = how many times channel c occurs in idx[b] (idx [batch, k]), the
 * selection of each token as dense counts for dip_int4_gemm_tc's epilogue 2
 * (the reference's index_select over idx, dip_stream_predispatch.py:199-203). */
DIP_API int dip_select_count(const int32_t* idx, int64_t batch, int64_t k, int64_t inter,
                             uint32_t* cnt, dip_stream_t stream);

/* ---- tensor-parallel exchanges over peer memory (config 4) ----------------------
 * The reference is single-GPU; the sharded layer (rank r of P owns channels
 * [r I/P, (r+1) I/P)) needs the full g on every rank and the sum of the P fp32
 * down partials.  These replace the NCCL all-gather / all-reduce with peer
 * stores over NVLink into per-rank mailboxes and per-call flags.
 * Set-up (once per rank): dip_p2p_alloc(dip_p2p_mailbox_bytes(...)) (zeroed),
 * dip_ipc_handle of it to the peers (64 bytes), dip_ipc_open of the peers'
 * handles.  mailboxes[q] = rank q's mailbox as this process maps it (its own
 * for q == rank), 256-byte aligned.  Every rank must make the same sequence of
 * calls.  dip_p2p_gather: g_local [n_local] -> the mailbox's g buffer (at byte
 * offset 512 of the mailbox) holds all P slices in rank order.
 * dip_p2p_reduce: y = bf16(sum over ranks in rank order of partial [hidden]),
 * identical on every rank.  Waits are bounded (device error word on timeout). */
DIP_API size_t dip_p2p_mailbox_bytes(int64_t inter, int64_t hidden, int64_t world);
DIP_API int dip_p2p_alloc(size_t bytes, void** ptr);
DIP_API int dip_p2p_free(void* ptr);
DIP_API int dip_ipc_handle(const void* ptr, void* handle64);
DIP_API int dip_ipc_open(const void* handle64, void** ptr);
DIP_API int dip_ipc_close(void* ptr);
DIP_API int dip_p2p_gather(int rank, int world, void* const* mailboxes, const dip_bf16* g_local,
                           int64_t n_local, int64_t hidden, dip_stream_t stream);
DIP_API int dip_p2p_reduce(int rank, int world, void* const* mailboxes, const float* partial,
                           int64_t inter, int64_t hidden, dip_bf16* y, dip_stream_t stream);
/* Mailboxes handed to dip_p2p_gather / dip_p2p_reduce / dip_mlp_decode_fused_tp
 * for peers must come from dip_p2p_alloc (own) or dip_ipc_open (peers): the
 * library records each range's size and rejects (DIP_ERR_ARG) a call whose
 * stores would not fit, instead of writing past another GPU's allocation. */

/* ---- a5..a10 sharded along I, one launch per rank: the tensor-parallel layer ----
 * StreamingDIPMlp.forward (dip_stream_predispatch.py:176-204) for one token with
 * the channels split over `world` GPUs: rank r holds rows [r I/P, (r+1) I/P) of
 * gate, up and the transposed down (`shard`, shard->inter = I/P) and runs one
 * cooperative kernel per layer that
 *   - computes its g slice and adds its |g| keys to every rank's histograms
 *     (remote reductions over NVLink), so every rank's coordinating CTA finds
 *     the same selection over all inter_total channels (indices identical to
 *     dip_mlp_decode_fused's on the whole layer);
 *   - gathers up / down over its own selected channels;
 *   - stores its fp32 partial of y into every rank's y slots (16-byte peer
 *     stores plus a tagged flag per CTA) and sums the slots in rank order:
 *     y is identical on every rank.
 * No NCCL, no multicast, no TMA on peer memory: peer stores, peer reductions
 * and local polls only.  workspaces[q] = rank q's workspace
 * (dip_mlp_fused_tp_workspace_bytes, zeroed before the first call, 256-byte
 * aligned; peers' mapped through dip_ipc_open).  Every rank makes the same
 * sequence of calls with the same shapes on GPUs with the same SM count.
 * opts as for dip_mlp_decode_fused_ex (h_out indexed by global channel id;
 * prefetch: the next layer's shard).
 * idx_out (optional, [k]) receives only the entries of this rank's channels
 * (global channel ids at their global positions; rank 0 also writes the zero
 * padding); g_out (optional) this rank's g slice.  Waits are bounded (device
 * error word; after a timeout zero every rank's workspace).  No counterpart in
 * the reference, which is single-GPU. */
DIP_API size_t dip_mlp_fused_tp_workspace_bytes(int64_t hidden, int64_t inter_total, int64_t k);
DIP_API int dip_mlp_decode_fused_tp(const dip_layer_t* shard, int64_t inter_total, int rank,
                                    int world, void* const* workspaces, size_t workspace_bytes,
                                    const dip_bf16* x, const dip_bf16* resid, float eps, int64_t k,
                                    dip_bf16* y, dip_bf16* g_out, int32_t* idx_out,
                                    dip_bf16* x_used, const dip_fused_opts_t* opts,
                                    dip_stream_t stream);

/* ---- a1/a3: weight format ---------------------------------------------------------
 * Symmetric int4 group-128 quantisation of a bf16 [rows, cols] matrix, bit
 * exact with scripts/quantize.py:32-64. */
DIP_API int dip_quantize_int4_g128(const dip_bf16* w, int64_t rows, int64_t cols, int8_t* qweight,
                           dip_bf16* scales, dip_stream_t stream);
/* dequantize -> transpose -> requantise along the new rows, bit exact with
 * dip_stream_predispatch.py:100-120.  down_qw [out_f, inter/2] ->
 * down_t_qw [inter, out_f/2], down_t_sc [inter, out_f/128]. */
DIP_API int dip_transpose_down_int4(const int8_t* down_qw, const dip_bf16* down_sc, int64_t out_f,
                            int64_t inter, int8_t* down_t_qw, dip_bf16* down_t_sc,
                            dip_stream_t stream);
/* Unpack + scale: w[r,c] = bf16(q*s), bit exact with qlinear.py:52-64. */
DIP_API int dip_dequantize_int4_g128(const int8_t* qweight, const dip_bf16* scales, int64_t rows,
                             int64_t cols, dip_bf16* w, dip_stream_t stream);

/* ---- tensor parallelism along the intermediate dimension (config 4) ----------
 * Not in the reference (single GPU only).  Rank r owns channels [lo, hi) of
 * gate, up and down_t.  After an all-gather of g every rank runs the same
 * dip_topk_select; dip_shard_select keeps the selected channels it owns
 * (local row ids, idx order) and their count on the device; the two kernels
 * below take that device-side count (grids are sized for max_k) and the down
 * projection returns fp32 partials for the all-reduce. */
DIP_API int dip_shard_select(const int32_t* idx, int64_t k, int64_t lo, int64_t hi,
                             int32_t* local_idx, int32_t* count, dip_stream_t stream);
DIP_API int dip_gather_up_h_count(const int8_t* up_qw, const dip_bf16* up_sc, int64_t n_rows,
                                  const dip_bf16* x, const dip_bf16* g, const int32_t* idx,
                                  const int32_t* count, int64_t max_k, int64_t in_features,
                                  dip_bf16* h, dip_stream_t stream);
DIP_API int dip_gather_down_partial(const int8_t* down_t, const dip_bf16* scales,
                                    int64_t n_rows, const dip_bf16* h, const int32_t* idx,
                                    const int32_t* count, int64_t max_k, int64_t out_features,
                                    void* workspace, size_t workspace_bytes, float* y_f32,
                                    dip_stream_t stream);

/* ---- inter-layer step of the synthetic decode stack ---------------------------
 * x_next = bf16(v * rsqrt(mean(v^2) + eps)), v = y + r (RMSNorm with unit
 * weight of a layer output plus a residual).  Not part of the reference's
 * MLP; it defines the per-layer inputs of the 64-layer benchmark stack. */
DIP_API int dip_residual_rmsnorm(const dip_bf16* y, const dip_bf16* r, int64_t n, float eps,
                                 dip_bf16* out, dip_stream_t stream);
/* The same for `rows` consecutive rows of n values (one normalisation per
 * row): the batched stack's per-token inter-layer step. */
DIP_API int dip_residual_rmsnorm_rows(const dip_bf16* y, const dip_bf16* r, int64_t rows, int64_t n,
                                      float eps, dip_bf16* out, dip_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* DIP_B200_H_ */
