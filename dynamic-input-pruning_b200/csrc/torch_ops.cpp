// torch_ops.cpp — thin torch extension over the C ABI (include/dip_b200.h).
//
// Registers the reference's five operator schemas unchanged, so code written
// against the reference keeps calling torch.ops.<ns>.<op>:
//   int4_ops::int4_gemv               kernels/int4_gemv/int4_gemv.cu:110-115
//   topk_ops::topk_select             kernels/topk_select/topk_select.cu:166-171
//   int4_gather_ops::int4_gather_gemv kernels/int4_gather/int4_gather_gemv.cu:110-115
//   int4_down_ops::int4_gather_down   kernels/int4_down/int4_gather_down.cu:97-102
//   ca_fused_ops::ca_fused_gemv       kernels/ca_fused/ca_fused_gemv.cu:107-112
// plus the fused B200 operators of namespace dip_b200.  Unlike the reference
// wrappers, every input is checked (device, dtype, shape, contiguity) and
// every launch goes to torch's current stream.  Only the CUDA dispatch key is
// implemented: there is no CPU kernel to fall back to.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <ATen/ATen.h>
#include <torch/library.h>

#include <map>
#include <mutex>
#include <vector>

#include "../../include/dip_b200.h"

namespace {

using at::Tensor;

void check_status(int st, const char* what) {
  TORCH_CHECK(st == DIP_OK, what, " failed: ", dip_status_string(st),
              st == DIP_ERR_CUDA ? std::string(" (") + dip_last_cuda_error() + ")" : "");
}

void check_cuda(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}
void check_dtype(const Tensor& t, c10::ScalarType dt, const char* name) {
  TORCH_CHECK(t.scalar_type() == dt, name, " must be ", dt, ", got ", t.scalar_type());
}
void check_packed(const Tensor& qw, const Tensor& sc, const char* name) {
  check_cuda(qw, name);
  check_cuda(sc, name);
  TORCH_CHECK(qw.dim() == 2 && sc.dim() == 2, name, ": qweight/scales must be 2-D");
  TORCH_CHECK(qw.scalar_type() == at::kChar || qw.scalar_type() == at::kByte, name,
              ": qweight must be int8");
  check_dtype(sc, at::kBFloat16, name);
  TORCH_CHECK(qw.size(0) == sc.size(0) && qw.size(1) * 2 == sc.size(1) * 128, name,
              ": qweight [rows, in/2] and scales [rows, in/128] disagree");
}
Tensor idx32(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == at::kInt || t.scalar_type() == at::kLong, name,
              " must be int32 or int64");
  return t.to(at::kInt).contiguous();
}
dip_stream_t cur_stream() {
  return reinterpret_cast<dip_stream_t>(at::cuda::getCurrentCUDAStream().stream());
}
const int8_t* i8(const Tensor& t) { return reinterpret_cast<const int8_t*>(t.data_ptr()); }
const dip_bf16* bf(const Tensor& t) { return reinterpret_cast<const dip_bf16*>(t.data_ptr()); }
dip_bf16* bfm(Tensor& t) { return reinterpret_cast<dip_bf16*>(t.data_ptr()); }
Tensor bf16_empty(int64_t n, const Tensor& like) {
  return at::empty({n}, like.options().dtype(at::kBFloat16));
}

// The histogram of dip_topk_select_ws must be zero on entry and is left
// zero, so one buffer per (device, stream) serves every call issued on that
// stream: it is allocated and zeroed once.  While the stream is being
// captured into a CUDA graph a fresh zeroed buffer is used instead (a buffer
// first zeroed inside a capture would only be zeroed at replay).
Tensor topk_hist_for(const Tensor& like) {
  const int64_t nb = (int64_t)dip_topk_hist_bytes();
  cudaStream_t st = at::cuda::getCurrentCUDAStream().stream();
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone)
    return at::zeros({nb}, like.options().dtype(at::kByte));
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, Tensor> cache;
  std::lock_guard<std::mutex> lk(mu);
  auto key = std::make_pair((int)like.device().index(), st);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  Tensor t = at::zeros({nb}, like.options().dtype(at::kByte));
  cache.emplace(key, t);
  return t;
}

// ---------------- reference schemas ----------------
Tensor int4_gemv(const Tensor& qweight, const Tensor& scales, const Tensor& x_in) {
  check_packed(qweight, scales, "int4_gemv");
  c10::cuda::CUDAGuard guard(qweight.device());
  Tensor x = x_in.contiguous();
  check_cuda(x, "x");
  check_dtype(x, at::kBFloat16, "x");
  TORCH_CHECK(x.numel() == qweight.size(1) * 2, "int4_gemv: x has ", x.numel(),
              " elements, expected ", qweight.size(1) * 2);
  Tensor out = bf16_empty(qweight.size(0), x);
  check_status(dip_int4_gemv(i8(qweight), bf(scales), bf(x), bfm(out), qweight.size(0),
                             qweight.size(1) * 2, 0, cur_stream()),
               "int4_gemv");
  return out;
}

Tensor topk_select(const Tensor& s_in, int64_t k) {
  Tensor s = s_in.contiguous();
  check_cuda(s, "s");
  check_dtype(s, at::kBFloat16, "s");
  c10::cuda::CUDAGuard guard(s.device());
  TORCH_CHECK(k >= 0, "topk_select: k must be >= 0");
  Tensor idx = at::empty({k}, s.options().dtype(at::kInt));
  if (k == 0) return idx;
  Tensor hist = topk_hist_for(s);
  check_status(dip_topk_select_ws(bf(s), s.numel(), k, idx.data_ptr<int32_t>(), hist.data_ptr(),
                                  cur_stream()),
               "topk_select");
  return idx;
}

Tensor int4_gather_gemv(const Tensor& qweight, const Tensor& scales, const Tensor& x_in,
                        const Tensor& indices_in) {
  check_packed(qweight, scales, "int4_gather_gemv");
  c10::cuda::CUDAGuard guard(qweight.device());
  Tensor x = x_in.contiguous();
  check_dtype(x, at::kBFloat16, "x");
  TORCH_CHECK(x.numel() == qweight.size(1) * 2, "int4_gather_gemv: x/qweight mismatch");
  Tensor ind = idx32(indices_in, "indices");
  Tensor out = bf16_empty(ind.numel(), x);
  check_status(dip_int4_gather_gemv(i8(qweight), bf(scales), qweight.size(0), bf(x),
                                    ind.data_ptr<int32_t>(), ind.numel(), qweight.size(1) * 2,
                                    bfm(out), cur_stream()),
               "int4_gather_gemv");
  return out;
}

Tensor int4_gather_down(const Tensor& down_t_sel, const Tensor& scales, const Tensor& h_in) {
  check_packed(down_t_sel, scales, "int4_gather_down");
  c10::cuda::CUDAGuard guard(down_t_sel.device());
  Tensor h = h_in.contiguous();
  check_dtype(h, at::kBFloat16, "h_sel");
  TORCH_CHECK(h.numel() == down_t_sel.size(0), "int4_gather_down: h_sel has ", h.numel(),
              " elements, down_t_sel has ", down_t_sel.size(0), " rows");
  const int64_t out_f = down_t_sel.size(1) * 2;
  Tensor y = bf16_empty(out_f, h);
  Tensor ws = at::empty({(int64_t)dip_gather_down_workspace_bytes(out_f)},
                        h.options().dtype(at::kByte));
  check_status(dip_int4_gather_down(i8(down_t_sel), bf(scales), down_t_sel.size(0), bf(h),
                                    nullptr, h.numel(), out_f, ws.data_ptr(), ws.numel(),
                                    bfm(y), cur_stream()),
               "int4_gather_down");
  return y;
}

Tensor ca_fused_gemv(const Tensor& res_qw, const Tensor& res_sc, const Tensor& str_qw,
                     const Tensor& str_sc, const Tensor& x_in, const Tensor& src_in,
                     const Tensor& row_in) {
  check_packed(res_qw, res_sc, "ca_fused_gemv(res)");
  check_packed(str_qw, str_sc, "ca_fused_gemv(str)");
  c10::cuda::CUDAGuard guard(res_qw.device());
  Tensor x = x_in.contiguous();
  check_dtype(x, at::kBFloat16, "x");
  const int64_t in_f = x.numel();  // the reference takes in_features from x
  TORCH_CHECK(res_qw.size(1) * 2 == in_f && str_qw.size(1) * 2 == in_f,
              "ca_fused_gemv: x length does not match the packed rows");
  Tensor src = idx32(src_in, "src"), row = idx32(row_in, "row");
  TORCH_CHECK(src.numel() == row.numel(), "ca_fused_gemv: src/row length mismatch");
  Tensor out = bf16_empty(src.numel(), x);
  check_status(dip_ca_fused_gemv(i8(res_qw), bf(res_sc), res_qw.size(0), i8(str_qw), bf(str_sc),
                                 str_qw.size(0), bf(x), src.data_ptr<int32_t>(),
                                 row.data_ptr<int32_t>(), src.numel(), in_f, bfm(out),
                                 cur_stream()),
               "ca_fused_gemv");
  return out;
}

// ---------------- B200 fused operators ----------------
Tensor gate_silu(const Tensor& qweight, const Tensor& scales, const Tensor& x_in) {
  check_packed(qweight, scales, "gate_silu");
  c10::cuda::CUDAGuard guard(qweight.device());
  Tensor x = x_in.contiguous();
  check_dtype(x, at::kBFloat16, "x");
  TORCH_CHECK(x.numel() == qweight.size(1) * 2, "gate_silu: x/qweight mismatch");
  Tensor out = bf16_empty(qweight.size(0), x);
  check_status(dip_int4_gemv(i8(qweight), bf(scales), bf(x), bfm(out), qweight.size(0),
                             qweight.size(1) * 2, 1, cur_stream()),
               "gate_silu");
  return out;
}

Tensor topk_select_batched(const Tensor& s_in, int64_t k) {
  Tensor s = s_in.contiguous();
  check_cuda(s, "s");
  check_dtype(s, at::kBFloat16, "s");
  TORCH_CHECK(s.dim() == 2, "topk_select_batched: s must be [B, n]");
  c10::cuda::CUDAGuard guard(s.device());
  Tensor idx = at::empty({s.size(0), k}, s.options().dtype(at::kInt));
  if (k == 0 || s.size(0) == 0) return idx;
  check_status(dip_topk_select_batched(bf(s), s.size(0), s.size(1), s.size(1), k,
                                       idx.data_ptr<int32_t>(), k, cur_stream()),
               "topk_select_batched");
  return idx;
}

Tensor gather_up_h(const Tensor& up_qw, const Tensor& up_sc, const Tensor& x_in,
                   const Tensor& g_in, const Tensor& idx_in) {
  check_packed(up_qw, up_sc, "gather_up_h");
  c10::cuda::CUDAGuard guard(up_qw.device());
  Tensor x = x_in.contiguous(), g = g_in.contiguous();
  check_dtype(x, at::kBFloat16, "x");
  check_dtype(g, at::kBFloat16, "g");
  TORCH_CHECK(x.numel() == up_qw.size(1) * 2, "gather_up_h: x/up_qw mismatch");
  TORCH_CHECK(g.numel() == up_qw.size(0), "gather_up_h: g must have one value per row");
  Tensor idx = idx32(idx_in, "idx");
  Tensor h = bf16_empty(idx.numel(), x);
  check_status(dip_gather_up_h(i8(up_qw), bf(up_sc), up_qw.size(0), bf(x), bf(g),
                               idx.data_ptr<int32_t>(), idx.numel(), up_qw.size(1) * 2, bfm(h),
                               cur_stream()),
               "gather_up_h");
  return h;
}

Tensor gather_down_idx(const Tensor& dt_qw, const Tensor& dt_sc, const Tensor& h_in,
                       const Tensor& idx_in) {
  check_packed(dt_qw, dt_sc, "gather_down_idx");
  c10::cuda::CUDAGuard guard(dt_qw.device());
  Tensor h = h_in.contiguous();
  check_dtype(h, at::kBFloat16, "h");
  Tensor idx = idx32(idx_in, "idx");
  TORCH_CHECK(h.numel() == idx.numel(), "gather_down_idx: h/idx length mismatch");
  const int64_t out_f = dt_qw.size(1) * 2;
  Tensor y = bf16_empty(out_f, h);
  Tensor ws = at::empty({(int64_t)dip_gather_down_workspace_bytes(out_f)},
                        h.options().dtype(at::kByte));
  check_status(dip_int4_gather_down(i8(dt_qw), bf(dt_sc), dt_qw.size(0), bf(h),
                                    idx.data_ptr<int32_t>(), idx.numel(), out_f, ws.data_ptr(),
                                    ws.numel(), bfm(y), cur_stream()),
               "gather_down_idx");
  return y;
}

std::tuple<Tensor, Tensor, Tensor, Tensor> ca_split(const Tensor& idx_in,
                                                    const Tensor& id2slot_in) {
  Tensor idx = idx32(idx_in, "idx");
  TORCH_CHECK(id2slot_in.is_cuda() && id2slot_in.scalar_type() == at::kLong,
              "ca_split: id2slot must be a CUDA int64 tensor");
  Tensor id2slot = id2slot_in.contiguous();
  c10::cuda::CUDAGuard guard(idx.device());
  const int64_t k = idx.numel();
  auto iopt = idx.options().dtype(at::kInt);
  Tensor comb = at::empty({k}, iopt), src = at::empty({k}, iopt), row = at::empty({k}, iopt);
  Tensor nhit = at::empty({1}, iopt);
  check_status(dip_ca_split(idx.data_ptr<int32_t>(), k, id2slot.data_ptr<int64_t>(),
                            id2slot.numel(), comb.data_ptr<int32_t>(), src.data_ptr<int32_t>(),
                            row.data_ptr<int32_t>(), nhit.data_ptr<int32_t>(), cur_stream()),
               "ca_split");
  return {comb, src, row, nhit};
}

Tensor srcrow_up_h(const Tensor& res_qw, const Tensor& res_sc, const Tensor& full_qw,
                   const Tensor& full_sc, const Tensor& x_in, const Tensor& g_in,
                   const Tensor& comb_in, const Tensor& src_in, const Tensor& row_in) {
  check_packed(full_qw, full_sc, "srcrow_up_h(full)");
  check_packed(res_qw, res_sc, "srcrow_up_h(res)");
  c10::cuda::CUDAGuard guard(full_qw.device());
  Tensor x = x_in.contiguous(), g = g_in.contiguous();
  check_dtype(x, at::kBFloat16, "x");
  check_dtype(g, at::kBFloat16, "g");
  TORCH_CHECK(x.numel() == full_qw.size(1) * 2 && res_qw.size(1) == full_qw.size(1),
              "srcrow_up_h: shape mismatch");
  Tensor comb = idx32(comb_in, "combined_ids"), src = idx32(src_in, "src"),
         row = idx32(row_in, "row");
  Tensor h = bf16_empty(src.numel(), x);
  check_status(dip_srcrow_up_h(i8(res_qw), bf(res_sc), res_qw.size(0), i8(full_qw), bf(full_sc),
                               full_qw.size(0), bf(x), bf(g), comb.data_ptr<int32_t>(),
                               src.data_ptr<int32_t>(), row.data_ptr<int32_t>(), src.numel(),
                               full_qw.size(1) * 2, bfm(h), cur_stream()),
               "srcrow_up_h");
  return h;
}

Tensor srcrow_down(const Tensor& res_dt, const Tensor& res_sc, const Tensor& full_dt,
                   const Tensor& full_sc, const Tensor& h_in, const Tensor& src_in,
                   const Tensor& row_in) {
  check_packed(full_dt, full_sc, "srcrow_down(full)");
  check_packed(res_dt, res_sc, "srcrow_down(res)");
  c10::cuda::CUDAGuard guard(full_dt.device());
  Tensor h = h_in.contiguous();
  check_dtype(h, at::kBFloat16, "h");
  Tensor src = idx32(src_in, "src"), row = idx32(row_in, "row");
  const int64_t out_f = full_dt.size(1) * 2;
  Tensor y = bf16_empty(out_f, h);
  Tensor ws = at::empty({(int64_t)dip_gather_down_workspace_bytes(out_f)},
                        h.options().dtype(at::kByte));
  check_status(dip_srcrow_down(i8(res_dt), bf(res_sc), res_dt.size(0), i8(full_dt), bf(full_sc),
                               full_dt.size(0), bf(h), src.data_ptr<int32_t>(),
                               row.data_ptr<int32_t>(), src.numel(), out_f, ws.data_ptr(),
                               ws.numel(), bfm(y), cur_stream()),
               "srcrow_down");
  return y;
}

std::tuple<Tensor, Tensor, Tensor> mlp_decode(const Tensor& gate_qw, const Tensor& gate_sc,
                                              const Tensor& up_qw, const Tensor& up_sc,
                                              const Tensor& dt_qw, const Tensor& dt_sc,
                                              const Tensor& x_in, int64_t k,
                                              const std::optional<Tensor>& ws_opt) {
  check_packed(gate_qw, gate_sc, "mlp_decode(gate)");
  check_packed(up_qw, up_sc, "mlp_decode(up)");
  check_packed(dt_qw, dt_sc, "mlp_decode(down_t)");
  c10::cuda::CUDAGuard guard(gate_qw.device());
  Tensor x = x_in.contiguous();
  check_dtype(x, at::kBFloat16, "x");
  const int64_t hidden = gate_qw.size(1) * 2, inter = gate_qw.size(0);
  TORCH_CHECK(x.numel() == hidden && up_qw.sizes() == gate_qw.sizes() &&
                  dt_qw.size(0) == inter && dt_qw.size(1) * 2 == hidden,
              "mlp_decode: shape mismatch");
  dip_layer_t L = {i8(gate_qw), bf(gate_sc), i8(up_qw), bf(up_sc), i8(dt_qw), bf(dt_sc),
                   hidden, inter};
  Tensor y = bf16_empty(hidden, x), g = bf16_empty(inter, x);
  Tensor idx = at::empty({k}, x.options().dtype(at::kInt));
  const size_t wsb = dip_mlp_workspace_bytes(hidden, inter, k);
  Tensor ws = ws_opt.has_value() ? *ws_opt : at::zeros({(int64_t)wsb}, x.options().dtype(at::kByte));
  TORCH_CHECK(ws.is_cuda() && ws.is_contiguous() && (size_t)ws.nbytes() >= wsb,
              "mlp_decode: workspace too small (need ", wsb, " bytes)");
  check_status(dip_mlp_decode(&L, bf(x), k, ws.data_ptr(), wsb, bfm(y), bfm(g),
                              idx.data_ptr<int32_t>(), cur_stream()),
               "mlp_decode");
  return {y, g, idx};
}

std::tuple<Tensor, Tensor> quantize_int4(const Tensor& w_in) {
  Tensor w = w_in.contiguous();
  check_cuda(w, "w");
  check_dtype(w, at::kBFloat16, "w");
  TORCH_CHECK(w.dim() == 2 && w.size(1) % 128 == 0, "quantize_int4: w must be [out, in%128==0]");
  c10::cuda::CUDAGuard guard(w.device());
  Tensor qw = at::empty({w.size(0), w.size(1) / 2}, w.options().dtype(at::kChar));
  Tensor sc = at::empty({w.size(0), w.size(1) / 128}, w.options());
  check_status(dip_quantize_int4_g128(bf(w), w.size(0), w.size(1),
                                      reinterpret_cast<int8_t*>(qw.data_ptr()), bfm(sc),
                                      cur_stream()),
               "quantize_int4");
  return {qw, sc};
}

Tensor dequantize_int4(const Tensor& qw, const Tensor& sc) {
  check_packed(qw, sc, "dequantize_int4");
  c10::cuda::CUDAGuard guard(qw.device());
  Tensor w = at::empty({qw.size(0), qw.size(1) * 2}, sc.options());
  check_status(dip_dequantize_int4_g128(i8(qw), bf(sc), qw.size(0), qw.size(1) * 2, bfm(w),
                                        cur_stream()),
               "dequantize_int4");
  return w;
}

std::tuple<Tensor, Tensor> transpose_down_int4(const Tensor& dqw, const Tensor& dsc) {
  check_packed(dqw, dsc, "transpose_down_int4");
  c10::cuda::CUDAGuard guard(dqw.device());
  const int64_t out_f = dqw.size(0), inter = dqw.size(1) * 2;
  TORCH_CHECK(out_f % 128 == 0, "transpose_down_int4: out_features must be a multiple of 128");
  Tensor tq = at::empty({inter, out_f / 2}, dqw.options().dtype(at::kChar));
  Tensor ts = at::empty({inter, out_f / 128}, dsc.options());
  check_status(dip_transpose_down_int4(i8(dqw), bf(dsc), out_f, inter,
                                       reinterpret_cast<int8_t*>(tq.data_ptr()), bfm(ts),
                                       cur_stream()),
               "transpose_down_int4");
  return {tq, ts};
}

Tensor residual_rmsnorm(const Tensor& y_in, const Tensor& r_in, double eps) {
  Tensor y = y_in.contiguous(), r = r_in.contiguous();
  check_cuda(y, "y");
  check_cuda(r, "r");
  check_dtype(y, at::kBFloat16, "y");
  check_dtype(r, at::kBFloat16, "r");
  TORCH_CHECK(y.numel() == r.numel(), "residual_rmsnorm: y/r size mismatch");
  TORCH_CHECK(y.dim() == 1 || y.dim() == 2, "residual_rmsnorm: y must be [n] or [rows, n]");
  c10::cuda::CUDAGuard guard(y.device());
  Tensor out = at::empty_like(y);
  const int64_t rows = y.dim() == 2 ? y.size(0) : 1;
  const int64_t n = y.dim() == 2 ? y.size(1) : y.numel();
  check_status(dip_residual_rmsnorm_rows(bf(y), bf(r), rows, n, (float)eps, bfm(out), cur_stream()),
               "residual_rmsnorm");
  return out;
}

// batched decode / dense forward on tcgen05: x [B, in] -> [B, rows]
Tensor gemm_tc(const Tensor& qweight, const Tensor& scales, const Tensor& x_in, int64_t epilogue,
               const c10::optional<Tensor>& g_in, const c10::optional<Tensor>& cnt_in,
               int64_t ksplit) {
  check_packed(qweight, scales, "gemm_tc");
  Tensor x = x_in.contiguous();
  check_cuda(x, "x");
  check_dtype(x, at::kBFloat16, "x");
  TORCH_CHECK(x.dim() == 2 && x.size(1) == qweight.size(1) * 2, "gemm_tc: x must be [B, in]");
  c10::cuda::CUDAGuard guard(x.device());
  Tensor out = at::empty({x.size(0), qweight.size(0)}, x.options());
  if (x.size(0) == 0) return out;
  Tensor g, cnt;
  const uint16_t* gp = nullptr;
  const uint32_t* cp = nullptr;
  if (epilogue == 2) {
    TORCH_CHECK(g_in.has_value() && cnt_in.has_value(), "gemm_tc: epilogue 2 needs g and cnt");
    g = g_in->contiguous();
    cnt = cnt_in->contiguous();
    check_dtype(g, at::kBFloat16, "g");
    check_dtype(cnt, at::kInt, "cnt");
    TORCH_CHECK(g.sizes() == out.sizes() && cnt.sizes() == out.sizes(), "gemm_tc: g / cnt must be [B, rows]");
    gp = bf(g);
    cp = reinterpret_cast<const uint32_t*>(cnt.data_ptr<int32_t>());
  }
  const size_t nws = dip_int4_gemm_tc_workspace_bytes(qweight.size(0), x.size(1), x.size(0));
  Tensor ws = at::empty({(int64_t)nws}, x.options().dtype(at::kByte));
  check_status(dip_int4_gemm_tc_split(i8(qweight), bf(scales), bf(x), qweight.size(0), x.size(1),
                                      x.size(0), (int)epilogue, gp, cp, (int)ksplit, ws.data_ptr(),
                                      nws, bfm(out), cur_stream()),
               "gemm_tc");
  return out;
}

// h [B, inter] -> fp32 y [B, hidden] (a tensor-parallel partial)
Tensor down_tc_f32(const Tensor& dt_qw, const Tensor& dt_sc, const Tensor& h_in) {
  check_packed(dt_qw, dt_sc, "down_tc_f32");
  Tensor h = h_in.contiguous();
  check_cuda(h, "h");
  check_dtype(h, at::kBFloat16, "h");
  TORCH_CHECK(h.dim() == 2 && h.size(1) == dt_qw.size(0), "down_tc_f32: h must be [B, inter]");
  c10::cuda::CUDAGuard guard(h.device());
  const int64_t out_f = dt_qw.size(1) * 2, B = h.size(0);
  Tensor y = at::empty({B, out_f}, h.options().dtype(at::kFloat));
  if (B == 0) return y;
  const size_t nws = dip_int4_down_tc_workspace_bytes(out_f, B);
  Tensor ws = at::empty({(int64_t)nws}, h.options().dtype(at::kByte));
  check_status(dip_int4_down_tc_f32(i8(dt_qw), bf(dt_sc), bf(h), dt_qw.size(0), out_f, B,
                                    ws.data_ptr(), nws, y.data_ptr<float>(), cur_stream()),
               "down_tc_f32");
  return y;
}

int64_t op_gemm_tc_auto_split(int64_t rows, int64_t in_features) {
  return dip_int4_gemm_tc_auto_split(rows, in_features);
}

// h [B, inter] -> y [B, hidden] over the transposed down weights
Tensor down_tc(const Tensor& dt_qw, const Tensor& dt_sc, const Tensor& h_in) {
  check_packed(dt_qw, dt_sc, "down_tc");
  Tensor h = h_in.contiguous();
  check_cuda(h, "h");
  check_dtype(h, at::kBFloat16, "h");
  TORCH_CHECK(h.dim() == 2 && h.size(1) == dt_qw.size(0), "down_tc: h must be [B, inter]");
  c10::cuda::CUDAGuard guard(h.device());
  const int64_t out_f = dt_qw.size(1) * 2, B = h.size(0);
  Tensor y = at::empty({B, out_f}, h.options());
  if (B == 0) return y;
  const size_t nws = dip_int4_down_tc_workspace_bytes(out_f, B);
  Tensor ws = at::empty({(int64_t)nws}, h.options().dtype(at::kByte));
  check_status(dip_int4_down_tc(i8(dt_qw), bf(dt_sc), bf(h), dt_qw.size(0), out_f, B, ws.data_ptr(),
                                nws, bfm(y), cur_stream()),
               "down_tc");
  return y;
}

// idx [B, k] -> cnt [B, inter] (int32 counts)
Tensor select_count(const Tensor& idx_in, int64_t inter) {
  Tensor idx = idx_in.contiguous();
  check_cuda(idx, "idx");
  check_dtype(idx, at::kInt, "idx");
  TORCH_CHECK(idx.dim() == 2, "select_count: idx must be [B, k]");
  c10::cuda::CUDAGuard guard(idx.device());
  Tensor cnt = at::empty({idx.size(0), inter}, idx.options());
  if (idx.size(0) == 0) return cnt;
  check_status(dip_select_count(idx.data_ptr<int32_t>(), idx.size(0), idx.size(1), inter,
                                reinterpret_cast<uint32_t*>(cnt.data_ptr<int32_t>()), cur_stream()),
               "select_count");
  return cnt;
}

// config 3: x [B, in] -> [B, rows] (gate GEMV with SiLU, or plain)
Tensor gemv_batched(const Tensor& qweight, const Tensor& scales, const Tensor& x_in, bool silu) {
  check_packed(qweight, scales, "gemv_batched");
  Tensor x = x_in.contiguous();
  check_cuda(x, "x");
  check_dtype(x, at::kBFloat16, "x");
  TORCH_CHECK(x.dim() == 2 && x.size(1) == qweight.size(1) * 2, "gemv_batched: x must be [B, in]");
  c10::cuda::CUDAGuard guard(x.device());
  Tensor out = at::empty({x.size(0), qweight.size(0)}, x.options());
  check_status(dip_int4_gemv_batched(i8(qweight), bf(scales), bf(x), bfm(out), qweight.size(0),
                                     x.size(1), x.size(0), silu ? 1 : 0, cur_stream()),
               "gemv_batched");
  return out;
}

std::tuple<Tensor, Tensor> shard_select(const Tensor& idx_in, int64_t lo, int64_t hi) {
  Tensor idx = idx32(idx_in, "idx");
  c10::cuda::CUDAGuard guard(idx.device());
  const int64_t k = idx.numel();
  auto iopt = idx.options().dtype(at::kInt);
  Tensor local = at::empty({std::max<int64_t>(1, std::min<int64_t>(k, hi - lo))}, iopt);
  Tensor count = at::empty({1}, iopt);
  check_status(dip_shard_select(idx.data_ptr<int32_t>(), k, lo, hi, local.data_ptr<int32_t>(),
                                count.data_ptr<int32_t>(), cur_stream()),
               "shard_select");
  return {local, count};
}

Tensor gather_up_h_count(const Tensor& up_qw, const Tensor& up_sc, const Tensor& x_in,
                         const Tensor& g_in, const Tensor& idx_in, const Tensor& count) {
  check_packed(up_qw, up_sc, "gather_up_h_count");
  c10::cuda::CUDAGuard guard(up_qw.device());
  Tensor x = x_in.contiguous(), g = g_in.contiguous();
  check_dtype(x, at::kBFloat16, "x");
  check_dtype(g, at::kBFloat16, "g");
  TORCH_CHECK(x.numel() == up_qw.size(1) * 2 && g.numel() == up_qw.size(0),
              "gather_up_h_count: shape mismatch");
  Tensor idx = idx32(idx_in, "idx");
  check_dtype(count, at::kInt, "count");
  Tensor h = bf16_empty(idx.numel(), x);
  check_status(dip_gather_up_h_count(i8(up_qw), bf(up_sc), up_qw.size(0), bf(x), bf(g),
                                     idx.data_ptr<int32_t>(), count.data_ptr<int32_t>(),
                                     idx.numel(), up_qw.size(1) * 2, bfm(h), cur_stream()),
               "gather_up_h_count");
  return h;
}

Tensor gather_down_partial(const Tensor& dt_qw, const Tensor& dt_sc, const Tensor& h_in,
                           const Tensor& idx_in, const Tensor& count) {
  check_packed(dt_qw, dt_sc, "gather_down_partial");
  c10::cuda::CUDAGuard guard(dt_qw.device());
  Tensor h = h_in.contiguous();
  check_dtype(h, at::kBFloat16, "h");
  Tensor idx = idx32(idx_in, "idx");
  check_dtype(count, at::kInt, "count");
  TORCH_CHECK(h.numel() == idx.numel(), "gather_down_partial: h/idx length mismatch");
  const int64_t out_f = dt_qw.size(1) * 2;
  Tensor y = at::empty({out_f}, h.options().dtype(at::kFloat));
  Tensor ws = at::empty({(int64_t)dip_gather_down_workspace_bytes(out_f)},
                        h.options().dtype(at::kByte));
  check_status(dip_gather_down_partial(i8(dt_qw), bf(dt_sc), dt_qw.size(0), bf(h),
                                       idx.data_ptr<int32_t>(), count.data_ptr<int32_t>(),
                                       idx.numel(), out_f, ws.data_ptr(), ws.numel(),
                                       y.data_ptr<float>(), cur_stream()),
               "gather_down_partial");
  return y;
}

// Optional extras of a fused-layer call: h_out [h_len] bf16; the next
// layer's gate weights (same shape as this layer's) for the L2 prefetch.
dip_fused_opts_t make_opts(const std::optional<Tensor>& h_out, const std::optional<Tensor>& next_gq,
                           const std::optional<Tensor>& next_gs, const Tensor& gate_qw,
                           const Tensor& gate_sc, int64_t h_len) {
  dip_fused_opts_t o = {nullptr, nullptr, nullptr};
  if (h_out.has_value()) {
    TORCH_CHECK(h_out->is_cuda() && h_out->is_contiguous() &&
                    h_out->scalar_type() == at::kBFloat16 && h_out->numel() == h_len,
                "h_out must be a contiguous CUDA bf16 tensor of ", h_len, " elements");
    o.h_out = reinterpret_cast<dip_bf16*>(h_out->data_ptr());
  }
  TORCH_CHECK(next_gq.has_value() == next_gs.has_value(),
              "next_gate_qw and next_gate_sc go together");
  if (next_gq.has_value()) {
    TORCH_CHECK(next_gq->is_cuda() && next_gq->is_contiguous() && next_gs->is_contiguous() &&
                    next_gq->sizes() == gate_qw.sizes() && next_gs->sizes() == gate_sc.sizes(),
                "next layer's gate weights must be contiguous CUDA tensors of this layer's shape");
    o.prefetch_gate_qw = i8(*next_gq);
    o.prefetch_gate_sc = bf(*next_gs);
  }
  return o;
}

std::tuple<Tensor, Tensor, Tensor> mlp_decode_fused_impl(
    const Tensor& gate_qw, const Tensor& gate_sc, const Tensor& up_qw, const Tensor& up_sc,
    const Tensor& dt_qw, const Tensor& dt_sc, const dip_ca_cache_t* cache, const Tensor& x_in,
    const std::optional<Tensor>& resid, double eps, int64_t k, const std::optional<Tensor>& ws_opt,
    const std::optional<Tensor>& h_out = std::nullopt,
    const std::optional<Tensor>& next_gq = std::nullopt,
    const std::optional<Tensor>& next_gs = std::nullopt) {
  check_packed(gate_qw, gate_sc, "mlp_decode_fused(gate)");
  check_packed(up_qw, up_sc, "mlp_decode_fused(up)");
  check_packed(dt_qw, dt_sc, "mlp_decode_fused(down_t)");
  c10::cuda::CUDAGuard guard(gate_qw.device());
  Tensor x = x_in.contiguous();
  check_dtype(x, at::kBFloat16, "x");
  const int64_t hidden = gate_qw.size(1) * 2, inter = gate_qw.size(0);
  TORCH_CHECK(x.numel() == hidden && up_qw.sizes() == gate_qw.sizes() &&
                  dt_qw.size(0) == inter && dt_qw.size(1) * 2 == hidden,
              "mlp_decode_fused: shape mismatch");
  Tensor r;
  if (resid.has_value()) {
    r = resid->contiguous();
    check_dtype(r, at::kBFloat16, "resid");
    TORCH_CHECK(r.numel() == hidden, "mlp_decode_fused: resid size");
  }
  dip_layer_t L = {i8(gate_qw), bf(gate_sc), i8(up_qw), bf(up_sc), i8(dt_qw), bf(dt_sc),
                   hidden, inter};
  Tensor y = bf16_empty(hidden, x), g = bf16_empty(inter, x);
  Tensor idx = at::empty({k}, x.options().dtype(at::kInt));
  const size_t wsb = dip_mlp_fused_workspace_bytes(hidden, inter, k);
  Tensor ws = ws_opt.has_value() ? *ws_opt : at::zeros({(int64_t)wsb}, x.options().dtype(at::kByte));
  TORCH_CHECK(ws.is_cuda() && ws.is_contiguous() && (size_t)ws.nbytes() >= wsb,
              "mlp_decode_fused: workspace too small (need ", wsb, " bytes)");
  const dip_fused_opts_t opts = make_opts(h_out, next_gq, next_gs, gate_qw, gate_sc, inter);
  check_status(dip_mlp_decode_fused_ex(&L, cache, bf(x), resid.has_value() ? bf(r) : nullptr,
                                       (float)eps, k, ws.data_ptr(), wsb, bfm(y), bfm(g),
                                       idx.data_ptr<int32_t>(), nullptr, &opts, cur_stream()),
               "mlp_decode_fused");
  return {y, g, idx};
}

std::tuple<Tensor, Tensor, Tensor> mlp_decode_fused(
    const Tensor& gate_qw, const Tensor& gate_sc, const Tensor& up_qw, const Tensor& up_sc,
    const Tensor& dt_qw, const Tensor& dt_sc, const Tensor& x_in, const std::optional<Tensor>& resid,
    double eps, int64_t k, const std::optional<Tensor>& ws_opt, const std::optional<Tensor>& h_out,
    const std::optional<Tensor>& next_gq, const std::optional<Tensor>& next_gs) {
  return mlp_decode_fused_impl(gate_qw, gate_sc, up_qw, up_sc, dt_qw, dt_sc, nullptr, x_in, resid,
                               eps, k, ws_opt, h_out, next_gq, next_gs);
}

// the cache-aware layer in one launch (dip_mlp_decode_fused_ca)
std::tuple<Tensor, Tensor, Tensor> mlp_decode_fused_ca(
    const Tensor& gate_qw, const Tensor& gate_sc, const Tensor& up_qw, const Tensor& up_sc,
    const Tensor& dt_qw, const Tensor& dt_sc, const Tensor& id2slot, const Tensor& res_up_qw,
    const Tensor& res_up_sc, const Tensor& res_dn_qw, const Tensor& res_dn_sc, const Tensor& x_in,
    const std::optional<Tensor>& resid, double eps, int64_t k,
    const std::optional<Tensor>& ws_opt, const std::optional<Tensor>& next_gq,
    const std::optional<Tensor>& next_gs) {
  TORCH_CHECK(id2slot.is_cuda() && id2slot.scalar_type() == at::kLong && id2slot.is_contiguous() &&
                  id2slot.numel() == gate_qw.size(0),
              "mlp_decode_fused_ca: id2slot must be a contiguous CUDA int64 [inter] tensor");
  check_packed(res_up_qw, res_up_sc, "mlp_decode_fused_ca(res_up)");
  check_packed(res_dn_qw, res_dn_sc, "mlp_decode_fused_ca(res_dn)");
  TORCH_CHECK(res_up_qw.size(1) == up_qw.size(1) && res_dn_qw.size(1) == dt_qw.size(1) &&
                  res_up_qw.size(0) == res_dn_qw.size(0),
              "mlp_decode_fused_ca: cache shape mismatch");
  dip_ca_cache_t c = {id2slot.data_ptr<int64_t>(), i8(res_up_qw), bf(res_up_sc), i8(res_dn_qw),
                      bf(res_dn_sc), res_up_qw.size(0)};
  return mlp_decode_fused_impl(gate_qw, gate_sc, up_qw, up_sc, dt_qw, dt_sc, &c, x_in, resid, eps,
                               k, ws_opt, std::nullopt, next_gq, next_gs);
}

// one tensor-parallel layer on this rank (dip_mlp_decode_fused_tp); the
// workspaces are raw device addresses (own + IPC-mapped peers)
std::tuple<Tensor, Tensor> mlp_decode_fused_tp(
    const Tensor& gate_qw, const Tensor& gate_sc, const Tensor& up_qw, const Tensor& up_sc,
    const Tensor& dt_qw, const Tensor& dt_sc, const Tensor& x_in, const std::optional<Tensor>& resid,
    double eps, int64_t k, int64_t inter_total, int64_t rank, int64_t world,
    at::IntArrayRef workspaces, int64_t workspace_bytes, const std::optional<Tensor>& idx_out,
    const std::optional<Tensor>& x_used, const std::optional<Tensor>& h_out,
    const std::optional<Tensor>& next_gq, const std::optional<Tensor>& next_gs) {
  check_packed(gate_qw, gate_sc, "mlp_decode_fused_tp(gate)");
  check_packed(up_qw, up_sc, "mlp_decode_fused_tp(up)");
  check_packed(dt_qw, dt_sc, "mlp_decode_fused_tp(down_t)");
  c10::cuda::CUDAGuard guard(gate_qw.device());
  Tensor x = x_in.contiguous();
  check_dtype(x, at::kBFloat16, "x");
  const int64_t hidden = gate_qw.size(1) * 2, inter = gate_qw.size(0);
  TORCH_CHECK(x.numel() == hidden && up_qw.sizes() == gate_qw.sizes() &&
                  dt_qw.size(0) == inter && dt_qw.size(1) * 2 == hidden,
              "mlp_decode_fused_tp: shape mismatch");
  TORCH_CHECK((int64_t)workspaces.size() == world, "mlp_decode_fused_tp: one workspace per rank");
  Tensor r;
  if (resid.has_value()) {
    r = resid->contiguous();
    check_dtype(r, at::kBFloat16, "resid");
    TORCH_CHECK(r.numel() == hidden, "mlp_decode_fused_tp: resid size");
  }
  int32_t* idxp = nullptr;
  if (idx_out.has_value()) {
    TORCH_CHECK(idx_out->is_cuda() && idx_out->is_contiguous() &&
                    idx_out->scalar_type() == at::kInt && idx_out->numel() == k,
                "mlp_decode_fused_tp: idx_out must be a contiguous CUDA int32 [k] tensor");
    idxp = idx_out->data_ptr<int32_t>();
  }
  dip_bf16* xu = nullptr;
  if (x_used.has_value()) {
    TORCH_CHECK(x_used->is_cuda() && x_used->is_contiguous() &&
                    x_used->scalar_type() == at::kBFloat16 && x_used->numel() == hidden,
                "mlp_decode_fused_tp: x_used must be a contiguous CUDA bf16 [hidden] tensor");
    xu = reinterpret_cast<dip_bf16*>(x_used->data_ptr());
  }
  dip_layer_t L = {i8(gate_qw), bf(gate_sc), i8(up_qw), bf(up_sc), i8(dt_qw), bf(dt_sc),
                   hidden, inter};
  std::vector<void*> ws(workspaces.size());
  for (size_t q = 0; q < ws.size(); ++q) ws[q] = reinterpret_cast<void*>(workspaces[q]);
  Tensor y = bf16_empty(hidden, x), g = bf16_empty(inter, x);
  const dip_fused_opts_t opts = make_opts(h_out, next_gq, next_gs, gate_qw, gate_sc, inter_total);
  check_status(dip_mlp_decode_fused_tp(&L, inter_total, (int)rank, (int)world, ws.data(),
                                       (size_t)workspace_bytes, bf(x),
                                       resid.has_value() ? bf(r) : nullptr, (float)eps, k, bfm(y),
                                       bfm(g), idxp, xu, &opts, cur_stream()),
               "mlp_decode_fused_tp");
  return {y, g};
}

int64_t op_mlp_fused_tp_workspace_bytes(int64_t hidden, int64_t inter_total, int64_t k) {
  return (int64_t)dip_mlp_fused_tp_workspace_bytes(hidden, inter_total, k);
}

int64_t op_set_spin_limit(int64_t polls) {
  check_status(dip_set_spin_limit((unsigned)polls), "set_spin_limit");
  return 0;
}

int64_t op_mlp_fused_workspace_bytes(int64_t hidden, int64_t inter, int64_t k) {
  return (int64_t)dip_mlp_fused_workspace_bytes(hidden, inter, k);
}

int64_t op_mlp_workspace_bytes(int64_t hidden, int64_t inter, int64_t k) {
  return (int64_t)dip_mlp_workspace_bytes(hidden, inter, k);
}

int64_t op_set_pdl(int64_t enable) { return dip_set_pdl((int)enable); }
int64_t op_set_gemv_variant(int64_t simple) { return dip_set_gemv_variant((int)simple); }
int64_t op_take_device_error() {
  unsigned int v = 0;
  check_status(dip_take_device_error(&v), "take_device_error");
  return (int64_t)v;
}

}  // namespace

TORCH_LIBRARY(int4_ops, m) { m.def("int4_gemv(Tensor qweight, Tensor scales, Tensor x) -> Tensor"); }
TORCH_LIBRARY_IMPL(int4_ops, CUDA, m) { m.impl("int4_gemv", &int4_gemv); }

TORCH_LIBRARY(topk_ops, m) { m.def("topk_select(Tensor s, int k) -> Tensor"); }
TORCH_LIBRARY_IMPL(topk_ops, CUDA, m) { m.impl("topk_select", &topk_select); }

TORCH_LIBRARY(int4_gather_ops, m) {
  m.def("int4_gather_gemv(Tensor qweight, Tensor scales, Tensor x, Tensor indices) -> Tensor");
}
TORCH_LIBRARY_IMPL(int4_gather_ops, CUDA, m) { m.impl("int4_gather_gemv", &int4_gather_gemv); }

TORCH_LIBRARY(int4_down_ops, m) {
  m.def("int4_gather_down(Tensor down_t_sel, Tensor scales, Tensor h_sel) -> Tensor");
}
TORCH_LIBRARY_IMPL(int4_down_ops, CUDA, m) { m.impl("int4_gather_down", &int4_gather_down); }

TORCH_LIBRARY(ca_fused_ops, m) {
  m.def(
      "ca_fused_gemv(Tensor res_qw, Tensor res_sc, Tensor str_qw, Tensor str_sc, Tensor x, "
      "Tensor src, Tensor row) -> Tensor");
}
TORCH_LIBRARY_IMPL(ca_fused_ops, CUDA, m) { m.impl("ca_fused_gemv", &ca_fused_gemv); }

TORCH_LIBRARY(dip_b200, m) {
  m.def("gate_silu(Tensor qweight, Tensor scales, Tensor x) -> Tensor");
  m.def("topk_select_batched(Tensor s, int k) -> Tensor");
  m.def("gather_up_h(Tensor up_qw, Tensor up_sc, Tensor x, Tensor g, Tensor idx) -> Tensor");
  m.def("gather_down_idx(Tensor down_t_qw, Tensor down_t_sc, Tensor h, Tensor idx) -> Tensor");
  m.def("ca_split(Tensor idx, Tensor id2slot) -> (Tensor, Tensor, Tensor, Tensor)");
  m.def(
      "srcrow_up_h(Tensor res_qw, Tensor res_sc, Tensor full_qw, Tensor full_sc, Tensor x, "
      "Tensor g, Tensor combined_ids, Tensor src, Tensor row) -> Tensor");
  m.def(
      "srcrow_down(Tensor res_dt, Tensor res_sc, Tensor full_dt, Tensor full_sc, Tensor h, "
      "Tensor src, Tensor row) -> Tensor");
  m.def(
      "mlp_decode(Tensor gate_qw, Tensor gate_sc, Tensor up_qw, Tensor up_sc, Tensor down_t_qw, "
      "Tensor down_t_sc, Tensor x, int k, Tensor? workspace=None) -> (Tensor, Tensor, Tensor)");
  m.def("mlp_workspace_bytes(int hidden, int inter, int k) -> int");
  m.def(
      "mlp_decode_fused(Tensor gate_qw, Tensor gate_sc, Tensor up_qw, Tensor up_sc, "
      "Tensor down_t_qw, Tensor down_t_sc, Tensor x, Tensor? resid, float eps, int k, "
      "Tensor? workspace=None, Tensor? h_out=None, Tensor? next_gate_qw=None, "
      "Tensor? next_gate_sc=None) -> (Tensor, Tensor, Tensor)");
  m.def("mlp_fused_workspace_bytes(int hidden, int inter, int k) -> int");
  m.def(
      "mlp_decode_fused_tp(Tensor gate_qw, Tensor gate_sc, Tensor up_qw, Tensor up_sc, "
      "Tensor down_t_qw, Tensor down_t_sc, Tensor x, Tensor? resid, float eps, int k, "
      "int inter_total, int rank, int world, int[] workspaces, int workspace_bytes, "
      "Tensor? idx_out=None, Tensor? x_used=None, Tensor? h_out=None, "
      "Tensor? next_gate_qw=None, Tensor? next_gate_sc=None) -> (Tensor, Tensor)");
  m.def("mlp_fused_tp_workspace_bytes(int hidden, int inter_total, int k) -> int");
  m.def("set_spin_limit(int polls) -> int");
  m.def(
      "mlp_decode_fused_ca(Tensor gate_qw, Tensor gate_sc, Tensor up_qw, Tensor up_sc, "
      "Tensor down_t_qw, Tensor down_t_sc, Tensor id2slot, Tensor res_up_qw, Tensor res_up_sc, "
      "Tensor res_dn_qw, Tensor res_dn_sc, Tensor x, Tensor? resid, float eps, int k, "
      "Tensor? workspace=None, Tensor? next_gate_qw=None, Tensor? next_gate_sc=None) "
      "-> (Tensor, Tensor, Tensor)");
  m.def("quantize_int4(Tensor w) -> (Tensor, Tensor)");
  m.def("dequantize_int4(Tensor qweight, Tensor scales) -> Tensor");
  m.def("transpose_down_int4(Tensor down_qw, Tensor down_sc) -> (Tensor, Tensor)");
  m.def("residual_rmsnorm(Tensor y, Tensor r, float eps) -> Tensor");
  m.def("gemv_batched(Tensor qweight, Tensor scales, Tensor x, bool silu) -> Tensor");
  m.def("gemm_tc(Tensor qweight, Tensor scales, Tensor x, int epilogue, Tensor? g=None, Tensor? cnt=None, int ksplit=0) -> Tensor");
  m.def("down_tc_f32(Tensor down_t_qw, Tensor down_t_sc, Tensor h) -> Tensor");
  m.def("gemm_tc_auto_split(int rows, int in_features) -> int");
  m.def("down_tc(Tensor down_t_qw, Tensor down_t_sc, Tensor h) -> Tensor");
  m.def("select_count(Tensor idx, int inter) -> Tensor");
  m.def("shard_select(Tensor idx, int lo, int hi) -> (Tensor, Tensor)");
  m.def(
      "gather_up_h_count(Tensor up_qw, Tensor up_sc, Tensor x, Tensor g, Tensor idx, "
      "Tensor count) -> Tensor");
  m.def(
      "gather_down_partial(Tensor down_t_qw, Tensor down_t_sc, Tensor h, Tensor idx, "
      "Tensor count) -> Tensor");
  m.def("set_pdl(int enable) -> int");
  m.def("set_gemv_variant(int simple) -> int");
  m.def("take_device_error() -> int");
}
TORCH_LIBRARY_IMPL(dip_b200, CUDA, m) {
  m.impl("gate_silu", &gate_silu);
  m.impl("topk_select_batched", &topk_select_batched);
  m.impl("gather_up_h", &gather_up_h);
  m.impl("gather_down_idx", &gather_down_idx);
  m.impl("ca_split", &ca_split);
  m.impl("srcrow_up_h", &srcrow_up_h);
  m.impl("srcrow_down", &srcrow_down);
  m.impl("mlp_decode", &mlp_decode);
  m.impl("mlp_decode_fused", &mlp_decode_fused);
  m.impl("mlp_decode_fused_ca", &mlp_decode_fused_ca);
  m.impl("mlp_decode_fused_tp", &mlp_decode_fused_tp);
  m.impl("quantize_int4", &quantize_int4);
  m.impl("dequantize_int4", &dequantize_int4);
  m.impl("transpose_down_int4", &transpose_down_int4);
  m.impl("residual_rmsnorm", &residual_rmsnorm);
  m.impl("gemv_batched", &gemv_batched);
  m.impl("gemm_tc", &gemm_tc);
  m.impl("down_tc", &down_tc);
  m.impl("down_tc_f32", &down_tc_f32);
  m.impl("select_count", &select_count);
  m.impl("shard_select", &shard_select);
  m.impl("gather_up_h_count", &gather_up_h_count);
  m.impl("gather_down_partial", &gather_down_partial);
}
TORCH_LIBRARY_IMPL(dip_b200, CompositeExplicitAutograd, m) {
  m.impl("set_pdl", &op_set_pdl);
  m.impl("mlp_workspace_bytes", &op_mlp_workspace_bytes);
  m.impl("mlp_fused_workspace_bytes", &op_mlp_fused_workspace_bytes);
  m.impl("mlp_fused_tp_workspace_bytes", &op_mlp_fused_tp_workspace_bytes);
  m.impl("set_spin_limit", &op_set_spin_limit);
  m.impl("gemm_tc_auto_split", &op_gemm_tc_auto_split);
  m.impl("set_gemv_variant", &op_set_gemv_variant);
  m.impl("take_device_error", &op_take_device_error);
}
