// fa8_torch.cpp — PyTorch-facing host layer above the C ABI (include/fa8.h).
//
// Mirrors the reference's extension module (csrc/attention_api.cpp:6-9,
// include/attention_api.h:9-10): the function `flash_attn_fp8_forward(q, k,
// v)` with e4m3 Q/K (B, H, S, D) and V pre-transposed to (B, H, D, S)
// (test.py:51-52). Like the reference it is causal with scale 1/sqrt(D)
// (csrc/flash_attention.cu:524, :292-304); unlike it, it returns fp16 O
// (the reference returns e4m3, :526), never blocks on the device (:539) and
// never exits the process. Input errors raise RuntimeError through
// TORCH_CHECK as in include/attention_api.cuh:20-26, with dtype / shape
// checks the reference lacks.
//
// flash_attn_fp8_forward_ex adds: non-causal mode, an explicit scale,
// V in BHSD layout, LSE output, e4m3 output, context-parallel offsets, the
// P-split threshold and caller-provided output buffers.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cmath>
#include <string>
#include <vector>

#include "fa8.h"

namespace {

void check_status(int st, const char* what) {
  TORCH_CHECK(st == FA8_OK, what, " failed: ", fa8_status_string(st), " (",
              fa8_last_error_message(), ")");
}

void check_fp8_input(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.device().is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == at::ScalarType::Float8_e4m3fn, name,
              " must be torch.float8_e4m3fn, got ", t.scalar_type());
  TORCH_CHECK(t.dim() == 4, name, " must be 4-D, got ", t.dim(), " dims");
  TORCH_CHECK(t.stride(3) == 1 || t.size(3) == 1, name, " must have a unit-stride last dim");
}

bool tma_ok(const torch::Tensor& t) {
  if (reinterpret_cast<uintptr_t>(t.data_ptr()) % 16) return false;
  for (int d = 0; d < 3; ++d)
    if (t.size(d) > 1 && (t.stride(d) % 16 != 0)) return false;
  return true;
}

std::vector<torch::Tensor> forward_impl(torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                        bool causal, double softmax_scale,
                                        const std::string& v_layout, bool return_lse,
                                        const std::string& out_dtype, int64_t q_offset,
                                        int64_t kv_offset, int64_t split_keys,
                                        c10::optional<torch::Tensor> out_opt,
                                        c10::optional<torch::Tensor> lse_opt,
                                        double descale_q = 1.0, double descale_k = 1.0,
                                        double descale_v = 1.0,
                                        c10::optional<torch::Tensor> descale_q_bh = c10::nullopt,
                                        c10::optional<torch::Tensor> descale_k_bh = c10::nullopt,
                                        c10::optional<torch::Tensor> descale_v_bh = c10::nullopt,
                                        int64_t sm_budget = 0) {
  check_fp8_input(q, "q");
  check_fp8_input(k, "k");
  check_fp8_input(v, "v");
  TORCH_CHECK(k.device() == q.device() && v.device() == q.device(),
              "q, k, v must be on the same device");
  TORCH_CHECK(v_layout == "bhds" || v_layout == "bhsd", "v_layout must be 'bhds' or 'bhsd'");
  TORCH_CHECK(out_dtype == "fp16" || out_dtype == "e4m3" || out_dtype == "fp32",
              "out_dtype must be 'fp16', 'e4m3' or 'fp32'");
  const int64_t B = q.size(0), H = q.size(1), Sq = q.size(2), D = q.size(3);
  const int64_t Hkv = k.size(1), Skv = k.size(2);
  TORCH_CHECK(D == 64 || D == 128, "head_dim must be 64 or 128, got ", D);
  TORCH_CHECK(k.size(0) == B && k.size(3) == D, "k must be (B, H_kv, S_kv, D)");
  TORCH_CHECK(Hkv > 0 && H % Hkv == 0, "H must be a multiple of H_kv");
  c10::cuda::CUDAGuard guard(q.device());
  auto stream = at::cuda::getCurrentCUDAStream(q.get_device());

  // V goes to the kernel as given: (B, H_kv, D, S) ("bhds", the reference's
  // pre-transposed layout) or (B, H_kv, S, D) ("bhsd", read by the PV product
  // as an MN-major operand). Only layouts the TMA cannot describe (a BHDS row
  // of S_kv % 16 != 0 keys, unaligned strides) are copied first.
  torch::Tensor vt;
  int v_code = FA8_V_BHDS;
  if (v_layout == "bhds") {
    TORCH_CHECK(v.size(0) == B && v.size(1) == Hkv && v.size(2) == D && v.size(3) == Skv,
                "v (bhds) must be (B, H_kv, D, S_kv)");
    vt = v;
    if (Skv % 16 != 0 || !tma_ok(vt) || vt.stride(3) != 1) {
      const int64_t Sp = (Skv + 15) / 16 * 16;
      auto vp = torch::empty({B, Hkv, D, Sp}, vt.options());
      vp.narrow(3, Skv, Sp - Skv).zero_();
      vp.narrow(3, 0, Skv).copy_(vt);
      vt = vp;
    }
  } else {
    TORCH_CHECK(v.size(0) == B && v.size(1) == Hkv && v.size(2) == Skv && v.size(3) == D,
                "v (bhsd) must be (B, H_kv, S_kv, D)");
    vt = tma_ok(v) && v.stride(3) == 1 ? v : v.contiguous();
    v_code = FA8_V_BHSD;
  }
  if (!tma_ok(q)) q = q.contiguous();
  if (!tma_ok(k)) k = k.contiguous();

  const at::ScalarType out_st = out_dtype == "e4m3"   ? at::ScalarType::Float8_e4m3fn
                                : out_dtype == "fp32" ? at::ScalarType::Float
                                                      : at::ScalarType::Half;
  torch::Tensor out;
  if (out_opt.has_value()) {
    out = *out_opt;
    TORCH_CHECK(out.device() == q.device(), "out must be on q's device");
    TORCH_CHECK(out.scalar_type() == out_st, "out has the wrong dtype");
    TORCH_CHECK(out.dim() == 4 && out.size(0) == B && out.size(1) == H && out.size(2) == Sq &&
                    out.size(3) == D && out.stride(3) == 1,
                "out must be (B, H, S_q, D) with unit last stride");
  } else {
    out = torch::empty({B, H, Sq, D}, q.options().dtype(out_st));
  }
  torch::Tensor lse;
  if (return_lse || lse_opt.has_value()) {
    if (lse_opt.has_value()) {
      lse = *lse_opt;
      TORCH_CHECK(lse.device() == q.device(), "lse must be on q's device");
      TORCH_CHECK(lse.scalar_type() == at::ScalarType::Float && lse.dim() == 3 &&
                      lse.size(0) == B && lse.size(1) == H && lse.size(2) == Sq &&
                      lse.stride(2) == 1,
                  "lse must be float32 (B, H, S_q) with unit last stride");
    } else {
      lse = torch::empty({B, H, Sq}, q.options().dtype(at::ScalarType::Float));
    }
  }

  fa8_fwd_params p;
  fa8_fwd_params_init(&p, B, H, Hkv, Sq, Skv, D);
  p.q = q.data_ptr();
  p.k = k.data_ptr();
  p.v = vt.data_ptr();
  p.o = out.data_ptr();
  p.lse = lse.defined() ? lse.data_ptr<float>() : nullptr;
  p.q_stride_b = q.stride(0);
  p.q_stride_h = q.stride(1);
  p.q_stride_s = q.stride(2);
  p.k_stride_b = k.stride(0);
  p.k_stride_h = k.stride(1);
  p.k_stride_s = k.stride(2);
  p.v_stride_b = vt.stride(0);
  p.v_stride_h = vt.stride(1);
  p.v_stride_r = vt.stride(2);
  p.v_layout = v_code;
  p.o_stride_b = out.stride(0);
  p.o_stride_h = out.stride(1);
  p.o_stride_s = out.stride(2);
  if (lse.defined()) {
    p.lse_stride_b = lse.stride(0);
    p.lse_stride_h = lse.stride(1);
  }
  p.softmax_scale = static_cast<float>(softmax_scale);
  p.causal = causal ? 1 : 0;
  p.out_dtype = out_dtype == "e4m3" ? FA8_OUT_E4M3 : (out_dtype == "fp32" ? FA8_OUT_F32 : FA8_OUT_F16);
  p.q_offset = q_offset;
  p.kv_offset = kv_offset;
  p.split_keys = static_cast<int32_t>(split_keys);
  p.descale_q = static_cast<float>(descale_q);
  p.descale_k = static_cast<float>(descale_k);
  p.descale_v = static_cast<float>(descale_v);
  // Per-(batch, head) factors: anything that broadcasts to (B, H) for Q and
  // (B, H_kv) for K/V, materialised as contiguous fp32 on the device.
  auto bh = [&](const c10::optional<torch::Tensor>& t, int64_t heads,
                const char* name) -> torch::Tensor {
    if (!t.has_value()) return torch::Tensor();
    TORCH_CHECK(t->device() == q.device(), name, " must be on q's device");
    return t->to(torch::kFloat32).expand({B, heads}).contiguous();
  };
  torch::Tensor dq = bh(descale_q_bh, H, "descale_q"), dk = bh(descale_k_bh, Hkv, "descale_k"),
                dv = bh(descale_v_bh, Hkv, "descale_v");
  if (dq.defined()) p.descale_q_bh = dq.data_ptr<float>();
  if (dk.defined()) p.descale_k_bh = dk.data_ptr<float>();
  if (dv.defined()) p.descale_v_bh = dv.data_ptr<float>();
  p.descale_q_stride_b = H;
  p.descale_q_stride_h = 1;
  p.descale_kv_stride_b = Hkv;
  p.descale_kv_stride_h = 1;
  TORCH_CHECK(sm_budget >= 0, "sm_budget must be >= 0");
  p.sm_budget = (int32_t)sm_budget;
  // Split-KV for calls too small to fill the GPU: a workspace from the caching
  // allocator whose leading counters start at zero.
  torch::Tensor ws;
  p.kv_splits = 0;
  const int64_t ws_bytes = fa8_fwd_workspace_size(&p);
  if (ws_bytes > 0) {
    ws = torch::empty({ws_bytes}, q.options().dtype(at::kByte));
    const int64_t qtiles = B * H * ((Sq + 127) / 128);
    ws.narrow(0, 0, (qtiles * 4 + 255) / 256 * 256).zero_();
    p.workspace = ws.data_ptr();
    p.workspace_bytes = ws_bytes;
  }
  check_status(fa8_fwd(&p, stream.stream()), "fa8_fwd");
  if (lse.defined()) return {out, lse};
  return {out};
}

}  // namespace

torch::Tensor flash_attn_fp8_forward(torch::Tensor q, torch::Tensor k, torch::Tensor v) {
  TORCH_CHECK(q.dim() == 4, "q must be (B, H, S, D)");
  const double scale = 1.0 / std::sqrt(static_cast<double>(q.size(3)));
  return forward_impl(q, k, v, /*causal=*/true, scale, "bhds", false, "fp16", 0, 0, -1,
                      c10::nullopt, c10::nullopt)[0];
}

std::vector<torch::Tensor> flash_attn_fp8_forward_ex(
    torch::Tensor q, torch::Tensor k, torch::Tensor v, bool causal,
    c10::optional<double> softmax_scale, std::string v_layout, bool return_lse,
    std::string out_dtype, int64_t q_offset, int64_t kv_offset, int64_t split_keys,
    c10::optional<torch::Tensor> out, c10::optional<torch::Tensor> lse, double descale_q,
    double descale_k, double descale_v, c10::optional<torch::Tensor> descale_q_bh,
    c10::optional<torch::Tensor> descale_k_bh, c10::optional<torch::Tensor> descale_v_bh,
    int64_t sm_budget) {
  TORCH_CHECK(q.dim() == 4, "q must be (B, H, S, D)");
  const double scale = softmax_scale.has_value()
                           ? *softmax_scale
                           : 1.0 / std::sqrt(static_cast<double>(q.size(3)));
  return forward_impl(q, k, v, causal, scale, v_layout, return_lse, out_dtype, q_offset,
                      kv_offset, split_keys, out, lse, descale_q, descale_k, descale_v,
                      descale_q_bh, descale_k_bh, descale_v_bh, sm_budget);
}

// Variable-length (packed) batches: q (total_q, H, D), k (total_kv, H_kv, D),
// v (total_kv, H_kv, D) ("thd", read in place as BHSD rows) or pre-transposed
// (H_kv, D, total_kv) ("hdt"); cu_seqlens_* int32 (batch + 1) on q's device.
// The offsets are never copied to the host: the kernel validates each
// sequence and reports refusals in the optional int32 `status` word.
// Returns [out (total_q, H, D)] (+ lse (H, total_q)).
std::vector<torch::Tensor> flash_attn_fp8_varlen_forward(
    torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor cu_seqlens_q,
    torch::Tensor cu_seqlens_kv, int64_t max_seqlen_q, bool causal,
    c10::optional<double> softmax_scale, std::string v_layout, bool return_lse,
    std::string out_dtype, c10::optional<torch::Tensor> status) {
  for (auto* t : {&q, &k, &v}) {
    TORCH_CHECK(t->device().is_cuda() && t->scalar_type() == at::ScalarType::Float8_e4m3fn,
                "q, k, v must be CUDA float8_e4m3fn tensors");
    TORCH_CHECK(t->dim() == 3, "q, k, v must be 3-D (packed)");
  }
  TORCH_CHECK(k.device() == q.device() && v.device() == q.device(),
              "q, k, v must be on the same device");
  TORCH_CHECK(v_layout == "thd" || v_layout == "hdt", "v_layout must be 'thd' or 'hdt'");
  TORCH_CHECK(out_dtype == "fp16" || out_dtype == "e4m3", "out_dtype must be 'fp16' or 'e4m3'");
  const int64_t Tq = q.size(0), H = q.size(1), D = q.size(2);
  const int64_t Tk = k.size(0), Hkv = k.size(1);
  TORCH_CHECK(D == 64 || D == 128, "head_dim must be 64 or 128");
  TORCH_CHECK(k.size(2) == D && Hkv > 0 && H % Hkv == 0, "k must be (total_kv, H_kv, D)");
  TORCH_CHECK(cu_seqlens_q.dim() == 1 && cu_seqlens_q.numel() >= 2 &&
                  cu_seqlens_kv.dim() == 1 && cu_seqlens_kv.numel() == cu_seqlens_q.numel(),
              "cu_seqlens_q / cu_seqlens_kv must be 1-D with batch + 1 entries");
  TORCH_CHECK(max_seqlen_q > 0 && max_seqlen_q <= Tq, "need 0 < max_seqlen_q <= total_q");
  const int64_t B = cu_seqlens_q.numel() - 1;
  c10::cuda::CUDAGuard guard(q.device());
  auto stream = at::cuda::getCurrentCUDAStream(q.get_device());
  // Offsets live on the device as int32; other dtypes / devices are converted
  // with device-side (or host-to-device) copies, never device-to-host.
  auto dev_i32 = [&](const torch::Tensor& t) {
    TORCH_CHECK(t.device().is_cpu() || t.device() == q.device(),
                "cu_seqlens must be on q's device (or on the host)");
    return t.to(q.device(), at::kInt).contiguous();
  };
  auto cuq_d = dev_i32(cu_seqlens_q);
  auto cuk_d = dev_i32(cu_seqlens_kv);
  if (!tma_ok(q) || q.stride(2) != 1) q = q.contiguous();
  if (!tma_ok(k) || k.stride(2) != 1) k = k.contiguous();
  torch::Tensor vt;
  int v_code;
  if (v_layout == "thd") {
    TORCH_CHECK(v.size(0) == Tk && v.size(1) == Hkv && v.size(2) == D, "v must be (total_kv, H_kv, D)");
    vt = tma_ok(v) && v.stride(2) == 1 ? v : v.contiguous();
    v_code = FA8_V_BHSD;
  } else {
    TORCH_CHECK(v.size(0) == Hkv && v.size(1) == D && v.size(2) == Tk, "v must be (H_kv, D, total_kv)");
    vt = v;
    if (Tk % 16 != 0 || !tma_ok(vt) || vt.stride(2) != 1) {
      const int64_t Tk_pad = (Tk + 15) / 16 * 16;
      auto vp = torch::empty({Hkv, D, Tk_pad}, v.options());
      vp.narrow(2, Tk, Tk_pad - Tk).zero_();
      vp.narrow(2, 0, Tk).copy_(v);
      vt = vp;
    }
    v_code = FA8_V_BHDS;
  }
  const bool e4m3_out = out_dtype == "e4m3";
  auto out = torch::empty({Tq, H, D}, q.options().dtype(e4m3_out ? at::ScalarType::Float8_e4m3fn
                                                                    : at::ScalarType::Half));
  torch::Tensor lse;
  if (return_lse) lse = torch::empty({H, Tq}, q.options().dtype(at::ScalarType::Float));
  int32_t* status_ptr = nullptr;
  if (status.has_value()) {
    TORCH_CHECK(status->device() == q.device() && status->scalar_type() == at::kInt &&
                    status->numel() >= 1 && status->is_contiguous(),
                "status must be a contiguous int32 CUDA tensor on q's device");
    status_ptr = status->data_ptr<int32_t>();
  }
  fa8_fwd_params p;
  fa8_fwd_params_init(&p, B, H, Hkv, Tq, Tk, D);
  p.q = q.data_ptr();
  p.k = k.data_ptr();
  p.v = vt.data_ptr();
  p.o = out.data_ptr();
  p.lse = return_lse ? lse.data_ptr<float>() : nullptr;
  p.status = status_ptr;
  p.q_stride_s = q.stride(0);  p.q_stride_h = q.stride(1);  p.q_stride_b = Tq * q.stride(0);
  p.k_stride_s = k.stride(0);  p.k_stride_h = k.stride(1);  p.k_stride_b = Tk * k.stride(0);
  if (v_code == FA8_V_BHSD) {
    p.v_stride_r = vt.stride(0); p.v_stride_h = vt.stride(1); p.v_stride_b = Tk * vt.stride(0);
  } else {
    p.v_stride_r = vt.stride(1); p.v_stride_h = vt.stride(0); p.v_stride_b = Hkv * vt.stride(0);
  }
  p.v_layout = v_code;
  p.o_stride_s = H * D;  p.o_stride_h = D;  p.o_stride_b = 0;
  p.lse_stride_h = Tq;   p.lse_stride_b = 0;
  p.softmax_scale = static_cast<float>(softmax_scale.has_value() ? *softmax_scale
                                                                 : 1.0 / std::sqrt((double)D));
  p.causal = causal ? 1 : 0;
  p.out_dtype = e4m3_out ? FA8_OUT_E4M3 : FA8_OUT_F16;
  p.cu_seqlens_q = cuq_d.data_ptr<int>();
  p.cu_seqlens_kv = cuk_d.data_ptr<int>();
  p.max_seqlen_q = max_seqlen_q;
  check_status(fa8_fwd(&p, stream.stream()), "fa8_fwd (varlen)");
  if (return_lse) return {out, lse};
  return {out};
}

std::vector<torch::Tensor> lse_merge(std::vector<torch::Tensor> outs,
                                     std::vector<torch::Tensor> lses) {
  TORCH_CHECK(!outs.empty() && outs.size() == lses.size() && outs.size() <= 16,
              "lse_merge takes 1..16 (out, lse) pairs");
  const auto& o0 = outs[0];
  TORCH_CHECK(o0.device().is_cuda(), "outs must be CUDA tensors");
  const bool f16 = o0.scalar_type() == at::ScalarType::Half;
  TORCH_CHECK(f16 || o0.scalar_type() == at::ScalarType::Float, "outs must be fp16 or fp32");
  const int64_t D = o0.size(-1);
  const int64_t rows = o0.numel() / D;
  std::vector<const void*> op;
  std::vector<const float*> lp;
  for (size_t i = 0; i < outs.size(); ++i) {
    TORCH_CHECK(outs[i].is_contiguous() && outs[i].sizes() == o0.sizes() &&
                    outs[i].scalar_type() == o0.scalar_type() && outs[i].device() == o0.device(),
                "all outs must be contiguous with one shape / dtype / device");
    TORCH_CHECK(lses[i].is_contiguous() && lses[i].scalar_type() == at::ScalarType::Float &&
                    lses[i].numel() == rows && lses[i].device() == o0.device(),
                "lse parts must be contiguous float32 on the outs' device, one entry per row");
    op.push_back(outs[i].data_ptr());
    lp.push_back(lses[i].data_ptr<float>());
  }
  c10::cuda::CUDAGuard guard(o0.device());
  auto out = torch::empty(o0.sizes(), o0.options().dtype(at::ScalarType::Half));
  auto lse = torch::empty(lses[0].sizes(), lses[0].options());
  check_status(fa8_lse_merge((int)outs.size(), op.data(), f16 ? 1 : 0, lp.data(), rows, D,
                             out.data_ptr(), D, lse.data_ptr<float>(),
                             at::cuda::getCurrentCUDAStream(o0.get_device()).stream()),
               "fa8_lse_merge");
  return {out, lse};
}

torch::Tensor quantize_e4m3(torch::Tensor x, double scale, bool transpose_last2) {
  TORCH_CHECK(x.device().is_cuda() && x.is_contiguous(), "x must be a contiguous CUDA tensor");
  TORCH_CHECK(x.scalar_type() == at::ScalarType::Half || x.scalar_type() == at::ScalarType::BFloat16,
              "x must be fp16 or bf16");
  TORCH_CHECK(x.dim() >= 2, "x must have at least 2 dims");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t rows = x.size(-2), cols = x.size(-1);
  const int64_t batch = rows * cols == 0 ? 0 : x.numel() / (rows * cols);
  auto sizes = x.sizes().vec();
  if (transpose_last2) std::swap(sizes[sizes.size() - 1], sizes[sizes.size() - 2]);
  auto y = torch::empty(sizes, x.options().dtype(at::ScalarType::Float8_e4m3fn));
  check_status(fa8_quantize_e4m3(x.data_ptr(), x.scalar_type() == at::ScalarType::Half ? 0 : 1,
                                 y.data_ptr(), batch, rows, cols, (float)scale,
                                 transpose_last2 ? 1 : 0,
                                 at::cuda::getCurrentCUDAStream(x.get_device()).stream()),
               "fa8_quantize_e4m3");
  return y;
}

// Backward: gradients for q, k, v (e4m3, contiguous after .contiguous()),
// given the forward's fp16 out and fp32 lse and the fp16 grad_out. Returns
// [dq, dk, dv] in fp32 (dk, dv with the K/V head count).
std::vector<torch::Tensor> flash_attn_fp8_backward(torch::Tensor q, torch::Tensor k,
                                                   torch::Tensor v, torch::Tensor out,
                                                   torch::Tensor grad_out, torch::Tensor lse,
                                                   bool causal, c10::optional<double> softmax_scale,
                                                   std::string v_layout) {
  for (auto* t : {&q, &k, &v})
    TORCH_CHECK(t->device().is_cuda() && t->scalar_type() == at::ScalarType::Float8_e4m3fn &&
                    t->dim() == 4,
                "q, k, v must be 4-D CUDA float8_e4m3fn tensors");
  TORCH_CHECK(v_layout == "bhds" || v_layout == "bhsd", "v_layout must be 'bhds' or 'bhsd'");
  const int64_t B = q.size(0), H = q.size(1), Sq = q.size(2), D = q.size(3);
  const int64_t Hkv = k.size(1), Skv = k.size(2);
  TORCH_CHECK(D == 64 || D == 128, "head_dim must be 64 or 128");
  TORCH_CHECK(k.size(0) == B && k.size(3) == D && Hkv > 0 && H % Hkv == 0,
              "k must be (B, H_kv, S_kv, D) with H % H_kv == 0");
  if (v_layout == "bhds") {
    TORCH_CHECK(v.sizes() == torch::IntArrayRef({B, Hkv, D, Skv}), "v must be (B, H_kv, D, S_kv)");
  } else {
    TORCH_CHECK(v.sizes() == k.sizes(), "v must be (B, H_kv, S_kv, D)");
  }
  for (auto* t : {&out, &grad_out}) {
    TORCH_CHECK(t->device() == q.device() && t->scalar_type() == at::ScalarType::Half &&
                    t->sizes() == q.sizes(),
                "out and grad_out must be fp16 (B, H, S_q, D) on q's device");
  }
  TORCH_CHECK(lse.device() == q.device() && lse.scalar_type() == at::ScalarType::Float &&
                  lse.sizes() == torch::IntArrayRef({B, H, Sq}),
              "lse must be float32 (B, H, S_q) on q's device");
  TORCH_CHECK(k.device() == q.device() && v.device() == q.device(), "q, k, v on one device");
  c10::cuda::CUDAGuard guard(q.device());
  auto stream = at::cuda::getCurrentCUDAStream(q.get_device());
  q = q.contiguous(); k = k.contiguous(); v = v.contiguous();
  out = out.contiguous(); grad_out = grad_out.contiguous(); lse = lse.contiguous();
  auto f32 = q.options().dtype(at::ScalarType::Float);
  auto dq = torch::empty({B, H, Sq, D}, f32);
  auto dk = torch::empty({B, Hkv, Skv, D}, f32);
  auto dv = torch::empty({B, Hkv, Skv, D}, f32);
  fa8_bwd_params p;
  fa8_bwd_params_init(&p, B, H, Hkv, Sq, Skv, D);
  p.q = q.data_ptr(); p.k = k.data_ptr(); p.v = v.data_ptr();
  p.o = out.data_ptr(); p.d_o = grad_out.data_ptr(); p.lse = lse.data_ptr<float>();
  p.dq = dq.data_ptr<float>(); p.dk = dk.data_ptr<float>(); p.dv = dv.data_ptr<float>();
  p.causal = causal ? 1 : 0;
  p.softmax_scale = static_cast<float>(softmax_scale.has_value() ? *softmax_scale
                                                                 : 1.0 / std::sqrt((double)D));
  p.v_layout = v_layout == "bhsd" ? FA8_V_BHSD : FA8_V_BHDS;
  const int64_t ws_bytes = fa8_bwd_workspace_size(&p);
  TORCH_CHECK(ws_bytes >= 0, "fa8_bwd_workspace_size: ", fa8_last_error_message());
  auto ws = torch::empty({std::max<int64_t>(ws_bytes, 1)}, q.options().dtype(at::kByte));
  check_status(fa8_bwd(&p, ws.data_ptr(), ws_bytes, stream.stream()), "fa8_bwd");
  return {dq, dk, dv};
}

int64_t launch_count() { return (int64_t)fa8_launch_count(); }

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("flash_attn_fp8_forward", &flash_attn_fp8_forward,
        "FP8 (e4m3) causal flash-attention forward on sm_100a; V in (B,H,D,S); returns fp16 O");
  m.def("flash_attn_fp8_forward_ex", &flash_attn_fp8_forward_ex, py::arg("q"), py::arg("k"),
        py::arg("v"), py::arg("causal") = true, py::arg("softmax_scale") = py::none(),
        py::arg("v_layout") = "bhds", py::arg("return_lse") = false,
        py::arg("out_dtype") = "fp16", py::arg("q_offset") = 0, py::arg("kv_offset") = 0,
        py::arg("split_keys") = -1, py::arg("out") = py::none(), py::arg("lse") = py::none(),
        py::arg("descale_q") = 1.0, py::arg("descale_k") = 1.0, py::arg("descale_v") = 1.0,
        py::arg("descale_q_bh") = py::none(), py::arg("descale_k_bh") = py::none(),
        py::arg("descale_v_bh") = py::none(), py::arg("sm_budget") = 0,
        "FP8 attention forward with options; returns [out] or [out, lse]");
  m.def("flash_attn_fp8_varlen_forward", &flash_attn_fp8_varlen_forward, py::arg("q"),
        py::arg("k"), py::arg("v"), py::arg("cu_seqlens_q"), py::arg("cu_seqlens_kv"),
        py::arg("max_seqlen_q"), py::arg("causal") = true, py::arg("softmax_scale") = py::none(),
        py::arg("v_layout") = "thd", py::arg("return_lse") = false,
        py::arg("out_dtype") = "fp16", py::arg("status") = py::none(),
        "FP8 attention over packed variable-length sequences; returns [out] or [out, lse]");
  m.def("lse_merge", &lse_merge, "log-sum-exp merge of partial attention outputs");
  m.def("quantize_e4m3", &quantize_e4m3, py::arg("x"), py::arg("scale") = 1.0,
        py::arg("transpose_last2") = false, "fp16/bf16 -> e4m3 (optionally transposed)");
  m.def("flash_attn_fp8_backward", &flash_attn_fp8_backward, py::arg("q"), py::arg("k"),
        py::arg("v"), py::arg("out"), py::arg("grad_out"), py::arg("lse"),
        py::arg("causal") = true, py::arg("softmax_scale") = py::none(),
        py::arg("v_layout") = "bhds", "gradients [dq, dk, dv] (fp32) of the FP8 attention");
  m.def("launch_count", &launch_count, "kernel launches issued by the C ABI so far");
}
