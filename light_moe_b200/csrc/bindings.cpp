// bindings.cpp -- the `_C` operator module: light-moe's operator surface
// (csrc/bindings.cpp:28-49 of the reference: grouped_gemm, fused_gate_topk,
// fused_gate_topk_permute, same argument names and return types) plus the new W4A16 and
// MoE-layer ops, all implemented by calling the C ABI in include/lmoe_b200.h.
//
// Host-side duties only: argument checks (TORCH_CHECK -> RuntimeError, like the
// reference's fused_moe_ops.cu:150-151 / grouped_gemm.cu:17-18), output allocation through
// the PyTorch caching allocator, the device guard, and launching on the *current* CUDA
// stream (the reference launches its kernel on the legacy default stream).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <optional>
#include <tuple>

#include "lmoe_b200.h"

namespace {

void check_status(int st, const char* what) {
  TORCH_CHECK(st == LMOE_OK, what, " failed: ", lmoe_status_string(st), " (status ", st, ")");
}

lmoe_stream_t cur_stream() { return reinterpret_cast<lmoe_stream_t>(at::cuda::getCurrentCUDAStream().stream()); }

torch::Tensor as_bf16_contig(const torch::Tensor& t) {
  return t.scalar_type() == torch::kBFloat16 ? t.contiguous() : t.to(torch::kBFloat16).contiguous();
}

// The operand as one of the library's element types: bf16, fp16 and fp32 pass unchanged;
// any other floating type becomes fp32, the type the reference converts every operand to
// (csrc/fused_moe_ops.cu:158-159).
torch::Tensor as_kernel_type(const torch::Tensor& t) {
  const auto st = t.scalar_type();
  if (st == torch::kBFloat16 || st == torch::kFloat16 || st == torch::kFloat32) return t.contiguous();
  return t.to(torch::kFloat32).contiguous();
}

int dtype_code(const torch::Tensor& t) {
  switch (t.scalar_type()) {
    case torch::kBFloat16: return LMOE_DTYPE_BF16;
    case torch::kFloat16: return LMOE_DTYPE_F16;
    case torch::kFloat32: return LMOE_DTYPE_F32;
    default: TORCH_CHECK(false, "unsupported dtype ", t.scalar_type());
  }
  return -1;
}

void check_cuda(const torch::Tensor& t, const char* name) { TORCH_CHECK(t.is_cuda(), name, " must be CUDA"); }

torch::Tensor workspace(int64_t bytes, const torch::Tensor& like) {
  return torch::empty({bytes > 0 ? bytes : 1}, like.options().dtype(torch::kUInt8));
}

struct Routed {
  torch::Tensor ids, weights, counts, offsets, sorted_idx, positions, logits, probs;
};

Routed route(const torch::Tensor& hidden_states, const torch::Tensor& gate_weight,
             const std::optional<torch::Tensor>& bias, int64_t top_k, bool perm, bool want_logits,
             bool want_probs = false) {
  check_cuda(hidden_states, "hidden_states");
  check_cuda(gate_weight, "gate_weight");
  TORCH_CHECK(hidden_states.dim() == 2 && gate_weight.dim() == 2, "hidden_states [T,d] and gate_weight [E,d]");
  TORCH_CHECK(hidden_states.size(1) == gate_weight.size(1), "hidden size mismatch");
  const c10::cuda::OptionalCUDAGuard guard(hidden_states.device());
  auto x = as_kernel_type(hidden_states);
  auto w = as_kernel_type(gate_weight);
  const int64_t T = x.size(0);
  const int64_t d = x.size(1);
  const int64_t E = w.size(0);
  torch::Tensor b;
  if (bias.has_value() && bias->defined()) {
    check_cuda(*bias, "bias");
    b = bias->to(torch::kFloat32).contiguous();
    TORCH_CHECK(b.numel() == E, "bias must have num_experts elements");
  }
  auto i32 = x.options().dtype(torch::kInt32);
  Routed r;
  r.ids = torch::empty({T, top_k}, i32);
  r.weights = torch::empty({T, top_k}, x.options().dtype(torch::kFloat32));
  if (perm) {
    r.counts = torch::empty({E}, i32);
    r.offsets = torch::empty({E + 1}, i32);
    r.sorted_idx = torch::empty({T * top_k}, i32);
    r.positions = torch::empty({T * top_k}, i32);
  }
  if (want_logits) r.logits = torch::empty({T, E}, x.options().dtype(torch::kFloat32));
  if (want_probs) r.probs = torch::empty({T, E}, x.options().dtype(torch::kFloat32));
  const int xdt = dtype_code(x), wdt = dtype_code(w);
  auto ws = workspace((int64_t)lmoe_router_workspace_bytes_typed(T, (int)E, xdt, wdt), x);
  int st = lmoe_fused_gate_topk_typed(x.data_ptr(), xdt, w.data_ptr(), wdt, b.defined() ? b.data_ptr<float>() : nullptr,
                                T, (int)d,
                                (int)E, (int)top_k, r.ids.data_ptr<int32_t>(), r.weights.data_ptr<float>(), nullptr,
                                perm ? r.counts.data_ptr<int32_t>() : nullptr,
                                perm ? r.offsets.data_ptr<int32_t>() : nullptr,
                                perm ? r.sorted_idx.data_ptr<int32_t>() : nullptr,
                                perm ? r.positions.data_ptr<int32_t>() : nullptr,
                                want_logits ? r.logits.data_ptr<float>() : nullptr,
                                want_probs ? r.probs.data_ptr<float>() : nullptr, ws.data_ptr(), ws.numel(),
                                cur_stream());
  check_status(st, "fused_gate_topk");
  return r;
}

// ---------------------------------------------------------------- reference surface

// light_moe._C.fused_gate_topk (csrc/bindings.cpp:38-42 of the reference)
std::tuple<torch::Tensor, torch::Tensor> fused_gate_topk(torch::Tensor hidden_states, torch::Tensor gate_weight,
                                                         int64_t top_k) {
  Routed r = route(hidden_states, gate_weight, std::nullopt, top_k, false, false);
  return {r.ids, r.weights.to(hidden_states.scalar_type())};
}

// light_moe._C.fused_gate_topk_permute (csrc/bindings.cpp:44-48 of the reference)
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor> fused_gate_topk_permute(
    torch::Tensor hidden_states, torch::Tensor gate_weight, int64_t top_k) {
  Routed r = route(hidden_states, gate_weight, std::nullopt, top_k, true, false);
  const c10::cuda::OptionalCUDAGuard guard(hidden_states.device());
  // the permuted rows are the caller's rows, copied unchanged in their own dtype
  auto x = hidden_states.contiguous();
  const int64_t T = x.size(0);
  const int64_t d = x.size(1);
  auto permuted = torch::empty({T * top_k, d}, x.options());
  const int esize = (int)x.element_size();
  int st = LMOE_OK;
  if ((esize == 2 || esize == 4) && (d * esize) % 16 == 0) {
    st = lmoe_permute_rows(x.data_ptr(), esize, r.sorted_idx.data_ptr<int32_t>(), T * top_k, (int)d, (int)top_k,
                           permuted.data_ptr(), cur_stream());
  } else {
    // other element sizes or row lengths: the same gather through ATen
    permuted = x.index_select(0, r.sorted_idx.to(torch::kInt64).floor_divide(top_k));
  }
  check_status(st, "fused_gate_topk_permute");
  return {permuted, r.ids, r.weights.to(hidden_states.scalar_type()),
          r.offsets.to(torch::kInt64), r.sorted_idx.to(torch::kInt64)};
}

// light_moe._C.grouped_gemm (csrc/bindings.cpp:32-36 of the reference)
torch::Tensor grouped_gemm(torch::Tensor input, torch::Tensor weights, torch::Tensor expert_offsets,
                           int64_t num_experts) {
  check_cuda(input, "input");
  check_cuda(weights, "weights");
  check_cuda(expert_offsets, "expert_offsets");
  TORCH_CHECK(input.dim() == 2 && weights.dim() == 3, "input [T,K], weights [E,N,K]");
  TORCH_CHECK(weights.size(0) >= num_experts && weights.size(2) == input.size(1), "shape mismatch");
  TORCH_CHECK(expert_offsets.numel() >= num_experts + 1, "expert_offsets must have num_experts + 1 entries");
  const c10::cuda::OptionalCUDAGuard guard(input.device());
  // computed in the input dtype (bf16 / fp16 on tensor cores, fp32 on CUDA cores), like the
  // reference's per-expert mm_out (csrc/grouped_gemm.cu:24-40); the weights follow the input
  auto x = as_kernel_type(input);
  auto w = weights.scalar_type() == x.scalar_type() ? weights.contiguous() : weights.to(x.scalar_type()).contiguous();
  auto off = expert_offsets.contiguous();
  TORCH_CHECK(off.scalar_type() == torch::kInt64 || off.scalar_type() == torch::kInt32, "offsets int64/int32");
  const int64_t T = x.size(0), K = x.size(1), N = w.size(1);
  auto out = torch::empty({T, N}, x.options());
  auto ws = workspace((int64_t)lmoe_gemm_workspace_bytes(), x);
  int st = lmoe_grouped_gemm(x.data_ptr(), dtype_code(x), T, (int)K, w.data_ptr(), (int)N, off.data_ptr(),
                             off.scalar_type() == torch::kInt64 ? 1 : 0, (int)num_experts, 1, out.data_ptr(),
                             ws.data_ptr(), ws.numel(), cur_stream());
  check_status(st, "grouped_gemm");
  return out.to(input.scalar_type());
}

// ---------------------------------------------------------------- new ops

std::vector<torch::Tensor> fused_gate_topk_ex(torch::Tensor hidden_states, torch::Tensor gate_weight, int64_t top_k,
                                              std::optional<torch::Tensor> bias, bool return_logits,
                                              bool return_probs) {
  Routed r = route(hidden_states, gate_weight, bias, top_k, true, return_logits, return_probs);
  std::vector<torch::Tensor> out = {r.ids, r.weights, r.counts, r.offsets, r.sorted_idx, r.positions};
  if (return_logits) out.push_back(r.logits);
  if (return_probs) out.push_back(r.probs);
  return out;
}

std::tuple<torch::Tensor, torch::Tensor> quantize_w4(torch::Tensor w, int64_t group_size) {
  check_cuda(w, "w");
  TORCH_CHECK(w.dim() >= 2, "w must be [..., N, K]");
  const c10::cuda::OptionalCUDAGuard guard(w.device());
  const bool f32 = w.scalar_type() == torch::kFloat32;
  auto wc = f32 ? w.contiguous() : as_bf16_contig(w);
  const int64_t K = wc.size(-1);
  TORCH_CHECK(K % group_size == 0 && group_size % 2 == 0, "K must be divisible by an even group_size");
  const int64_t rows = wc.numel() / K;
  auto qshape = wc.sizes().vec();
  qshape.back() = K / 2;
  auto sshape = wc.sizes().vec();
  sshape.back() = K / group_size;
  auto q = torch::empty(qshape, wc.options().dtype(torch::kUInt8));
  auto s = torch::empty(sshape, wc.options().dtype(torch::kFloat16));
  int st = lmoe_quantize_w4(wc.data_ptr(), f32 ? 1 : 0, rows, (int)K, (int)group_size, q.data_ptr<uint8_t>(),
                            reinterpret_cast<uint16_t*>(s.data_ptr()), cur_stream());
  check_status(st, "quantize_w4");
  return {q, s};
}

torch::Tensor dequantize_w4(torch::Tensor qweight, torch::Tensor scales, int64_t group_size) {
  check_cuda(qweight, "qweight");
  check_cuda(scales, "scales");
  TORCH_CHECK(qweight.scalar_type() == torch::kUInt8 && scales.scalar_type() == torch::kFloat16, "uint8 / fp16");
  const c10::cuda::OptionalCUDAGuard guard(qweight.device());
  auto q = qweight.contiguous();
  auto s = scales.contiguous();
  const int64_t K = q.size(-1) * 2;
  const int64_t rows = q.numel() / (K / 2);
  TORCH_CHECK(s.numel() == rows * (K / group_size), "scales shape mismatch");
  auto shape = q.sizes().vec();
  shape.back() = K;
  auto out = torch::empty(shape, q.options().dtype(torch::kBFloat16));
  int st = lmoe_dequantize_w4(q.data_ptr<uint8_t>(), reinterpret_cast<const uint16_t*>(s.data_ptr()), rows, (int)K,
                              (int)group_size, out.data_ptr(), cur_stream());
  check_status(st, "dequantize_w4");
  return out;
}

torch::Tensor prepack_w4(torch::Tensor qweight, torch::Tensor scales, int64_t group_size,
                         std::optional<torch::Tensor> qweight_up, std::optional<torch::Tensor> scales_up) {
  check_cuda(qweight, "qweight");
  TORCH_CHECK(qweight.dim() == 3, "qweight must be [E, N, K/2]");
  const c10::cuda::OptionalCUDAGuard guard(qweight.device());
  auto q = qweight.contiguous();
  auto s = scales.contiguous();
  const bool paired = qweight_up.has_value() && qweight_up->defined();
  torch::Tensor qb, sb;
  if (paired) {
    qb = qweight_up->contiguous();
    sb = scales_up.value().contiguous();
    TORCH_CHECK(qb.sizes() == q.sizes() && sb.sizes() == s.sizes(), "gate and up shapes differ");
  }
  const int64_t E = q.size(0), N = q.size(1), K = q.size(2) * 2;
  size_t pb = 0;
  check_status(lmoe_w4_prepacked_bytes((int)E, (int)N, (int)K, (int)group_size, paired ? 1 : 0, &pb), "prepack_w4");
  auto packed = torch::empty({(int64_t)pb}, q.options());
  int st = lmoe_prepack_w4(q.data_ptr<uint8_t>(), reinterpret_cast<const uint16_t*>(s.data_ptr()),
                           paired ? qb.data_ptr<uint8_t>() : nullptr,
                           paired ? reinterpret_cast<const uint16_t*>(sb.data_ptr()) : nullptr, (int)E, (int)N,
                           (int)K, (int)group_size, packed.data_ptr<uint8_t>(), cur_stream());
  check_status(st, "prepack_w4");
  return packed;
}

torch::Tensor w4a16_grouped_gemm(torch::Tensor input, torch::Tensor packed, torch::Tensor expert_offsets, int64_t num_experts, int64_t N, int64_t group_size,
                                 int64_t epilogue, std::optional<torch::Tensor> dest_rows,
                                 std::optional<torch::Tensor> row_scale, int64_t out_rows,
                                 int64_t max_rows_per_expert, std::optional<torch::Tensor> segment_expert) {
  check_cuda(input, "input");
  check_cuda(packed, "packed");
  const c10::cuda::OptionalCUDAGuard guard(input.device());
  auto x = as_bf16_contig(input);
  auto off = expert_offsets.contiguous();
  const int64_t T = x.size(0), K = x.size(1);
  const int64_t ncols = epilogue == 1 ? N / 2 : N;
  const int64_t rows_out = out_rows > 0 ? out_rows : T;
  auto out = epilogue == 2 ? torch::zeros({rows_out, ncols}, x.options()) : torch::empty({rows_out, ncols}, x.options());
  torch::Tensor dr, rs;
  if (dest_rows.has_value() && dest_rows->defined()) dr = dest_rows->to(torch::kInt32).contiguous();
  if (row_scale.has_value() && row_scale->defined()) rs = row_scale->to(torch::kFloat32).contiguous();
  torch::Tensor se;
  if (segment_expert.has_value() && segment_expert->defined()) se = segment_expert->to(torch::kInt32).contiguous();
  // weight matrices held by `packed` (each N x K in the prepacked layout)
  size_t per = 0;
  check_status(lmoe_w4_prepacked_bytes(1, (int)N, (int)K, (int)group_size, 0, &per), "w4a16_grouped_gemm");
  TORCH_CHECK(per > 0 && packed.numel() % (int64_t)per == 0, "packed size is not a whole number of matrices");
  const int num_w = (int)(packed.numel() / (int64_t)per);
  auto ws = workspace((int64_t)lmoe_gemm_workspace_bytes(), x);
  int st = lmoe_w4a16_grouped_gemm(
      x.data_ptr(), T, (int)K, packed.data_ptr<uint8_t>(), (int)N, (int)group_size, off.data_ptr(), off.scalar_type() == torch::kInt64 ? 1 : 0, (int)num_experts,
      se.defined() ? se.data_ptr<int32_t>() : nullptr, num_w, (int)epilogue, dr.defined() ? dr.data_ptr<int32_t>() : nullptr, rs.defined() ? rs.data_ptr<float>() : nullptr,
      max_rows_per_expert, out.data_ptr(), ncols, ws.data_ptr(), ws.numel(), cur_stream());
  check_status(st, "w4a16_grouped_gemm");
  return out;
}

torch::Tensor combine_rows(torch::Tensor rows, torch::Tensor positions, torch::Tensor weights, int64_t num_tokens,
                           int64_t top_k, std::optional<torch::Tensor> extra_rows, int64_t num_extra) {
  check_cuda(rows, "rows");
  const c10::cuda::OptionalCUDAGuard guard(rows.device());
  auto r = as_bf16_contig(rows);
  auto p = positions.to(torch::kInt32).contiguous();
  auto w = weights.to(torch::kFloat32).contiguous();
  const int64_t d = r.size(1);
  torch::Tensor ex;
  if (extra_rows.has_value() && extra_rows->defined()) ex = as_bf16_contig(*extra_rows);
  auto y = torch::empty({num_tokens, d}, r.options());
  int st = lmoe_combine_rows(r.data_ptr(), p.data_ptr<int32_t>(), w.data_ptr<float>(), num_tokens, (int)top_k, (int)d,
                             ex.defined() ? ex.data_ptr() : nullptr, ex.defined() ? (int)num_extra : 0, y.data_ptr(),
                             cur_stream());
  check_status(st, "combine_rows");
  return y;
}

std::vector<torch::Tensor> moe_layer_w4a16(torch::Tensor x, torch::Tensor gate_weight, torch::Tensor w13_packed,
                                           torch::Tensor w2_packed, int64_t top_k, int64_t ffn_size,
                                           int64_t group_size, int64_t num_shared,
                                           std::optional<torch::Tensor> gate_bias) {
  check_cuda(x, "x");
  const c10::cuda::OptionalCUDAGuard guard(x.device());
  auto xb = as_bf16_contig(x);
  auto gw = as_bf16_contig(gate_weight);
  const int64_t T = xb.size(0), d = xb.size(1), E = gw.size(0);
  torch::Tensor b;
  if (gate_bias.has_value() && gate_bias->defined()) b = gate_bias->to(torch::kFloat32).contiguous();
  auto y = torch::empty({T, d}, xb.options());
  auto ids = torch::empty({T, top_k}, xb.options().dtype(torch::kInt32));
  auto wts = torch::empty({T, top_k}, xb.options().dtype(torch::kFloat32));
  auto ws = workspace((int64_t)lmoe_moe_layer_workspace_bytes(T, (int)d, (int)ffn_size, (int)E, (int)top_k,
                                                               (int)num_shared),
                      xb);
  int st = lmoe_moe_layer_w4a16(xb.data_ptr(), T, (int)d, gw.data_ptr(), b.defined() ? b.data_ptr<float>() : nullptr,
                                (int)E, (int)top_k, (int)num_shared, w13_packed.data_ptr<uint8_t>(),
                                w2_packed.data_ptr<uint8_t>(), (int)ffn_size, (int)group_size, y.data_ptr(), ids.data_ptr<int32_t>(),
                                wts.data_ptr<float>(), ws.data_ptr(), ws.numel(), cur_stream());
  check_status(st, "moe_layer_w4a16");
  return {y, ids, wts};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "light-moe operator surface on B200 (sm_100a): router, grouped GEMMs, W4A16 MoE layer";
  m.def("grouped_gemm", &grouped_gemm, "Grouped GEMM for MoE experts (bf16, offsets read on the device)",
        py::arg("input"), py::arg("weights"), py::arg("expert_offsets"), py::arg("num_experts"));
  m.def("fused_gate_topk", &fused_gate_topk, "Gate projection + softmax + top-k in one kernel",
        py::arg("hidden_states"), py::arg("gate_weight"), py::arg("top_k"));
  m.def("fused_gate_topk_permute", &fused_gate_topk_permute,
        "Gate + top-k + counts/offsets/stable permutation + row gather", py::arg("hidden_states"),
        py::arg("gate_weight"), py::arg("top_k"));
  m.def("fused_gate_topk_ex", &fused_gate_topk_ex,
        "Router with fp32 weights, int32 counts/offsets/sorted_idx and optional logits / probabilities",
        py::arg("hidden_states"), py::arg("gate_weight"), py::arg("top_k"), py::arg("bias") = py::none(),
        py::arg("return_logits") = false, py::arg("return_probs") = false);
  m.def("quantize_w4", &quantize_w4, "Symmetric per-group int4 quantisation", py::arg("w"), py::arg("group_size"));
  m.def("dequantize_w4", &dequantize_w4, "int4 -> bf16", py::arg("qweight"), py::arg("scales"),
        py::arg("group_size"));
  m.def("prepack_w4", &prepack_w4, "Canonical int4 -> GEMM device layout", py::arg("qweight"), py::arg("scales"),
        py::arg("group_size"), py::arg("qweight_up") = py::none(), py::arg("scales_up") = py::none());
  m.def("w4a16_grouped_gemm", &w4a16_grouped_gemm, "W4A16 grouped GEMM", py::arg("input"), py::arg("packed"),
        py::arg("expert_offsets"), py::arg("num_experts"), py::arg("N"),
        py::arg("group_size"), py::arg("epilogue") = 0, py::arg("dest_rows") = py::none(),
        py::arg("row_scale") = py::none(), py::arg("out_rows") = 0, py::arg("max_rows_per_expert") = 0,
        py::arg("segment_expert") = py::none());
  m.def("combine_rows", &combine_rows, "Weighted combine of slot rows back to tokens", py::arg("rows"),
        py::arg("positions"), py::arg("weights"), py::arg("num_tokens"), py::arg("top_k"),
        py::arg("extra_rows") = py::none(), py::arg("num_extra") = 0);
  m.def("moe_layer_w4a16", &moe_layer_w4a16, "W4A16 MoE layer", py::arg("x"), py::arg("gate_weight"),
        py::arg("w13_packed"), py::arg("w2_packed"), py::arg("top_k"),
        py::arg("ffn_size"), py::arg("group_size"), py::arg("num_shared") = 0, py::arg("gate_bias") = py::none());
}
