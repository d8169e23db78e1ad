// PyTorch dispatcher ops over the C ABI of libduplex_b200.so (include/duplex_b200.h):
// TORCH_LIBRARY(duplex_b200, ...) with CUDA implementations that pass data pointers,
// sizes and the current CUDA stream to the extern "C" entry points and raise on a
// non-zero status.  The ops are visible to the dispatcher, the profiler (by name) and
// torch.compile (as opaque custom ops); the reference-named Python modules call the
// same entry points through ctypes.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include "duplex_b200.h"

namespace {

void check(int rc, const char* what) {
  TORCH_CHECK(rc == DUPLEX_OK, "duplex_b200::", what, " failed: status ", rc, ": ",
              duplex_error_string(rc));
}

void* stream() { return c10::cuda::getCurrentCUDAStream().stream(); }

int act_code(const at::ScalarType t) {
  if (t == at::kHalf) return DUPLEX_DTYPE_F16;
  if (t == at::kBFloat16) return DUPLEX_DTYPE_BF16;
  if (t == at::kFloat) return DUPLEX_DTYPE_F32;
  TORCH_CHECK(false, "duplex_b200: unsupported dtype ", t);
  return -1;
}

void require(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), "duplex_b200: ", name, " must be a CUDA tensor (no CPU path)");
  TORCH_CHECK(t.is_contiguous(), "duplex_b200: ", name, " must be contiguous");
}

const void* opt_ptr(const std::optional<at::Tensor>& t) {
  return t.has_value() ? t->data_ptr() : nullptr;
}

// unpack4 (reference fused_packed_moe.py:54-65)
at::Tensor unpack4(const at::Tensor& packed, int64_t out_cols) {
  require(packed, "packed");
  const c10::cuda::CUDAGuard guard(packed.device());
  const int64_t C = packed.size(-1), rows = packed.numel() / C;
  auto sizes = packed.sizes().vec();
  sizes.back() = out_cols;
  at::Tensor out = at::empty(sizes, packed.options().dtype(at::kInt));
  check(duplex_unpack4(packed.data_ptr<int32_t>(), rows, (int32_t)C, (int32_t)out_cols,
                       out.data_ptr<int32_t>(), stream()),
        "unpack4");
  return out;
}

// FusedPackedMoE._dequant / dequantize_weight (fused_packed_moe.py:183-189)
at::Tensor dequant(const at::Tensor& packed, const at::Tensor& scale,
                   const std::optional<at::Tensor>& zeros, int64_t cols, at::ScalarType out_dtype) {
  require(packed, "packed");
  require(scale, "scale");
  const c10::cuda::CUDAGuard guard(packed.device());
  const int64_t G = scale.size(-1), rows = packed.numel() / packed.size(-1);
  TORCH_CHECK(cols % G == 0, "duplex_b200::dequant: cols not divisible by the scale groups");
  auto sizes = packed.sizes().vec();
  sizes.back() = cols;
  at::Tensor out = at::empty(sizes, packed.options().dtype(out_dtype));
  const int32_t* z = zeros.has_value() ? zeros->data_ptr<int32_t>() : nullptr;
  check(duplex_dequant(packed.data_ptr<int32_t>(), scale.data_ptr(), act_code(scale.scalar_type()),
                       z, rows, (int32_t)cols, (int32_t)(cols / G), out.data_ptr(),
                       act_code(out_dtype), stream()),
        "dequant");
  return out;
}

// dequant_gemv (triton_dequant_gemv.py:85-113) over tile records
at::Tensor dequant_gemv(const at::Tensor& x, const at::Tensor& tiles, int64_t E, int64_t R,
                        int64_t K, int64_t group, bool has_zeros, at::ScalarType scale_dtype,
                        const at::Tensor& sel) {
  require(x, "x");
  require(tiles, "tiles");
  require(sel, "sel");
  TORCH_CHECK(sel.scalar_type() == at::kInt, "duplex_b200::dequant_gemv: sel must be int32");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t k = sel.numel();
  at::Tensor out = at::empty({k, R}, x.options().dtype(at::kFloat));
  const int64_t slot_stride = x.dim() == 1 ? 0 : K;
  check(duplex_dq_gemv(x.data_ptr(), act_code(x.scalar_type()), slot_stride, tiles.data_ptr(),
                       act_code(scale_dtype), has_zeros ? 1 : 0, (int32_t)E, (int32_t)R,
                       (int32_t)K, (int32_t)group, sel.data_ptr<int32_t>(), (int32_t)k,
                       out.data_ptr<float>(), nullptr, stream()),
        "dequant_gemv");
  return out;
}

// TritonPackedLinear.forward (triton_dequant_gemv.py:151-159), B <= 8 rows per launch
at::Tensor packed_linear(const at::Tensor& x, const at::Tensor& tiles, int64_t R, int64_t K,
                         int64_t group, bool has_zeros, at::ScalarType scale_dtype,
                         const std::optional<at::Tensor>& bias,
                         const std::optional<at::Tensor>& residual, double rms_eps) {
  require(x, "x");
  require(tiles, "tiles");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t B = x.numel() / K;
  at::Tensor out = at::empty({B, R}, x.options());
  for (int64_t r0 = 0; r0 < B; r0 += 8) {
    const int64_t b = B - r0 < 8 ? B - r0 : 8;
    const auto* xb = static_cast<const uint8_t*>(x.data_ptr()) + r0 * K * x.element_size();
    auto* ob = static_cast<uint8_t*>(out.data_ptr()) + r0 * R * out.element_size();
    const uint8_t* rb = residual.has_value()
                            ? static_cast<const uint8_t*>(residual->data_ptr()) +
                                  r0 * R * residual->element_size()
                            : nullptr;
    check(duplex_packed_linear(xb, act_code(x.scalar_type()), (int32_t)b, K, tiles.data_ptr(),
                               act_code(scale_dtype), has_zeros ? 1 : 0, (int32_t)R, (int32_t)K,
                               (int32_t)group, opt_ptr(bias), rb, R, ob, R, (float)rms_eps, 0,
                               stream()),
          "packed_linear");
  }
  auto sizes = x.sizes().vec();
  sizes.back() = R;
  return out.view(sizes);
}

// FusedPackedMoE.forward (fused_packed_moe.py:191-275) for T <= 8 tokens
at::Tensor moe_forward(const at::Tensor& x, const at::Tensor& gate_w,
                       const std::optional<at::Tensor>& gate_b, const at::Tensor& gu_tiles,
                       const at::Tensor& dn_tiles, int64_t I, int64_t top_k, bool norm_topk,
                       int64_t group, bool has_zeros, const at::Tensor& workspace,
                       const at::Tensor& err, const std::optional<at::Tensor>& residual,
                       double rms_eps) {
  require(x, "x");
  require(gate_w, "gate_w");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t T = x.size(0), H = x.size(1), E = gate_w.size(0);
  at::Tensor out = at::empty_like(x);
  check(duplex_moe_forward(x.data_ptr(), act_code(x.scalar_type()), (int32_t)T, gate_w.data_ptr(),
                           opt_ptr(gate_b), (int32_t)E, (int32_t)H, (int32_t)I, (int32_t)top_k,
                           norm_topk ? 1 : 0, gu_tiles.data_ptr(), dn_tiles.data_ptr(),
                           act_code(x.scalar_type()), has_zeros ? 1 : 0, (int32_t)group,
                           opt_ptr(residual), out.data_ptr(), nullptr, nullptr, workspace.data_ptr(),
                           (size_t)workspace.numel(), err.data_ptr<int32_t>(), (float)rms_eps, 1,
                           stream()),
        "moe_forward");
  return out;
}

// the batched-decode layer (duplex_moe_grouped) for T <= 512 tokens
at::Tensor moe_grouped(const at::Tensor& x, const at::Tensor& gate_w,
                       const std::optional<at::Tensor>& gate_b, const at::Tensor& gu_tiles,
                       const at::Tensor& dn_tiles, int64_t I, int64_t top_k, bool norm_topk,
                       int64_t group, bool has_zeros, const at::Tensor& workspace,
                       const at::Tensor& err, const std::optional<at::Tensor>& residual) {
  require(x, "x");
  require(gate_w, "gate_w");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t T = x.size(0), H = x.size(1), E = gate_w.size(0);
  at::Tensor out = at::empty_like(x);
  check(duplex_moe_grouped(x.data_ptr(), act_code(x.scalar_type()), (int32_t)T, gate_w.data_ptr(),
                           opt_ptr(gate_b), nullptr, (int32_t)E, (int32_t)H, (int32_t)I,
                           (int32_t)top_k, norm_topk ? 1 : 0, gu_tiles.data_ptr(),
                           dn_tiles.data_ptr(), act_code(x.scalar_type()), has_zeros ? 1 : 0,
                           (int32_t)group, opt_ptr(residual), out.data_ptr(), nullptr, nullptr,
                           workspace.data_ptr(), (size_t)workspace.numel(),
                           err.data_ptr<int32_t>(), stream()),
        "moe_grouped");
  return out;
}

// expert-parallel dispatch pack (into caller buffers) and combine
void ep_dispatch(const at::Tensor& rows, int64_t top_k, int64_t E, int64_t n_ranks,
                 int64_t ids_offset, at::Tensor& send, at::Tensor& slot_of) {
  require(rows, "rows");
  const c10::cuda::CUDAGuard guard(rows.device());
  check(duplex_ep_dispatch_pack(rows.data_ptr(), rows.stride(0), (int32_t)rows.size(0),
                                (int32_t)top_k, (int32_t)E, (int32_t)n_ranks, ids_offset,
                                send.data_ptr(), slot_of.data_ptr<int32_t>(), stream()),
        "ep_dispatch");
}

at::Tensor ep_combine(const at::Tensor& partials, const at::Tensor& slot_of,
                      const std::optional<at::Tensor>& residual, at::ScalarType out_dtype) {
  require(partials, "partials");
  const c10::cuda::CUDAGuard guard(partials.device());
  const int64_t N = partials.size(0), T = partials.size(1), H = partials.size(2);
  at::Tensor out = at::empty({T, H}, partials.options().dtype(out_dtype));
  check(duplex_ep_combine(partials.data_ptr<float>(), slot_of.data_ptr<int32_t>(), (int32_t)T,
                          (int32_t)N, (int32_t)H, opt_ptr(residual), out.data_ptr(),
                          act_code(out_dtype), stream()),
        "ep_combine");
  return out;
}

// the router of FusedPackedMoE.forward (fused_packed_moe.py:195-199), T <= 8 tokens:
// (w [T, top_k] fp32, sel [T, top_k] int32); workspace from duplex_moe_workspace_bytes,
// zero-filled once
std::tuple<at::Tensor, at::Tensor> moe_route(const at::Tensor& x, const at::Tensor& gate_w,
                                             const std::optional<at::Tensor>& gate_b, int64_t top_k,
                                             bool norm_topk, const at::Tensor& workspace) {
  require(x, "x");
  require(gate_w, "gate_w");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t T = x.size(0), H = x.size(1), E = gate_w.size(0);
  at::Tensor w = at::empty({T, top_k}, x.options().dtype(at::kFloat));
  at::Tensor sel = at::empty({T, top_k}, x.options().dtype(at::kInt));
  check(duplex_moe_route(x.data_ptr(), act_code(x.scalar_type()), (int32_t)T, gate_w.data_ptr(),
                         opt_ptr(gate_b), (int32_t)E, (int32_t)H, (int32_t)top_k, norm_topk ? 1 : 0,
                         w.data_ptr<float>(), sel.data_ptr<int32_t>(), workspace.data_ptr(),
                         (size_t)workspace.numel(), 0.f, 0, stream()),
        "moe_route");
  return {w, sel};
}

// the Talker's MoE block (fused_moe.py:40-141), T <= 8 tokens
at::Tensor talker_moe(const at::Tensor& x, const at::Tensor& gate_w, const at::Tensor& gate_up,
                      const at::Tensor& down, const std::optional<at::Tensor>& gu_scale,
                      const std::optional<at::Tensor>& dn_scale, int64_t top_k, bool norm_topk,
                      const std::optional<at::Tensor>& sh_gate, const std::optional<at::Tensor>& sh_up,
                      const std::optional<at::Tensor>& sh_down,
                      const std::optional<at::Tensor>& sh_gate_w, const at::Tensor& workspace,
                      const at::Tensor& err) {
  require(x, "x");
  require(gate_up, "gate_up");
  require(down, "down");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t T = x.size(0), H = x.size(1), E = gate_up.size(0), I = gate_up.size(1) / 2;
  const int64_t S = sh_gate.has_value() ? sh_gate->size(0) : 0;
  at::Tensor out = at::empty_like(x);
  check(duplex_talker_moe_forward(
            x.data_ptr(), act_code(x.scalar_type()), (int32_t)T, gate_w.data_ptr(), (int32_t)E,
            (int32_t)H, (int32_t)I, (int32_t)top_k, norm_topk ? 1 : 0, gate_up.data_ptr(),
            down.data_ptr(), gate_up.scalar_type() == at::kChar ? 1 : 0, opt_ptr(gu_scale),
            opt_ptr(dn_scale), opt_ptr(sh_gate), opt_ptr(sh_up), opt_ptr(sh_down), (int32_t)S,
            opt_ptr(sh_gate_w), out.data_ptr(), nullptr, nullptr, workspace.data_ptr(),
            (size_t)workspace.numel(), err.data_ptr<int32_t>(), stream()),
        "talker_moe");
  return out;
}

}  // namespace

TORCH_LIBRARY(duplex_b200, m) {
  m.def("unpack4(Tensor packed, int out_cols) -> Tensor");
  m.def("dequant(Tensor packed, Tensor scale, Tensor? zeros, int cols, ScalarType out_dtype) -> Tensor");
  m.def("dequant_gemv(Tensor x, Tensor tiles, int E, int R, int K, int group, bool has_zeros, "
        "ScalarType scale_dtype, Tensor sel) -> Tensor");
  m.def("packed_linear(Tensor x, Tensor tiles, int R, int K, int group, bool has_zeros, "
        "ScalarType scale_dtype, Tensor? bias, Tensor? residual, float rms_eps) -> Tensor");
  m.def("moe_forward(Tensor x, Tensor gate_w, Tensor? gate_b, Tensor gu_tiles, Tensor dn_tiles, "
        "int I, int top_k, bool norm_topk, int group, bool has_zeros, Tensor workspace, "
        "Tensor err, Tensor? residual, float rms_eps) -> Tensor");
  m.def("moe_grouped(Tensor x, Tensor gate_w, Tensor? gate_b, Tensor gu_tiles, Tensor dn_tiles, "
        "int I, int top_k, bool norm_topk, int group, bool has_zeros, Tensor workspace, "
        "Tensor err, Tensor? residual) -> Tensor");
  m.def("ep_dispatch(Tensor rows, int top_k, int E, int n_ranks, int ids_offset, "
        "Tensor(a!) send, Tensor(b!) slot_of) -> ()");
  m.def("ep_combine(Tensor partials, Tensor slot_of, Tensor? residual, ScalarType out_dtype) "
        "-> Tensor");
  m.def("moe_route(Tensor x, Tensor gate_w, Tensor? gate_b, int top_k, bool norm_topk, "
        "Tensor workspace) -> (Tensor, Tensor)");
  m.def("talker_moe(Tensor x, Tensor gate_w, Tensor gate_up, Tensor down, Tensor? gu_scale, "
        "Tensor? dn_scale, int top_k, bool norm_topk, Tensor? sh_gate, Tensor? sh_up, "
        "Tensor? sh_down, Tensor? sh_gate_w, Tensor workspace, Tensor err) -> Tensor");
}

TORCH_LIBRARY_IMPL(duplex_b200, CUDA, m) {
  m.impl("unpack4", &unpack4);
  m.impl("dequant", &dequant);
  m.impl("dequant_gemv", &dequant_gemv);
  m.impl("packed_linear", &packed_linear);
  m.impl("moe_forward", &moe_forward);
  m.impl("moe_grouped", &moe_grouped);
  m.impl("ep_dispatch", &ep_dispatch);
  m.impl("ep_combine", &ep_combine);
  m.impl("moe_route", &moe_route);
  m.impl("talker_moe", &talker_moe);
}
