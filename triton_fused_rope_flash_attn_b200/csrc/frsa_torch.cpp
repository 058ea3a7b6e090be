// PyTorch C++ extension over the C ABI (include/frsa.h): the host side of the
// product path. It does in C++ what the reference's autograd wrapper does in
// Python before its Triton launches (fa_rope_full .py:1011-1138): shape and
// dtype checks, output and scratch allocation (torch's caching allocator, on
// the tensors' device), and the launch on torch's current stream. The C-ABI
// entry points are bound at run time from the loaded libfrsa.so (bind()), so
// this module has no link-time dependency on it.
//
// Each function returns its tensors plus the FRSA status code; the Python
// layer turns a non-zero code into FrsaError, as it does for direct C-ABI
// calls.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cmath>
#include <cstdint>

#include "frsa.h"

namespace {

using FwdFn = int (*)(const frsa_attn_args*, void*);
using WsFn = size_t (*)(const frsa_attn_args*);

FwdFn g_fwd = nullptr;
FwdFn g_bwd = nullptr;
WsFn g_ws = nullptr;

void bind(int64_t fwd, int64_t bwd, int64_t ws) {
  g_fwd = reinterpret_cast<FwdFn>(fwd);
  g_bwd = reinterpret_cast<FwdFn>(bwd);
  g_ws = reinterpret_cast<WsFn>(ws);
}

int32_t dtype_code(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kBFloat16: return FRSA_DTYPE_BF16;
    case at::kHalf: return FRSA_DTYPE_F16;
    case at::kFloat: return FRSA_DTYPE_F32;
    default: TORCH_CHECK_TYPE(false, "unsupported compute dtype ", t.scalar_type());
  }
  return -1;
}

void check_inputs(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                  const at::Tensor& cosp, const at::Tensor& sinp, int64_t flags) {
  TORCH_CHECK(g_fwd && g_bwd && g_ws, "frsa extension: C ABI not bound (call bind first)");
  TORCH_CHECK(q.is_cuda(), "q must be a CUDA tensor (there is no CPU path)");
  TORCH_CHECK(q.dim() == 4, "q must be [B, H, N, D]");
  TORCH_CHECK(k.sizes() == q.sizes() && v.sizes() == q.sizes(), "q, k, v shapes differ");
  TORCH_CHECK_TYPE(k.scalar_type() == q.scalar_type() && v.scalar_type() == q.scalar_type(),
                   "q, k, v dtypes differ");
  TORCH_CHECK(k.device() == q.device() && v.device() == q.device(), "q, k, v devices differ");
  if (flags & FRSA_FLAG_NO_ROPE) return;   // tables unused
  TORCH_CHECK_TYPE(cosp.scalar_type() == at::kFloat && sinp.scalar_type() == at::kFloat,
                   "COSP/SINP must be float32");
  TORCH_CHECK(cosp.device() == q.device() && sinp.device() == q.device(),
              "RoPE tables must be on the same device as Q");
  TORCH_CHECK(cosp.dim() == 2 && cosp.sizes() == sinp.sizes(), "COSP/SINP must be [N_pos, D/2]");
}

// q, k and v are read in place through strided TMA maps when their d stride
// is 1, their other strides are multiples of 16 bytes and their data 16-byte
// aligned (e.g. the q, k, v views of a [B, N, 3, H, D] projection output);
// otherwise a contiguous copy is made.
bool tma_strided_ok(const at::Tensor& t) {
  if (t.stride(3) != 1) return false;
  const int64_t e = t.element_size();
  for (int d = 0; d < 3; ++d)
    if (t.size(d) > 1 && (t.stride(d) < 1 || (t.stride(d) * e) % 16 != 0)) return false;
  return (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15u) == 0;
}

at::Tensor readable(const at::Tensor& t) { return tma_strided_ok(t) ? t : t.contiguous(); }

void set_strides(int64_t* dst, const at::Tensor& t) {
  if (t.is_contiguous()) {
    dst[0] = dst[1] = dst[2] = 0;
    return;
  }
  // Size-1 dimensions may carry any stride; give them a valid one.
  const int64_t e = t.element_size(), unit = 16 / e;
  for (int d = 0; d < 3; ++d) dst[d] = (t.size(d) > 1) ? t.stride(d) : unit;
}

void fill_shape(frsa_attn_args& a, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                const at::Tensor& cosp, const at::Tensor& sinp, bool has_cls, double scale,
                int64_t flags) {
  a.q = q.data_ptr();
  a.k = k.data_ptr();
  a.v = v.data_ptr();
  set_strides(a.q_strides, q);
  set_strides(a.k_strides, k);
  set_strides(a.v_strides, v);
  a.flags = static_cast<int32_t>(flags);
  const bool rope = (flags & FRSA_FLAG_NO_ROPE) == 0;
  a.cosp = rope ? cosp.data_ptr<float>() : nullptr;
  a.sinp = rope ? sinp.data_ptr<float>() : nullptr;
  a.B = q.size(0);
  a.H = q.size(1);
  a.N = q.size(2);
  a.D = q.size(3);
  a.n_pos = rope ? cosp.size(0) : 0;
  a.has_cls = has_cls ? 1 : 0;
  a.io_dtype = a.compute_dtype = dtype_code(q);
  a.scale = scale > 0 ? static_cast<float>(scale) : static_cast<float>(1.0 / std::sqrt(double(a.D)));
}

// O and LSE of softmax(R(q) R(k)^T * scale) v. scale <= 0: 1/sqrt(D).
std::tuple<at::Tensor, at::Tensor, int64_t> fwd(const at::Tensor& q_in, const at::Tensor& k_in,
                                                const at::Tensor& v_in, const at::Tensor& cosp_in,
                                                const at::Tensor& sinp_in, bool has_cls,
                                                double scale, int64_t flags) {
  check_inputs(q_in, k_in, v_in, cosp_in, sinp_in, flags);
  const c10::cuda::CUDAGuard guard(q_in.device());
  const at::Tensor q = readable(q_in), k = readable(k_in), v = readable(v_in);
  const bool rope = (flags & FRSA_FLAG_NO_ROPE) == 0;
  const at::Tensor cosp = rope ? cosp_in.contiguous() : cosp_in;
  const at::Tensor sinp = rope ? sinp_in.contiguous() : sinp_in;
  at::Tensor o = at::empty(q.sizes(), q.options());
  at::Tensor lse = at::empty({q.size(0), q.size(1), q.size(2)}, q.options().dtype(at::kFloat));
  frsa_attn_args a{};
  fill_shape(a, q, k, v, cosp, sinp, has_cls, scale, flags);
  a.o = o.data_ptr();
  a.lse = lse.data_ptr<float>();
  const int rc = g_fwd(&a, at::cuda::getCurrentCUDAStream().stream());
  return {o, lse, rc};
}

// dQ, dK, dV (and Delta into delta_out when given). scale <= 0: 1/sqrt(D).
std::tuple<at::Tensor, at::Tensor, at::Tensor, int64_t> bwd(
    const at::Tensor& q_in, const at::Tensor& k_in, const at::Tensor& v_in,
    const at::Tensor& o_in, const at::Tensor& lse_in, const at::Tensor& do_in,
    const at::Tensor& cosp_in, const at::Tensor& sinp_in, bool has_cls,
    const c10::optional<at::Tensor>& delta_out, double scale, int64_t flags) {
  check_inputs(q_in, k_in, v_in, cosp_in, sinp_in, flags);
  TORCH_CHECK(o_in.sizes() == q_in.sizes() && do_in.sizes() == q_in.sizes(),
              "o and dO must have q's shape");
  TORCH_CHECK_TYPE(o_in.scalar_type() == q_in.scalar_type() &&
                       do_in.scalar_type() == q_in.scalar_type(),
                   "o and dO must have q's dtype");
  TORCH_CHECK_TYPE(lse_in.scalar_type() == at::kFloat, "lse must be float32");
  const c10::cuda::CUDAGuard guard(q_in.device());
  const at::Tensor q = readable(q_in), k = readable(k_in), v = readable(v_in);
  const at::Tensor o = o_in.contiguous(), lse = lse_in.contiguous(), d_o = do_in.contiguous();
  const bool rope = (flags & FRSA_FLAG_NO_ROPE) == 0;
  const at::Tensor cosp = rope ? cosp_in.contiguous() : cosp_in;
  const at::Tensor sinp = rope ? sinp_in.contiguous() : sinp_in;
  at::Tensor dq = at::empty(q.sizes(), q.options()), dk = at::empty(k.sizes(), k.options()),
             dv = at::empty(v.sizes(), v.options());
  frsa_attn_args a{};
  fill_shape(a, q, k, v, cosp, sinp, has_cls, scale, flags);
  a.o = const_cast<void*>(o.data_ptr());
  a.lse = const_cast<float*>(lse.data_ptr<float>());
  a.d_o = d_o.data_ptr();
  a.dq = dq.data_ptr();
  a.dk = dk.data_ptr();
  a.dv = dv.data_ptr();
  if (delta_out.has_value()) {
    TORCH_CHECK(delta_out->is_contiguous() && delta_out->scalar_type() == at::kFloat &&
                    delta_out->numel() == q.size(0) * q.size(1) * q.size(2),
                "delta_out must be a contiguous float32 [B, H, N] tensor");
    a.delta = delta_out->data_ptr<float>();
  }
  at::Tensor ws;
  const size_t ws_bytes = g_ws(&a);
  if (ws_bytes > 0) {
    ws = at::empty({static_cast<int64_t>((ws_bytes + 3) / 4)}, q.options().dtype(at::kFloat));
    a.workspace = ws.data_ptr();
    a.workspace_bytes = ws_bytes;
  }
  const int rc = g_bwd(&a, at::cuda::getCurrentCUDAStream().stream());
  return {dq, dk, dv, rc};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "PyTorch host side of the fused 2D-RoPE attention (C ABI include/frsa.h)";
  m.def("bind", &bind, "bind the C-ABI entry points (frsa_fwd, frsa_bwd, frsa_bwd_workspace_bytes)");
  m.def("fwd", &fwd, "forward: (o, lse, status)");
  m.def("bwd", &bwd, "backward: (dq, dk, dv, status)");
}
