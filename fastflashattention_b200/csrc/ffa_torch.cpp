// ffa_torch.cpp — the torch-facing host path of the library, in C++.
//
// The reference's host path is Python: `fastflash_attn` (fastflash_attention/_kernel.py:282-318)
// prepares the tensors and launches the forward, and the autograd Function `FastFlashAttn`
// (:773-906) saves q, k, v, o, lse and launches the backward.  At short sequences that host
// work, not the kernels, sets the step time (the reference measured launch and autograd
// overhead at about 68 % of wall time, :820-821).  This file does the same work in C++ and
// registers it as torch operators, so a call costs one dispatcher entry instead of dozens of
// Python-level tensor operations and a ctypes call:
//
//   ffa_b200::forward(q, k, v, causal, scale)          -> o            (no LSE, no grad)
//   ffa_b200::forward_lse(q, k, v, causal, scale)      -> (o, lse)
//   ffa_b200::backward(q, k, v, o, do, lse, causal, scale) -> (dq, dk, dv)
//   ffa_b200::attention(q, k, v, causal, scale)        -> o, differentiable (C++ autograd node)
//
// q, k, v are [B, H, S, D] bf16 CUDA tensors with D a power of two <= 128 (the Python layer
// has already checked the contract and raised UnsupportedConfig otherwise).  Outputs come from
// the torch caching allocator on the inputs' device and every launch goes on the current
// stream, as in the reference.  D < 64 is zero-padded to 64 (exact).  Errors from the C ABI
// raise RuntimeError with the library's message.  The kernels are reached only through the
// C ABI of libffa_sm100.so (include/ffa.h).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/autograd.h>
#include <torch/library.h>

#include <cmath>

#include "../../include/ffa.h"

namespace {

using at::Tensor;

void check(int rc, const char* fn) {
  if (rc != FFA_OK) {
    char buf[256];
    ffa_last_error(buf, sizeof(buf));
    TORCH_CHECK(false, fn, " failed with status ", rc, ": ", buf);
  }
}

int64_t kernel_dim(int64_t d) { return d <= 64 ? 64 : 128; }

// [B, H, S, D] -> contiguous [B*H, S, kd] (zero-padded along D when D < kd)
Tensor prep(const Tensor& t, int64_t kd) {
  Tensor c = t.contiguous();
  if (c.size(3) != kd) c = at::constant_pad_nd(c, {0, kd - c.size(3)}, 0);
  return c.view({c.size(0) * c.size(1), c.size(2), kd});
}

// [B*H, S, kd] -> [B, H, S, D]
Tensor unprep(const Tensor& t, int64_t B, int64_t H, int64_t D) {
  Tensor r = t.view({B, H, t.size(1), t.size(2)});
  return r.size(3) == D ? r : r.narrow(3, 0, D).contiguous();
}

double softmax_scale(int64_t D, const c10::optional<double>& scale) {
  return scale.has_value() ? *scale : 1.0 / std::sqrt(static_cast<double>(D));
}

void* stream_of(const Tensor& t) { return at::cuda::getCurrentCUDAStream(t.device().index()).stream(); }

std::tuple<Tensor, Tensor> fwd_impl(const Tensor& q, const Tensor& k, const Tensor& v, bool causal,
                                    const c10::optional<double>& scale, bool with_lse) {
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda(), "q, k, v must be CUDA tensors");
  TORCH_CHECK(q.dim() == 4 && q.sizes() == k.sizes() && q.sizes() == v.sizes(), "q, k, v must share a [B,H,S,D] shape");
  const int64_t B = q.size(0), H = q.size(1), S = q.size(2), D = q.size(3);
  const c10::cuda::CUDAGuard guard(q.device());
  const int64_t kd = kernel_dim(D);
  Tensor qf = prep(q, kd), kf = prep(k, kd), vf = prep(v, kd);
  Tensor o = at::empty_like(qf);
  Tensor lse;
  if (with_lse) lse = at::empty({B * H, S}, q.options().dtype(at::kFloat));
  check(ffa_fwd(qf.data_ptr(), kf.data_ptr(), vf.data_ptr(), o.data_ptr(), with_lse ? lse.data_ptr<float>() : nullptr,
                static_cast<int>(B * H), static_cast<int>(S), static_cast<int>(kd), qf.stride(0), qf.stride(1),
                softmax_scale(D, scale), causal ? 1 : 0, stream_of(q)),
        "ffa_fwd");
  return {unprep(o, B, H, D), with_lse ? lse.view({B, H, S}) : lse};
}

Tensor forward_op(const Tensor& q, const Tensor& k, const Tensor& v, bool causal, c10::optional<double> scale) {
  return std::get<0>(fwd_impl(q, k, v, causal, scale, false));
}

std::tuple<Tensor, Tensor> forward_lse_op(const Tensor& q, const Tensor& k, const Tensor& v, bool causal,
                                          c10::optional<double> scale) {
  return fwd_impl(q, k, v, causal, scale, true);
}

std::tuple<Tensor, Tensor, Tensor> backward_op(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& o,
                                               const Tensor& dout, const Tensor& lse, bool causal,
                                               c10::optional<double> scale) {
  const int64_t B = q.size(0), H = q.size(1), S = q.size(2), D = q.size(3);
  const c10::cuda::CUDAGuard guard(q.device());
  const int64_t kd = kernel_dim(D);
  Tensor qf = prep(q, kd), kf = prep(k, kd), vf = prep(v, kd), of = prep(o, kd), dof = prep(dout, kd);
  Tensor lf = lse.contiguous();
  Tensor dq = at::empty_like(qf), dk = at::empty_like(kf), dv = at::empty_like(vf);
  Tensor delta = at::empty({B * H, S}, q.options().dtype(at::kFloat));
  check(ffa_bwd(qf.data_ptr(), kf.data_ptr(), vf.data_ptr(), of.data_ptr(), dof.data_ptr(), lf.data_ptr<float>(),
                delta.data_ptr<float>(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), static_cast<int>(B * H),
                static_cast<int>(S), static_cast<int>(kd), qf.stride(0), qf.stride(1), softmax_scale(D, scale),
                causal ? 1 : 0, stream_of(q)),
        "ffa_bwd");
  return {unprep(dq, B, H, D), unprep(dk, B, H, D), unprep(dv, B, H, D)};
}

// The autograd node of ffa_b200::attention: forward with LSE, saved q, k, v, o, lse, and the
// deterministic backward (reference FastFlashAttn, _kernel.py:773-906).
class Attention : public torch::autograd::Function<Attention> {
 public:
  static Tensor forward(torch::autograd::AutogradContext* ctx, const Tensor& q, const Tensor& k, const Tensor& v,
                        bool causal, c10::optional<double> scale) {
    auto [o, lse] = fwd_impl(q, k, v, causal, scale, true);
    ctx->save_for_backward({q, k, v, o, lse});
    ctx->saved_data["causal"] = causal;
    ctx->saved_data["has_scale"] = scale.has_value();
    ctx->saved_data["scale"] = scale.has_value() ? *scale : 0.0;
    return o;
  }

  static torch::autograd::tensor_list backward(torch::autograd::AutogradContext* ctx,
                                               torch::autograd::tensor_list grads) {
    const auto saved = ctx->get_saved_variables();
    const bool causal = ctx->saved_data["causal"].toBool();
    c10::optional<double> scale;
    if (ctx->saved_data["has_scale"].toBool()) scale = ctx->saved_data["scale"].toDouble();
    auto [dq, dk, dv] = backward_op(saved[0], saved[1], saved[2], saved[3], grads[0], saved[4], causal, scale);
    return {dq, dk, dv, Tensor(), Tensor()};
  }
};

Tensor attention_op(const Tensor& q, const Tensor& k, const Tensor& v, bool causal, c10::optional<double> scale) {
  return Attention::apply(q, k, v, causal, scale);
}

}  // namespace

TORCH_LIBRARY(ffa_b200, m) {
  m.def("forward(Tensor q, Tensor k, Tensor v, bool causal, float? scale) -> Tensor");
  m.def("forward_lse(Tensor q, Tensor k, Tensor v, bool causal, float? scale) -> (Tensor, Tensor)");
  m.def("backward(Tensor q, Tensor k, Tensor v, Tensor o, Tensor dout, Tensor lse, bool causal, float? scale)"
        " -> (Tensor, Tensor, Tensor)");
  m.def("attention(Tensor q, Tensor k, Tensor v, bool causal, float? scale) -> Tensor");
}

TORCH_LIBRARY_IMPL(ffa_b200, CUDA, m) {
  m.impl("attention", forward_op);  // reached only where autograd is off (inference mode)
  m.impl("forward", forward_op);
  m.impl("forward_lse", forward_lse_op);
  m.impl("backward", backward_op);
}

TORCH_LIBRARY_IMPL(ffa_b200, Autograd, m) { m.impl("attention", attention_op); }
