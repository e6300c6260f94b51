// sy_torch.cpp -- the thin PyTorch C++ extension over the C ABI.
//
// The Python autograd functions of switchyard.triton_op (forward and backward
// of _BlockAttnResTriton, src/switchyard/triton_op.py:504-589 in the
// reference) call these instead of several Python-level steps: one call does
// the output/statistics/partial-row allocations (torch's caching allocator, on
// the tensor's device and its current stream), the launches through
// include/switchyard_b200.h, and the status check. Arguments arrive already
// validated by the Python layer (which keeps the reference's exception types
// and messages); only the invariants the kernels rely on are checked here.
#include <torch/extension.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <string>
#include <tuple>

#include "switchyard_b200.h"

namespace {

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kBFloat16:
      return SY_BF16;
    case at::kHalf:
      return SY_F16;
    case at::kFloat:
      return SY_F32;
    default:
      TORCH_CHECK(false, "switchyard kernels take bfloat16, float16 or float32 tensors, got ", t);
  }
  return -1;
}

void check(int status, const char* what) {
  TORCH_CHECK(status == SY_OK, "switchyard: ", what, " failed (status ", status,
              "): ", sy_status_string(status));
}

sy_stream_t stream_of(const at::Tensor& t) {
  return static_cast<sy_stream_t>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

void need_cuda_contiguous(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous(), "switchyard: ", name,
              " must be a contiguous CUDA tensor");
}

// out [B, T, D] in v's dtype and the fp32 statistics [B*T, SW], plus the kernel
// family the planner picked (sy_plan_kind; -1 when nothing was launched).
std::tuple<at::Tensor, at::Tensor, int64_t> forward(const at::Tensor& v, const at::Tensor& w,
                                                    double eps) {
  need_cuda_contiguous(v, "v");
  need_cuda_contiguous(w, "w");
  TORCH_CHECK(v.dim() == 4 && w.dim() == 1 && w.size(0) == v.size(3), "switchyard: bad shapes");
  const c10::cuda::CUDAGuard guard(v.device());
  const int64_t n = v.size(0), b = v.size(1), t = v.size(2), d = v.size(3), bt = b * t;
  at::Tensor out = at::empty({b, t, d}, v.options());
  at::Tensor stats = at::empty({bt, sy_stats_stride(n)}, v.options().dtype(at::kFloat));
  int64_t kind = -1;
  if (bt > 0 && d > 0) {
    const int vd = dtype_code(v.scalar_type());
    check(sy_fwd(v.data_ptr(), w.data_ptr(), out.data_ptr(), stats.data_ptr<float>(), n, bt, d,
                 vd, dtype_code(w.scalar_type()), static_cast<float>(eps), stream_of(v)),
          "sy_fwd");
    kind = sy_plan_kind(0, n, bt, d, 1, vd);
  }
  return {out, stats, kind};
}

// dv [N, B, T, D] and the fp32 dw partial rows [P, D] (undefined when D == 0).
std::tuple<at::Tensor, at::Tensor> backward_partials(const at::Tensor& v, const at::Tensor& w,
                                                     const at::Tensor& stats,
                                                     const at::Tensor& grad_out, double eps) {
  need_cuda_contiguous(v, "v");
  need_cuda_contiguous(w, "w");
  need_cuda_contiguous(stats, "stats");
  const c10::cuda::CUDAGuard guard(v.device());
  const at::Tensor g = grad_out.to(v.scalar_type()).contiguous();
  const int64_t n = v.size(0), bt = v.size(1) * v.size(2), d = v.size(3);
  TORCH_CHECK(g.numel() == bt * d, "switchyard: gradient of the wrong size");
  at::Tensor dv = at::empty_like(v);
  if (d == 0) return {dv, at::Tensor()};
  const int vd = dtype_code(v.scalar_type());
  const int64_t p = sy_bwd_partials(n, bt, d, vd);
  TORCH_CHECK(p >= 1, "switchyard: sy_bwd_partials failed (status ", -p, "): ",
              sy_status_string(static_cast<int>(-p)));
  at::Tensor part = at::empty({p, d}, v.options().dtype(at::kFloat));
  check(sy_bwd(v.data_ptr(), w.data_ptr(), g.data_ptr(), stats.data_ptr<float>(), dv.data_ptr(),
               part.data_ptr<float>(), p, n, bt, d, vd, dtype_code(w.scalar_type()),
               static_cast<float>(eps), stream_of(v)),
        "sy_bwd");
  return {dv, part};
}

// dv and dw = the fixed-order sum of the partial rows, in `dw_dtype`.
std::tuple<at::Tensor, at::Tensor> backward(const at::Tensor& v, const at::Tensor& w,
                                            const at::Tensor& stats, const at::Tensor& grad_out,
                                            double eps, at::ScalarType dw_dtype) {
  auto [dv, part] = backward_partials(v, w, stats, grad_out, eps);
  const c10::cuda::CUDAGuard guard(v.device());
  at::Tensor dw = at::empty({w.size(0)}, w.options().dtype(dw_dtype));
  if (part.defined())
    check(sy_dw_reduce(part.data_ptr<float>(), part.size(0), part.size(1), dw.data_ptr(),
                       dtype_code(dw_dtype), stream_of(v)),
          "sy_dw_reduce");
  return {dv, dw};
}

// With the module's gain, q = w * gain: dv, and dw = dq * gain, dgain = dq * w
// in one reduction launch (either may be skipped: undefined tensor returned).
std::tuple<at::Tensor, at::Tensor, at::Tensor> backward_gain(
    const at::Tensor& v, const at::Tensor& q, const at::Tensor& stats, const at::Tensor& grad_out,
    const at::Tensor& w, const at::Tensor& gain, double eps, bool need_dw, bool need_dg) {
  need_cuda_contiguous(w, "w");
  need_cuda_contiguous(gain, "gain");
  auto [dv, part] = backward_partials(v, q, stats, grad_out, eps);
  const c10::cuda::CUDAGuard guard(v.device());
  at::Tensor dw = need_dw ? at::empty_like(w) : at::Tensor();
  at::Tensor dg = need_dg ? at::empty_like(gain) : at::Tensor();
  if (!part.defined()) {
    if (need_dw) dw.zero_();
    if (need_dg) dg.zero_();
  } else if (need_dw || need_dg) {
    check(sy_dw_reduce_gain(part.data_ptr<float>(), part.size(0), part.size(1), w.data_ptr(),
                            gain.data_ptr(), need_dw ? dw.data_ptr() : nullptr,
                            need_dg ? dg.data_ptr() : nullptr, dtype_code(w.scalar_type()),
                            stream_of(v)),
          "sy_dw_reduce_gain");
  }
  return {dv, dw, dg};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "switchyard B200: PyTorch C++ extension over the C ABI of libswitchyard_b200.so";
  m.def("forward", &forward, "sy_fwd: (out, stats, plan kind)");
  m.def("backward_partials", &backward_partials, "sy_bwd: (dv, dw partial rows)");
  m.def("backward", &backward, "sy_bwd + sy_dw_reduce: (dv, dw)");
  m.def("backward_gain", &backward_gain, "sy_bwd + sy_dw_reduce_gain: (dv, dw, dgain)");
  m.def("version", []() { return std::string(sy_version()); });
}
