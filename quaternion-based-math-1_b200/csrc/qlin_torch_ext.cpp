// Inference forward of the package's modules in C++ (torch extension).
//
// fused_quaternion_linear without autograd spends most of a decode call's
// time on host-side argument handling when written in Python (about 25 us
// against a 6-7 us device call).  This function performs the same checks,
// in the same order and with the same error classes as the reference
// (shape problems -> ValueError, quaternion/packing.py:45-52 and
// quaternion/linear.py:55-61; device, dtype and launch problems ->
// RuntimeError), allocates the output, picks the workspace and calls
// qlin_forward_ex on the current stream.  The library does the rest.
//
// Workspaces: calls of at most 4 tokens (16-bit) use a zero-filled buffer
// kept per (device, stream) and pass QLIN_FLAG_ZEROED_WORKSPACE (calls on one
// stream are ordered and leave its counter bytes at zero); a buffer that
// must grow while the stream is being captured into a CUDA graph is not
// grown -- that call takes a plain workspace from the caching allocator.
// A buffer that is replaced by a larger one is never released: a CUDA graph
// captured earlier on that stream still holds its address and would write
// its counters and partial sums into whatever memory reused it.
#include <torch/extension.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAGraphsC10Utils.h>

#include <map>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "qlin_b200.h"

namespace {

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return QLIN_F32;
    case at::kBFloat16: return QLIN_BF16;
    case at::kHalf: return QLIN_F16;
    default:
      TORCH_CHECK(false, "unsupported dtype ", t,
                  "; the B200 quaternion kernels take float32, bfloat16 or float16");
  }
  return -1;
}

constexpr int64_t kZeroedMaxTokens = 4;

std::mutex g_ws_mutex;
std::map<std::pair<int, uintptr_t>, at::Tensor> g_zeroed;
std::vector<at::Tensor> g_zeroed_retired;  // superseded buffers, kept alive for captured graphs

at::Tensor zeroed_workspace(const at::Device& dev, cudaStream_t stream, size_t bytes) {
  const auto key = std::make_pair(static_cast<int>(dev.index()), reinterpret_cast<uintptr_t>(stream));
  std::lock_guard<std::mutex> lock(g_ws_mutex);
  auto it = g_zeroed.find(key);
  if (it != g_zeroed.end() && static_cast<size_t>(it->second.numel()) >= bytes) return it->second;
  if (c10::cuda::currentStreamCaptureStatusMayInitCtx() != c10::cuda::CaptureStatus::None) return at::Tensor();
  at::Tensor buf = at::zeros({static_cast<int64_t>(std::max<size_t>(bytes, 64 * 1024))},
                             at::TensorOptions().dtype(at::kByte).device(dev));
  if (it != g_zeroed.end()) g_zeroed_retired.push_back(it->second);
  g_zeroed[key] = buf;
  return buf;
}

void shape_error(const std::string& msg) { throw pybind11::value_error(msg); }

at::Tensor forward(const at::Tensor& x, const at::Tensor& wr, const at::Tensor& wi, const at::Tensor& wj,
                   const at::Tensor& wk, const c10::optional<at::Tensor>& bias_opt,
                   const c10::optional<at::Tensor>& lora_a_opt, const c10::optional<at::Tensor>& lora_b_opt,
                   double lora_scale, bool static_weights, const c10::optional<at::Tensor>& packed_opt) {
  // shapes first, as the reference validates them before touching devices
  const int64_t K = x.dim() > 0 ? x.size(-1) : 0;
  if (x.dim() == 0 || K % 4 != 0)
    shape_error("in_features must be divisible by 4 (quaternion packing), got " + std::to_string(K));
  const int64_t in_groups = K / 4;
  for (const at::Tensor* w : {&wr, &wi, &wj, &wk})
    if (w->dim() != 2) shape_error("weight components must be 2D [out_groups, in_groups]");
  if (wr.size(1) != in_groups)
    shape_error("weight in_groups (" + std::to_string(wr.size(1)) + ") must match input in_groups (" +
                std::to_string(in_groups) + ")");
  if (wr.sizes() != wi.sizes() || wr.sizes() != wj.sizes() || wr.sizes() != wk.sizes())
    shape_error("all four weight components must share the same shape");
  const int64_t out_groups = wr.size(0);
  const bool has_bias = bias_opt.has_value() && bias_opt->defined();
  if (has_bias && (bias_opt->dim() != 1 || bias_opt->size(0) != 4 * out_groups))
    shape_error("bias must be [" + std::to_string(4 * out_groups) + "]");
  const bool has_a = lora_a_opt.has_value() && lora_a_opt->defined();
  const bool has_b = lora_b_opt.has_value() && lora_b_opt->defined();
  if (has_a != has_b) shape_error("LoRA needs both A and B");
  int64_t rank = 0;
  if (has_a) {
    rank = lora_a_opt->size(0);
    if (lora_a_opt->dim() != 2 || lora_a_opt->size(1) != 4 * in_groups || lora_b_opt->dim() != 2 ||
        lora_b_opt->size(0) != 4 * out_groups || lora_b_opt->size(1) != rank)
      shape_error("LoRA shapes must be A [r, " + std::to_string(4 * in_groups) + "] and B [" +
                  std::to_string(4 * out_groups) + ", r]");
  }
  // devices and dtypes
  TORCH_CHECK(x.is_cuda(),
              "the B200 quaternion linear kernels require CUDA tensors (there is no CPU path); got a tensor on ",
              x.device());
  const int code = dtype_code(x.scalar_type());
  std::vector<const at::Tensor*> all = {&wr, &wi, &wj, &wk};
  if (has_bias) all.push_back(&*bias_opt);
  if (has_a) {
    all.push_back(&*lora_a_opt);
    all.push_back(&*lora_b_opt);
  }
  // the packed weight cache [out_groups, in_groups, 4] (the module's, or none)
  const bool has_packed = packed_opt.has_value() && packed_opt->defined();
  if (has_packed) {
    TORCH_CHECK(packed_opt->dim() == 3 && packed_opt->size(0) == out_groups && packed_opt->size(1) == in_groups &&
                    packed_opt->size(2) == 4 && packed_opt->is_contiguous(),
                "packed weights must be a contiguous [out_groups, in_groups, 4] tensor");
    all.push_back(&*packed_opt);
  }
  for (const at::Tensor* t : all) {
    TORCH_CHECK(t->is_cuda(),
                "the B200 quaternion linear kernels require CUDA tensors (there is no CPU path); got a tensor on ",
                t->device());
    TORCH_CHECK(t->device() == x.device(), "all tensors must be on one device, got ", x.device(), " and ",
                t->device());
    TORCH_CHECK(t->scalar_type() == x.scalar_type(), "all tensors must share one dtype, got ",
                x.scalar_type(), " and ", t->scalar_type());
  }
  // layouts: rows of x, K-major weights sharing one row stride
  at::Tensor x2 = x.is_contiguous() ? x.view({-1, K}) : x.reshape({-1, K}).contiguous();
  const int64_t M = x2.size(0);
  at::Tensor w[4] = {wr, wi, wj, wk};
  int64_t ld_w = in_groups;
  if (!(wr.is_contiguous() && wi.is_contiguous() && wj.is_contiguous() && wk.is_contiguous()))
    for (auto& t : w) t = t.contiguous();
  at::Tensor b = has_bias ? bias_opt->contiguous() : at::Tensor();
  at::Tensor la = has_a ? lora_a_opt->contiguous() : at::Tensor();
  at::Tensor lb = has_a ? lora_b_opt->contiguous() : at::Tensor();
  if (rank % 8 != 0 && code != QLIN_F32) {
    // zero-padding the rank to a multiple of 8 keeps the tensor-core path
    // (TMA rows of rank elements) and adds exact zeros
    const int64_t pad = 8 - rank % 8;
    la = at::cat({la, la.new_zeros({pad, la.size(1)})}, 0);
    lb = at::cat({lb, lb.new_zeros({lb.size(0), pad})}, 1).contiguous();
    rank += pad;
  }
  std::vector<int64_t> out_shape(x.sizes().begin(), x.sizes().end());
  out_shape.back() = 4 * out_groups;
  at::Tensor y = at::empty({M, 4 * out_groups}, x.options());
  if (M > 0) {
    c10::cuda::CUDAGuard guard(x.device());
    cudaStream_t stream = at::cuda::getCurrentCUDAStream(x.device().index()).stream();
    size_t ws_bytes = 0;
    int st = qlin_workspace_size(code, M, in_groups, out_groups, static_cast<int>(rank), &ws_bytes);
    TORCH_CHECK(st == QLIN_OK, "qlin_workspace_size: ", qlin_status_string(st));
    int flags = static_weights ? QLIN_FLAG_STATIC_WEIGHTS : 0;
    at::Tensor ws;
    if (ws_bytes > 0 && code != QLIN_F32 && M <= kZeroedMaxTokens) {
      ws = zeroed_workspace(x.device(), stream, ws_bytes);
      if (ws.defined()) flags |= QLIN_FLAG_ZEROED_WORKSPACE;
    }
    if (!ws.defined() && ws_bytes > 0)
      ws = at::empty({static_cast<int64_t>(ws_bytes)}, at::TensorOptions().dtype(at::kByte).device(x.device()));
    if (has_packed)
      st = qlin_forward_packed(code, x2.data_ptr(), x2.stride(0), packed_opt->data_ptr(), in_groups,
                               w[0].data_ptr(), w[1].data_ptr(), w[2].data_ptr(), w[3].data_ptr(), ld_w,
                               has_bias ? b.data_ptr() : nullptr, rank ? la.data_ptr() : nullptr,
                               rank ? lb.data_ptr() : nullptr, static_cast<int>(rank),
                               static_cast<float>(lora_scale), y.data_ptr(), 4 * out_groups, M, in_groups,
                               out_groups, ws.defined() ? ws.data_ptr() : nullptr, ws_bytes, flags, stream);
    else
      st = qlin_forward_ex(code, x2.data_ptr(), x2.stride(0), w[0].data_ptr(), w[1].data_ptr(), w[2].data_ptr(),
                           w[3].data_ptr(), ld_w, has_bias ? b.data_ptr() : nullptr, rank ? la.data_ptr() : nullptr,
                           rank ? lb.data_ptr() : nullptr, static_cast<int>(rank), static_cast<float>(lora_scale),
                           y.data_ptr(), 4 * out_groups, M, in_groups, out_groups,
                           ws.defined() ? ws.data_ptr() : nullptr, ws_bytes, QLIN_ALGO_AUTO, flags, stream);
    if (st == QLIN_ERR_SHAPE) shape_error(std::string("qlin_forward: ") + qlin_status_string(st));
    TORCH_CHECK(st == QLIN_OK, "qlin_forward: ", qlin_status_string(st), " (status ", st, ")");
  }
  return y.view(out_shape);
}

// The zero-filled decode workspaces currently cached (tests read their
// counter bytes).
std::vector<at::Tensor> workspaces() {
  std::lock_guard<std::mutex> lock(g_ws_mutex);
  std::vector<at::Tensor> out;
  for (auto& kv : g_zeroed) out.push_back(kv.second);
  return out;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("forward", &forward, "fused quaternion linear inference forward (see qlin_b200.h)", pybind11::arg("x"),
        pybind11::arg("wr"), pybind11::arg("wi"), pybind11::arg("wj"), pybind11::arg("wk"),
        pybind11::arg("bias") = pybind11::none(), pybind11::arg("lora_a") = pybind11::none(),
        pybind11::arg("lora_b") = pybind11::none(), pybind11::arg("lora_scale") = 0.0,
        pybind11::arg("static_weights") = false, pybind11::arg("packed") = pybind11::none());
  m.def("workspaces", &workspaces, "the cached zero-filled decode workspaces");
}
