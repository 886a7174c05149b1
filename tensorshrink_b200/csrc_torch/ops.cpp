// torch.ops.tensorshrink.qlinear: the fused dequant-GEMM as a PyTorch
// operator over the C ABI of libtensorshrink_b200 (ts_qlinear).
//
// The reference's kernel seam is `fused_quantized_linear(x, packed, scale,
// gmin, bias, bits, group_size, cols, out_features, compute_dtype, ...)`
// (triton_kernels.py:714-739), called from QuantLinear.forward with kwargs
// prebuilt per device (modules.py:473-515). This operator takes the same
// QuantLinear buffers as tensors and runs on the current CUDA stream, so a
// module's forward is one dispatcher call: no Python-side workspace lookup,
// struct packing or ctypes marshalling per call. The decode workspace is a
// per-(device, stream) buffer from the caching allocator, zeroed once and
// grown when a call needs more (kernels leave it zeroed). A Meta
// implementation gives shapes to tracing.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <map>
#include <mutex>
#include <utility>

#include "tensorshrink_b200.h"

namespace {

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kHalf: return TS_F16;
    case at::kBFloat16: return TS_BF16;
    case at::kFloat: return TS_F32;
    default: TORCH_CHECK(false, "tensorshrink: unsupported dtype ", t);
  }
  return -1;
}

const void* ptr_or_null(const c10::optional<at::Tensor>& t) {
  return t.has_value() && t->defined() ? t->data_ptr() : nullptr;
}

void check_on(const c10::optional<at::Tensor>& t, const at::Device& dev, const char* name) {
  if (!t.has_value() || !t->defined()) return;
  TORCH_CHECK(t->device() == dev, "tensorshrink.qlinear: ", name, " is on ", t->device(), ", x on ", dev);
  TORCH_CHECK(t->is_contiguous(), "tensorshrink.qlinear: ", name, " must be contiguous");
}

std::mutex g_ws_mu;
std::map<std::pair<int, cudaStream_t>, at::Tensor> g_ws;

// The workspace of (device, stream), at least `bytes` long. Buffers are kept
// for the life of the process (a captured CUDA graph may still use one).
at::Tensor workspace(const at::Device& dev, cudaStream_t s, size_t bytes) {
  std::lock_guard<std::mutex> lk(g_ws_mu);
  auto& w = g_ws[{dev.index(), s}];
  if (!w.defined() || (size_t)w.numel() < bytes) {
    static std::vector<at::Tensor> keep;   // superseded buffers may live on in captured graphs
    if (w.defined()) keep.push_back(w);
    w = at::zeros({(int64_t)std::max<size_t>(bytes, 1 << 16)}, at::TensorOptions().dtype(at::kByte).device(dev));
  }
  return w;
}

at::Tensor qlinear_cuda(const at::Tensor& x, const at::Tensor& packed, const c10::optional<at::Tensor>& scale,
                        const c10::optional<at::Tensor>& gmin, const c10::optional<at::Tensor>& dq_scale_codes,
                        const c10::optional<at::Tensor>& dq_scale_meta, const c10::optional<at::Tensor>& dq_gmin_codes,
                        const c10::optional<at::Tensor>& dq_gmin_meta, const c10::optional<at::Tensor>& codebook,
                        const c10::optional<at::Tensor>& outlier_row_ptr,
                        const c10::optional<at::Tensor>& outlier_col,
                        const c10::optional<at::Tensor>& outlier_delta, const c10::optional<at::Tensor>& bias,
                        int64_t bits, int64_t group_size, int64_t cols, int64_t rows, int64_t n_groups,
                        int64_t dq_group_size, c10::optional<at::ScalarType> out_dtype) {
  TORCH_CHECK(x.is_cuda(), "tensorshrink.qlinear: x must be a CUDA tensor");
  const at::Device dev = x.device();
  c10::cuda::CUDAGuard guard(dev);
  TORCH_CHECK(packed.device() == dev && packed.is_contiguous() && packed.dim() == 2,
              "tensorshrink.qlinear: packed must be a contiguous 2-D tensor on x's device");
  check_on(scale, dev, "scale");
  check_on(gmin, dev, "gmin");
  check_on(dq_scale_codes, dev, "dq_scale_codes");
  check_on(dq_scale_meta, dev, "dq_scale_meta");
  check_on(dq_gmin_codes, dev, "dq_gmin_codes");
  check_on(dq_gmin_meta, dev, "dq_gmin_meta");
  check_on(codebook, dev, "codebook");
  check_on(outlier_row_ptr, dev, "outlier_row_ptr");
  check_on(outlier_col, dev, "outlier_col");
  check_on(outlier_delta, dev, "outlier_delta");
  check_on(bias, dev, "bias");
  TORCH_CHECK(x.size(-1) == cols, "tensorshrink.qlinear: x has ", x.size(-1), " features, the layer ", cols);
  at::Tensor x2d = x.reshape({-1, cols});
  if (!x2d.is_contiguous()) x2d = x2d.contiguous();
  const int64_t M = x2d.size(0);
  const at::ScalarType odt = out_dtype.value_or(x.scalar_type());
  std::vector<int64_t> oshape(x.sizes().begin(), x.sizes().end());
  oshape.back() = rows;
  at::Tensor out = at::empty({M, rows}, x.options().dtype(odt));
  if (M == 0) return out.reshape(oshape);

  const bool dq = ptr_or_null(dq_scale_codes) != nullptr;
  ts_qweight w{};
  w.rows = rows;
  w.cols = cols;
  w.n_groups = n_groups;
  w.padded_cols = n_groups * group_size;
  w.packed_row_bytes = packed.stride(0);
  w.bits = (int32_t)bits;
  w.group_size = (int32_t)group_size;
  w.packed = static_cast<const uint8_t*>(packed.data_ptr());
  w.scale = dq ? nullptr : static_cast<const uint16_t*>(ptr_or_null(scale));
  w.gmin = dq ? nullptr : static_cast<const uint16_t*>(ptr_or_null(gmin));
  w.dq_scale_codes = static_cast<const uint8_t*>(ptr_or_null(dq_scale_codes));
  w.dq_scale_meta = static_cast<const uint16_t*>(ptr_or_null(dq_scale_meta));
  w.dq_gmin_codes = static_cast<const uint8_t*>(ptr_or_null(dq_gmin_codes));
  w.dq_gmin_meta = static_cast<const uint16_t*>(ptr_or_null(dq_gmin_meta));
  w.dq_group_size = dq ? (int32_t)dq_group_size : 0;
  w.codebook = static_cast<const float*>(ptr_or_null(codebook));
  const int64_t n_out = outlier_delta.has_value() && outlier_delta->defined() ? outlier_delta->numel() : 0;
  w.n_outliers = n_out;
  if (n_out) {
    w.outlier_row_ptr = static_cast<const int32_t*>(ptr_or_null(outlier_row_ptr));
    w.outlier_col = static_cast<const int32_t*>(ptr_or_null(outlier_col));
    w.outlier_delta = static_cast<const uint16_t*>(ptr_or_null(outlier_delta));
  }
  cudaStream_t s = at::cuda::getCurrentCUDAStream(dev.index()).stream();
  at::Tensor ws = workspace(dev, s, ts_qlinear_workspace_size(&w, M));
  const int bdt = bias.has_value() && bias->defined() ? dtype_code(bias->scalar_type()) : 0;
  const int rc = ts_qlinear(&w, x2d.data_ptr(), dtype_code(x2d.scalar_type()), M, x2d.stride(0),
                            ptr_or_null(bias), bdt, out.data_ptr(), dtype_code(odt), out.stride(0), ws.data_ptr(),
                            (size_t)ws.numel(), s);
  TORCH_CHECK(rc == 0, "tensorshrink.qlinear: ", ts_last_error());
  return out.reshape(oshape);
}

at::Tensor qlinear_meta(const at::Tensor& x, const at::Tensor& packed, const c10::optional<at::Tensor>&,
                        const c10::optional<at::Tensor>&, const c10::optional<at::Tensor>&,
                        const c10::optional<at::Tensor>&, const c10::optional<at::Tensor>&,
                        const c10::optional<at::Tensor>&, const c10::optional<at::Tensor>&,
                        const c10::optional<at::Tensor>&, const c10::optional<at::Tensor>&,
                        const c10::optional<at::Tensor>&, const c10::optional<at::Tensor>&, int64_t, int64_t,
                        int64_t, int64_t rows, int64_t, int64_t, c10::optional<at::ScalarType> out_dtype) {
  std::vector<int64_t> oshape(x.sizes().begin(), x.sizes().end());
  oshape.back() = rows;
  return at::empty(oshape, x.options().dtype(out_dtype.value_or(x.scalar_type())));
}

// ts_qlinear_status over every workspace of `device` this operator made:
// raises if a bounded wait in a kernel ran out since the last check.
void device_status(int64_t device, bool clear) {
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  cudaStream_t s = at::cuda::getCurrentCUDAStream((c10::DeviceIndex)device).stream();
  std::vector<at::Tensor> bufs;
  {
    std::lock_guard<std::mutex> lk(g_ws_mu);
    for (auto& kv : g_ws)
      if (kv.first.first == device) bufs.push_back(kv.second);
  }
  for (auto& b : bufs) {
    const int rc = ts_qlinear_status(b.data_ptr(), (size_t)b.numel(), clear ? 1 : 0, s);
    TORCH_CHECK(rc == 0, "tensorshrink: ", ts_last_error());
  }
}

}  // namespace

TORCH_LIBRARY(tensorshrink, m) {
  m.def("device_status(int device, bool clear=True) -> ()", &device_status);
  m.def(
      "qlinear(Tensor x, Tensor packed, Tensor? scale, Tensor? gmin, Tensor? dq_scale_codes, "
      "Tensor? dq_scale_meta, Tensor? dq_gmin_codes, Tensor? dq_gmin_meta, Tensor? codebook, "
      "Tensor? outlier_row_ptr, Tensor? outlier_col, Tensor? outlier_delta, Tensor? bias, int bits, "
      "int group_size, int cols, int rows, int n_groups, int dq_group_size, ScalarType? out_dtype=None) -> Tensor");
}

TORCH_LIBRARY_IMPL(tensorshrink, CUDA, m) { m.impl("qlinear", &qlinear_cuda); }
TORCH_LIBRARY_IMPL(tensorshrink, Meta, m) { m.impl("qlinear", &qlinear_meta); }
