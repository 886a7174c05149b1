// Dense dequantization, the standalone outlier correction, and the generic
// (any group size / row stride) fused GEMV used when the fast decode kernel's
// 16-byte layout conditions do not hold.
#include "common.cuh"

namespace ts {

// ---- dense reconstruction (triton_kernels.py:1003-1186) --------------------
// One thread per output element; values in fp32 (cb?[code]*scale + gmin as a
// multiply then an add, codec.py:789), rounded once to the output dtype.
__global__ void dequant_kernel(const QW q, void* out, int out_dtype, int64_t out_stride) {
  const int64_t n = q.rows * q.cols;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / q.cols, c = i - r * q.cols;
    const int code = load_code(q, r, c);
    const float v = q.codebook ? __ldg(q.codebook + code) : (float)code;
    const float2 sg = load_scale_gmin(q, r, c / q.group_size);
    store_f(out, out_dtype, r * out_stride + c, __fadd_rn(__fmul_rn(v, sg.x), sg.y));
  }
}

// Outlier positions get base + delta in fp32 (modules.py:912-919).
__global__ void dequant_outliers_kernel(const QW q, void* out, int out_dtype, int64_t out_stride) {
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < q.n_outliers;
       j += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = q.orow[j], c = q.ocol[j];
    const int code = load_code(q, r, c);
    const float v = q.codebook ? __ldg(q.codebook + code) : (float)code;
    const float2 sg = load_scale_gmin(q, r, c / q.group_size);
    const float base = __fadd_rn(__fmul_rn(v, sg.x), sg.y);
    store_f(out, out_dtype, r * out_stride + c, base + __half2float(q.odelta[j]));
  }
}

int run_dequant(const ts_qweight& w, void* out, int out_dtype, int64_t out_stride,
                int apply_outliers, cudaStream_t stream) {
  const QW q = make_qw(w);
  const int64_t n = w.rows * w.cols;
  if (n > 0) {
    const int blocks = (int)std::min<int64_t>((n + 255) / 256, (int64_t)sm_count() * 16);
    dequant_kernel<<<blocks, 256, 0, stream>>>(q, out, out_dtype, out_stride);
    TS_LAUNCH_CHECK();
  }
  if (apply_outliers && w.n_outliers > 0) {
    const int blocks = (int)std::min<int64_t>((w.n_outliers + 255) / 256, (int64_t)sm_count() * 4);
    dequant_outliers_kernel<<<blocks, 256, 0, stream>>>(q, out, out_dtype, out_stride);
    TS_LAUNCH_CHECK();
  }
  return TS_OK;
}

// ---- standalone outlier correction (triton_kernels.py:543-576) -------------
__global__ void outlier_atomic_kernel(float* out, int64_t M, int64_t out_stride, const void* x,
                                      int x_dtype, int64_t x_stride, const int32_t* row,
                                      const int32_t* col, const __half* delta, int64_t n) {
  const int64_t total = n * M;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / n, k = i - m * n;
    const float v = load_f(x, x_dtype, m * x_stride + col[k]) * __half2float(delta[k]);
    atomicAdd(out + m * out_stride + row[k], v);
  }
}

int run_outlier_atomic(float* out, int64_t M, int64_t out_stride, const void* x, int x_dtype,
                       int64_t x_stride, const int32_t* row, const int32_t* col,
                       const uint16_t* delta, int64_t n, cudaStream_t stream) {
  if (n == 0 || M == 0) return TS_OK;
  const int64_t total = n * M;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, (int64_t)sm_count() * 8);
  outlier_atomic_kernel<<<blocks, 256, 0, stream>>>(out, M, out_stride, x, x_dtype, x_stride, row, col,
                                                    reinterpret_cast<const __half*>(delta), n);
  TS_LAUNCH_CHECK();
  return TS_OK;
}

// ---- generic fused GEMV -----------------------------------------------------
// One warp per (row, token): lanes stride over columns in fp32. Slow but
// layout-agnostic (any group size, odd packed strides); the fast kernels cover
// every layout the reference's fused path accepts.
__global__ void generic_qlinear_kernel(const QW q, const void* x, int x_dtype, int64_t x_stride,
                                       int64_t M, const void* bias, int bias_dtype, void* out,
                                       int out_dtype, int64_t out_stride) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t t = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); t < q.rows * M;
       t += warps) {
    const int64_t row = t / M, m = t - row * M;
    float acc = 0.f;
    for (int64_t c = lane; c < q.cols; c += 32) {
      const int code = load_code(q, row, c);
      const float v = q.codebook ? __ldg(q.codebook + code) : (float)code;
      const float2 sg = load_scale_gmin(q, row, c / q.group_size);
      acc = fmaf(load_f(x, x_dtype, m * x_stride + c), __fadd_rn(__fmul_rn(v, sg.x), sg.y), acc);
    }
    if (q.n_outliers > 0) {
      const int o0 = q.orow_ptr[row], o1 = q.orow_ptr[row + 1];
      for (int j = o0 + lane; j < o1; j += 32)
        acc += load_f(x, x_dtype, m * x_stride + q.ocol[j]) * __half2float(q.odelta[j]);
    }
    acc = warp_sum(acc);
    if (lane == 0) {
      if (bias) acc += load_f(bias, bias_dtype, row);
      store_f(out, out_dtype, m * out_stride + row, acc);
    }
  }
}

int run_generic_qlinear(const ts_qweight& w, const void* x, int x_dtype, int64_t M,
                        int64_t x_stride, const void* bias, int bias_dtype, void* out,
                        int out_dtype, int64_t out_stride, cudaStream_t stream) {
  const int64_t work = w.rows * M;
  if (work == 0) return TS_OK;
  const int blocks = (int)std::min<int64_t>((work + 7) / 8, (int64_t)sm_count() * 8);
  generic_qlinear_kernel<<<blocks, 256, 0, stream>>>(make_qw(w), x, x_dtype, x_stride, M, bias,
                                                     bias_dtype, out, out_dtype, out_stride);
  TS_LAUNCH_CHECK();
  return TS_OK;
}

}  // namespace ts
