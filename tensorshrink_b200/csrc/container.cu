// Outlier tables of a container entry, built on the device.
//
// The reference container stores a weight's outliers row-sorted as
// (row delta, column, value) with 16- or 32-bit unsigned indices
// (container.py:98-153 `_encode_outliers` / `_decode_outliers`); QuantLinear
// needs int32 row/column tables, CSR row offsets and fp16 deltas against the
// group-affine reconstruction (modules.py:414-448, 649-715). One block scans
// the row deltas (inclusive prefix sum, 1024 entries per pass); a grid pass
// then writes the CSR offsets and the deltas
//   delta = f16(f32(value) - (cb?[code] * scale + gmin)),
// a separately rounded multiply and add in fp32 with the double-quant
// scale/min reconstructed in fp32 as QuantLinear does.
#include <algorithm>

#include "common.cuh"

namespace ts {
namespace ctr {

constexpr int kScanThreads = 1024;

template <typename IDX>
__global__ void __launch_bounds__(kScanThreads) row_scan_kernel(const IDX* row_delta, const IDX* col, int64_t n,
                                                                int32_t* row, int32_t* col_out) {
  __shared__ int64_t warp_sums[kScanThreads / 32];
  __shared__ int64_t carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t base = 0; base < n; base += kScanThreads) {
    const int64_t i = base + threadIdx.x;
    int64_t v = i < n ? (int64_t)row_delta[i] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t t = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += t;
    }
    if (lane == 31) warp_sums[warp] = v;
    __syncthreads();
    if (warp == 0) {
      int64_t s = warp_sums[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int64_t t = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += t;
      }
      warp_sums[lane] = s;
    }
    __syncthreads();
    const int64_t incl = v + (warp > 0 ? warp_sums[warp - 1] : 0) + carry;
    if (i < n) {
      row[i] = (int32_t)incl;
      col_out[i] = (int32_t)col[i];
    }
    __syncthreads();
    if (threadIdx.x == kScanThreads - 1) carry = incl;
    __syncthreads();
  }
}

__global__ void tables_kernel(const QW q, const int32_t* row, const int32_t* col, const uint16_t* val, int64_t n,
                              uint16_t* delta, int32_t* row_ptr, int* bad) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    const int r = row[i], c = col[i];
    const int prev = i > 0 ? row[i - 1] : -1;
    if (r < 0 || r >= q.rows || c < 0 || c >= q.cols || r < prev) {
      atomicExch(bad, 1);
      continue;
    }
    for (int k = prev + 1; k <= r; ++k) row_ptr[k] = (int32_t)i;   // rows (prev, r] start here
    const int code = load_code(q, r, c);
    const float v = q.codebook ? q.codebook[code] : (float)code;
    const float2 sg = load_scale_gmin(q, r, c / q.group_size);
    const float base = __fadd_rn(__fmul_rn(v, sg.x), sg.y);
    delta[i] = f2h(__fsub_rn(h2f(val[i]), base));
  }
  // rows after the last outlier
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int last = n > 0 ? row[n - 1] : -1;
  for (int64_t k = last + 1 + t; k <= q.rows; k += stride) row_ptr[k] = (int32_t)n;
}

}  // namespace ctr
}  // namespace ts

using namespace ts;

extern "C" int ts_outlier_tables_from_stream(const ts_qweight* w, const void* row_delta, const void* col,
                                             int index_bytes, const uint16_t* val, int64_t n, int32_t* row_out,
                                             int32_t* col_out, uint16_t* delta_out, int32_t* row_ptr_out,
                                             int* bad_flag, void* stream) {
  TS_REQUIRE(w != nullptr && row_ptr_out != nullptr && bad_flag != nullptr, "NULL pointer");
  TS_REQUIRE(index_bytes == 2 || index_bytes == 4, "index_bytes must be 2 or 4");
  TS_REQUIRE(n >= 0 && n < (int64_t(1) << 31), "bad outlier count");
  TS_REQUIRE(n == 0 || (row_delta && col && val && row_out && col_out && delta_out), "NULL outlier pointer");
  TS_REQUIRE(w->bits == 2 || w->bits == 4 || w->bits == 8, "bits must be 2, 4 or 8");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const QW q = make_qw(*w);
  TS_CUDA_TRY(cudaMemsetAsync(bad_flag, 0, sizeof(int), st));
  if (n > 0) {
    if (index_bytes == 2)
      ctr::row_scan_kernel<uint16_t><<<1, ctr::kScanThreads, 0, st>>>(
          reinterpret_cast<const uint16_t*>(row_delta), reinterpret_cast<const uint16_t*>(col), n, row_out, col_out);
    else
      ctr::row_scan_kernel<uint32_t><<<1, ctr::kScanThreads, 0, st>>>(
          reinterpret_cast<const uint32_t*>(row_delta), reinterpret_cast<const uint32_t*>(col), n, row_out, col_out);
    TS_LAUNCH_CHECK();
  }
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)sm_count() * 4));
  ctr::tables_kernel<<<blocks, 256, 0, st>>>(q, row_out, col_out, val, n, delta_out, row_ptr_out, bad_flag);
  TS_LAUNCH_CHECK();
  return TS_OK;
}
