// Shared device/host helpers for the tensorshrink_b200 kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "tensorshrink_b200.h"

namespace ts {

// ---- error reporting (thread-local message, see ts_last_error) -------------
void set_error(const char* fmt, ...);
void count_launch(int n = 1);

#define TS_REQUIRE(cond, ...)            \
  do {                                   \
    if (!(cond)) {                       \
      ::ts::set_error(__VA_ARGS__);      \
      return TS_ERR_INVALID;             \
    }                                    \
  } while (0)

#define TS_UNSUPPORTED(cond, ...)        \
  do {                                   \
    if (!(cond)) {                       \
      ::ts::set_error(__VA_ARGS__);      \
      return TS_ERR_UNSUPPORTED;         \
    }                                    \
  } while (0)

#define TS_CUDA_TRY(expr)                                                        \
  do {                                                                           \
    cudaError_t _e = (expr);                                                     \
    if (_e != cudaSuccess) {                                                     \
      ::ts::set_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e),  \
                      __FILE__, __LINE__);                                       \
      return TS_ERR_CUDA;                                                        \
    }                                                                            \
  } while (0)

// Checks the launch that was just issued (configuration errors only; the
// kernel itself runs asynchronously).
#define TS_LAUNCH_CHECK()                                                        \
  do {                                                                           \
    cudaError_t _e = cudaGetLastError();                                         \
    if (_e != cudaSuccess) {                                                     \
      ::ts::set_error("kernel launch failed: %s (%s:%d)", cudaGetErrorString(_e), \
                      __FILE__, __LINE__);                                       \
      return TS_ERR_CUDA;                                                        \
    }                                                                            \
    ::ts::count_launch();                                                        \
  } while (0)

int sm_count();            // SMs of the current device (cached per device)
// Limit of every bounded barrier wait in the kernels (2 s unless a test
// stall asked for less), and whether the next launch is a test stall (its
// copy producer issues nothing, so the first waits run out; see
// ts_test_inject_stall). take_test_stall() consumes the request.
uint64_t wait_limit_ns();
bool take_test_stall();
int max_smem_optin();      // opt-in shared memory per block of the current device

inline bool is_aligned(const void* p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// ---- dtype helpers ---------------------------------------------------------
__device__ __forceinline__ float load_f(const void* p, int dtype, int64_t i) {
  if (dtype == TS_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  if (dtype == TS_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

// the same through L2 only (data another CTA of the running kernel wrote)
__device__ __forceinline__ float load_f_cg(const void* p, int dtype, int64_t i) {
  if (dtype == TS_F16) return __half2float(__ushort_as_half(__ldcg(reinterpret_cast<const unsigned short*>(p) + i)));
  if (dtype == TS_BF16) return __uint_as_float((uint32_t)__ldcg(reinterpret_cast<const unsigned short*>(p) + i) << 16);
  return __ldcg(reinterpret_cast<const float*>(p) + i);
}

__device__ __forceinline__ void store_f(void* p, int dtype, int64_t i, float v) {
  if (dtype == TS_F16)
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else if (dtype == TS_BF16)
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<float*>(p)[i] = v;
}

__device__ __forceinline__ float h2f(uint16_t bits) {
  return __half2float(__ushort_as_half(bits));
}

__device__ __forceinline__ uint16_t f2h(float v) {
  return __half_as_ushort(__float2half_rn(v));
}

// Streaming 16-byte load of weights that are read exactly once per call:
// skip L1 and ask L2 to prefetch the neighbouring 256-byte sector group.
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue, and wait for the previous kernel's results before reading them.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_primary() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Decoded view of ts_qweight used by device code.
// One decode-kernel layer call: y = W x (+ bias) (+ residual), x optionally
// staged as silu(gate) * up of a [gate | up] row (gated) or as the RMSNorm of
// an fp32 row (norm_w), rounded to act_dtype.
struct GemvOp {
  const ts_qweight* w;
  const void* x;
  int x_dtype;
  int64_t x_stride;
  const void* bias;
  int bias_dtype;
  void* out;
  int out_dtype;
  int64_t out_stride;
  int gated;
  const float* norm_w;
  float norm_eps;
  int act_dtype;
  const float* residual;
  int64_t residual_stride;
};

struct QW {
  const uint8_t* packed;
  const __half* scale;
  const __half* gmin;
  const uint8_t* dqs_codes;
  const __half2* dqs_meta;
  const uint8_t* dqg_codes;
  const __half2* dqg_meta;
  const float* codebook;
  const int32_t* orow_ptr;
  const int32_t* orow;
  const int32_t* ocol;
  const __half* odelta;
  int64_t rows, cols, padded_cols, n_groups, row_bytes, n_outliers;
  int bits, group_size, dq_gs;
};

inline QW make_qw(const ts_qweight& w) {
  QW q;
  q.packed = w.packed;
  q.scale = reinterpret_cast<const __half*>(w.scale);
  q.gmin = reinterpret_cast<const __half*>(w.gmin);
  q.dqs_codes = w.dq_scale_codes;
  q.dqs_meta = reinterpret_cast<const __half2*>(w.dq_scale_meta);
  q.dqg_codes = w.dq_gmin_codes;
  q.dqg_meta = reinterpret_cast<const __half2*>(w.dq_gmin_meta);
  q.codebook = w.codebook;
  q.orow_ptr = w.outlier_row_ptr;
  q.orow = w.outlier_row;
  q.ocol = w.outlier_col;
  q.odelta = reinterpret_cast<const __half*>(w.outlier_delta);
  q.rows = w.rows;
  q.cols = w.cols;
  q.padded_cols = w.padded_cols;
  q.n_groups = w.n_groups;
  q.row_bytes = w.packed_row_bytes;
  q.n_outliers = w.n_outliers;
  q.bits = w.bits;
  q.group_size = w.group_size;
  q.dq_gs = w.dq_group_size;
  return q;
}

// fp32 (scale, gmin) of (row, group): plain fp16 metadata, or the
// double-quantized reconstruction code * meta_scale + meta_min evaluated as a
// separately rounded multiply and add (modules.py:573-580).
__device__ __forceinline__ float2 load_scale_gmin(const QW& q, int64_t row, int64_t g) {
  const int64_t flat = row * q.n_groups + g;
  if (q.dqs_codes != nullptr) {
    const int64_t sup = flat / q.dq_gs;
    const float2 ms = __half22float2(q.dqs_meta[sup]);
    const float2 mg = __half22float2(q.dqg_meta[sup]);
    const float s = __fadd_rn(__fmul_rn((float)q.dqs_codes[flat], ms.x), ms.y);
    const float m = __fadd_rn(__fmul_rn((float)q.dqg_codes[flat], mg.x), mg.y);
    return make_float2(s, m);
  }
  return make_float2(__half2float(q.scale[flat]), __half2float(q.gmin[flat]));
}

// Code of element (row, col) from the packed layout.
__device__ __forceinline__ int load_code(const QW& q, int64_t row, int64_t col) {
  const uint8_t* p = q.packed + row * q.row_bytes;
  if (q.bits == 4) return (p[col >> 1] >> ((col & 1) * 4)) & 0xF;
  if (q.bits == 2) return (p[col >> 2] >> ((col & 3) * 2)) & 0x3;
  return p[col];
}

}  // namespace ts
