/*
 * tensorshrink_b200 — C ABI of the B200 (sm_100a) QuantLinear hot path.
 *
 * Plain pointers and sizes only: every pointer argument named "device" is a
 * CUDA device address on the current device, and `stream` is a cudaStream_t
 * passed as void* (NULL = legacy default stream). No entry point allocates
 * device memory; scratch comes from caller-provided workspaces whose sizes
 * the *_workspace_size() functions report. All launches are asynchronous on
 * `stream`. Functions return TS_OK (0) or a negative ts_status; the message
 * of the last failure on the calling thread is in ts_last_error().
 *
 * Packed-weight layout is the reference's `QuantLinear` buffer layout,
 * unchanged (tensorshrink codec.py:102-151, modules.py:337-448):
 *   packed   uint8 [rows, padded_cols*bits/8]; 4-bit: byte = c[2j] | c[2j+1]<<4;
 *            2-bit: byte = c[4j] | c[4j+1]<<2 | c[4j+2]<<4 | c[4j+3]<<6; 8-bit raw.
 *   scale/gmin fp16 [rows, n_groups]   (or the double-quantized form:
 *   dq_*_codes uint8 flattened row-major over [rows, n_groups], one
 *   (meta_scale, meta_min) fp16 pair per dq_group_size entries).
 *   codebook fp32 [1<<bits] (NF / Lloyd-Max levels) or NULL.
 *   outliers: row-sorted int32 row/col, fp16 delta, plus CSR row offsets.
 * Reconstruction: w[r,c] = cb?[code] * scale[r,g] + gmin[r,g] (+ delta at
 * outlier positions), g = c / group_size.
 */
#ifndef TENSORSHRINK_B200_H
#define TENSORSHRINK_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TS_API __attribute__((visibility("default")))
#else
#define TS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum ts_dtype {
  TS_F16 = 0,
  TS_BF16 = 1,
  TS_F32 = 2
} ts_dtype;

typedef enum ts_status {
  TS_OK = 0,
  TS_ERR_INVALID = -1,     /* bad argument (shape, pointer, alignment) */
  TS_ERR_UNSUPPORTED = -2, /* valid but not covered (bit width, dtype) */
  TS_ERR_CUDA = -3,        /* a CUDA runtime call failed */
  TS_ERR_WORKSPACE = -4,   /* workspace missing or too small */
  TS_ERR_TIMEOUT = -5      /* a bounded wait in a kernel ran out (ts_qlinear_status) */
} ts_status;

/* One quantized weight matrix as resident on the device (QuantLinear's
 * buffers). Exactly one of {scale,gmin} / {dq_*} is set. */
typedef struct ts_qweight {
  int64_t rows;             /* out_features (N) */
  int64_t cols;             /* in_features (K), unpadded */
  int64_t padded_cols;      /* cols rounded up to a multiple of group_size */
  int64_t n_groups;         /* padded_cols / group_size */
  int64_t packed_row_bytes; /* row stride of `packed` in bytes */
  int32_t bits;             /* 2, 4 or 8 */
  int32_t group_size;
  const uint8_t* packed;
  const uint16_t* scale;    /* fp16 [rows, n_groups] or NULL */
  const uint16_t* gmin;     /* fp16 [rows, n_groups] or NULL */
  const uint8_t* dq_scale_codes;
  const uint16_t* dq_scale_meta; /* fp16 [n_super, 2] */
  const uint8_t* dq_gmin_codes;
  const uint16_t* dq_gmin_meta;
  int32_t dq_group_size;
  int32_t reserved0;
  const float* codebook;    /* fp32 [1<<bits] or NULL */
  int64_t n_outliers;
  const int32_t* outlier_row_ptr; /* [rows+1] CSR offsets into the tables */
  const int32_t* outlier_row;     /* row-sorted */
  const int32_t* outlier_col;
  const uint16_t* outlier_delta;  /* fp16 */
} ts_qweight;

/* ---------------------------------------------------------------------------
 * Fused dequant-GEMM:  out[M, rows] = x[M, cols] . W^T (+ outliers) (+ bias)
 *
 * Replaces triton_kernels.py:714-945 `fused_quantized_linear` (and, for
 * M > 64, the modules.py:898-922 dequantize_weight + F.linear path). Same
 * arguments in the same meaning; the output is written directly in
 * `out_dtype` (fp16, bf16 or fp32) instead of an fp32 pool buffer plus a
 * cast, and outliers are folded into the kernel's epilogue through the CSR
 * row offsets instead of an atomic post-pass.
 * x: device [M, cols] rows `x_row_stride` elements apart, fp16 or bf16.
 * bias: device [rows] in `bias_dtype`, or NULL. out: device [M, rows].
 * workspace: device memory of ts_qlinear_workspace_size() bytes, zero-filled
 * before its first use; calls leave it zeroed again. Calls that run
 * concurrently must use distinct workspaces.
 */
TS_API size_t ts_qlinear_workspace_size(const ts_qweight* w, int64_t M);

TS_API int ts_qlinear(const ts_qweight* w, const void* x, int x_dtype, int64_t M,
               int64_t x_row_stride, const void* bias, int bias_dtype, void* out,
               int out_dtype, int64_t out_row_stride, void* workspace,
               size_t workspace_bytes, void* stream);

/*
 * Gated MLP projection: out = (silu(gate) * up) . W^T (+ outliers)(+ bias),
 * with gate_up [M, 2 * cols] holding gate in columns [0, cols) and up in
 * [cols, 2 cols) (the output of a fused gate/up projection). silu(gate) and
 * the product are rounded to x_dtype as the unfused F.silu(gate) * up
 * rounds them. Decode-sized calls only (the decode kernel computes the
 * product while staging the activations): TS_ERR_UNSUPPORTED otherwise,
 * and the caller runs the product and ts_qlinear. Replaces the
 * `F.silu(gate) * up` elementwise pass in front of the reference's down
 * projection (the reference has no fused form). Workspace as ts_qlinear.
 */
TS_API int ts_qlinear_gated(const ts_qweight* w, const void* gate_up, int x_dtype, int64_t M,
               int64_t x_row_stride, const void* bias, int bias_dtype, void* out,
               int out_dtype, int64_t out_row_stride, void* workspace,
               size_t workspace_bytes, void* stream);

/*
 * One layer of a fused decode call. The reference runs each of these as a
 * QuantLinear.forward (modules.py:819-940) between plain torch ops of its
 * model (RMSNorm in front, the residual add behind); here they are folded
 * into the decode kernel:
 *   flags & TS_OP_GATED:   x rows hold [gate | up] (2 * cols): the input is
 *                          silu(gate) * up (as ts_qlinear_gated);
 *   flags & TS_OP_RMSNORM: x rows are fp32 (x_dtype TS_F32): the input is
 *                          F.rms_norm(x, norm_weight, norm_eps) rounded to
 *                          act_dtype, each token's mean square reduced in the
 *                          kernel;
 *   residual != NULL:      fp32 [M, rows] added to the result (may alias out).
 * act_dtype: the activation dtype the staged input is rounded to (fp16/bf16;
 * x_dtype for plain 16-bit inputs).
 */
#define TS_OP_GATED 1
#define TS_OP_RMSNORM 2
typedef struct ts_qlinear_op {
  const ts_qweight* w;
  const void* x;
  int64_t x_row_stride;
  int32_t x_dtype;
  int32_t flags;
  const void* bias;
  int32_t bias_dtype;
  int32_t out_dtype;
  void* out;
  int64_t out_row_stride;
  const float* norm_weight;
  float norm_eps;
  int32_t act_dtype;
  const float* residual;
  int64_t residual_row_stride;
} ts_qlinear_op;

/*
 * One fused layer call (decode-sized M; TS_ERR_UNSUPPORTED for calls the
 * decode kernel does not take: then run the unfused ops and ts_qlinear).
 * A call with no flags and no residual is ts_qlinear. Workspace as ts_qlinear.
 */
TS_API int ts_qlinear_ex(const ts_qlinear_op* op, int64_t M, void* workspace, size_t workspace_bytes,
                         void* stream);

/*
 * A chain of n_ops layers where op i + 1 reads what op i wrote (an MLP:
 * gate_up then the gated down projection; or consecutive blocks). Results
 * equal n_ops ts_qlinear_ex calls in stream order; every op is validated
 * before any runs. persistent = 0: one decode launch per layer (each starts
 * streaming its weights while the previous one finishes, by programmatic
 * dependent launch). persistent != 0, when every layer takes the decode
 * kernel in one pass with the same code layout (bits, group size, codebook,
 * double quant) and n_ops <= ts_qlinear_chain_max(): ONE launch, in which
 * layer i + 1 waits (bounded) on a grid-wide counter for layer i while the
 * weight tiles of the following layers already stream into shared memory.
 * The workspace must cover ts_qlinear_workspace_size() of every layer.
 */
TS_API int ts_qlinear_chain(const ts_qlinear_op* ops, int n_ops, int64_t M, int persistent, void* workspace,
                            size_t workspace_bytes, void* stream);
TS_API int ts_qlinear_chain_max(void);

/*
 * Allocation-free variant of ts_qlinear (no counterpart in the reference):
 * same arguments minus the workspace. The decode kernel's scratch lives in a
 * fixed per-device array of ts_qlinear_noalloc_max_scratch() bytes (512 KiB)
 * inside the library, for callers that cannot allocate device memory. A
 * call that takes the decode kernel (fewer than 65 tokens, or a layout the
 * tensor-core kernel does not cover) with a weight whose
 * ts_qlinear_workspace_size() exceeds that returns TS_ERR_UNSUPPORTED. The
 * first call on each device loads the array there and must happen before
 * any stream capture. Calls that may overlap on one device race on the
 * shared array and must be serialized.
 */
TS_API size_t ts_qlinear_noalloc_max_scratch(void);

TS_API int ts_qlinear_noalloc(const ts_qweight* w, const void* x, int x_dtype, int64_t M,
               int64_t x_row_stride, const void* bias, int bias_dtype, void* out,
               int out_dtype, int64_t out_row_stride, void* stream);

/*
 * Device error status of the qlinear kernels. Every barrier wait inside the
 * kernels is bounded (2 s); a wait that runs out makes the kernel unwind
 * (its results are then invalid) and records a code in the workspace's flag
 * (decode kernel) or in a per-device flag (tensor-core kernel). This call
 * synchronizes `stream`, reads both flags and returns TS_OK when neither is
 * set, else TS_ERR_TIMEOUT with the codes in ts_last_error(). With
 * clear != 0 it also resets the flags and the workspace's row-block
 * counters, so the workspace is usable again. workspace == NULL checks the
 * ts_qlinear_noalloc scratch array instead. No counterpart in the reference
 * (its Triton kernels have no waits).
 */
TS_API int ts_qlinear_status(void* workspace, size_t workspace_bytes, int clear, void* stream);

/* Test hook: the next qlinear kernel launch on the calling thread runs with
 * its copy producer disabled and every barrier wait limited to
 * `wait_limit_ns` (at most 2 s), so its first waits run out and the kernel
 * reports TS_ERR_TIMEOUT through ts_qlinear_status. Nothing faults or hangs:
 * the kernel returns within a few wait limits. */
TS_API int ts_test_inject_stall(uint64_t wait_limit_ns);

/* Standalone outlier correction into an fp32 result:
 *   out[m, row[k]] += x[m, col[k]] * delta[k]   for every k (any order).
 * Replaces triton_kernels.py:948-991 `apply_outlier_correction` (the path the
 * reference takes for unsorted or very large outlier tables). */
TS_API int ts_apply_outlier_correction(float* out, int64_t M, int64_t N, int64_t out_row_stride,
                                const void* x, int x_dtype, int64_t x_row_stride,
                                const int32_t* row, const int32_t* col,
                                const uint16_t* delta, int64_t n_outliers, void* stream);

/* QuantLinear outlier tables from a container's outlier stream.
 * Replaces the host decode of container.py:142-153 `_decode_outliers` plus
 * the table build of modules.py:414-448, 649-715. Inputs: the weight
 * (packed codes and metadata set; outlier fields ignored) and the stream as
 * stored: row deltas and columns as unsigned 16- or 32-bit integers
 * (index_bytes), values fp16, n entries, rows non-decreasing. Outputs
 * (device): int32 rows (prefix sums of the deltas) and columns, fp16 deltas
 * f16(value - (cb?[code] * scale + gmin)) in fp32 with the double-quant
 * metadata reconstructed in fp32, and CSR offsets row_ptr[rows + 1].
 * *bad_flag (device int) is set to 1 when an entry lies outside the weight. */
TS_API int ts_outlier_tables_from_stream(const ts_qweight* w, const void* row_delta, const void* col,
                                         int index_bytes, const uint16_t* val, int64_t n, int32_t* row_out,
                                         int32_t* col_out, uint16_t* delta_out, int32_t* row_ptr_out,
                                         int* bad_flag, void* stream);

/* ---------------------------------------------------------------------------
 * One-shot all-reduce over NVLink peer memory for tensor-parallel layers.
 * Replaces, for the row-parallel partial sums, the torch.distributed
 * all_reduce the reference's multi-GPU path would use (the reference itself
 * has no tensor parallelism; its layers run on one device).
 * Each rank allocates one exchange buffer (ts_peer_alloc, zeroed; bytes from
 * ts_peer_buffer_bytes), shares its CUDA IPC handle (ts_ipc_get_handle, 64
 * bytes) and maps the others (ts_ipc_open). ts_allreduce_oneshot then sums
 * `n` floats of `in` over the ranks (rank order, identical on every rank)
 * plus an optional `residual`, into `out` (which may alias either). Every
 * rank must make the same sequence of calls with the same n; n <= cap.
 * Waits for peers are bounded (2 s); on expiry *err_flag (device int) is
 * set to a non-zero code and the output is invalid.
 */
TS_API size_t ts_peer_buffer_bytes(int world, int64_t cap);
TS_API int ts_peer_alloc(int world, int64_t cap, void** ptr);
TS_API int ts_peer_free(void* ptr);
TS_API int ts_ipc_get_handle(void* ptr, void* handle_out);
TS_API int ts_ipc_open(const void* handle, void** ptr);
TS_API int ts_ipc_close(void* ptr);
TS_API int ts_allreduce_oneshot(void* const* peer_bufs, int rank, int world, int64_t cap, const float* in,
                                const float* residual, float* out, int64_t n, int* err_flag, void* stream);

/*
 * Decode-step attention of the Llama-shaped decoder used to measure decode
 * tok/s (no counterpart in the reference, whose models keep their own
 * attention): for each of `batch` sequences, rotary embedding of the new q
 * and k (rope_cos / rope_sin: fp32 [max_seq, head_dim / 2]), append of k and
 * v to the bf16 caches at position *pos (device int64), and grouped-query
 * attention over cache positions [0, min(attn_len, *pos + 1)).
 * qkv: bf16 [batch, (n_q + 2 n_kv) head_dim] (q heads, then k, then v);
 * caches: bf16 [batch][n_kv][max_seq][head_dim] with the given element
 * strides; out: bf16 [batch, n_q head_dim].
 */
TS_API int ts_decode_attention(const void* qkv, int64_t qkv_row_stride, int batch, int n_q, int n_kv,
                               int head_dim, const int64_t* pos, const float* rope_cos, const float* rope_sin,
                               void* k_cache, void* v_cache, int64_t cache_batch_stride,
                               int64_t cache_head_stride, int attn_len, int max_seq, void* out,
                               int64_t out_row_stride, void* stream);

/* Dense reconstruction W[rows, cols] in `out_dtype`.
 * Replaces triton_kernels.py:1114-1186 `dequantize_weight` (which covers only
 * 4/8-bit; this covers 2/4/8 and the double-quantized metadata). With
 * apply_outliers != 0 the outlier positions get base + delta, computed in
 * fp32, as modules.py:912-919 does before its F.linear. */
TS_API int ts_dequantize_weight(const ts_qweight* w, void* out, int out_dtype, int64_t out_row_stride,
                         int apply_outliers, void* stream);

/* ---------------------------------------------------------------------------
 * GPU quantize + pack (GOAP), replacing gpu_quantize.py:52-166
 * `quantize_tensor_gpu` and the tensor work of codec.py:453-675
 * `quantize_tensor`: top-k |w| outlier extraction and clamp, per-group affine
 * parameters, uniform / codebook / Lloyd-Max code assignment, bit packing,
 * double quantization of scale/gmin, and QuantLinear's row-sorted outlier
 * tables with their fp16 deltas (modules.py:414-448, 649-715).
 * Bit-identical to the reference codec on the same input, except that ties
 * at the top-k threshold keep the lowest flat indices.
 */
typedef enum ts_qmode {
  TS_QMODE_UNIFORM = 0,  /* round-half-even on the integer grid */
  TS_QMODE_CODEBOOK = 1, /* nearest entry of a given sorted fp32 codebook (NF) */
  TS_QMODE_LLOYD = 2     /* fit a Lloyd-Max codebook on the device, then assign */
} ts_qmode;

typedef struct ts_quant_params {
  int64_t rows, cols;
  int32_t bits, group_size;
  int64_t k_outliers;        /* codec.py:530: max(1, int(n*frac)) or 0 */
  int32_t double_quant;      /* 0/1 */
  int32_t dq_group_size;
  int32_t mode;              /* ts_qmode */
  int32_t lloyd_iters;       /* codec.py:258 default 12 */
  const float* codebook;     /* device fp32 [1<<bits], sorted (TS_QMODE_CODEBOOK) */
  const int64_t* lloyd_sample; /* device flat indices into the padded
                                  [rows, padded_cols] grid, or NULL = all */
  int64_t lloyd_n_sample;
} ts_quant_params;

typedef struct ts_quant_outputs {
  uint8_t* packed;           /* [rows, padded_cols*bits/8] */
  uint16_t* scale;           /* fp16 [rows, n_groups]; DQ-reconstructed when double_quant */
  uint16_t* gmin;
  uint8_t* dq_scale_codes;   /* [n_super*dq_group_size] (double_quant only) */
  uint16_t* dq_scale_meta;   /* fp16 [n_super, 2] */
  uint8_t* dq_gmin_codes;
  uint16_t* dq_gmin_meta;
  float* codebook_out;       /* fp32 [1<<bits]: levels the codes were assigned
                                against (Lloyd: the fitted levels), or NULL */
  uint16_t* codebook_f16;    /* fp16 [1<<bits] stored codebook (Lloyd-Max: required;
                                codebook mode: optional, and when given the
                                outlier deltas are taken against these fp16
                                levels, as for a companded weight), or NULL */
  int32_t* outlier_idx;      /* [k] flat indices, ascending */
  uint16_t* outlier_val;     /* fp16 [k] original values */
  int32_t* outlier_row;      /* [k] row-sorted (ascending flat index order) */
  int32_t* outlier_col;
  uint16_t* outlier_delta;   /* fp16 [k] val - base */
  int32_t* outlier_row_ptr;  /* [rows+1] */
  float* threshold;          /* [1] clipping magnitude (0 when no outliers), or NULL */
} ts_quant_outputs;

TS_API size_t ts_quantize_workspace_size(const ts_quant_params* p);

TS_API int ts_quantize_pack(const void* w, int w_dtype, const ts_quant_params* p,
                     const ts_quant_outputs* o, void* workspace, size_t workspace_bytes,
                     void* stream);

/* Lloyd-Max 1-D fit on device values, codec.py:320-361 (on a given sample):
 * levels_out = sorted fp32 [n_levels] after `iters` Lloyd iterations started
 * from linspace(min, max). */
TS_API size_t ts_lloyd_fit_workspace_size(int64_t n, int n_levels);
TS_API int ts_lloyd_fit(const float* values, int64_t n, int n_levels, int iters, float* levels_out,
                 void* workspace, size_t workspace_bytes, void* stream);

/* Diagnostics. */
TS_API const char* ts_last_error(void);
TS_API const char* ts_version(void);
/* Number of kernels this library launched on the calling thread since the
 * last reset (bench bookkeeping). */
TS_API int64_t ts_launch_count(int reset);

#ifdef __cplusplus
}
#endif

#endif /* TENSORSHRINK_B200_H */
