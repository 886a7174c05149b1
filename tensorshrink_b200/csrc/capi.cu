// C ABI entry points (include/tensorshrink_b200.h): argument validation,
// dispatch to the kernels, error reporting.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace ts {

// implemented in qgemv.cu / dequant.cu / quantize.cu / qgemm_sm100.cu
// the two builds of qgemv.cu: one CTA per SM (v1) and two CTAs per SM (v2)
#define TS_DECLARE_GEMV(ns)                                                                          \
  namespace ns {                                                                                     \
  bool gemv_supported(const ts_qweight& w);                                                          \
  size_t gemv_workspace_size(const ts_qweight& w);                                                   \
  size_t gemv_error_flag_offset();                                                                   \
  int gemv_max_tokens(const ts_qweight& w);                                                          \
  int run_gemv(const GemvOp& op, int64_t M, void* workspace, size_t ws_bytes, cudaStream_t stream);  \
  bool gemv_chain_ok(const GemvOp* ops, int n, int64_t M);                                           \
  int run_gemv_chain(const GemvOp* ops, int n, int64_t M, void* workspace, size_t ws_bytes,          \
                     cudaStream_t stream);                                                           \
  }
TS_DECLARE_GEMV(gemv_v1)
TS_DECLARE_GEMV(gemv_v2)
#undef TS_DECLARE_GEMV
static bool gemv_supported(const ts_qweight& w) { return gemv_v1::gemv_supported(w); }
// Workspace covering either build (v2 runs twice the CTAs, so its partial-sum
// area is larger).
static size_t gemv_workspace_size(const ts_qweight& w) {
  size_t n = gemv_v1::gemv_workspace_size(w);
  if (gemv_v2::gemv_supported(w)) n = std::max(n, gemv_v2::gemv_workspace_size(w));
  return n;
}
// Two CTAs per SM when that build takes all M tokens in one pass and the
// workspace covers it; one CTA per SM otherwise.
static int run_gemv(const GemvOp& op, int64_t M, void* workspace, size_t ws_bytes, cudaStream_t stream) {
  const ts_qweight& w = *op.w;
  // A gated input is staged from twice the columns (the silu product is
  // formed per element): one CTA per SM stages it once per SM, not twice
  // (measured 10% faster on the 14336-column down projection).
  // TS_GEMV_CTAS_PER_SM=1 selects the one-CTA build for every call (tuning knob).
  const char* knob = getenv("TS_GEMV_CTAS_PER_SM");
  const bool force_v1 = (knob && knob[0] == '1') || op.gated;
  if (!force_v1 && gemv_v2::gemv_supported(w) && M <= gemv_v2::gemv_max_tokens(w) &&
      ws_bytes >= gemv_v2::gemv_workspace_size(w))
    return gemv_v2::run_gemv(op, M, workspace, ws_bytes, stream);
  return gemv_v1::run_gemv(op, M, workspace, ws_bytes, stream);
}
static GemvOp plain_op(const ts_qweight& w, const void* x, int x_dtype, int64_t x_stride, const void* bias,
                       int bias_dtype, void* out, int out_dtype, int64_t out_stride, int gated) {
  GemvOp op{};
  op.w = &w;
  op.x = x;
  op.x_dtype = x_dtype;
  op.x_stride = x_stride;
  op.bias = bias;
  op.bias_dtype = bias_dtype;
  op.out = out;
  op.out_dtype = out_dtype;
  op.out_stride = out_stride;
  op.gated = gated;
  op.act_dtype = x_dtype;
  return op;
}
int run_generic_qlinear(const ts_qweight& w, const void* x, int x_dtype, int64_t M,
                        int64_t x_stride, const void* bias, int bias_dtype, void* out,
                        int out_dtype, int64_t out_stride, cudaStream_t stream);
bool qgemm_supported(const ts_qweight& w, const void* x, int64_t x_stride);
size_t qgemm_workspace_extra(const ts_qweight& w, int64_t M, size_t counters_bytes_gemv);
bool qgemm_split_fits(const ts_qweight& w, int64_t M, size_t counters_off, size_t ws_bytes);
int run_qgemm(const ts_qweight& w, const void* x, int x_dtype, int64_t M, int64_t x_stride, const void* bias,
              int bias_dtype, void* out, int out_dtype, int64_t out_stride, void* workspace, size_t counters_off,
              size_t ws_bytes, cudaStream_t stream);
// Token counts from this one up always go to the tensor-core kernel.
constexpr int64_t kQgemmMinTokens = 65;
// From this one up they go there too when the workspace holds the split
// plan's partial sums (the GEMV takes at most 8 tokens per pass over the
// weights; the split tensor-core kernel reads the weights once for any M,
// and is the faster of the two from three GEMV passes on).
constexpr int64_t kSplitMinTokens = 17;
int qgemm_error_flag(int* code, bool clear, cudaStream_t stream);
int run_dequant(const ts_qweight& w, void* out, int out_dtype, int64_t out_stride,
                int apply_outliers, cudaStream_t stream);
int run_outlier_atomic(float* out, int64_t M, int64_t out_stride, const void* x, int x_dtype,
                       int64_t x_stride, const int32_t* row, const int32_t* col,
                       const uint16_t* delta, int64_t n, cudaStream_t stream);
size_t quantize_ws_size(const ts_quant_params& p, int dtype);
int run_quantize(const void* w, int dtype, const ts_quant_params& p, const ts_quant_outputs& o,
                 char* ws, size_t ws_bytes, cudaStream_t stream);
size_t lloyd_ws_size();
int run_lloyd_standalone(const float* vals, int64_t n, int n_levels, int iters, float* out, char* ws,
                         size_t ws_bytes, cudaStream_t stream);

namespace {
thread_local char g_err[1024] = "";
thread_local int64_t g_launches = 0;
// default limit of every bounded wait in the kernels
constexpr uint64_t kDefaultWaitNs = 2000000000ull;
// test stall requested by ts_test_inject_stall for the next launch on this thread
thread_local bool g_stall_next = false;
thread_local uint64_t g_stall_wait_ns = kDefaultWaitNs;

struct DevInfo {
  int sms = 0;
  int smem_optin = 0;
};
std::mutex g_dev_mu;
std::vector<DevInfo> g_dev;

const DevInfo& dev_info() {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if ((int)g_dev.size() <= dev) g_dev.resize(dev + 1);
  DevInfo& d = g_dev[dev];
  if (d.sms == 0) {
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (d.sms <= 0) d.sms = 148;
    if (d.smem_optin <= 0) d.smem_optin = 227 * 1024;
  }
  return d;
}
}  // namespace

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

void count_launch(int n) { g_launches += n; }
uint64_t wait_limit_ns() { return g_stall_next ? g_stall_wait_ns : kDefaultWaitNs; }
bool take_test_stall() {
  const bool s = g_stall_next;
  g_stall_next = false;
  return s;
}
int sm_count() { return dev_info().sms; }
int max_smem_optin() { return dev_info().smem_optin; }

static bool valid_act_dtype(int d) { return d == TS_F16 || d == TS_BF16; }
static bool valid_dtype(int d) { return d == TS_F16 || d == TS_BF16 || d == TS_F32; }

// Shape/pointer checks shared by every entry point taking a ts_qweight.
static int check_qweight(const ts_qweight* w) {
  TS_REQUIRE(w != nullptr, "qweight is NULL");
  TS_UNSUPPORTED(w->bits == 2 || w->bits == 4 || w->bits == 8,
                 "bits=%d not supported (2, 4 or 8)", w->bits);
  TS_REQUIRE(w->rows >= 0 && w->cols >= 0 && w->group_size > 0, "bad weight shape");
  TS_REQUIRE(w->padded_cols >= w->cols && w->padded_cols % w->group_size == 0 &&
                 w->n_groups == w->padded_cols / w->group_size,
             "inconsistent padded_cols/n_groups (cols=%lld padded=%lld gs=%d n_groups=%lld)",
             (long long)w->cols, (long long)w->padded_cols, w->group_size, (long long)w->n_groups);
  TS_REQUIRE(w->packed_row_bytes * 8 >= w->padded_cols * w->bits, "packed rows too short");
  TS_REQUIRE(w->packed != nullptr || w->rows * w->cols == 0, "packed is NULL");
  const bool plain = w->scale != nullptr && w->gmin != nullptr;
  const bool dq = w->dq_scale_codes && w->dq_scale_meta && w->dq_gmin_codes && w->dq_gmin_meta;
  TS_REQUIRE(plain != dq, "exactly one of scale/gmin or the four dq_* buffers must be given");
  TS_REQUIRE(!dq || w->dq_group_size > 0, "dq_group_size must be > 0");
  TS_REQUIRE(w->n_outliers == 0 ||
                 ((w->outlier_row_ptr || w->outlier_row) && w->outlier_col && w->outlier_delta),
             "outlier tables missing");
  return TS_OK;
}

}  // namespace ts

using namespace ts;

extern "C" {

const char* ts_last_error(void) { return g_err; }

const char* ts_version(void) { return "tensorshrink_b200 0.1.0 (sm_100a)"; }

int ts_test_inject_stall(uint64_t wait_limit_ns) {
  TS_REQUIRE(wait_limit_ns > 0 && wait_limit_ns <= kDefaultWaitNs, "wait limit must be in (0, 2 s]");
  g_stall_next = true;
  g_stall_wait_ns = wait_limit_ns;
  return TS_OK;
}

int64_t ts_launch_count(int reset) {
  const int64_t v = g_launches;
  if (reset) g_launches = 0;
  return v;
}

size_t ts_qlinear_workspace_size(const ts_qweight* w, int64_t M) {
  if (!w) return 0;
  const size_t head = gemv_v1::gemv_error_flag_offset() + 256;   // partial sums of the GEMV + error flag
  const size_t base = gemv_supported(*w) ? std::max(gemv_workspace_size(*w), head) : head;
  // split tensor-core plans serve calls of kSplitMinTokens tokens and more
  const bool gemv_fits = gemv_supported(*w) && gemv_v1::gemv_max_tokens(*w) > 0;
  const int64_t Ms = gemv_fits ? M : std::max<int64_t>(M, kSplitMinTokens);
  return base + (Ms >= kSplitMinTokens ? qgemm_workspace_extra(*w, Ms, base - head) : 0);
}

int ts_qlinear(const ts_qweight* w, const void* x, int x_dtype, int64_t M, int64_t x_row_stride,
               const void* bias, int bias_dtype, void* out, int out_dtype, int64_t out_row_stride,
               void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_qweight(w);
  if (rc != TS_OK) return rc;
  TS_UNSUPPORTED(valid_act_dtype(x_dtype), "x dtype must be fp16 or bf16");
  TS_UNSUPPORTED(valid_dtype(out_dtype), "out dtype must be fp16, bf16 or fp32");
  TS_REQUIRE(bias == nullptr || valid_dtype(bias_dtype), "bad bias dtype");
  TS_REQUIRE(M >= 0, "M < 0");
  if (M == 0 || w->rows == 0) return TS_OK;
  TS_REQUIRE(x != nullptr && out != nullptr, "x/out is NULL");
  TS_REQUIRE(x_row_stride >= w->cols && out_row_stride >= w->rows, "row strides too small");
  TS_REQUIRE(w->n_outliers == 0 || w->outlier_row_ptr != nullptr,
             "qlinear needs the CSR outlier_row_ptr table");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const size_t counters_off = gemv_v1::gemv_error_flag_offset() + 256;
  if (qgemm_supported(*w, x, x_row_stride)) {
    const bool split_ok = workspace != nullptr && qgemm_split_fits(*w, M, counters_off, workspace_bytes);
    if (M >= kQgemmMinTokens || (M >= kSplitMinTokens && split_ok))
      return run_qgemm(*w, x, x_dtype, M, x_row_stride, bias, bias_dtype, out, out_dtype, out_row_stride,
                       split_ok ? workspace : nullptr, counters_off, workspace_bytes, s);
  }
  // activations too long for the decode kernel's shared-memory staging:
  // the split tensor-core kernel when the workspace holds it, else the
  // generic kernel below
  const bool gemv_fits = gemv_supported(*w) && gemv_v1::gemv_max_tokens(*w) > 0;
  if (!gemv_fits && qgemm_supported(*w, x, x_row_stride) && workspace != nullptr &&
      qgemm_split_fits(*w, std::max<int64_t>(M, kSplitMinTokens), counters_off, workspace_bytes))
    return run_qgemm(*w, x, x_dtype, M, x_row_stride, bias, bias_dtype, out, out_dtype, out_row_stride, workspace,
                     counters_off, workspace_bytes, s);
  if (gemv_fits) {
    TS_REQUIRE(workspace != nullptr, "workspace is NULL (size %zu needed)", gemv_workspace_size(*w));
    return run_gemv(plain_op(*w, x, x_dtype, x_row_stride, bias, bias_dtype, out, out_dtype, out_row_stride, 0), M,
                    workspace, workspace_bytes, s);
  }
  return run_generic_qlinear(*w, x, x_dtype, M, x_row_stride, bias, bias_dtype, out, out_dtype,
                             out_row_stride, s);
}

int ts_qlinear_gated(const ts_qweight* w, const void* gate_up, int x_dtype, int64_t M, int64_t x_row_stride,
                     const void* bias, int bias_dtype, void* out, int out_dtype, int64_t out_row_stride,
                     void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_qweight(w);
  if (rc != TS_OK) return rc;
  TS_UNSUPPORTED(valid_act_dtype(x_dtype), "x dtype must be fp16 or bf16");
  TS_UNSUPPORTED(valid_dtype(out_dtype), "out dtype must be fp16, bf16 or fp32");
  TS_REQUIRE(M >= 0, "M < 0");
  if (M == 0 || w->rows == 0) return TS_OK;
  TS_REQUIRE(gate_up != nullptr && out != nullptr && workspace != nullptr, "NULL pointer");
  TS_REQUIRE(x_row_stride >= 2 * w->cols && out_row_stride >= w->rows, "row strides too small");
  TS_REQUIRE(w->n_outliers == 0 || w->outlier_row_ptr != nullptr, "qlinear needs the CSR outlier_row_ptr table");
  TS_UNSUPPORTED(gemv_supported(*w) && M <= gemv_v1::gemv_max_tokens(*w),
                 "gated qlinear runs in the decode kernel only (M=%lld)", (long long)M);
  return run_gemv(plain_op(*w, gate_up, x_dtype, x_row_stride, bias, bias_dtype, out, out_dtype, out_row_stride, 1),
                  M, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

// Validates one fused op and converts it to the decode kernel's form;
// TS_ERR_UNSUPPORTED when the decode kernel does not take it.
static int fused_op(const ts_qlinear_op* o, int64_t M, GemvOp& op) {
  TS_REQUIRE(o != nullptr, "op is NULL");
  int rc = check_qweight(o->w);
  if (rc != TS_OK) return rc;
  const ts_qweight& w = *o->w;
  const bool gated = (o->flags & TS_OP_GATED) != 0, norm = (o->flags & TS_OP_RMSNORM) != 0;
  TS_REQUIRE((o->flags & ~(TS_OP_GATED | TS_OP_RMSNORM)) == 0, "unknown op flags 0x%x", o->flags);
  TS_UNSUPPORTED(!(gated && norm), "an op is gated or normalized, not both");
  TS_UNSUPPORTED(valid_dtype(o->out_dtype), "out dtype must be fp16, bf16 or fp32");
  TS_UNSUPPORTED(valid_act_dtype(o->act_dtype), "act dtype must be fp16 or bf16");
  if (norm) {
    TS_UNSUPPORTED(o->x_dtype == TS_F32, "RMSNorm ops take fp32 rows");
    TS_REQUIRE(o->norm_weight != nullptr, "norm_weight is NULL");
  } else {
    TS_UNSUPPORTED(valid_act_dtype(o->x_dtype), "x dtype must be fp16 or bf16");
    TS_UNSUPPORTED(o->x_dtype == o->act_dtype, "act dtype must equal x dtype for 16-bit inputs");
  }
  TS_REQUIRE(o->bias == nullptr || valid_dtype(o->bias_dtype), "bad bias dtype");
  TS_REQUIRE(o->x != nullptr && o->out != nullptr, "x/out is NULL");
  TS_REQUIRE(o->x_row_stride >= (gated ? 2 : 1) * w.cols && o->out_row_stride >= w.rows, "row strides too small");
  TS_REQUIRE(o->residual == nullptr || o->residual_row_stride >= w.rows, "residual stride too small");
  TS_REQUIRE(o->residual == nullptr || o->out_dtype == TS_F32 || o->residual != o->out,
             "a residual aliasing out needs an fp32 out");
  TS_REQUIRE(w.n_outliers == 0 || w.outlier_row_ptr != nullptr, "qlinear needs the CSR outlier_row_ptr table");
  TS_UNSUPPORTED(gemv_supported(w) && M <= gemv_v1::gemv_max_tokens(w),
                 "fused qlinear ops run in the decode kernel only (M=%lld)", (long long)M);
  op = plain_op(w, o->x, o->x_dtype, o->x_row_stride, o->bias, o->bias_dtype, o->out, o->out_dtype,
                o->out_row_stride, gated ? 1 : 0);
  op.act_dtype = o->act_dtype;
  op.norm_w = norm ? o->norm_weight : nullptr;
  op.norm_eps = o->norm_eps;
  op.residual = o->residual;
  op.residual_stride = o->residual_row_stride;
  return TS_OK;
}

int ts_qlinear_ex(const ts_qlinear_op* o, int64_t M, void* workspace, size_t workspace_bytes, void* stream) {
  TS_REQUIRE(o != nullptr, "op is NULL");
  TS_REQUIRE(M >= 0, "M < 0");
  if (o->flags == 0 && o->residual == nullptr && o->x_dtype != TS_F32)
    return ts_qlinear(o->w, o->x, o->x_dtype, M, o->x_row_stride, o->bias, o->bias_dtype, o->out, o->out_dtype,
                      o->out_row_stride, workspace, workspace_bytes, stream);
  if (M == 0 || (o->w && o->w->rows == 0)) return TS_OK;
  GemvOp op;
  const int rc = fused_op(o, M, op);
  if (rc != TS_OK) return rc;
  TS_REQUIRE(workspace != nullptr, "workspace is NULL");
  return run_gemv(op, M, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int ts_qlinear_chain_max(void) { return 8; }

int ts_qlinear_chain(const ts_qlinear_op* ops, int n_ops, int64_t M, int persistent, void* workspace,
                     size_t workspace_bytes, void* stream) {
  TS_REQUIRE(ops != nullptr && n_ops >= 0, "bad op list");
  TS_REQUIRE(M >= 0, "M < 0");
  if (n_ops == 0 || M == 0) return TS_OK;
  TS_REQUIRE(workspace != nullptr, "workspace is NULL");
  // every op is validated before any runs: a chain runs whole or not at all
  std::vector<GemvOp> g(n_ops);
  for (int i = 0; i < n_ops; ++i) {
    const int rc = fused_op(&ops[i], M, g[i]);
    if (rc != TS_OK) return rc;
    TS_REQUIRE(ops[i].w->rows > 0, "empty layer in a chain");
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (persistent && n_ops > 1 && n_ops <= ts_qlinear_chain_max() && gemv_v1::gemv_chain_ok(g.data(), n_ops, M)) {
    // the two-CTA-per-SM build when every layer fits it, else the one-CTA
    // one; TS_CHAIN_CTAS_PER_SM=1 selects the one-CTA build (tuning knob)
    const char* knob = getenv("TS_CHAIN_CTAS_PER_SM");
    bool v2 = !(knob && knob[0] == '1');
    for (int i = 0; i < n_ops && v2; ++i)
      v2 = gemv_v2::gemv_supported(*g[i].w) && M <= gemv_v2::gemv_max_tokens(*g[i].w) &&
           workspace_bytes >= gemv_v2::gemv_workspace_size(*g[i].w);
    if (v2 && gemv_v2::gemv_chain_ok(g.data(), n_ops, M))
      return gemv_v2::run_gemv_chain(g.data(), n_ops, M, workspace, workspace_bytes, s);
    return gemv_v1::run_gemv_chain(g.data(), n_ops, M, workspace, workspace_bytes, s);
  }
  for (int i = 0; i < n_ops; ++i) {
    const int rc = run_gemv(g[i], M, workspace, workspace_bytes, s);
    if (rc != TS_OK) return rc;
  }
  return TS_OK;
}

int ts_apply_outlier_correction(float* out, int64_t M, int64_t N, int64_t out_row_stride,
                                const void* x, int x_dtype, int64_t x_row_stride,
                                const int32_t* row, const int32_t* col, const uint16_t* delta,
                                int64_t n_outliers, void* stream) {
  TS_UNSUPPORTED(valid_act_dtype(x_dtype) || x_dtype == TS_F32, "bad x dtype");
  TS_REQUIRE(M >= 0 && N >= 0 && n_outliers >= 0, "negative size");
  if (n_outliers == 0 || M == 0) return TS_OK;
  TS_REQUIRE(out && x && row && col && delta, "NULL pointer");
  TS_REQUIRE(out_row_stride >= N, "out stride too small");
  return run_outlier_atomic(out, M, out_row_stride, x, x_dtype, x_row_stride, row, col, delta,
                            n_outliers, reinterpret_cast<cudaStream_t>(stream));
}

int ts_dequantize_weight(const ts_qweight* w, void* out, int out_dtype, int64_t out_row_stride,
                         int apply_outliers, void* stream) {
  int rc = check_qweight(w);
  if (rc != TS_OK) return rc;
  TS_UNSUPPORTED(valid_dtype(out_dtype), "out dtype must be fp16, bf16 or fp32");
  TS_REQUIRE(out != nullptr || w->rows * w->cols == 0, "out is NULL");
  TS_REQUIRE(out_row_stride >= w->cols, "out stride too small");
  TS_REQUIRE(!apply_outliers || w->n_outliers == 0 || w->outlier_row != nullptr,
             "outlier_row needed to apply outliers");
  return run_dequant(*w, out, out_dtype, out_row_stride, apply_outliers,
                     reinterpret_cast<cudaStream_t>(stream));
}

static int check_qparams(const ts_quant_params* p) {
  TS_REQUIRE(p != nullptr, "params is NULL");
  TS_UNSUPPORTED(p->bits == 2 || p->bits == 4 || p->bits == 8, "bits=%d not supported", p->bits);
  const int gs = p->group_size;
  TS_UNSUPPORTED(gs >= 8 && gs <= 256 && (gs & (gs - 1)) == 0,
                 "group_size=%d not supported by the GPU quantizer (power of two in [8, 256])", gs);
  TS_REQUIRE(p->rows > 0 && p->cols > 0, "empty weight");
  TS_REQUIRE(p->rows * p->cols < (1ll << 31), "weight too large for int32 outlier indices");
  TS_REQUIRE(p->k_outliers >= 0, "k_outliers < 0");
  TS_REQUIRE(!p->double_quant || p->dq_group_size > 0, "dq_group_size must be > 0");
  TS_REQUIRE(p->mode >= 0 && p->mode <= 2, "bad mode");
  TS_REQUIRE(p->mode != TS_QMODE_LLOYD || (p->lloyd_iters >= 0), "bad lloyd_iters");
  return TS_OK;
}

size_t ts_quantize_workspace_size(const ts_quant_params* p) {
  if (!p) return 0;
  // sized for the widest key (fp32 input)
  return quantize_ws_size(*p, TS_F32);
}

int ts_quantize_pack(const void* w, int w_dtype, const ts_quant_params* p, const ts_quant_outputs* o,
                     void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_qparams(p);
  if (rc != TS_OK) return rc;
  TS_UNSUPPORTED(valid_dtype(w_dtype), "weight dtype must be fp16, bf16 or fp32");
  TS_REQUIRE(w && o && o->packed && o->scale && o->gmin && o->outlier_row_ptr, "NULL pointer");
  const bool outl = p->k_outliers > 0 && p->k_outliers < p->rows * p->cols;
  TS_REQUIRE(!outl || (o->outlier_idx && o->outlier_val && o->outlier_row && o->outlier_col &&
                       o->outlier_delta),
             "outlier outputs missing");
  TS_REQUIRE(!p->double_quant || (o->dq_scale_codes && o->dq_scale_meta && o->dq_gmin_codes &&
                                  o->dq_gmin_meta),
             "double-quant outputs missing");
  TS_REQUIRE(is_aligned(o->packed, 8), "packed output must be 8-byte aligned");
  TS_REQUIRE(workspace != nullptr, "workspace is NULL");
  return run_quantize(w, w_dtype, *p, *o, reinterpret_cast<char*>(workspace), workspace_bytes,
                      reinterpret_cast<cudaStream_t>(stream));
}

size_t ts_lloyd_fit_workspace_size(int64_t n, int n_levels) {
  (void)n;
  (void)n_levels;
  return lloyd_ws_size();
}

int ts_lloyd_fit(const float* values, int64_t n, int n_levels, int iters, float* levels_out,
                 void* workspace, size_t workspace_bytes, void* stream) {
  TS_REQUIRE(values && levels_out && workspace, "NULL pointer");
  return run_lloyd_standalone(values, n, n_levels, iters, levels_out,
                              reinterpret_cast<char*>(workspace), workspace_bytes,
                              reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ---- tensor-map encoding via the driver entry point ------------------------
#include <cudaTypedefs.h>
#include "sm100.cuh"

namespace ts {

int encode_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t inner,
                   uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                   CUtensorMapSwizzle swizzle) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  TS_REQUIRE(fn != nullptr, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TS_REQUIRE(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (%d): inner=%llu outer=%llu stride=%llu box=%ux%u",
             (int)r, (unsigned long long)inner, (unsigned long long)outer,
             (unsigned long long)row_stride_bytes, box_inner, box_outer);
  return TS_OK;
}

}  // namespace ts

// ---- allocation-free decode entry point -------------------------------------
// Callers that may not allocate device memory at all (a serving loop replaying
// pre-recorded work under a fixed memory budget, or a host whose allocator is
// owned by another runtime and cannot be called from the decode thread) have
// no place to put the fast decode kernel's split-row counters and partial
// sums. This variant keeps them in a fixed per-device array compiled into the
// library instead of a caller workspace. Module loading zero-fills the array;
// every call that completes leaves the counters at zero again, which is the
// state the next call needs. One array per device means two calls that may
// overlap on the device (different streams, or different host threads) race
// on it: serialize them.
namespace ts {
namespace {
constexpr size_t kNoAllocScratchBytes = 512u << 10;
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the current device's scratch array. The host-side name
// of a __device__ array is only a stand-in, so the address is asked of the
// runtime on every call (cheap once the module is loaded; no stale pointer
// survives a context reset). The first call on a device loads the module
// there, which a stream capture does not allow: make it before capturing.
int noalloc_scratch(void** out) {
  void* p = nullptr;
  TS_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
  *out = p;
  return TS_OK;
}
}  // namespace
}  // namespace ts

extern "C" size_t ts_qlinear_noalloc_max_scratch(void) { return ts::kNoAllocScratchBytes; }

extern "C" int ts_qlinear_noalloc(const ts_qweight* w, const void* x, int x_dtype, int64_t M,
                                  int64_t x_row_stride, const void* bias, int bias_dtype, void* out,
                                  int out_dtype, int64_t out_row_stride, void* stream) {
  int rc = check_qweight(w);
  if (rc != TS_OK) return rc;
  void* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc != TS_OK) return rc;
  // only the decode kernel uses scratch; the tensor-core kernel takes the
  // calls of kQgemmMinTokens tokens and more whose layout it supports
  const bool gemv_path = !(M >= kQgemmMinTokens && qgemm_supported(*w, x, x_row_stride)) && gemv_supported(*w);
  // (the fixed array is too small for the split tensor-core plan's partial
  // sums, so 9..64-token calls take the decode kernel here)
  const size_t need = gemv_path ? gemv_workspace_size(*w) : 0;
  TS_UNSUPPORTED(need <= kNoAllocScratchBytes,
                 "ts_qlinear_noalloc: weight of %lld rows needs %zu bytes of scratch, above the "
                 "fixed %zu; use ts_qlinear with a caller workspace",
                 (long long)w->rows, need, kNoAllocScratchBytes);
  return ts_qlinear(w, x, x_dtype, M, x_row_stride, bias, bias_dtype, out, out_dtype,
                    out_row_stride, scratch, kNoAllocScratchBytes, stream);
}

// ---- device error status -------------------------------------------------------
extern "C" int ts_qlinear_status(void* workspace, size_t workspace_bytes, int clear, void* stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  char* ws = reinterpret_cast<char*>(workspace);
  if (ws == nullptr) {
    void* p = nullptr;
    int rc = noalloc_scratch(&p);
    if (rc != TS_OK) return rc;
    ws = reinterpret_cast<char*>(p);
    workspace_bytes = kNoAllocScratchBytes;
  }
  const size_t flag_off = gemv_v1::gemv_error_flag_offset();
  TS_REQUIRE(workspace_bytes >= flag_off + 256, "workspace of %zu bytes is smaller than any GEMV workspace",
             workspace_bytes);
  int gemv_code = 0, gemm_code = 0;
  TS_CUDA_TRY(cudaMemcpyAsync(&gemv_code, ws + flag_off, sizeof(int), cudaMemcpyDeviceToHost, st));
  TS_CUDA_TRY(cudaStreamSynchronize(st));
  int rc = qgemm_error_flag(&gemm_code, clear != 0, st);
  if (rc != TS_OK) return rc;
  if (gemv_code == 0 && gemm_code == 0) return TS_OK;
  if (clear && gemv_code != 0) {
    // the flag, and the row-block counters a CTA that gave up may have left
    // non-zero (partial sums need no reset: each slot is written before it is read)
    TS_CUDA_TRY(cudaMemsetAsync(ws + flag_off, 0, workspace_bytes - flag_off, st));
    TS_CUDA_TRY(cudaStreamSynchronize(st));
  }
  set_error("a bounded wait on the device ran out (decode kernel code %d, tensor-core kernel code %d); "
            "the outputs of the calls since the last status check are not valid",
            gemv_code, gemm_code);
  return TS_ERR_TIMEOUT;
}
