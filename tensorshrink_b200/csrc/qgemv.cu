// Decode-shaped fused dequant-GEMV (M <= 8 tokens per pass) on CUDA cores.
//
// Replaces the reference's `_fused_dequant_matmul_{2,4,8}bit` Triton kernels
// (tensorshrink triton_kernels.py:278-541) for decode shapes, with the
// outlier correction of `_add_outlier_tile` / `_outlier_correction_kernel`
// (triton_kernels.py:154-232, 543-576) folded into the row epilogue.
//
// Work decomposition. The packed matrix is cut into "units": R consecutive
// rows x one 512-byte chunk of each row. A warp processes a unit with one
// 16-byte streaming load per lane per row (LDG.128, L1 bypassed), so a lane
// always covers exactly one 16-byte span of one quantization group. Units are
// numbered row-group-major and every warp of the persistent grid takes an
// equal contiguous range, so HBM traffic is balanced to within one unit. Rows
// wholly inside one warp's range are finished by that warp; a row split
// between warps is finished by whichever piece arrives last (per-row counter
// in the workspace), which sums the pieces' partials in warp order, so the
// result is deterministic.
//
// Arithmetic. Per (row, group) the reconstruction is w = v(code)*s + g, so
//   sum_k x_k w_k = s * sum_k x_k (v_k - C) + (g + C*s) * sum_k x_k
// with a centring constant C. The activations are staged once per CTA in
// shared memory as fp16 scaled by a power of two per 16-byte span (exact
// rescale, keeps every partial product in fp16 range), together with the
// span's fp32 sum. Codes are turned into fp16 (v - C) values either with the
// exponent-bias trick (uniform grids: integer codes OR-ed into the mantissa
// of 1024.0) or through a per-lane-replicated byte lookup table in shared
// memory (NF / Lloyd-Max codebooks); products are accumulated with HFMA2 over
// one 32-bit word of codes and then in fp32.
#include "common.cuh"

namespace ts {
namespace gemv {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kR = 2;  // rows per unit

template <int BITS>
struct Geo {
  static constexpr int SPAN = 128 / BITS;      // weights per lane per unit (16 bytes)
  static constexpr int VEC = SPAN / 8;         // 16-byte fp16 activation vectors per span
  static constexpr int WORD_W = 32 / BITS;     // weights per 32-bit word of codes
  static constexpr int CHUNK_W = 32 * SPAN;    // weights per 512-byte chunk
};

struct Args {
  QW q;
  const void* x;
  int x_dtype;
  int64_t x_stride;
  int64_t m0;      // first token of this pass
  int mt;          // tokens in this pass (<= MT)
  const void* bias;
  int bias_dtype;
  void* out;
  int out_dtype;
  int64_t out_stride;
  float* partials;
  int* counters;
  uint32_t units;      // n_rowgroups * chunks
  uint32_t chunks;     // 512-byte chunks per row
  uint32_t total_warps;
  int n_chunks_x;      // chunks covering padded_cols (activation staging)
  int x_vec16;         // rows of x are 16-byte aligned (vector staging loads)
  int gbytes_shift;    // log2(bytes of packed codes per group)
  int dq_shift;        // log2(dq_group_size) when a power of two, else -1
  float center;        // C in the identity above (uniform grids; codebooks use their midpoint)
};

// Position of weight offset j (0..WORD_W-1) inside the fp16 activation block
// that matches the order in which codes come out of a 32-bit word.
template <int BITS, bool CB>
__device__ __forceinline__ int word_pos(int j) {
  if (CB || BITS == 8) return j;
  constexpr int H = Geo<BITS>::WORD_W / 2;  // the trick yields pairs (j, j+H)
  return j < H ? 2 * j : 2 * (j - H) + 1;
}

__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(orv));  // (a & b) | c
  return r;
}

__device__ __forceinline__ half2 u2h2(uint32_t v) { return *reinterpret_cast<half2*>(&v); }
__device__ __forceinline__ uint32_t h22u(half2 v) { return *reinterpret_cast<uint32_t*>(&v); }

// One 32-bit word of codes dotted with its activations; returns the half2
// partial (lanes of the pair summed later in fp32). `xv` points at the span's
// fp16 activation vectors (uint4 = 8 halves).
template <int BITS, bool CB>
__device__ __forceinline__ half2 word_dot(uint32_t q, const uint4* xv, int w, const char* lut) {
  if constexpr (!CB && BITS == 4) {
    // (1024 + n) with n at the low nibble of each 16-bit half; then /16 for
    // the nibble sitting at bits 4-7. Centre C = 8.
    const uint4 xa = xv[w];
    const uint32_t t0 = lop_and_or(q, 0x000F000Fu, 0x64006400u);
    const uint32_t t1 = lop_and_or(q, 0x00F000F0u, 0x64006400u);
    const uint32_t q2 = q >> 8;
    const uint32_t t2 = lop_and_or(q2, 0x000F000Fu, 0x64006400u);
    const uint32_t t3 = lop_and_or(q2, 0x00F000F0u, 0x64006400u);
    const half2 c0 = __hsub2(u2h2(t0), u2h2(0x64086408u));                      // n - 8
    const half2 c1 = __hfma2(u2h2(t1), u2h2(0x2C002C00u), u2h2(0xD480D480u));   // (1024+16n)/16 - 72
    const half2 c2 = __hsub2(u2h2(t2), u2h2(0x64086408u));
    const half2 c3 = __hfma2(u2h2(t3), u2h2(0x2C002C00u), u2h2(0xD480D480u));
    half2 a = __hmul2(c0, u2h2(xa.x));
    a = __hfma2(c1, u2h2(xa.y), a);
    a = __hfma2(c2, u2h2(xa.z), a);
    a = __hfma2(c3, u2h2(xa.w), a);
    return a;
  } else if constexpr (!CB && BITS == 2) {
    // 16 crumbs: pairs (j, j+8); crumb at bits 2i of each half scaled by 4^-i.
    const uint4 xa = xv[2 * w];
    const uint4 xb = xv[2 * w + 1];
    const uint32_t q2 = q >> 8;
    const half2 c0 = __hsub2(u2h2(lop_and_or(q, 0x00030003u, 0x64006400u)), u2h2(0x64026402u));
    const half2 c1 = __hfma2(u2h2(lop_and_or(q, 0x000C000Cu, 0x64006400u)), u2h2(0x34003400u), u2h2(0xDC08DC08u));
    const half2 c2 = __hfma2(u2h2(lop_and_or(q, 0x00300030u, 0x64006400u)), u2h2(0x2C002C00u), u2h2(0xD420D420u));
    const half2 c3 = __hfma2(u2h2(lop_and_or(q, 0x00C000C0u, 0x64006400u)), u2h2(0x24002400u), u2h2(0xCC80CC80u));
    const half2 c4 = __hsub2(u2h2(lop_and_or(q2, 0x00030003u, 0x64006400u)), u2h2(0x64026402u));
    const half2 c5 = __hfma2(u2h2(lop_and_or(q2, 0x000C000Cu, 0x64006400u)), u2h2(0x34003400u), u2h2(0xDC08DC08u));
    const half2 c6 = __hfma2(u2h2(lop_and_or(q2, 0x00300030u, 0x64006400u)), u2h2(0x2C002C00u), u2h2(0xD420D420u));
    const half2 c7 = __hfma2(u2h2(lop_and_or(q2, 0x00C000C0u, 0x64006400u)), u2h2(0x24002400u), u2h2(0xCC80CC80u));
    half2 a = __hmul2(c0, u2h2(xa.x));
    a = __hfma2(c1, u2h2(xa.y), a);
    a = __hfma2(c2, u2h2(xa.z), a);
    a = __hfma2(c3, u2h2(xa.w), a);
    a = __hfma2(c4, u2h2(xb.x), a);
    a = __hfma2(c5, u2h2(xb.y), a);
    a = __hfma2(c6, u2h2(xb.z), a);
    a = __hfma2(c7, u2h2(xb.w), a);
    return a;
  } else if constexpr (!CB && BITS == 8) {
    // (1024 + b) by byte permute into the fp16 mantissa, centre 128.
    const uint4 xa = xv[w >> 1];
    const uint32_t xlo = (w & 1) ? xa.z : xa.x;
    const uint32_t xhi = (w & 1) ? xa.w : xa.y;
    const uint32_t t0 = __byte_perm(q, 0x64646464u, 0x5140);
    const uint32_t t1 = __byte_perm(q, 0x64646464u, 0x5342);
    const half2 c0 = __hsub2(u2h2(t0), u2h2(0x64806480u));
    const half2 c1 = __hsub2(u2h2(t1), u2h2(0x64806480u));
    half2 a = __hmul2(c0, u2h2(xlo));
    a = __hfma2(c1, u2h2(xhi), a);
    return a;
  } else if constexpr (CB && BITS == 4) {
    // lut: [256 bytes][32 lanes] half2 (v(lo)-C, v(hi)-C); `lut` is lane-offset.
    const uint4 xa = xv[w];
    const uint32_t xs[4] = {xa.x, xa.y, xa.z, xa.w};
    half2 a = __float2half2_rn(0.f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t b = (q >> (8 * i)) & 0xFFu;
      const uint32_t v = *reinterpret_cast<const uint32_t*>(lut + b * 128u);
      a = __hfma2(u2h2(v), u2h2(xs[i]), a);
    }
    return a;
  } else if constexpr (CB && BITS == 2) {
    // lut: [256][32 lanes] uint2 = two half2 (crumbs 0,1 | 2,3).
    const uint4 xa = xv[2 * w];
    const uint4 xb = xv[2 * w + 1];
    const uint32_t xs[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
    half2 a = __float2half2_rn(0.f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t b = (q >> (8 * i)) & 0xFFu;
      const uint2 v = *reinterpret_cast<const uint2*>(lut + b * 256u);
      a = __hfma2(u2h2(v.x), u2h2(xs[2 * i]), a);
      a = __hfma2(u2h2(v.y), u2h2(xs[2 * i + 1]), a);
    }
    return a;
  } else {
    // CB && BITS == 8: lut [256][32 lanes] u32 holding one fp16 in the low half.
    const uint4 xa = xv[w >> 1];
    const uint32_t xlo = (w & 1) ? xa.z : xa.x;
    const uint32_t xhi = (w & 1) ? xa.w : xa.y;
    const uint32_t v0 = *reinterpret_cast<const uint32_t*>(lut + (q & 0xFFu) * 128u);
    const uint32_t v1 = *reinterpret_cast<const uint32_t*>(lut + ((q >> 8) & 0xFFu) * 128u);
    const uint32_t v2 = *reinterpret_cast<const uint32_t*>(lut + ((q >> 16) & 0xFFu) * 128u);
    const uint32_t v3 = *reinterpret_cast<const uint32_t*>(lut + (q >> 24) * 128u);
    half2 a = __hmul2(u2h2(__byte_perm(v0, v1, 0x5410)), u2h2(xlo));
    a = __hfma2(u2h2(__byte_perm(v2, v3, 0x5410)), u2h2(xhi), a);
    return a;
  }
}

// Raw (not yet decoded) metadata of one (row, group), loaded ahead of use.
struct MetaRaw {
  uint32_t a, b, c;
};

template <bool DQ>
__device__ __forceinline__ MetaRaw load_meta(const QW& q, uint32_t flat, int dq_shift) {
  MetaRaw m;
  if constexpr (DQ) {
    const uint32_t sup = dq_shift >= 0 ? (flat >> dq_shift) : flat / (uint32_t)q.dq_gs;
    m.a = (uint32_t)__ldg(q.dqs_codes + flat) | ((uint32_t)__ldg(q.dqg_codes + flat) << 8);
    m.b = h22u(__ldg(q.dqs_meta + sup));
    m.c = h22u(__ldg(q.dqg_meta + sup));
  } else {
    m.a = __half_as_ushort(__ldg(q.scale + flat));
    m.b = __half_as_ushort(__ldg(q.gmin + flat));
    m.c = 0;
  }
  return m;
}

template <bool DQ>
__device__ __forceinline__ float2 decode_meta(const MetaRaw& m) {
  if constexpr (DQ) {
    const float2 ms = __half22float2(u2h2(m.b));
    const float2 mg = __half22float2(u2h2(m.c));
    const float s = __fadd_rn(__fmul_rn((float)(m.a & 0xFFu), ms.x), ms.y);
    const float g = __fadd_rn(__fmul_rn((float)(m.a >> 8), mg.x), mg.y);
    return make_float2(s, g);
  } else {
    return make_float2(h2f((uint16_t)m.a), h2f((uint16_t)m.b));
  }
}

struct Stage {
  uint4 w[kR];
  MetaRaw m[kR];
};

// Unit position (row group, 512-byte chunk), advanced incrementally so the
// streaming loop does no integer division.
struct Cursor {
  uint32_t rg, ch;
};

template <int BITS, bool DQ>
__device__ __forceinline__ void load_stage(Stage& st, const Args& a, const Cursor c, int lane) {
  const uint32_t boff = c.ch * 512u + lane * 16u;
  const bool valid = boff < (uint32_t)a.q.row_bytes;
  const uint32_t g = boff >> a.gbytes_shift;
#pragma unroll
  for (int r = 0; r < kR; ++r) {
    const uint32_t row = c.rg * kR + r;
    if (valid && row < (uint32_t)a.q.rows) {
      st.w[r] = ldg_stream_v4(a.q.packed + (size_t)row * (size_t)a.q.row_bytes + boff);
      st.m[r] = load_meta<DQ>(a.q, row * (uint32_t)a.q.n_groups + g, a.dq_shift);
    } else {
      st.w[r] = make_uint4(0, 0, 0, 0);
      st.m[r] = MetaRaw{0, 0, 0};
    }
  }
}

__device__ __forceinline__ void advance(Cursor& c, uint32_t chunks) {
  if (++c.ch == chunks) {
    c.ch = 0;
    ++c.rg;
  }
}

// Index of the warp whose unit range contains unit u (ranges are
// [floor(U*w/W), floor(U*(w+1)/W))).
__device__ __forceinline__ uint32_t warp_of(uint64_t u, uint64_t U, uint64_t W) {
  return (uint32_t)(((u + 1) * W + U - 1) / U - 1);
}

template <int MT>
__device__ void finish_rows(const Args& a, uint32_t rg, float (&tot)[kR][MT], int lane) {
  // Outlier correction (CSR walk, lanes split the row's entries), bias, store.
#pragma unroll
  for (int r = 0; r < kR; ++r) {
    const int64_t row = (int64_t)rg * kR + r;
    if (row >= a.q.rows) break;
    float c[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) c[m] = 0.f;
    if (a.q.n_outliers > 0) {
      const int o0 = __ldg(a.q.orow_ptr + row), o1 = __ldg(a.q.orow_ptr + row + 1);
      for (int j = o0 + lane; j < o1; j += 32) {
        const int64_t col = __ldg(a.q.ocol + j);
        const float d = __half2float(__ldg(a.q.odelta + j));
#pragma unroll
        for (int m = 0; m < MT; ++m)
          if (m < a.mt) c[m] += load_f(a.x, a.x_dtype, (a.m0 + m) * a.x_stride + col) * d;
      }
#pragma unroll
      for (int m = 0; m < MT; ++m) c[m] = warp_sum(c[m]);
    }
    const float b = a.bias ? load_f(a.bias, a.bias_dtype, row) : 0.f;
#pragma unroll
    for (int m = 0; m < MT; ++m)
      if (lane == m && m < a.mt)
        store_f(a.out, a.out_dtype, (a.m0 + m) * a.out_stride + row, tot[r][m] + c[m] + b);
  }
}

template <int BITS, bool CB, bool DQ, int MT>
__global__ void __launch_bounds__(kThreads, 2) qgemv_kernel(const Args a) {
  using G = Geo<BITS>;
  extern __shared__ __align__(16) char smem[];
  constexpr int LUT_BYTES = !CB ? 0 : (BITS == 2 ? 256 * 32 * 8 : 256 * 32 * 4);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const uint32_t gw = blockIdx.x * kWarps + warp;
  const uint64_t U = a.units, W = a.total_warps;
  const uint32_t u_begin = (uint32_t)(U * gw / W);
  const uint32_t u_end = (uint32_t)(U * (gw + 1) / W);

  char* lut = smem;
  __half* xs = reinterpret_cast<__half*>(smem + LUT_BYTES);
  const int64_t x_tok = (int64_t)a.n_chunks_x * G::CHUNK_W;  // halves per token
  float2* sx = reinterpret_cast<float2*>(xs + MT * x_tok);
  const int n_spans = a.n_chunks_x * 32;

  // 1. Start streaming this warp's first weights (independent of x).
  constexpr int D = 3;
  Stage st[D];
  const uint32_t first_rg = u_begin / a.chunks;
  Cursor pf{first_rg, u_begin - first_rg * a.chunks};  // prefetch cursor
#pragma unroll
  for (int d = 0; d < D; ++d)
    if (u_begin + d < u_end) {
      load_stage<BITS, DQ>(st[d], a, pf, lane);
      advance(pf, a.chunks);
    }

  // 2. Codebook lookup table (per-lane copies: conflict-free random access).
  //    Centre C = midpoint of the codebook range keeps the fp16 levels small.
  float center = a.center;
  if constexpr (CB) {
    const float* cb = a.q.codebook;
    center = 0.5f * (__ldg(cb) + __ldg(cb + (1 << BITS) - 1));
    for (int i = threadIdx.x; i < 256 * 32; i += kThreads) {
      const int b = i >> 5, l = i & 31;
      if constexpr (BITS == 4) {
        const half2 v = __floats2half2_rn(__ldg(cb + (b & 15)) - center, __ldg(cb + (b >> 4)) - center);
        reinterpret_cast<uint32_t*>(lut)[b * 32 + l] = h22u(v);
      } else if constexpr (BITS == 2) {
        const half2 v0 = __floats2half2_rn(__ldg(cb + (b & 3)) - center, __ldg(cb + ((b >> 2) & 3)) - center);
        const half2 v1 = __floats2half2_rn(__ldg(cb + ((b >> 4) & 3)) - center, __ldg(cb + (b >> 6)) - center);
        reinterpret_cast<uint2*>(lut)[b * 32 + l] = make_uint2(h22u(v0), h22u(v1));
      } else {
        reinterpret_cast<uint32_t*>(lut)[b * 32 + l] = f2h(__ldg(cb + b) - center);
      }
    }
  }

  // 3. Wait for the producer of x (programmatic dependent launch), stage it:
  //    one thread per 8 consecutive activations; the SPAN/8 threads of a span
  //    (an aligned lane group) reduce its max |x| and sum with shuffles.
  pdl_wait_primary();
  {
    constexpr int TPS = G::SPAN / 8;
    const uint32_t per_tok = (uint32_t)(a.q.padded_cols / 8);
    const uint32_t items = MT * per_tok;
    for (uint32_t base = 0; base < items; base += kThreads) {
      const uint32_t it = base + threadIdx.x;
      const bool live = it < items;
      const uint32_t m = live ? it / per_tok : 0;
      const uint32_t k0 = live ? (it - m * per_tok) * 8 : 0;
      const bool tok = live && (int)m < a.mt;
      const int64_t xoff = (a.m0 + m) * a.x_stride + k0;
      float v[8];
      if (tok && a.x_vec16 && k0 + 8 <= (uint32_t)a.q.cols) {
        const uint4 raw = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(a.x) + xoff));
        const uint32_t r4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (a.x_dtype == TS_F16) {
            const float2 f = __half22float2(u2h2(r4[j]));
            v[2 * j] = f.x;
            v[2 * j + 1] = f.y;
          } else {
            v[2 * j] = __uint_as_float(r4[j] << 16);
            v[2 * j + 1] = __uint_as_float(r4[j] & 0xFFFF0000u);
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          v[j] = (tok && k0 + j < (uint32_t)a.q.cols) ? load_f(a.x, a.x_dtype, xoff + j) : 0.f;
      }
      float mx = 0.f, sum = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        mx = fmaxf(mx, fabsf(v[j]));
        sum += v[j];
      }
#pragma unroll
      for (int o = TPS / 2; o > 0; o >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        sum += __shfl_xor_sync(0xffffffffu, sum, o);
      }
      int e = 0;
      if (mx > 0.f) frexpf(mx, &e);
      if (live) {
        const uint32_t sp = k0 / G::SPAN;          // span index within the token
        const int j0 = (int)(k0 - sp * G::SPAN);   // this thread's offset in the span
        if (j0 == 0) sx[m * n_spans + sp] = make_float2(ldexpf(1.f, e), sum);
        __half* dst = xs + m * x_tok + (int64_t)(sp >> 5) * G::CHUNK_W;
        const int l = (int)(sp & 31);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int jj = j0 + j;
          const int word = jj / G::WORD_W, jw = jj - word * G::WORD_W;
          const int o = word * G::WORD_W + word_pos<BITS, CB>(jw);
          dst[((o >> 3) * 32 + l) * 8 + (o & 7)] = __float2half_rn(ldexpf(v[j], -e));
        }
      }
    }
  }
  __syncthreads();
  pdl_launch_dependents();

  if (u_begin >= u_end) return;
  const char* lut_lane = lut + lane * (BITS == 2 ? 8 : 4);

  float acc[kR][MT];
#pragma unroll
  for (int r = 0; r < kR; ++r)
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[r][m] = 0.f;

  uint32_t rg = first_rg;
  uint32_t ch = u_begin - rg * a.chunks;
  bool started_here = ch == 0;

  for (uint32_t base = u_begin; base < u_end; base += D) {
#pragma unroll
    for (int d = 0; d < D; ++d) {
      const uint32_t u = base + d;
      if (u < u_end) {
        const Stage cur = st[d];
        if (u + D < u_end) {
          load_stage<BITS, DQ>(st[d], a, pf, lane);
          advance(pf, a.chunks);
        }
        const uint32_t boff = ch * 512u + lane * 16u;
        if (boff < (uint32_t)a.q.row_bytes) {
          const uint32_t sp = ch * 32 + lane;
          float2 fx[MT];
#pragma unroll
          for (int m = 0; m < MT; ++m) fx[m] = sx[m * n_spans + sp];
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            if (m < a.mt) {
              const uint4* xv = reinterpret_cast<const uint4*>(xs + m * x_tok + (int64_t)ch * G::CHUNK_W) + lane;
              uint4 xl[G::VEC];  // vector v of this lane sits v*32 uint4s further
#pragma unroll
              for (int v = 0; v < G::VEC; ++v) xl[v] = xv[v * 32];
#pragma unroll
              for (int r = 0; r < kR; ++r) {
                const uint32_t wq[4] = {cur.w[r].x, cur.w[r].y, cur.w[r].z, cur.w[r].w};
                float p0 = 0.f, p1 = 0.f;
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                  const float2 f2 = __half22float2(word_dot<BITS, CB>(wq[w], xl, w, lut_lane));
                  p0 += f2.x;
                  p1 += f2.y;
                }
                const float2 sg = decode_meta<DQ>(cur.m[r]);
                const float gprime = fmaf(center, sg.x, sg.y);
                acc[r][m] = fmaf(sg.x * fx[m].x, p0 + p1, fmaf(gprime, fx[m].y, acc[r][m]));
              }
            }
          }
        }
        const bool last_chunk = ch == a.chunks - 1;
        if (last_chunk || u == u_end - 1) {
          // ---- flush this row group ----
          float tot[kR][MT];
#pragma unroll
          for (int r = 0; r < kR; ++r)
#pragma unroll
            for (int m = 0; m < MT; ++m) {
              tot[r][m] = warp_sum(acc[r][m]);
              acc[r][m] = 0.f;
            }
          if (started_here && last_chunk) {
            finish_rows<MT>(a, rg, tot, lane);
          } else {
            const int slot = (rg == first_rg) ? 0 : 1;
            float* mine = a.partials + ((size_t)gw * 2 + slot) * (kR * MT);
#pragma unroll
            for (int r = 0; r < kR; ++r)
#pragma unroll
              for (int m = 0; m < MT; ++m)
                if (lane == r * MT + m) mine[r * MT + m] = tot[r][m];
            __threadfence();
            __syncwarp();
            int old = 0;
            if (lane == 0) old = atomicAdd(a.counters + rg, 1);
            old = __shfl_sync(0xffffffffu, old, 0);
            // pieces = distinct non-empty warps owning this row group's units
            const uint64_t u0 = (uint64_t)rg * a.chunks;
            int pieces = 1;
            for (uint32_t c = 1, prev = warp_of(u0, U, W); c < a.chunks; ++c) {
              const uint32_t w = warp_of(u0 + c, U, W);
              pieces += w != prev;
              prev = w;
            }
            if (old == pieces - 1) {
              __threadfence();
#pragma unroll
              for (int r = 0; r < kR; ++r)
#pragma unroll
                for (int m = 0; m < MT; ++m) tot[r][m] = 0.f;
              for (uint32_t c = 0, prev = 0xFFFFFFFFu; c < a.chunks; ++c) {
                const uint32_t pw = warp_of(u0 + c, U, W);
                if (pw == prev) continue;
                prev = pw;
                const uint32_t pfirst = (uint32_t)((U * pw / W) / a.chunks);
                const float* src = a.partials + ((size_t)pw * 2 + (rg == pfirst ? 0 : 1)) * (kR * MT);
#pragma unroll
                for (int r = 0; r < kR; ++r)
#pragma unroll
                  for (int m = 0; m < MT; ++m) tot[r][m] += __ldcg(src + r * MT + m);
              }
              finish_rows<MT>(a, rg, tot, lane);
              if (lane == 0) a.counters[rg] = 0;
            }
          }
        }
        if (last_chunk) {
          ++rg;
          ch = 0;
          started_here = true;
        } else {
          ++ch;
        }
      }
    }
  }
}

}  // namespace gemv

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

template <int BITS, bool CB, bool DQ, int MT>
int launch_one(const gemv::Args& a, int blocks_per_sm_cap, cudaStream_t stream, size_t smem) {
  auto kern = gemv::qgemv_kernel<BITS, CB, DQ, MT>;
  static thread_local int configured_dev = -1;
  static thread_local size_t configured_smem = 0;
  int dev = 0;
  TS_CUDA_TRY(cudaGetDevice(&dev));
  if (configured_dev != dev || configured_smem < smem) {
    TS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    configured_dev = dev;
    configured_smem = smem;
  }
  const int grid = (int)(a.total_warps / gemv::kWarps);
  (void)blocks_per_sm_cap;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(gemv::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  TS_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a));
  count_launch();
  return TS_OK;
}

template <int BITS, bool CB, bool DQ>
int launch_mt(int mt, const gemv::Args& a, cudaStream_t s, size_t smem) {
  if (mt <= 1) return launch_one<BITS, CB, DQ, 1>(a, 0, s, smem);
  if (mt <= 2) return launch_one<BITS, CB, DQ, 2>(a, 0, s, smem);
  return launch_one<BITS, CB, DQ, 4>(a, 0, s, smem);
}

template <int BITS>
int launch_bits(bool cb, bool dq, int mt, const gemv::Args& a, cudaStream_t s, size_t smem) {
  if (cb) return dq ? launch_mt<BITS, true, true>(mt, a, s, smem) : launch_mt<BITS, true, false>(mt, a, s, smem);
  return dq ? launch_mt<BITS, false, true>(mt, a, s, smem) : launch_mt<BITS, false, false>(mt, a, s, smem);
}

int pick_mt(int64_t tokens) {
  return tokens <= 1 ? 1 : tokens <= 2 ? 2 : 4;
}

}  // namespace

static int ilog2(int64_t v) {
  int r = 0;
  while ((int64_t(1) << (r + 1)) <= v) ++r;
  return r;
}

// Whether the fast GEMV covers this weight layout.
bool gemv_supported(const ts_qweight& w) {
  const int64_t gbytes = (int64_t)w.group_size * w.bits / 8;
  return (w.bits == 2 || w.bits == 4 || w.bits == 8) && gbytes % 16 == 0 &&
         (gbytes & (gbytes - 1)) == 0 && w.rows * w.n_groups < (int64_t(1) << 31) &&
         w.packed_row_bytes < (int64_t(1) << 30) &&
         w.packed_row_bytes % 16 == 0 && is_aligned(w.packed, 16) &&
         w.padded_cols % (128 / w.bits) == 0 && w.packed_row_bytes * 8 / w.bits >= w.padded_cols;
}

static int gemv_grid_warps() { return sm_count() * 2 * gemv::kWarps; }

size_t gemv_workspace_size(const ts_qweight& w) {
  const int64_t rgs = (w.rows + gemv::kR - 1) / gemv::kR;
  return align_up((size_t)rgs * sizeof(int), 256) +
         (size_t)gemv_grid_warps() * 2 * gemv::kR * 4 * sizeof(float);
}

static size_t gemv_smem(const ts_qweight& w, int mt) {
  const int span = 128 / w.bits;
  const int64_t chunk_w = 32 * span;
  const int64_t n_chunks = (w.padded_cols + chunk_w - 1) / chunk_w;
  size_t lut = w.codebook ? (w.bits == 2 ? 256 * 32 * 8 : 256 * 32 * 4) : 0;
  return lut + (size_t)mt * n_chunks * chunk_w * 2 + (size_t)mt * n_chunks * 32 * sizeof(float2);
}

// Largest token count per pass whose staged activations fit in shared memory.
int gemv_max_tokens(const ts_qweight& w) {
  const size_t cap = (size_t)std::min(max_smem_optin(), 200 * 1024);
  for (int mt : {4, 2, 1})
    if (gemv_smem(w, mt) <= cap) return mt;
  return 0;
}

int run_gemv(const ts_qweight& w, const void* x, int x_dtype, int64_t M, int64_t x_stride,
             const void* bias, int bias_dtype, void* out, int out_dtype, int64_t out_stride,
             void* workspace, size_t ws_bytes, cudaStream_t stream) {
  const int max_mt = gemv_max_tokens(w);
  TS_UNSUPPORTED(max_mt > 0, "qlinear: activations of %lld columns do not fit in shared memory",
                 (long long)w.cols);
  TS_REQUIRE(ws_bytes >= gemv_workspace_size(w), "qlinear: workspace too small (%zu < %zu)",
             ws_bytes, gemv_workspace_size(w));
  gemv::Args a;
  a.q = make_qw(w);
  a.x = x;
  a.x_dtype = x_dtype;
  a.x_stride = x_stride;
  a.bias = bias;
  a.bias_dtype = bias_dtype;
  a.out = out;
  a.out_dtype = out_dtype;
  a.out_stride = out_stride;
  const int64_t rgs = (w.rows + gemv::kR - 1) / gemv::kR;
  a.counters = reinterpret_cast<int*>(workspace);
  a.partials = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) +
                                        align_up((size_t)rgs * sizeof(int), 256));
  a.chunks = (uint32_t)((w.packed_row_bytes + 511) / 512);
  a.units = (uint32_t)(rgs * a.chunks);
  a.total_warps = (uint32_t)gemv_grid_warps();
  const int64_t chunk_w = 32 * (128 / w.bits);
  a.n_chunks_x = (int)((w.padded_cols + chunk_w - 1) / chunk_w);
  a.center = w.bits == 4 ? 8.f : w.bits == 2 ? 2.f : 128.f;  // codebooks: set in-kernel
  a.x_vec16 = is_aligned(x, 16) && (x_stride * 2) % 16 == 0;
  a.gbytes_shift = ilog2((int64_t)w.group_size * w.bits / 8);
  a.dq_shift = (w.dq_scale_codes && (w.dq_group_size & (w.dq_group_size - 1)) == 0)
                   ? ilog2(w.dq_group_size) : -1;
  for (int64_t m0 = 0; m0 < M; m0 += max_mt) {
    const int64_t tokens = std::min<int64_t>(max_mt, M - m0);
    const int mt = pick_mt(tokens);
    a.m0 = m0;
    a.mt = (int)tokens;
    const size_t smem = gemv_smem(w, mt);
    int rc;
    if (w.bits == 4)
      rc = launch_bits<4>(w.codebook != nullptr, w.dq_scale_codes != nullptr, mt, a, stream, smem);
    else if (w.bits == 2)
      rc = launch_bits<2>(w.codebook != nullptr, w.dq_scale_codes != nullptr, mt, a, stream, smem);
    else
      rc = launch_bits<8>(w.codebook != nullptr, w.dq_scale_codes != nullptr, mt, a, stream, smem);
    if (rc != TS_OK) return rc;
  }
  return TS_OK;
}

}  // namespace ts
