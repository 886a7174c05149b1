// GOAP quantize + pack on the GPU.
//
// Restates, as a handful of bandwidth-bound passes over the weight, the
// reference codec (tensorshrink codec.py:453-675) that gpu_quantize.py:52-166
// runs as a chain of torch ops:
//
//   pass A  stats_kernel      per-group min/max of the unclamped weight and
//                             the first-level histogram of |w| bit patterns
//   (fp32)  prefix_hist       second-level histogram (31-bit keys only)
//   pass B  cta_hist_kernel   last-level histogram, one per CTA row range
//   select  finalize_select   exact threshold T = k-th largest |w|, and each
//                             CTA's output offset and share of the ties
//   pass C  quantize_kernel   clamp to +-T, group affine, code assignment,
//                             bit packing, fp16 scale/gmin, ordered outlier
//                             index/value compaction
//   pass D  double_quant      double quantization of scale/gmin
//   pass E  outlier_tables    row/col split, fp16 delta, CSR row offsets
//
// Top-k is a radix select over the magnitude bit pattern (|w| as an unsigned
// integer orders like |w| as a float). Clipping commutes with min/max, so the
// group range of the clamped weight is clamp(range of the raw weight) and
// pass A need not wait for T. Ties at T keep the lowest flat indices.
// Every floating-point step uses explicitly rounded intrinsics in the
// reference's order (subtract, then IEEE divide; round-half-even), so codes,
// packed bytes, double-quant codes and deltas are bit-identical to it.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"

namespace ts {

int run_lloyd(const float* vals, int64_t n, int n_levels, int iters, float* out, uint16_t* out16,
              char* ws, cudaStream_t stream, size_t off_state, size_t off_mm);

namespace qz {

constexpr int kThreads = 256;

__host__ __device__ __forceinline__ int64_t i64max(int64_t a, int64_t b) { return a > b ? a : b; }
__host__ __device__ __forceinline__ int64_t i64min(int64_t a, int64_t b) { return a < b ? a : b; }

template <int DT>
struct Elem;
template <>
struct Elem<TS_F16> {
  static constexpr int KEY_BITS = 15, L1_BITS = 8, L2_BITS = 0, LAST_BITS = 7;
  __device__ static float val(const void* p, int64_t i) {
    return __half2float(reinterpret_cast<const __half*>(p)[i]);
  }
  __device__ static uint32_t key(const void* p, int64_t i) {
    return reinterpret_cast<const uint16_t*>(p)[i] & 0x7FFFu;
  }
};
template <>
struct Elem<TS_BF16> {
  static constexpr int KEY_BITS = 15, L1_BITS = 8, L2_BITS = 0, LAST_BITS = 7;
  __device__ static float val(const void* p, int64_t i) {
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  }
  __device__ static uint32_t key(const void* p, int64_t i) {
    return reinterpret_cast<const uint16_t*>(p)[i] & 0x7FFFu;
  }
};
template <>
struct Elem<TS_F32> {
  static constexpr int KEY_BITS = 31, L1_BITS = 11, L2_BITS = 10, LAST_BITS = 10;
  __device__ static float val(const void* p, int64_t i) { return reinterpret_cast<const float*>(p)[i]; }
  __device__ static uint32_t key(const void* p, int64_t i) {
    return reinterpret_cast<const uint32_t*>(p)[i] & 0x7FFFFFFFu;
  }
};

// Radix-select state shared between the passes (device workspace).
struct SelState {
  uint32_t prefix;      // selected key bits above the current level
  int64_t k_rem;        // rank still to be found below `prefix`
  uint32_t t_key;       // final threshold key
  float t_val;          // |w| at the threshold
  int64_t n_gt;         // elements strictly above T
  int64_t need_eq;      // ties to keep
  uint32_t floor_bin;   // pass A histograms only first-level bins >= this (a sampled lower bound of T)
  int redo;             // the bound was too high: the bins below it are counted by the redo pass
};

struct Geometry {
  const void* w;
  int64_t rows, cols, padded_cols, n_groups, n8;  // n8 = padded_cols / 8 (items per row)
  int gs, bits;
  int gs_shift;       // log2(gs) (group sizes are powers of two)
  uint64_t n8_magic;  // ceil(2^64 / n8) (0 when n8 == 1): row of item i = umul64hi(i, magic)
  int vec;            // rows are whole 16-byte vectors of 8 elements (cols % 8 == 0, aligned)
};

// Row of a flat item index: exact for i * n8 < 2^64 (multiply-high by the
// rounded-up reciprocal instead of a 64-bit division per item).
__device__ __forceinline__ int64_t row_of(const Geometry& g, int64_t i) {
  return g.n8_magic ? (int64_t)__umul64hi((uint64_t)i, g.n8_magic) : i;
}

// 8 consecutive elements of row r starting at column c0 as fp32 values and
// magnitude keys; columns past the end repeat the last column (codec.py:556
// pads with the last column).
template <int DT>
__device__ __forceinline__ void load8(const Geometry& g, int64_t r, int64_t c0, float (&v)[8], uint32_t (&k)[8]) {
  if (g.vec && c0 + 8 <= g.cols) {
    const int64_t e0 = r * g.cols + c0;
    if (DT == TS_F32) {
      const uint4 u0 = ldg_stream_v4(reinterpret_cast<const float*>(g.w) + e0);
      const uint4 u1 = ldg_stream_v4(reinterpret_cast<const float*>(g.w) + e0 + 4);
      const uint32_t b[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[j] = __uint_as_float(b[j]);
        k[j] = b[j] & 0x7FFFFFFFu;
      }
    } else {
      const uint4 u = ldg_stream_v4(reinterpret_cast<const uint16_t*>(g.w) + e0);
      const uint32_t b[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t h = (b[j >> 1] >> (16 * (j & 1))) & 0xFFFFu;
        v[j] = DT == TS_F16 ? __half2float(__ushort_as_half((uint16_t)h)) : __uint_as_float(h << 16);
        k[j] = h & 0x7FFFu;
      }
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int64_t c = c0 + j;
    const int64_t src = r * g.cols + (c < g.cols ? c : g.cols - 1);
    v[j] = Elem<DT>::val(g.w, src);
    k[j] = Elem<DT>::key(g.w, src);
  }
}

__device__ __forceinline__ float group_reduce_min(float v, int width) {
  for (int o = width / 2; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float group_reduce_max(float v, int width) {
  for (int o = width / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---- pass A ------------------------------------------------------------------
// Per-group min/max of the raw weight, and the first-level histogram of the
// magnitude keys. Only bins >= st->floor_bin are counted: the threshold lies
// at or above that bin whenever the counted elements number at least k
// (checked by the first select, which otherwise has the redo pass count the
// bins below). Few elements clear the bound, so few shared-memory atomics
// are issued.
template <int DT>
__global__ void __launch_bounds__(kThreads) stats_kernel(const Geometry g, float* gmin_raw,
                                                         float* gmax_raw, uint32_t* hist1,
                                                         int do_hist, const SelState* st) {
  using E = Elem<DT>;
  constexpr int NB = 1 << E::L1_BITS;
  constexpr int SH = E::KEY_BITS - E::L1_BITS;
  __shared__ uint32_t h[NB];
  if (do_hist)
    for (int i = threadIdx.x; i < NB; i += kThreads) h[i] = 0;
  __syncthreads();
  const uint32_t floor_bin = do_hist ? st->floor_bin : 0u;
  const int gw = g.gs / 8;  // threads per group (power of two <= 32)
  const int64_t items = g.rows * g.n8;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  for (int64_t base = (int64_t)blockIdx.x * kThreads; base < items; base += stride) {
    const int64_t it = base + threadIdx.x;
    float mn = INFINITY, mx = -INFINITY;
    int64_t r = 0, c0 = 0;
    if (it < items) {
      r = row_of(g, it);
      c0 = (it - r * g.n8) * 8;
      if (DT != TS_F32 && g.vec && c0 + 8 <= g.cols) {
        // 8 16-bit values: min/max on packed pairs (exact), keys from the raw bits
        const uint4 u = ldg_stream_v4(reinterpret_cast<const uint16_t*>(g.w) + r * g.cols + c0);
        const uint32_t b[4] = {u.x, u.y, u.z, u.w};
        if (DT == TS_F16) {
          __half2 lo = __hmin2(__hmin2(*reinterpret_cast<const __half2*>(&b[0]), *reinterpret_cast<const __half2*>(&b[1])),
                               __hmin2(*reinterpret_cast<const __half2*>(&b[2]), *reinterpret_cast<const __half2*>(&b[3])));
          __half2 hi = __hmax2(__hmax2(*reinterpret_cast<const __half2*>(&b[0]), *reinterpret_cast<const __half2*>(&b[1])),
                               __hmax2(*reinterpret_cast<const __half2*>(&b[2]), *reinterpret_cast<const __half2*>(&b[3])));
          mn = fminf(__low2float(lo), __high2float(lo));
          mx = fmaxf(__low2float(hi), __high2float(hi));
        } else {
          using B2 = __nv_bfloat162;
          B2 lo = __hmin2(__hmin2(*reinterpret_cast<const B2*>(&b[0]), *reinterpret_cast<const B2*>(&b[1])),
                          __hmin2(*reinterpret_cast<const B2*>(&b[2]), *reinterpret_cast<const B2*>(&b[3])));
          B2 hi = __hmax2(__hmax2(*reinterpret_cast<const B2*>(&b[0]), *reinterpret_cast<const B2*>(&b[1])),
                          __hmax2(*reinterpret_cast<const B2*>(&b[2]), *reinterpret_cast<const B2*>(&b[3])));
          mn = fminf(__low2float(lo), __high2float(lo));
          mx = fmaxf(__low2float(hi), __high2float(hi));
        }
        if (do_hist) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t bin = ((b[j >> 1] >> (16 * (j & 1))) & 0x7FFFu) >> SH;
            if (bin >= floor_bin) atomicAdd(&h[bin], 1u);
          }
        }
      } else {
        float v[8];
        uint32_t k[8];
        load8<DT>(g, r, c0, v, k);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          mn = fminf(mn, v[j]);
          mx = fmaxf(mx, v[j]);
          if (do_hist && c0 + j < g.cols && (k[j] >> SH) >= floor_bin) atomicAdd(&h[k[j] >> SH], 1u);
        }
      }
    }
    mn = group_reduce_min(mn, gw);
    mx = group_reduce_max(mx, gw);
    if (it < items && (threadIdx.x & (gw - 1)) == 0) {
      const int64_t grp = c0 >> g.gs_shift;
      gmin_raw[r * g.n_groups + grp] = mn;
      gmax_raw[r * g.n_groups + grp] = mx;
    }
  }
  if (do_hist) {
    __syncthreads();
    for (int i = threadIdx.x; i < NB; i += kThreads)
      if (h[i]) atomicAdd(hist1 + i, h[i]);
  }
}

// Lower bound of the threshold's first-level bin from a fixed, evenly spaced
// sample of the keys (one block): the highest bin b such that the sampled
// keys in bins >= b are at least 8x the expected share of the k largest plus
// 64. Pass A then counts exactly the elements in bins >= b; if those number
// fewer than k (the sample misled), the redo pass counts the rest, so the
// selected threshold is exact either way.
constexpr int kSampleThreads = 1024;
constexpr int kSamplePerThread = 4;
constexpr int kSample = kSampleThreads * kSamplePerThread;

template <int DT>
__global__ void __launch_bounds__(kSampleThreads) sample_bound_kernel(const Geometry g, int64_t k, SelState* st) {
  using E = Elem<DT>;
  constexpr int NB = 1 << E::L1_BITS;
  constexpr int SH = E::KEY_BITS - E::L1_BITS;
  __shared__ uint32_t h[NB];
  for (int i = threadIdx.x; i < NB; i += kSampleThreads) h[i] = 0;
  __syncthreads();
  const int64_t n = g.rows * g.cols;
  const int64_t S = n < kSample ? n : kSample;
  const int64_t step = n / S;   // sample si is element si * step
  uint32_t kk[kSamplePerThread];
#pragma unroll
  for (int j = 0; j < kSamplePerThread; ++j) {   // all loads first, then the counts
    const int64_t si = threadIdx.x + (int64_t)j * kSampleThreads;
    kk[j] = si < S ? E::key(g.w, si * step) : 0xFFFFFFFFu;
  }
#pragma unroll
  for (int j = 0; j < kSamplePerThread; ++j)
    if (kk[j] != 0xFFFFFFFFu) atomicAdd(&h[kk[j] >> SH], 1u);
  __syncthreads();
  if (threadIdx.x == 0) {
    const double want = 8.0 * (double)k * (double)S / (double)n + 64.0;
    uint32_t b = 0;
    if (want < (double)S) {
      uint64_t acc = 0;
      for (int bb = NB - 1; bb >= 0; --bb) {
        acc += h[bb];
        if ((double)acc >= want) { b = (uint32_t)bb; break; }
      }
    }
    st->floor_bin = b;
    st->redo = 0;
  }
}

// Redo pass: counts the first-level bins below the sampled bound when the
// bins above it held fewer than k elements (never, in practice; every CTA
// returns at once otherwise).
template <int DT>
__global__ void __launch_bounds__(kThreads) redo_hist_kernel(const Geometry g, uint32_t* hist1, const SelState* st) {
  if (!st->redo) return;
  using E = Elem<DT>;
  constexpr int NB = 1 << E::L1_BITS;
  constexpr int SH = E::KEY_BITS - E::L1_BITS;
  __shared__ uint32_t h[NB];
  for (int i = threadIdx.x; i < NB; i += kThreads) h[i] = 0;
  __syncthreads();
  const uint32_t floor_bin = st->floor_bin;
  const int64_t n = g.rows * g.cols;
  for (int64_t i = blockIdx.x * (int64_t)kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads) {
    const uint32_t bin = E::key(g.w, i) >> SH;
    if (bin < floor_bin) atomicAdd(&h[bin], 1u);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < NB; i += kThreads)
    if (h[i]) atomicAdd(hist1 + i, h[i]);
}

// Find the bin holding rank k (1-based, counted from the largest) of a
// histogram, given the count already above it. One block.
__device__ void select_bin(const uint32_t* hist, int nb, int64_t k, int* bin_out, int64_t* above_out) {
  __shared__ int64_t s_above;
  __shared__ int s_bin;
  if (threadIdx.x == 0) {
    int64_t acc = 0;
    int b = nb - 1;
    for (; b >= 0; --b) {
      if (acc + hist[b] >= k) break;
      acc += hist[b];
    }
    s_bin = b < 0 ? 0 : b;
    s_above = acc;
  }
  __syncthreads();
  *bin_out = s_bin;
  *above_out = s_above;
}

__global__ void select_level_kernel(const uint32_t* hist, int nb, SelState* st, int first,
                                    int64_t k, int level_bits) {
  int b;
  int64_t above;
  const int64_t kk = first ? k : st->k_rem;
  // one warp: lane t sums the t-th chunk of bins counted from the top, an
  // inclusive scan finds the chunk where the count from the top reaches kk,
  // and that lane walks its chunk
  const int lane = threadIdx.x;
  const int chunk = (nb + 31) / 32;
  const int hi = nb - lane * chunk, lo = max(0, hi - chunk);
  int64_t sum = 0;
  for (int i = lo; i < hi; ++i) sum += hist[i];
  int64_t incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  const int64_t tot = __shfl_sync(0xffffffffu, incl, 31);
  if (first) {
    // the first level's histogram counts only bins >= floor_bin: it must
    // hold at least k elements, else the redo pass adds the bins below
    if (tot < kk) {
      if (lane == 0) st->redo = 1;
      return;
    }
    if (lane == 0) st->redo = 0;
  }
  const unsigned hit = __ballot_sync(0xffffffffu, incl >= kk);
  const int owner = hit ? __ffs(hit) - 1 : 31;
  b = 0;
  above = tot;
  if (lane == owner) {
    int64_t acc = incl - sum;
    for (int i = hi - 1; i >= lo; --i) {
      if (acc + hist[i] >= kk) { b = i; break; }
      acc += hist[i];
    }
    above = acc;
  }
  b = __shfl_sync(0xffffffffu, b, owner);
  above = __shfl_sync(0xffffffffu, above, owner);
  if (threadIdx.x == 0) {
    st->prefix = first ? (uint32_t)b : ((st->prefix << level_bits) | (uint32_t)b);
    st->k_rem = kk - above;
  }
}

// ---- fp32 only: second level ---------------------------------------------------
__global__ void __launch_bounds__(kThreads) prefix_hist_kernel(const Geometry g, const SelState* st,
                                                               uint32_t* hist2) {
  using E = Elem<TS_F32>;
  constexpr int NB = 1 << E::L2_BITS;
  __shared__ uint32_t h[NB];
  for (int i = threadIdx.x; i < NB; i += kThreads) h[i] = 0;
  __syncthreads();
  const uint32_t prefix = st->prefix;
  const int64_t n = g.rows * g.cols;
  for (int64_t i = blockIdx.x * (int64_t)kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads) {
    const uint32_t key = E::key(g.w, i);
    if ((key >> (E::KEY_BITS - E::L1_BITS)) == prefix)
      atomicAdd(&h[(key >> E::LAST_BITS) & (NB - 1)], 1u);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < NB; i += kThreads)
    if (h[i]) atomicAdd(hist2 + i, h[i]);
}

// CTA c of passes B and C owns rows [c*rows_per_cta, ...).
struct CtaPlan {
  int64_t rows_per_cta;
  int n_cta;
};

// ---- pass B --------------------------------------------------------------------
template <int DT>
__global__ void __launch_bounds__(kThreads) cta_hist_kernel(const Geometry g, const CtaPlan plan,
                                                            const SelState* st, uint32_t* cta_hist) {
  using E = Elem<DT>;
  constexpr int NB = 1 << E::LAST_BITS;
  __shared__ uint32_t h[NB + 1];
  for (int i = threadIdx.x; i <= NB; i += kThreads) h[i] = 0;
  __syncthreads();
  const uint32_t prefix = st->prefix;
  const int64_t r0 = blockIdx.x * plan.rows_per_cta;
  const int64_t r1 = min(g.rows, r0 + plan.rows_per_cta);
  uint32_t above = 0;
  if (g.vec) {
    // 8 keys per 16/32-byte vector (the range starts on a row, rows are whole vectors)
    // two vectors per thread per iteration, both loads issued first
    const int64_t e_end = r1 * g.cols;
    for (int64_t e0 = r0 * g.cols + 8 * (int64_t)threadIdx.x; e0 < e_end; e0 += 16 * kThreads) {
      uint32_t k[2][8];
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int64_t e = e0 + h2 * 8 * kThreads;
        if (e >= e_end) {
#pragma unroll
          for (int j = 0; j < 8; ++j) k[h2][j] = 0u;
          continue;
        }
        if (DT == TS_F32) {
          const uint4 u0 = ldg_stream_v4(reinterpret_cast<const float*>(g.w) + e);
          const uint4 u1 = ldg_stream_v4(reinterpret_cast<const float*>(g.w) + e + 4);
          const uint32_t b[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
          for (int j = 0; j < 8; ++j) k[h2][j] = b[j] & 0x7FFFFFFFu;
        } else {
          const uint4 u = ldg_stream_v4(reinterpret_cast<const uint16_t*>(g.w) + e);
          const uint32_t b[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int j = 0; j < 8; ++j) k[h2][j] = (b[j >> 1] >> (16 * (j & 1))) & 0x7FFFu;
        }
      }
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        if (e0 + h2 * 8 * kThreads >= e_end) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t hi = k[h2][j] >> E::LAST_BITS;
          if (hi > prefix)
            ++above;
          else if (hi == prefix)
            atomicAdd(&h[k[h2][j] & (NB - 1)], 1u);
        }
      }
    }
  } else {
    for (int64_t i = r0 * g.cols + threadIdx.x; i < r1 * g.cols; i += kThreads) {
      const uint32_t key = E::key(g.w, i);
      const uint32_t hi = key >> E::LAST_BITS;
      if (hi > prefix)
        ++above;
      else if (hi == prefix)
        atomicAdd(&h[key & (NB - 1)], 1u);
    }
  }
  atomicAdd(&h[NB], above);
  __syncthreads();
  uint32_t* dst = cta_hist + (size_t)blockIdx.x * (NB + 1);
  for (int i = threadIdx.x; i <= NB; i += kThreads) dst[i] = h[i];
}

// ---- select: threshold, per-CTA offsets and tie shares ----------------------
// One block of 1024 threads (n_cta <= 1024 by the CTA plan). The bin totals
// are summed by (bin, CTA slice) pairs; the threshold bin is found by one
// thread walking at most 1024 bins in shared memory; each thread then counts
// one CTA's elements above the threshold and ties at it, and two block-wide
// exclusive scans turn those into output offsets and tie shares (ties are
// granted in CTA order, i.e. lowest flat indices first).
constexpr int kSelThreads = 1024;

__device__ __forceinline__ int64_t block_excl_scan64(int64_t v, int64_t* warp_tot /* [32] */) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int64_t incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) warp_tot[wid] = incl;
  __syncthreads();
  if (wid == 0) {
    int64_t w = lane < (int)(blockDim.x >> 5) ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t t = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += t;
    }
    warp_tot[lane] = w;   // inclusive prefix over warps
  }
  __syncthreads();
  const int64_t r = incl - v + (wid > 0 ? warp_tot[wid - 1] : 0);
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kSelThreads) finalize_select_kernel(const uint32_t* cta_hist, int nb, int n_cta,
                                                                      SelState* st,
                                                                      int64_t* cta_info /* [n_cta][2] */,
                                                                      int key_bits, int dtype) {
  extern __shared__ uint32_t tot[];  // nb
  __shared__ int64_t warp_tot[32];
  for (int b = threadIdx.x; b < nb; b += blockDim.x) tot[b] = 0;
  __syncthreads();
  {
    const int slices = blockDim.x >= (unsigned)nb ? (int)blockDim.x / nb : 1;
    const int b = threadIdx.x % nb, sl = threadIdx.x / nb;
    if (sl < slices) {
      uint32_t sum = 0;
      for (int c = sl; c < n_cta; c += slices) sum += cta_hist[(size_t)c * (nb + 1) + b];
      atomicAdd(&tot[b], sum);
    }
    for (int bb = b + slices * nb; bb < nb; bb += blockDim.x) {   // nb > blockDim: remaining bins
      uint32_t sum2 = 0;
      for (int c = 0; c < n_cta; ++c) sum2 += cta_hist[(size_t)c * (nb + 1) + bb];
      atomicAdd(&tot[bb], sum2);
    }
  }
  __syncthreads();
  int bin;
  int64_t above_in_level;
  select_bin(tot, nb, st->k_rem, &bin, &above_in_level);
  const int64_t need = st->k_rem - above_in_level;  // ties needed within the bin
  int64_t gt = 0, eq = 0;
  const int c = threadIdx.x;
  if (c < n_cta) {
    const uint32_t* h = cta_hist + (size_t)c * (nb + 1);
    gt = h[nb];
#pragma unroll 8
    for (int b = bin + 1; b < nb; ++b) gt += h[b];
    eq = h[bin];
  }
  const int64_t eq_before = block_excl_scan64(eq, warp_tot);
  const int64_t take = i64max(0, i64min(eq, need - eq_before));
  const int64_t off = block_excl_scan64(gt + take, warp_tot);
  const int64_t n_gt_before = block_excl_scan64(gt, warp_tot);
  if (c < n_cta) {
    cta_info[2 * c] = off;
    cta_info[2 * c + 1] = take;
  }
  if (c == n_cta - 1) st->n_gt = n_gt_before + gt;
  if (threadIdx.x == 0) {
    const uint32_t tkey = (st->prefix << (31 - __clz(nb))) | (uint32_t)bin;
    st->t_key = tkey;
    if (dtype == TS_F16)
      st->t_val = __half2float(__ushort_as_half((uint16_t)tkey));
    else if (dtype == TS_BF16)
      st->t_val = __bfloat162float(__ushort_as_bfloat16((uint16_t)tkey));
    else
      st->t_val = __uint_as_float(tkey);
    (void)key_bits;
    st->need_eq = need;
  }
}

// ---- pass C ----------------------------------------------------------------------
struct QuantArgs {
  Geometry g;
  CtaPlan plan;
  const SelState* st;       // nullptr when there are no outliers
  const int64_t* cta_info;
  const float* gmin_raw;
  const float* gmax_raw;
  const float* cb;          // sorted fp32 codebook for assignment or nullptr (uniform)
  int n_levels;
  uint8_t* packed;
  int64_t row_bytes;
  uint16_t* scale;
  uint16_t* gmin;
  int32_t* out_idx;
  uint16_t* out_val;
  int w_dtype;
  int prefetch;             // issue the next item's loads before processing this one
};

template <int DT>
__device__ __forceinline__ uint32_t elem_key(const void* w, int64_t i) {
  return Elem<DT>::key(w, i);
}

__device__ __forceinline__ int block_excl_scan(int v, int* total) {
  __shared__ int warp_tot[kThreads / 32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) warp_tot[wid] = incl;
  __syncthreads();
  int wbase = 0, all = 0;
  for (int i = 0; i < kThreads / 32; ++i) {
    if (i < wid) wbase += warp_tot[i];
    all += warp_tot[i];
  }
  __syncthreads();
  *total = all;
  return wbase + incl - v;
}

template <int DT>
__global__ void __launch_bounds__(kThreads) quantize_kernel(const QuantArgs a) {
  using E = Elem<DT>;
  const Geometry& g = a.g;
  __shared__ float s_cb_mid[256];
  __shared__ float s_cb[256];
  if (a.cb) {
    for (int i = threadIdx.x; i < a.n_levels; i += kThreads) s_cb[i] = a.cb[i];
    __syncthreads();
    for (int i = threadIdx.x; i + 1 < a.n_levels; i += kThreads)
      s_cb_mid[i] = __fmul_rn(__fadd_rn(s_cb[i], s_cb[i + 1]), 0.5f);  // codec.py:370
    __syncthreads();
  }
  const bool has_t = a.st != nullptr;
  const uint32_t tkey = has_t ? a.st->t_key : 0xFFFFFFFFu;
  const float tval = has_t ? a.st->t_val : INFINITY;
  int64_t out_pos = 0, tie_left = 0;
  if (has_t) {
    out_pos = a.cta_info[2 * blockIdx.x];
    tie_left = a.cta_info[2 * blockIdx.x + 1];
  }
  const float levels = (float)((1 << g.bits) - 1);
  const int levels_i = (1 << g.bits) - 1;
  const int64_t r0 = blockIdx.x * a.plan.rows_per_cta;
  const int64_t r1 = min(g.rows, r0 + a.plan.rows_per_cta);
  const int64_t it0 = r0 * g.n8, it1 = r1 * g.n8;
  // software pipeline (a.prefetch): the next item's loads are issued before
  // this item is processed, so two loads per thread are in flight
  float vn[8];
  uint32_t kn[8];
  if (a.prefetch && it0 + threadIdx.x < it1) {
    const int64_t rr = row_of(g, it0 + threadIdx.x);
    load8<DT>(g, rr, (it0 + threadIdx.x - rr * g.n8) * 8, vn, kn);
  }
  for (int64_t base = it0; base < it1; base += kThreads) {
    const int64_t it = base + threadIdx.x;
    const bool live = it < it1;
    int64_t r = 0, c0 = 0;
    float v[8];
    uint32_t keys[8];
    if (a.prefetch) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[j] = vn[j];
        keys[j] = kn[j];
      }
      if (it + kThreads < it1) {
        const int64_t rn = row_of(g, it + kThreads);
        load8<DT>(g, rn, (it + kThreads - rn * g.n8) * 8, vn, kn);
      }
    } else if (live) {
      const int64_t rl = row_of(g, it);
      load8<DT>(g, rl, (it - rl * g.n8) * 8, v, keys);
    }
    int sel_gt = 0, n_eq = 0;
    if (live) {
      r = row_of(g, it);
      c0 = (it - r * g.n8) * 8;
      if (has_t) {
        // almost every item lies wholly below the threshold: one max first
        uint32_t kmax = keys[0];
#pragma unroll
        for (int j = 1; j < 8; ++j) kmax = max(kmax, keys[j]);
        if (kmax >= tkey) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (c0 + j < g.cols) {
              sel_gt += keys[j] > tkey;
              n_eq += keys[j] == tkey;
            }
          }
        }
      }
    }
    // ---- codes ----
    if (live) {
      const int64_t grp = c0 >> g.gs_shift;
      const int64_t gi = r * g.n_groups + grp;
      // clamp(min) / clamp(max) of the raw range == range of the clamped group
      const float gmn = fminf(fmaxf(a.gmin_raw[gi], -tval), tval);
      const float gmx = fminf(fmaxf(a.gmax_raw[gi], -tval), tval);
      float scale = __fdiv_rn(__fsub_rn(gmx, gmn), levels);   // codec.py:570
      scale = fmaxf(scale, 1e-8f);                            // codec.py:571
      // t = (x - gmin) / scale must be the correctly rounded quotient
      // (codec.py:579-580). A product with the reciprocal is within a few
      // ulps of it, so it picks the same code unless it lies within a few
      // ulps of a rounding boundary (a half-integer, or a codebook midpoint);
      // only then is the exact IEEE division done.
      const float rs = __frcp_rn(scale);
      uint32_t codes[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float x = fminf(fmaxf(v[j], -tval), tval);      // codec.py:543
        const float d = __fsub_rn(x, gmn);
        float t = __fmul_rn(d, rs);
        const float tol = fmaxf(fabsf(t), 1.f) * 1e-6f;      // >= 8 ulps of t
        if (a.cb) {
          int lo = 0, hi = a.n_levels - 1;                    // count of mids < t
          while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (s_cb_mid[mid] < t) lo = mid + 1; else hi = mid;
          }
          const bool near = (lo > 0 && fabsf(t - s_cb_mid[lo - 1]) <= tol) ||
                            (lo < a.n_levels - 1 && fabsf(t - s_cb_mid[lo]) <= tol);
          if (near) {
            t = __fdiv_rn(d, scale);
            lo = 0;
            hi = a.n_levels - 1;
            while (lo < hi) {
              const int mid = (lo + hi) >> 1;
              if (s_cb_mid[mid] < t) lo = mid + 1; else hi = mid;
            }
          }
          codes[j] = (uint32_t)lo;
        } else {
          // t >= 0 (x >= the group minimum). Adding 1.5 * 2^23 rounds t to
          // the nearest integer, ties to even, as rintf does, and leaves it
          // in the low mantissa bits; t - rint(t) is exact, and t is within
          // tol of a half-integer exactly when 0.5 - |t - rint(t)| <= tol.
          constexpr float kMagic = 12582912.f;
          float r = __fadd_rn(t, kMagic);
          if (0.5f - fabsf(__fsub_rn(t, __fsub_rn(r, kMagic))) <= tol) {
            t = __fdiv_rn(d, scale);
            r = __fadd_rn(t, kMagic);
          }
          codes[j] = min(__float_as_uint(r) - 0x4B400000u, (uint32_t)levels_i);
        }
      }
      uint8_t* prow = a.packed + r * a.row_bytes;
      if (g.bits == 4) {
        uint32_t wv = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) wv |= codes[j] << (4 * j);
        *reinterpret_cast<uint32_t*>(prow + c0 / 2) = wv;
      } else if (g.bits == 2) {
        uint32_t wv = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) wv |= codes[j] << (2 * j);
        *reinterpret_cast<uint16_t*>(prow + c0 / 4) = (uint16_t)wv;
      } else {
        uint2 wv = make_uint2(0, 0);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          wv.x |= codes[j] << (8 * j);
          wv.y |= codes[j + 4] << (8 * j);
        }
        *reinterpret_cast<uint2*>(prow + c0) = wv;
      }
      if ((c0 & (g.gs - 1)) == 0) {
        a.scale[gi] = f2h(scale);                              // codec.py:637-638
        a.gmin[gi] = f2h(gmn);
      }
    }
    // ---- ordered outlier compaction (index order == thread order) ----
    // One scan of (elements above T) | (ties at T) << 16: a thread's first
    // output slot is the count above T before it plus the ties granted
    // before it (ties go to the lowest indices, up to tie_left).
    if (has_t) {
      int tot;
      const int before = block_excl_scan(sel_gt | (n_eq << 16), &tot);
      const int gt_before = before & 0xFFFF, eq_before = before >> 16;
      const int gt_total = tot & 0xFFFF, eq_total = tot >> 16;
      const int64_t ties_before = i64min((int64_t)eq_before, tie_left);
      int64_t allow = i64max(0, i64min((int64_t)n_eq, tie_left - eq_before));  // ties this thread takes
      if (live && sel_gt + allow > 0) {
        int64_t p = out_pos + gt_before + ties_before;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int64_t c = c0 + j;
          if (c >= g.cols) break;
          bool take = keys[j] > tkey;
          if (!take && keys[j] == tkey && allow > 0) {
            take = true;
            --allow;
          }
          if (take) {
            a.out_idx[p] = (int32_t)(r * g.cols + c);
            a.out_val[p] = f2h(v[j]);
            ++p;
          }
        }
      }
      const int64_t ties_taken = i64min((int64_t)eq_total, tie_left);
      out_pos += gt_total + ties_taken;
      tie_left -= ties_taken;
    }
  }
}

// ---- pass D: double quantization (codec.py:380-417) ---------------------------
// One block per super-group. Reads the fp16 values written by pass C and
// replaces them with their fp16 reconstruction, as codec.py:651-652 does.
__global__ void double_quant_kernel(uint16_t* vals, int64_t n, int dq_gs, uint8_t* codes,
                                    uint16_t* meta) {
  __shared__ float smin[kThreads / 32], smax[kThreads / 32];
  __shared__ float s_ms, s_mn;
  const int64_t s0 = (int64_t)blockIdx.x * dq_gs;
  float mn = INFINITY, mx = -INFINITY;
  for (int i = threadIdx.x; i < dq_gs; i += blockDim.x) {
    const int64_t f = s0 + i;
    const float v = h2f(vals[f < n ? f : n - 1]);
    mn = fminf(mn, v);
    mx = fmaxf(mx, v);
  }
  mn = group_reduce_min(mn, 32);
  mx = group_reduce_max(mx, 32);
  if ((threadIdx.x & 31) == 0) {
    smin[threadIdx.x >> 5] = mn;
    smax[threadIdx.x >> 5] = mx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) {
      mn = fminf(mn, smin[i]);
      mx = fmaxf(mx, smax[i]);
    }
    float ms = __fdiv_rn(__fsub_rn(mx, mn), 255.0f);
    ms = fmaxf(ms, 1e-8f);
    s_ms = ms;
    s_mn = mn;
    meta[2 * blockIdx.x] = f2h(ms);
    meta[2 * blockIdx.x + 1] = f2h(mn);
  }
  __syncthreads();
  const float ms = s_ms, mnv = s_mn;
  const float ms16 = h2f(f2h(ms)), mn16 = h2f(f2h(mnv));
  // every thread reads its values before any thread overwrites them
  float mine[8];
  int cnt = 0;
  for (int i = threadIdx.x; i < dq_gs && cnt < 8; i += blockDim.x) {
    const int64_t f = s0 + i;
    mine[cnt++] = h2f(vals[f < n ? f : n - 1]);
  }
  __syncthreads();
  cnt = 0;
  for (int i = threadIdx.x; i < dq_gs; i += blockDim.x) {
    const int64_t f = s0 + i;
    const float v = cnt < 8 ? mine[cnt] : h2f(vals[f < n ? f : n - 1]);
    ++cnt;
    float c = rintf(__fdiv_rn(__fsub_rn(v, mnv), ms));
    c = fminf(fmaxf(c, 0.f), 255.f);
    codes[f] = (uint8_t)c;
    if (f < n) vals[f] = f2h(__fadd_rn(__fmul_rn(c, ms16), mn16));  // codec.py:404-417
  }
}

// ---- pass E: QuantLinear outlier tables (modules.py:414-448, 649-715) --------------
struct TableArgs {
  int64_t k, cols, rows;
  const int32_t* idx;
  int32_t* row;
  int32_t* col;
  uint16_t* delta;
  const uint16_t* val;
  const uint8_t* packed;
  int64_t row_bytes;
  int bits, gs;
  int64_t n_groups;
  const uint16_t* scale;  // fp16 (plain) or nullptr
  const uint16_t* gmin;
  const uint8_t* dqs_codes;
  const uint16_t* dqs_meta;
  const uint8_t* dqg_codes;
  const uint16_t* dqg_meta;
  int dq_gs;
  const float* cb_delta;  // reconstruction levels used by the kernels, or nullptr
  const uint16_t* cb_f16; // Lloyd: the stored fp16 levels (take precedence)
};

__global__ void outlier_tables_kernel(const TableArgs a) {
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < a.k;
       j += (int64_t)gridDim.x * blockDim.x) {
    const int64_t f = a.idx[j];
    const int64_t r = f / a.cols, c = f - r * a.cols;
    a.row[j] = (int32_t)r;
    a.col[j] = (int32_t)c;
    const uint8_t* p = a.packed + r * a.row_bytes;
    int code;
    if (a.bits == 4) code = (p[c >> 1] >> ((c & 1) * 4)) & 0xF;
    else if (a.bits == 2) code = (p[c >> 2] >> ((c & 3) * 2)) & 0x3;
    else code = p[c];
    float cv = (float)code;
    if (a.cb_f16) cv = h2f(a.cb_f16[code]);
    else if (a.cb_delta) cv = a.cb_delta[code];
    const int64_t gi = r * a.n_groups + c / a.gs;
    float s, m;
    if (a.dqs_codes) {
      const int64_t sup = gi / a.dq_gs;
      s = __fadd_rn(__fmul_rn((float)a.dqs_codes[gi], h2f(a.dqs_meta[2 * sup])), h2f(a.dqs_meta[2 * sup + 1]));
      m = __fadd_rn(__fmul_rn((float)a.dqg_codes[gi], h2f(a.dqg_meta[2 * sup])), h2f(a.dqg_meta[2 * sup + 1]));
    } else {
      s = h2f(a.scale[gi]);
      m = h2f(a.gmin[gi]);
    }
    const float base = __fadd_rn(__fmul_rn(cv, s), m);
    a.delta[j] = f2h(__fsub_rn(h2f(a.val[j]), base));
  }
}

__global__ void row_ptr_kernel(const int32_t* idx, int64_t k, int64_t cols, int64_t rows, int32_t* ptr) {
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r <= rows;
       r += (int64_t)gridDim.x * blockDim.x) {
    // first j with idx[j] >= r*cols (indices are ascending => rows ascending)
    const int64_t key = r * cols;
    int64_t lo = 0, hi = k;
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if ((int64_t)idx[mid] < key) lo = mid + 1; else hi = mid;
    }
    ptr[r] = (int32_t)lo;
  }
}

// ---- Lloyd-Max fit (codec.py:320-361) -----------------------------------------------
// The reference accumulates each level's values with index_add_, which on CPU
// adds them one after the other in element order in float32. The fit here
// does exactly that (one thread per level walking the values in order), so
// the fitted levels are bit-identical to the reference's CPU fit on the same
// sample.
struct LloydState {
  float lo, hi;
  int n_levels;
  int pad;
  float cent[256];   // current centroids (unsorted positions, like the reference)
  float mids[256];   // decision boundaries of the sorted centroids
  int order[256];    // sorted position -> centroid index
};

__global__ void lloyd_minmax_kernel(const float* v, int64_t n, float* mm /* [2*blocks] */) {
  float lo = INFINITY, hi = -INFINITY;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    lo = fminf(lo, v[i]);
    hi = fmaxf(hi, v[i]);
  }
  lo = group_reduce_min(lo, 32);
  hi = group_reduce_max(hi, 32);
  __shared__ float sl[32], sh[32];
  if ((threadIdx.x & 31) == 0) {
    sl[threadIdx.x >> 5] = lo;
    sh[threadIdx.x >> 5] = hi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) {
      lo = fminf(lo, sl[i]);
      hi = fmaxf(hi, sh[i]);
    }
    mm[2 * blockIdx.x] = lo;
    mm[2 * blockIdx.x + 1] = hi;
  }
}

// Sort the current centroids (stable rank sort, as torch.sort orders equal
// keys by position) and derive the decision boundaries (a + b) / 2.
__device__ void lloyd_prepare(LloydState* s) {
  const int L = s->n_levels;
  __shared__ float sc[256];
  for (int i = threadIdx.x; i < L; i += blockDim.x) sc[i] = s->cent[i];
  __syncthreads();
  for (int i = threadIdx.x; i < L; i += blockDim.x) {
    int rank = 0;
    for (int j = 0; j < L; ++j) rank += (sc[j] < sc[i]) || (sc[j] == sc[i] && j < i);
    s->order[rank] = i;
  }
  __syncthreads();
  for (int i = threadIdx.x; i + 1 < L; i += blockDim.x)
    s->mids[i] = __fmul_rn(__fadd_rn(sc[s->order[i]], sc[s->order[i + 1]]), 0.5f);
  __syncthreads();
}

__global__ void lloyd_init_kernel(const float* mm, int nblk, int64_t n, int n_levels, LloydState* s) {
  if (threadIdx.x == 0) {
    float lo = INFINITY, hi = -INFINITY;
    for (int i = 0; i < nblk; ++i) {
      lo = fminf(lo, mm[2 * i]);
      hi = fmaxf(hi, mm[2 * i + 1]);
    }
    s->lo = lo;
    s->hi = hi;
    const int L = (int)i64min(n_levels, n);
    s->n_levels = L;
    // linspace(lo, hi, L) the way ATen computes it in float32
    if (L == 1) {
      s->cent[0] = lo;
    } else {
      const float step = __fdiv_rn(__fsub_rn(hi, lo), (float)(L - 1));
      const int half = L / 2;
      for (int i = 0; i < L; ++i)
        s->cent[i] = i < half ? __fadd_rn(lo, __fmul_rn(step, (float)i))
                              : __fsub_rn(hi, __fmul_rn(step, (float)(L - i - 1)));
    }
  }
  __syncthreads();
  lloyd_prepare(s);
}

// All `iters` Lloyd iterations in one block of 256 threads. Per iteration the
// values stream through shared memory in chunks: every thread assigns a
// share of the chunk (searchsorted over the boundaries, left side, then the
// sorted position's centroid index), then thread c walks the whole chunk in
// order and adds the values assigned to centroid c to its float32 sum and
// count. New centroid = sum / count; an empty centroid keeps its value.
constexpr int kLloydChunk = 4096;
__global__ void __launch_bounds__(256) lloyd_fit_kernel(const float* v, int64_t n, LloydState* s, int iters) {
  __shared__ float cv[kLloydChunk];
  __shared__ uint8_t ca[kLloydChunk];
  __shared__ float mids[256];
  __shared__ int order[256];
  const int L = s->n_levels;
  const int c = threadIdx.x;
  for (int it = 0; it < iters; ++it) {
    for (int i = threadIdx.x; i < L; i += blockDim.x) {
      mids[i] = s->mids[i];
      order[i] = s->order[i];
    }
    __syncthreads();
    float sum = 0.f, cnt = 0.f;
    for (int64_t base = 0; base < n; base += kLloydChunk) {
      const int m = (int)i64min(kLloydChunk, n - base);
      for (int j = threadIdx.x; j < m; j += blockDim.x) {
        const float x = v[base + j];
        int lo = 0, hi = L - 1;   // first boundary >= x (the count of boundaries below x)
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          if (mids[mid] < x) lo = mid + 1; else hi = mid;
        }
        cv[j] = x;
        ca[j] = (uint8_t)order[lo];
      }
      __syncthreads();
      if (c < L) {
        for (int j = 0; j < m; ++j) {
          const bool mine = ca[j] == c;
          const float t = __fadd_rn(sum, cv[j]);
          sum = mine ? t : sum;
          cnt = mine ? __fadd_rn(cnt, 1.f) : cnt;
        }
      }
      __syncthreads();
    }
    if (c < L && cnt > 0.f) s->cent[c] = __fdiv_rn(sum, cnt);
    __syncthreads();
    lloyd_prepare(s);
  }
}

__global__ void lloyd_output_kernel(const LloydState* s, int n_levels, float* out, uint16_t* out16) {
  // sorted centroids; unused trailing levels (fewer values than levels) repeat the last
  for (int i = threadIdx.x; i < n_levels; i += blockDim.x) {
    const int j = min(i, s->n_levels - 1);
    const float c = s->cent[s->order[j]];
    if (out) out[i] = c;
    if (out16) out16[i] = f2h(c);
  }
}

// Normalized values (x - gmin) / scale at given flat indices of the padded
// grid (Lloyd-Max fit input, codec.py:593 fits on `grouped`).
template <int DT>
__global__ void lloyd_gather_kernel(const Geometry g, const SelState* st, const float* gmin_raw,
                                    const float* gmax_raw, const int64_t* sample, int64_t n_sample,
                                    float* out) {
  using E = Elem<DT>;
  const float tval = st ? st->t_val : INFINITY;
  const float levels = (float)((1 << g.bits) - 1);
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < n_sample;
       j += (int64_t)gridDim.x * blockDim.x) {
    const int64_t f = sample ? sample[j] : j;
    const int64_t r = f / g.padded_cols, c = f - r * g.padded_cols;
    const int64_t gi = r * g.n_groups + (c >> g.gs_shift);
    const float gmn = fminf(fmaxf(gmin_raw[gi], -tval), tval);
    const float gmx = fminf(fmaxf(gmax_raw[gi], -tval), tval);
    const float scale = fmaxf(__fdiv_rn(__fsub_rn(gmx, gmn), levels), 1e-8f);
    const float x = fminf(fmaxf(E::val(g.w, r * g.cols + (c < g.cols ? c : g.cols - 1)), -tval), tval);
    out[j] = __fdiv_rn(__fsub_rn(x, gmn), scale);
  }
}

__global__ void to_half_kernel(const float* src, int n, uint16_t* dst) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = f2h(src[i]);
}

// ---- workspace layout ------------------------------------------------------------
struct WsLayout {
  size_t gmin_raw, gmax_raw, hist1, hist2, sel, cta_hist, cta_info, lloyd_vals, lloyd_state,
      lloyd_mm, cb32, total;
};

constexpr int kLloydBlocks = 296;

inline int last_bins(int dtype) { return dtype == TS_F32 ? 1024 : 128; }

inline CtaPlan make_plan(int64_t rows) {
  CtaPlan p;
  // 256-thread CTAs per SM for passes B and C (the select step takes at most
  // 1024 CTAs); TS_QZ_CTAS_PER_SM overrides the default of 4 (tuning knob)
  static const int per_sm = [] {
    const char* k = getenv("TS_QZ_CTAS_PER_SM");
    const int v = k ? atoi(k) : 0;
    return v >= 1 && v <= 8 ? v : 4;
  }();
  const int64_t target = qz::i64max(1, qz::i64min(1024, (int64_t)sm_count() * per_sm));
  p.rows_per_cta = qz::i64max(1, (rows + target - 1) / target);
  p.n_cta = (int)((rows + p.rows_per_cta - 1) / p.rows_per_cta);
  return p;
}

inline WsLayout layout(const ts_quant_params& p, int dtype) {
  WsLayout l;
  const int64_t gs = p.group_size;
  const int64_t padded = (p.cols + gs - 1) / gs * gs;
  const int64_t ng = padded / gs;
  const int64_t groups = p.rows * ng;
  const CtaPlan plan = make_plan(p.rows);
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + bytes, 256);
    return at;
  };
  l.gmin_raw = take(groups * 4);
  l.gmax_raw = take(groups * 4);
  l.hist1 = take(2048 * 4);
  l.hist2 = take(1024 * 4);
  l.sel = take(sizeof(SelState));
  l.cta_hist = take((size_t)plan.n_cta * (last_bins(dtype) + 1) * 4);
  l.cta_info = take((size_t)plan.n_cta * 2 * 8);
  const int64_t n_fit = p.mode == TS_QMODE_LLOYD
                            ? (p.lloyd_sample ? p.lloyd_n_sample : p.rows * padded)
                            : 0;
  l.lloyd_vals = take(n_fit * 4);
  l.lloyd_state = take(sizeof(LloydState));
  l.lloyd_mm = take(kLloydBlocks * 2 * 4);
  l.cb32 = take(256 * 4);
  l.total = o;
  return l;
}

template <int DT>
int run_quantize(const void* w, const ts_quant_params& p, const ts_quant_outputs& o, char* ws,
                 size_t ws_bytes, cudaStream_t stream) {
  const WsLayout L = layout(p, DT);
  TS_REQUIRE(ws_bytes >= L.total, "quantize_pack: workspace too small (%zu < %zu)", ws_bytes, L.total);
  Geometry g;
  g.w = w;
  g.rows = p.rows;
  g.cols = p.cols;
  g.gs = p.group_size;
  g.gs_shift = 0;
  while ((1 << g.gs_shift) < p.group_size) ++g.gs_shift;
  g.bits = p.bits;
  g.padded_cols = (p.cols + p.group_size - 1) / p.group_size * p.group_size;
  g.n_groups = g.padded_cols / p.group_size;
  g.n8 = g.padded_cols / 8;
  g.n8_magic = g.n8 > 1 ? ~0ull / (uint64_t)g.n8 + 1 : 0;
  {
    const int esz = DT == TS_F32 ? 4 : 2;
    g.vec = p.cols % 8 == 0 && is_aligned(w, 16) && ((p.cols * esz) % 16 == 0);
  }
  const int64_t n = p.rows * p.cols;
  const bool outliers = p.k_outliers > 0 && p.k_outliers < n;
  float* gmin_raw = reinterpret_cast<float*>(ws + L.gmin_raw);
  float* gmax_raw = reinterpret_cast<float*>(ws + L.gmax_raw);
  uint32_t* hist1 = reinterpret_cast<uint32_t*>(ws + L.hist1);
  uint32_t* hist2 = reinterpret_cast<uint32_t*>(ws + L.hist2);
  SelState* st = reinterpret_cast<SelState*>(ws + L.sel);
  uint32_t* cta_hist = reinterpret_cast<uint32_t*>(ws + L.cta_hist);
  int64_t* cta_info = reinterpret_cast<int64_t*>(ws + L.cta_info);
  const CtaPlan plan = make_plan(p.rows);
  using E = Elem<DT>;
  const int sms = sm_count();

  if (outliers) TS_CUDA_TRY(cudaMemsetAsync(ws + L.hist1, 0, L.sel - L.hist1, stream));
  {
    const int64_t items = g.rows * g.n8;
    const int blocks = (int)qz::i64min((items + kThreads - 1) / kThreads, (int64_t)sms * 8);
    if (outliers) {
      sample_bound_kernel<DT><<<1, kSampleThreads, 0, stream>>>(g, p.k_outliers, st);
      TS_LAUNCH_CHECK();
    }
    stats_kernel<DT><<<std::max(blocks, 1), kThreads, 0, stream>>>(g, gmin_raw, gmax_raw, hist1, outliers, st);
    TS_LAUNCH_CHECK();
  }
  if (outliers) {
    select_level_kernel<<<1, 32, 0, stream>>>(hist1, 1 << E::L1_BITS, st, 1, p.k_outliers, E::L1_BITS);
    TS_LAUNCH_CHECK();
    {
      const int blocks = (int)qz::i64min((n + kThreads - 1) / kThreads, (int64_t)sms * 8);
      redo_hist_kernel<DT><<<blocks, kThreads, 0, stream>>>(g, hist1, st);
      TS_LAUNCH_CHECK();
      select_level_kernel<<<1, 32, 0, stream>>>(hist1, 1 << E::L1_BITS, st, 1, p.k_outliers, E::L1_BITS);
      TS_LAUNCH_CHECK();
    }
    if (E::L2_BITS) {
      const int blocks = (int)qz::i64min((n + kThreads - 1) / kThreads, (int64_t)sms * 8);
      prefix_hist_kernel<<<blocks, kThreads, 0, stream>>>(g, st, hist2);
      TS_LAUNCH_CHECK();
      select_level_kernel<<<1, 32, 0, stream>>>(hist2, 1 << E::L2_BITS, st, 0, 0, E::L2_BITS);
      TS_LAUNCH_CHECK();
    }
    cta_hist_kernel<DT><<<plan.n_cta, kThreads, 0, stream>>>(g, plan, st, cta_hist);
    TS_LAUNCH_CHECK();
    const int nb = 1 << E::LAST_BITS;
    TS_REQUIRE(plan.n_cta <= kSelThreads, "quantize_pack: %d row ranges exceed the select block", plan.n_cta);
    finalize_select_kernel<<<1, kSelThreads, nb * sizeof(uint32_t), stream>>>(cta_hist, nb, plan.n_cta, st,
                                                                              cta_info, E::KEY_BITS, DT);
    TS_LAUNCH_CHECK();
  }
  if (o.threshold) {
    if (outliers) {
      TS_CUDA_TRY(cudaMemcpyAsync(o.threshold, &st->t_val, sizeof(float), cudaMemcpyDeviceToDevice, stream));
    } else {
      TS_CUDA_TRY(cudaMemsetAsync(o.threshold, 0, sizeof(float), stream));
    }
  }

  // code assignment levels
  const float* cb_assign = nullptr;
  const int n_levels = 1 << p.bits;
  if (p.mode == TS_QMODE_CODEBOOK) {
    TS_REQUIRE(p.codebook != nullptr, "quantize_pack: codebook mode needs a codebook");
    cb_assign = p.codebook;
  } else if (p.mode == TS_QMODE_LLOYD) {
    float* vals = reinterpret_cast<float*>(ws + L.lloyd_vals);
    const int64_t n_fit = p.lloyd_sample ? p.lloyd_n_sample : p.rows * g.padded_cols;
    const int blocks = (int)qz::i64min((n_fit + kThreads - 1) / kThreads, (int64_t)sms * 8);
    lloyd_gather_kernel<DT><<<std::max(blocks, 1), kThreads, 0, stream>>>(
        g, outliers ? st : nullptr, gmin_raw, gmax_raw, p.lloyd_sample, n_fit, vals);
    TS_LAUNCH_CHECK();
    float* cb32 = o.codebook_out ? o.codebook_out : reinterpret_cast<float*>(ws + L.cb32);
    const int rc = run_lloyd(vals, n_fit, n_levels, p.lloyd_iters, cb32, o.codebook_f16, ws, stream,
                             L.lloyd_state, L.lloyd_mm);
    if (rc != TS_OK) return rc;
    cb_assign = cb32;
  }
  if (p.mode == TS_QMODE_CODEBOOK && o.codebook_out)
    TS_CUDA_TRY(cudaMemcpyAsync(o.codebook_out, p.codebook, n_levels * 4, cudaMemcpyDeviceToDevice, stream));
  if (p.mode == TS_QMODE_CODEBOOK && o.codebook_f16) {
    // companded weights with caller-given levels store (and reconstruct
    // from) their fp16 rounding, codec.py:596
    to_half_kernel<<<1, 256, 0, stream>>>(p.codebook, n_levels, o.codebook_f16);
    TS_LAUNCH_CHECK();
  }

  QuantArgs qa;
  qa.g = g;
  qa.plan = plan;
  qa.st = outliers ? st : nullptr;
  qa.cta_info = cta_info;
  qa.gmin_raw = gmin_raw;
  qa.gmax_raw = gmax_raw;
  qa.cb = cb_assign;
  qa.n_levels = n_levels;
  qa.packed = o.packed;
  qa.row_bytes = g.padded_cols * p.bits / 8;
  qa.scale = o.scale;
  qa.gmin = o.gmin;
  qa.out_idx = o.outlier_idx;
  qa.out_val = o.outlier_val;
  qa.w_dtype = DT;
  {
    static const int prefetch = [] {   // TS_QZ_PREFETCH=1 turns the pass-C pipeline on (tuning knob)
      const char* k = getenv("TS_QZ_PREFETCH");
      return k && k[0] == '1' ? 1 : 0;
    }();
    qa.prefetch = prefetch;
  }
  quantize_kernel<DT><<<plan.n_cta, kThreads, 0, stream>>>(qa);
  TS_LAUNCH_CHECK();

  if (p.double_quant) {
    const int64_t ng = p.rows * g.n_groups;
    const int64_t n_super = (ng + p.dq_group_size - 1) / p.dq_group_size;
    double_quant_kernel<<<(int)n_super, kThreads, 0, stream>>>(o.scale, ng, p.dq_group_size,
                                                              o.dq_scale_codes, o.dq_scale_meta);
    TS_LAUNCH_CHECK();
    double_quant_kernel<<<(int)n_super, kThreads, 0, stream>>>(o.gmin, ng, p.dq_group_size,
                                                              o.dq_gmin_codes, o.dq_gmin_meta);
    TS_LAUNCH_CHECK();
  }

  const int64_t k = outliers ? p.k_outliers : 0;
  if (k > 0) {
    TableArgs t;
    t.k = k;
    t.cols = p.cols;
    t.rows = p.rows;
    t.idx = o.outlier_idx;
    t.row = o.outlier_row;
    t.col = o.outlier_col;
    t.delta = o.outlier_delta;
    t.val = o.outlier_val;
    t.packed = o.packed;
    t.row_bytes = qa.row_bytes;
    t.bits = p.bits;
    t.gs = p.group_size;
    t.n_groups = g.n_groups;
    t.scale = p.double_quant ? nullptr : o.scale;
    t.gmin = p.double_quant ? nullptr : o.gmin;
    t.dqs_codes = p.double_quant ? o.dq_scale_codes : nullptr;
    t.dqs_meta = o.dq_scale_meta;
    t.dqg_codes = o.dq_gmin_codes;
    t.dqg_meta = o.dq_gmin_meta;
    t.dq_gs = p.dq_group_size;
    t.cb_delta = cb_assign;
    t.cb_f16 = p.mode != TS_QMODE_UNIFORM ? o.codebook_f16 : nullptr;
    TS_REQUIRE(p.mode != TS_QMODE_LLOYD || o.codebook_f16 != nullptr,
               "quantize_pack: Lloyd mode needs codebook_f16 output");
    const int blocks = (int)qz::i64min((k + 255) / 256, (int64_t)sms * 4);
    outlier_tables_kernel<<<blocks, 256, 0, stream>>>(t);
    TS_LAUNCH_CHECK();
  }
  {
    const int blocks = (int)qz::i64min((p.rows + 1 + 255) / 256, (int64_t)sms * 4);
    row_ptr_kernel<<<blocks, 256, 0, stream>>>(o.outlier_idx, k, p.cols, p.rows, o.outlier_row_ptr);
    TS_LAUNCH_CHECK();
  }
  return TS_OK;
}

}  // namespace qz

int run_lloyd(const float* vals, int64_t n, int n_levels, int iters, float* out, uint16_t* out16,
              char* ws, cudaStream_t stream, size_t off_state, size_t off_mm) {
  using namespace qz;
  TS_REQUIRE(n > 0, "lloyd_fit: no values");
  TS_REQUIRE(n_levels >= 1 && n_levels <= 256, "lloyd_fit: n_levels must be in [1, 256]");
  LloydState* s = reinterpret_cast<LloydState*>(ws + off_state);
  float* mm = reinterpret_cast<float*>(ws + off_mm);
  const int blocks = (int)qz::i64min((n + 255) / 256, (int64_t)kLloydBlocks);
  lloyd_minmax_kernel<<<blocks, 256, 0, stream>>>(vals, n, mm);
  TS_LAUNCH_CHECK();
  lloyd_init_kernel<<<1, 256, 0, stream>>>(mm, blocks, n, n_levels, s);
  TS_LAUNCH_CHECK();
  if (iters > 0) {
    lloyd_fit_kernel<<<1, 256, 0, stream>>>(vals, n, s, iters);
    TS_LAUNCH_CHECK();
  }
  lloyd_output_kernel<<<1, 256, 0, stream>>>(s, n_levels, out, out16);
  TS_LAUNCH_CHECK();
  return TS_OK;
}

size_t lloyd_ws_size() {
  return align_up(sizeof(qz::LloydState), 256) + align_up(qz::kLloydBlocks * 2 * 4, 256) + 1024;
}

int run_lloyd_standalone(const float* vals, int64_t n, int n_levels, int iters, float* out, char* ws,
                         size_t ws_bytes, cudaStream_t stream) {
  TS_REQUIRE(ws_bytes >= lloyd_ws_size(), "lloyd_fit: workspace too small");
  const size_t st = 0;
  const size_t mm = align_up(sizeof(qz::LloydState), 256);
  return run_lloyd(vals, n, n_levels, iters, out, nullptr, ws, stream, st, mm);
}

size_t quantize_ws_size(const ts_quant_params& p, int dtype) { return qz::layout(p, dtype).total; }

int run_quantize(const void* w, int dtype, const ts_quant_params& p, const ts_quant_outputs& o,
                 char* ws, size_t ws_bytes, cudaStream_t stream) {
  if (dtype == TS_F16) return qz::run_quantize<TS_F16>(w, p, o, ws, ws_bytes, stream);
  if (dtype == TS_BF16) return qz::run_quantize<TS_BF16>(w, p, o, ws, ws_bytes, stream);
  return qz::run_quantize<TS_F32>(w, p, o, ws, ws_bytes, stream);
}

}  // namespace ts
