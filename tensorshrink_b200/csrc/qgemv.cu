// Decode-shaped fused dequant-GEMV (up to 8 tokens per pass) for sm_100a.
//
// Replaces the reference's `_fused_dequant_matmul_{2,4,8}bit` Triton kernels
// (tensorshrink triton_kernels.py:278-541) for decode shapes, with the
// outlier correction of `_add_outlier_tile` / `_outlier_correction_kernel`
// (triton_kernels.py:154-232, 543-576) and the bias folded into the epilogue.
//
// Streaming. The packed matrix is cut into tiles of 16 rows x 2 KB. Each
// persistent CTA owns an equal contiguous range of tiles (row-block major), so
// HBM traffic is balanced to within one tile. A producer warp streams each
// tile row with a 1-D bulk copy (16 lanes, one row each) and the tile's
// group metadata with 4-byte async copies into a ring of shared-memory stages
// guarded by mbarriers (full: all bytes landed; empty: consumers done), so
// the bytes in flight do not depend on how fast the math runs. Rows are
// stored with a 2064-byte pitch, which makes the fragment reads below
// bank-conflict-free.
//
// Math. Consumer warp w owns the 128-byte slice [128w, 128w+128) of every
// tile row: 8 chunks of 16 bytes, each one m16 x k tensor-core step. Lane
// (q, l) = (lane/4, lane%4) holds rows q and q+8 and reads the 4-byte word at
// 4l of a chunk, so the k of every MMA come from one chunk and hence one
// quantization group. The k order inside an MMA is free, so the activations
// (B) are staged in exactly the order the code words unpack. Per (row, group)
// the reconstruction is w = v*s + g, so
//   sum_k x_k w_k = s * sum_k x_k (v_k - C) + (g + C*s) * sum_k x_k ,
// applied once per group segment with the segment's fp32 activation sum.
//  - Uniform grids (C = 0, v = the integer code): codes are masked out of
//    the word as bytes (one AND, or shift + AND, per 4 codes) and feed
//    mma.sync m16n8k32 u8 x s8 with exact s32 accumulation. Activations are
//    staged as 15-bit fixed point per segment, x = f (256 hi + lo) with f a
//    power of two and hi, lo signed bytes; hi and lo of a token are two
//    adjacent B columns, so one MMA serves 4 tokens (two MMAs for 5..8).
//  - NF / Lloyd-Max codebooks: a per-lane byte lookup table in shared memory
//    gives fp16 (v - C) pairs for mma.sync m16n8k16 with fp32 accumulation;
//    the 8 columns are the tokens, staged as fp16 scaled by a power of two
//    per segment (exact rescale into [-1, 1]).
//
// Row blocks wholly inside one CTA's range are finished by that CTA; a row
// block split between CTAs is finished by whichever CTA arrives last (per
// row-block counter in the workspace), which sums the pieces' partials in CTA
// order, so results are deterministic. The outlier correction
// (x[:, col] * delta over the CSR row slice) and the bias of every row block
// whose first tile a CTA owns are computed in the prologue while the
// producer fills the first stages.
#include <mutex>

#include "common.cuh"
#include "sm100.cuh"

// This file is compiled twice: as is (16 consumer warps, one CTA per SM,
// namespace ts::gemv_v1) and from qgemv_x2.cu (8 consumer warps, two CTAs per
// SM, namespace ts::gemv_v2). The entry point picks per call.
#ifndef TS_GEMV_NS
#define TS_GEMV_NS gemv_v1
#endif

namespace ts {
namespace TS_GEMV_NS {
namespace gemv {

#ifndef TS_GEMV_CW
#define TS_GEMV_CW 16
#endif
#ifndef TS_GEMV_CPS
#define TS_GEMV_CPS 1
#endif
constexpr int kConsumerWarps = TS_GEMV_CW;   // consumer warps per CTA
constexpr int kCtasPerSm = TS_GEMV_CPS;      // resident CTAs per SM (grid = SMs x this)
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;   // + one producer warp
constexpr int kTileRows = 16;
#ifndef TS_GEMV_TILEK
#define TS_GEMV_TILEK 2048
#endif
constexpr int kTileK = TS_GEMV_TILEK;              // packed bytes per row per tile
constexpr int kSlice = kTileK / kConsumerWarps;    // 128 bytes per warp per row
constexpr int kPitch = kTileK + 16;                // smem row pitch (conflict-free)
constexpr int kMaxStages = 6;
constexpr int kMaxTok = 8;
constexpr int kMaxSupers = 64;                     // double-quant super-groups per tile
#ifndef TS_GEMV_OUTCAP
#define TS_GEMV_OUTCAP 2048
#endif
constexpr int kOutCap = TS_GEMV_OUTCAP;                      // outliers preloaded per CTA (more: read in place)

template <int BITS>
struct Geo {
  static constexpr int PPW = 16 / BITS;       // fp16 pairs per 32-bit code word
  static constexpr int MPW = PPW / 2;         // MMAs per word (per 16-byte chunk)
  static constexpr int KPW = 32 / BITS;       // codes per word
  static constexpr int KPC = 128 / BITS;      // codes per 16-byte chunk
};

__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(orv));  // (a & b) | c
  return r;
}
// fp32 -> the activation dtype -> fp32 (round to nearest even)
__device__ __forceinline__ float round_act(float v, int dtype) {
  return dtype == TS_F16 ? __half2float(__float2half_rn(v)) : __bfloat162float(__float2bfloat16_rn(v));
}
__device__ __forceinline__ half2 u2h2(uint32_t v) { return *reinterpret_cast<half2*>(&v); }
__device__ __forceinline__ uint32_t h22u(half2 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ uint32_t hsub(uint32_t a, uint32_t b) { return h22u(__hsub2(u2h2(a), u2h2(b))); }
__device__ __forceinline__ uint32_t hfma(uint32_t a, uint32_t b, uint32_t c) {
  return h22u(__hfma2(u2h2(a), u2h2(b), u2h2(c)));
}

// Codebook codes of one 32-bit word as PPW fp16 pairs (v - C) of consecutive
// codes, in the order the MMAs consume them. `lut` points at this lane's
// lookup-table column.
template <int BITS>
__device__ __forceinline__ void expand_cb(uint32_t q, const char* lut, uint32_t (&P)[Geo<BITS>::PPW]) {
  if constexpr (BITS == 4) {
    // lut: [256 bytes][32 lanes] half2 (v(lo)-C, v(hi)-C)
#pragma unroll
    for (int i = 0; i < 4; ++i) P[i] = *reinterpret_cast<const uint32_t*>(lut + ((q >> (8 * i)) & 0xFFu) * 128u);
  } else if constexpr (BITS == 2) {
    // lut: [256][32 lanes] uint2 = two half2 (crumbs 0,1 | 2,3)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint2 v = *reinterpret_cast<const uint2*>(lut + ((q >> (8 * i)) & 0xFFu) * 256u);
      P[2 * i] = v.x;
      P[2 * i + 1] = v.y;
    }
  } else {
    // CB && BITS == 8: lut [256][32 lanes] u32 holding one fp16 in the low half
    const uint32_t v0 = *reinterpret_cast<const uint32_t*>(lut + (q & 0xFFu) * 128u);
    const uint32_t v1 = *reinterpret_cast<const uint32_t*>(lut + ((q >> 8) & 0xFFu) * 128u);
    const uint32_t v2 = *reinterpret_cast<const uint32_t*>(lut + ((q >> 16) & 0xFFu) * 128u);
    const uint32_t v3 = *reinterpret_cast<const uint32_t*>(lut + (q >> 24) * 128u);
    P[0] = __byte_perm(v0, v1, 0x5410);
    P[1] = __byte_perm(v2, v3, 0x5410);
  }
}

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Integer MMA: u8 codes (A, 16 rows x 32 k) times s8 activation bytes
// (B, 32 k x 8 columns), exact s32 accumulation.
__device__ __forceinline__ void imma16832(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Four ints' low bytes packed into one word (byte 0 first).
__device__ __forceinline__ uint32_t pack_bytes(int b0, int b1, int b2, int b3) {
  return __byte_perm(__byte_perm((uint32_t)b0, (uint32_t)b1, 0x0040), __byte_perm((uint32_t)b2, (uint32_t)b3, 0x0040),
                     0x5410);
}

struct Args {
  // 2-D tensor maps of the metadata arrays ([rows, n_groups]: fp16 scale/min,
  // or the double-quant code bytes), used when meta_bulk is set
  CUtensorMap smap;
  CUtensorMap gmap;
  QW q;
  const void* x;
  int x_dtype;
  int64_t x_stride;
  int64_t m0;          // first token of this pass
  int mt;              // tokens in this pass (<= kMaxTok)
  const void* bias;
  int bias_dtype;
  void* out;
  int out_dtype;
  int64_t out_stride;
  float* partials;     // [grid][2][kTileRows][kMaxTok]
  int* counters;       // [row blocks]
  int* err;            // wait-timeout flag (read back by ts_qlinear_status)
  uint64_t wait_ns;    // limit of every barrier wait
  int stall;           // test hook: the producer issues no copies, so the first waits run out
  int gated;           // x rows hold [gate | up] (2 * cols): the input is silu(gate) * up
  uint32_t tiles;      // row_blocks * kgroups
  uint32_t kgroups;    // tiles per row block
  uint32_t grid;
  uint32_t quantum;    // tiles per unit of the CTA ranges (1, or kgroups: whole row blocks)
  int stages;          // ring depth
  int stage_bytes;     // packed rows + metadata of one stage
  int meta_row_words;  // 32-bit words per metadata row slot (per array)
  int n_chunks;        // 16-byte chunks covering padded_cols
  int seg_chunks;      // chunks per scale segment: min(4, group bytes / 16)
  int gpt;             // groups per full tile row
  int gbytes_shift;    // log2(bytes of packed codes per group)
  int max_owned_rows;  // capacity of the per-CTA epilogue table
  int x_vec16;         // activation rows are 16-byte aligned
  int meta_bulk;       // metadata rows are 16-byte multiples: one 2-D copy per array per tile
  int dq_shift;        // log2(dq_group_size) when it is a power of two, else -1
  int act_dtype;       // dtype the staged activations are rounded to (after the gate / the norm)
  const float* norm_w; // RMSNorm weight: x rows are the fp32 residual stream, normalized while staged
  float norm_eps;
  const float* residual;     // fp32 [M, rows] added to the output, or nullptr
  int64_t residual_stride;
};

// A chain of layers run by one persistent launch: layer i + 1 starts reading
// its activations once every CTA has finished layer i (a grid-wide counter
// in the workspace), while the producer warps keep streaming weight tiles of
// the following layers into the ring. NL bounds the chain length.
template <int NL>
struct Chain {
  Args L[NL];
  int n;
  int* sync;   // workspace: [done counter per layer boundary][exit counter]
};
constexpr int kMaxChain = 8;

// super-group index of a flat (row, group) index
__device__ __forceinline__ uint32_t dq_div(uint32_t flat, const Args& a) {
  return a.dq_shift >= 0 ? flat >> a.dq_shift : flat / (uint32_t)a.q.dq_gs;
}

__device__ __forceinline__ uint32_t cta_of(uint64_t t, uint64_t U, uint64_t G) {
  return (uint32_t)(((t + 1) * G + U - 1) / U - 1);
}

// shared memory ahead of the stage ring: the ring's mbarriers and the CTA flags
constexpr int kHeadBytes = 256;

#ifdef TS_GEMV_PROF
// Phase timings of an instrumented build (never the shipped library), per
// CTA: [start clock, tile-loop start clock, cycles in full-stage waits, in
// math, in flushes, tiles, producer cycles in empty-stage waits, end clock]
// (consumer warp 0; clocks are per SM).
__device__ unsigned long long g_gemv_prof[1024][8];
#define TS_PROF(...) __VA_ARGS__
#else
#define TS_PROF(...)
#endif

// Waits (bounded) until every CTA of the launch has finished the previous
// layer of a chain: consumer thread 0 polls the layer's counter, the other
// consumer threads wait at the named barrier.
__device__ __forceinline__ void chain_wait(const int* done, const Args& a, volatile int* s_abort) {
  if (threadIdx.x == 0) {
    const uint64_t t_start = globaltimer_ns();
    while (ld_acquire_gpu(done) < (int)gridDim.x) {
      if (*s_abort) break;
      if (globaltimer_ns() - t_start > a.wait_ns) {
        atomicExch(a.err, 4);
        *s_abort = 1;
        break;
      }
      __nanosleep(64);
    }
  }
  named_bar_sync(1, kConsumerThreads);
}

// One layer of the launch, run by every warp of the CTA in its role. The ring
// position (rs, rph) and the count of issued stages carry over from layer to
// layer, so the producer streams the next layer's tiles as soon as stages
// free up.
template <int BITS, bool CB, bool DQ, int SEG>
__device__ __forceinline__ void gemv_layer(const Args& a, char* smem, uint64_t* full, uint64_t* empty, int* s_flag,
                                           float* s_rstd, int& rs, uint32_t& rph, uint32_t& issued, int layer,
                                           const int* chain_done) {
  using G = Geo<BITS>;
  constexpr int LUT_BYTES = !CB ? 0 : (BITS == 2 ? 256 * 32 * 8 : 256 * 32 * 4);
  constexpr int E = DQ ? 4 : 2;                      // metadata elements per 32-bit word
  const int S = a.stages;
  // layout: [stages: rows | meta][LUT][B fragments][segment (f, sum)][epilogue][reduction][barriers]
  char* stages = smem;
  char* lut = smem + S * a.stage_bytes;
  const int n_mma = a.n_chunks * G::MPW;
  const int tok_stride = n_mma * 4 + 4;              // uint2 per token (+32 B pad)
  const int xcols = 2 * a.mt;                        // integer path: B columns (hi, lo per token) per MMA
  uint2* xb = reinterpret_cast<uint2*>(lut + LUT_BYTES);
  const int n_seg = a.n_chunks / a.seg_chunks;
  // per (token, segment): (activation scale, sum x, 0, 0)
  float4* sx = reinterpret_cast<float4*>(xb + a.mt * tok_stride);
  float* epi = reinterpret_cast<float*>(sx + a.mt * n_seg);
  float* red = epi + a.max_owned_rows * kMaxTok;
  int* o_ptr = reinterpret_cast<int*>(red + kConsumerWarps * kTileRows * kMaxTok);   // [owned rows + 1]
  int* o_col = o_ptr + a.max_owned_rows + 4;                                            // [kOutCap]
  uint32_t* o_dw = reinterpret_cast<uint32_t*>(o_col + kOutCap);   // [kOutCap / 2 + 1] fp16 deltas as words
  float* o_bias = reinterpret_cast<float*>(o_dw + kOutCap);                             // [owned rows]
  // set by the first wait that runs out: every role stops waiting and
  // unwinds (the producer first lets its copies in flight land)
  volatile int* s_abort = s_flag + 1;
  // per-stage metadata region (after the packed rows): plain: scale rows,
  // gmin rows; DQ: scale codes, gmin codes, scale supers, gmin supers
  const int mrw = a.meta_row_words;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // CTA b owns units [UQ b / G, UQ (b+1) / G) of `quantum` tiles each
  // (CTAs past this layer's grid, in a chain sized for a larger layer, own none)
  const uint64_t Q = a.quantum, UQ = a.tiles / a.quantum, GR = a.grid;
  const bool in_grid = blockIdx.x < a.grid;
  const uint32_t t0 = in_grid ? (uint32_t)(UQ * blockIdx.x / GR * Q) : 0u;
  const uint32_t t1 = in_grid ? (uint32_t)(UQ * (blockIdx.x + 1) / GR * Q) : 0u;
  const uint32_t KG = a.kgroups;
  const uint32_t NGR = (uint32_t)a.q.n_groups;

  // ------------------------------------------------------------------ producer
  if (warp == kConsumerWarps) {
    if (a.stall) return;
    uint32_t rb = t0 / KG, kg = t0 - rb * KG;
    int s = rs;
    uint32_t ph = rph;        // phase of the ring pass that stage s belongs to
    for (uint32_t i = 0; t0 + i < t1; ++i) {
      // warp-uniform decisions: every lane takes part in the __syncwarp below
      TS_PROF(long long pf_e = clock64();)
      if (issued >= (uint32_t)S && !__all_sync(0xffffffffu, mbar_wait_hint(empty + s, ph ^ 1, a.err, 1, a.wait_ns))) {
        *s_abort = 1;
        break;
      }
      TS_PROF(if (lane == 0) g_gemv_prof[blockIdx.x][6] += clock64() - pf_e;)
      if (__any_sync(0xffffffffu, *s_abort != 0)) break;
      char* st = stages + s * a.stage_bytes;
      uint32_t* meta = reinterpret_cast<uint32_t*>(st + kTileRows * kPitch);
      const uint32_t row0 = rb * kTileRows;
      const uint32_t nrows = (uint32_t)(a.q.rows - (int64_t)row0 < kTileRows ? a.q.rows - (int64_t)row0 : kTileRows);
      const uint32_t rbytes = (uint32_t)(a.q.row_bytes - (int64_t)kg * kTileK < kTileK ? a.q.row_bytes - (int64_t)kg * kTileK : kTileK);
      const uint32_t g0 = kg * (uint32_t)a.gpt;
      if (a.meta_bulk) {
        // aligned metadata: one bulk copy per (array, row) + one per super array
        const uint32_t ng = min((uint32_t)a.gpt, NGR - g0);            // groups in this tile
        uint32_t sup_al = 0, sup_bytes = 0;
        if constexpr (DQ) {
          const uint32_t s_lo = dq_div(row0 * NGR + g0, a);
          const uint32_t s_hi = dq_div((row0 + nrows - 1) * NGR + g0 + ng - 1, a);
          sup_al = s_lo & ~3u;
          sup_bytes = ((s_hi - sup_al + 4) & ~3u) * 4u;
          const uint32_t n_sup_all = (uint32_t)((a.q.rows * (int64_t)NGR + a.q.dq_gs - 1) / a.q.dq_gs);
          sup_bytes = min(sup_bytes, (n_sup_all - sup_al) * 4u);
        }
        // metadata: one [16 rows x gpt groups] box per array (rows past the end
        // and groups past n_groups arrive as zeros; the box is counted whole)
        const uint32_t box_bytes = (uint32_t)kTileRows * (uint32_t)a.gpt * (DQ ? 1u : 2u);
        if (lane == 0) mbar_arrive_expect_tx(full + s, nrows * rbytes + 2 * box_bytes + 2 * sup_bytes);
        __syncwarp();
        if (lane < (int)nrows)
          bulk_load(st + lane * kPitch,
                    a.q.packed + (size_t)(row0 + lane) * (size_t)a.q.row_bytes + (size_t)kg * kTileK, rbytes, full + s);
        if (lane == 0) {
          tma_load_2d(meta, &a.smap, (int)g0, (int)row0, full + s);
          tma_load_2d(meta + kTileRows * mrw, &a.gmap, (int)g0, (int)row0, full + s);
        }
        if constexpr (DQ) {
          if (lane < 2)
            bulk_load(meta + 2 * kTileRows * mrw + lane * kMaxSupers,
                      (lane == 0 ? a.q.dqs_meta : a.q.dqg_meta) + sup_al, sup_bytes, full + s);
        }
      } else {
        // unaligned metadata: 4-byte async copies of the aligned-down words
        for (int ar = 0; ar < 2 * kTileRows; ++ar) {
          const int arr = ar / kTileRows, r = ar - arr * kTileRows;
          const uint32_t row = row0 + r;
          const bool v = row < (uint32_t)a.q.rows;
          const uint32_t e0 = v ? ((row * NGR + g0) & ~(uint32_t)(E - 1)) : 0u;
          for (int wd = lane; wd < mrw; wd += 32) {
            const uint32_t e = e0 + wd * E;
            const bool in = v && e < (uint32_t)(a.q.rows * NGR);
            const void* src;
            if constexpr (DQ)
              src = (arr == 0 ? a.q.dqs_codes : a.q.dqg_codes) + (in ? e : 0u);
            else
              src = (arr == 0 ? a.q.scale : a.q.gmin) + (in ? e : 0u);
            cp_async4(meta + ar * mrw + wd, src, in ? 4 : 0);
          }
        }
        if constexpr (DQ) {
          uint32_t* sup = meta + 2 * kTileRows * mrw;
          const uint32_t s_al = (dq_div(row0 * NGR + g0, a)) & ~3u;
          const uint32_t n_sup_all = (uint32_t)((a.q.rows * (int64_t)NGR + a.q.dq_gs - 1) / a.q.dq_gs);
          for (int j = lane; j < kMaxSupers; j += 32) {
            const uint32_t sidx = s_al + j;
            const bool in = sidx < n_sup_all;
            cp_async4(sup + j, a.q.dqs_meta + (in ? sidx : 0u), in ? 4 : 0);
            cp_async4(sup + kMaxSupers + j, a.q.dqg_meta + (in ? sidx : 0u), in ? 4 : 0);
          }
        }
        // every lane's copies are tracked by the barrier (each registers a
        // pending arrival now) before lane 0's own arrival can end the phase
        cp_async_arrive_inc(full + s);
        __syncwarp();
        if (lane == 0) mbar_arrive_expect_tx(full + s, nrows * rbytes);
        __syncwarp();
        if (lane < (int)nrows)
          bulk_load(st + lane * kPitch,
                    a.q.packed + (size_t)(row0 + lane) * (size_t)a.q.row_bytes + (size_t)kg * kTileK, rbytes, full + s);
      }
      ++issued;
      if (++kg == KG) {
        kg = 0;
        ++rb;
      }
      if (++s == S) { s = 0; ph ^= 1; }
    }
    rs = s;
    rph = ph;
    return;
  }

  // ------------------------------------------------------------------ consumers
  float center = 0.f;   // codebooks: the midpoint C of the table
  if constexpr (CB) {
    const float* cb = a.q.codebook;
    center = 0.5f * (__ldg(cb) + __ldg(cb + (1 << BITS) - 1));
    for (int i = threadIdx.x; i < 256 * 32; i += kConsumerThreads) {
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

  // row blocks whose first tile this CTA owns (it adds their bias and outliers)
  const uint32_t rb_own0 = (t0 + KG - 1) / KG, rb_own1 = (t1 + KG - 1) / KG;
  const int n_own = (int)(rb_own1 - rb_own0) * kTileRows;

  // outlier slice (CSR bounds, columns, deltas) and bias of the owned rows:
  // constant buffers, loaded before waiting on the producer of x
  const int64_t own_row0 = (int64_t)rb_own0 * kTileRows;
  const int64_t rows_left = a.q.rows - own_row0;
  const int n_own_rows = rows_left <= 0 ? 0 : (rows_left < n_own ? (int)rows_left : n_own);
  for (int i = threadIdx.x; i <= n_own_rows; i += kConsumerThreads)
    o_ptr[i] = a.q.n_outliers > 0 ? __ldg(a.q.orow_ptr + own_row0 + i) : 0;
  for (int i = threadIdx.x; i < n_own_rows; i += kConsumerThreads)
    o_bias[i] = a.bias ? load_f(a.bias, a.bias_dtype, own_row0 + i) : 0.f;
  named_bar_sync(1, kConsumerThreads);
  const int o_base = n_own_rows > 0 ? o_ptr[0] : 0;
  const int o_cnt = n_own_rows > 0 ? o_ptr[n_own_rows] - o_base : 0;
  // the first kOutCap outliers of the slice into shared memory with async
  // copies, in flight while the activations load: columns as 4-byte words,
  // deltas as the 4-byte words covering them (o_dw holds delta j at half
  // index j + dl_off), zero-filled past the end of the array
  const int n_pre = min(o_cnt, kOutCap);
  const int dl_off = o_base & 1;
  for (int j = threadIdx.x; j < n_pre; j += kConsumerThreads) cp_async4(o_col + j, a.q.ocol + o_base + j, 4);
  if ((reinterpret_cast<uintptr_t>(a.q.odelta) & 3) == 0) {
    const int64_t h0 = (int64_t)o_base - dl_off;
    const int nw = (n_pre + dl_off + 1) >> 1;
    for (int w = threadIdx.x; w < nw; w += kConsumerThreads) {
      const int64_t left = a.q.n_outliers - (h0 + 2 * w);   // halves from this word to the end
      cp_async4(o_dw + w, a.q.odelta + h0 + 2 * w, left >= 2 ? 4 : 2);
    }
  } else {
    for (int j = threadIdx.x; j < n_pre; j += kConsumerThreads)
      reinterpret_cast<__half*>(o_dw)[j + dl_off] = __ldg(a.q.odelta + o_base + j);
  }

  // x is produced by the previous kernel in the stream (programmatic launch),
  // or, in a chain, by the previous layer of this launch
  if (layer == 0)
    pdl_wait_primary();
  else
    chain_wait(chain_done + layer - 1, a, s_abort);
  if (a.norm_w) {
    // RMSNorm of each token's fp32 row: 1 / sqrt(mean(h^2) + eps), reduced
    // over the consumer threads (warp shuffles, then the flush scratch)
    float ss[kMaxTok];
#pragma unroll
    for (int n = 0; n < kMaxTok; ++n) ss[n] = 0.f;
    const int64_t C = a.q.cols;
#pragma unroll
    for (int n = 0; n < kMaxTok; ++n) {
      if (n >= a.mt) break;
      const float* h = reinterpret_cast<const float*>(a.x) + (a.m0 + n) * a.x_stride;
      if (a.x_vec16 && C % 4 == 0) {
        const float4* h4 = reinterpret_cast<const float4*>(h);
#pragma unroll 4
        for (int64_t k = threadIdx.x; k < C / 4; k += kConsumerThreads) {
          const float4 v = __ldcg(h4 + k);
          ss[n] = fmaf(v.x, v.x, ss[n]);
          ss[n] = fmaf(v.y, v.y, ss[n]);
          ss[n] = fmaf(v.z, v.z, ss[n]);
          ss[n] = fmaf(v.w, v.w, ss[n]);
        }
      } else {
        for (int64_t k = threadIdx.x; k < C; k += kConsumerThreads) {
          const float v = __ldcg(h + k);
          ss[n] = fmaf(v, v, ss[n]);
        }
      }
    }
    float* red0 = red;   // the flush scratch, free until the first flush
#pragma unroll
    for (int n = 0; n < kMaxTok; ++n) {
      float v = ss[n];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) red0[warp * kMaxTok + n] = v;
    }
    named_bar_sync(1, kConsumerThreads);
    if (threadIdx.x < a.mt) {
      float t = 0.f;
      for (int w = 0; w < kConsumerWarps; ++w) t += red0[w * kMaxTok + threadIdx.x];
      s_rstd[threadIdx.x] = rsqrtf(t / (float)C + a.norm_eps);
    }
    named_bar_sync(1, kConsumerThreads);
  }
  {
    // one thread per 16 consecutive activations of one token: load, reduce the
    // segment's max |x| and sum across its threads, write the B fragments
    const int seg_k = a.seg_chunks * G::KPC;
    const int tps = seg_k / 16;                      // threads per segment (power of two)
    const uint32_t per_tok = (uint32_t)(a.q.padded_cols / 16);
    const uint32_t items = a.mt * per_tok;
    // kU items per thread per round, loads first (one item measured fastest:
    // more raise register pressure); x was written by the previous kernel,
    // or by this launch in a chain, so the loads are L2-coherent
    constexpr int kU = 1;
    for (uint32_t base0 = 0; base0 < items; base0 += kU * kConsumerThreads) {
    uint4 raw[kU][4];
#pragma unroll
    for (int jr = 0; jr < kU; ++jr) {
      const uint32_t it = base0 + jr * kConsumerThreads + threadIdx.x;
      const bool live = it < items;
      const uint32_t n = live ? it / per_tok : 0;
      const uint32_t k0 = live ? (it - n * per_tok) * 16 : 0;
      const int64_t xo = (a.m0 + n) * a.x_stride + k0;
      if (live && a.x_vec16 && k0 + 16 <= (uint32_t)a.q.cols) {
        if (a.x_dtype == TS_F32) {
          const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(a.x) + xo);
#pragma unroll
          for (int c = 0; c < 4; ++c) raw[jr][c] = __ldcg(p + c);
        } else {
          const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(a.x) + xo);
          raw[jr][0] = __ldcg(p);
          raw[jr][1] = __ldcg(p + 1);
          if (a.gated) {
            const uint4* pu = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(a.x) + xo + a.q.cols);
            raw[jr][2] = __ldcg(pu);
            raw[jr][3] = __ldcg(pu + 1);
          }
        }
      }
    }
#pragma unroll
    for (int jr = 0; jr < kU; ++jr) {
      const uint32_t it = base0 + jr * kConsumerThreads + threadIdx.x;
      const bool live = it < items;
      const uint32_t n = live ? it / per_tok : 0;
      const uint32_t k0 = live ? (it - n * per_tok) * 16 : 0;
      const int64_t xo = (a.m0 + n) * a.x_stride + k0;
      float v[16];
      // 16 activations at element offset `off` of the token's row (part 1:
      // the up half of a gated row)
      auto load16 = [&](int64_t off, int part, float (&o)[16]) {
        if (live && a.x_vec16 && k0 + 16 <= (uint32_t)a.q.cols && a.x_dtype == TS_F32) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            o[4 * j] = __uint_as_float(raw[jr][j].x);
            o[4 * j + 1] = __uint_as_float(raw[jr][j].y);
            o[4 * j + 2] = __uint_as_float(raw[jr][j].z);
            o[4 * j + 3] = __uint_as_float(raw[jr][j].w);
          }
        } else if (live && a.x_vec16 && k0 + 16 <= (uint32_t)a.q.cols) {
          const uint4 r0 = raw[jr][2 * part], r1 = raw[jr][2 * part + 1];
          const uint32_t rw[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (a.x_dtype == TS_F16) {
              const float2 f = __half22float2(u2h2(rw[j]));
              o[2 * j] = f.x;
              o[2 * j + 1] = f.y;
            } else {
              o[2 * j] = __uint_as_float(rw[j] << 16);
              o[2 * j + 1] = __uint_as_float(rw[j] & 0xFFFF0000u);
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            o[j] = (live && k0 + j < (uint32_t)a.q.cols) ? load_f_cg(a.x, a.x_dtype, off + j) : 0.f;
        }
      };
      load16(xo, 0, v);
      if (a.gated) {
        // gated MLP input: x = silu(gate) * up with gate, up the two halves of
        // the row, each rounded to the activation dtype as the unfused
        // F.silu(gate) * up would round them
        float u[16];
        load16(xo + a.q.cols, 1, u);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float sl = round_act(__fdividef(v[j], 1.f + __expf(-v[j])), a.act_dtype);
          v[j] = round_act(sl * u[j], a.act_dtype);
        }
      } else if (a.norm_w) {
        // x = (h * rstd) * w, rounded to the activation dtype, as
        // F.rms_norm(h, w).to(dtype) rounds it
        const float rs = live ? s_rstd[n] : 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j)
          v[j] = (live && k0 + j < (uint32_t)a.q.cols) ? round_act(v[j] * rs * __ldg(a.norm_w + k0 + j), a.act_dtype)
                                                         : 0.f;
      }
      float mx = 0.f, sum = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        mx = fmaxf(mx, fabsf(v[j]));
        sum += v[j];
      }
      for (int o = tps / 2; o > 0; o >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        sum += __shfl_xor_sync(0xffffffffu, sum, o);
      }
      // power-of-two scale 2^e with max|x| / 2^e in [0.5, 1): exponent bits
      const int e = mx > 0.f ? min(126, (int)((__float_as_uint(mx) >> 23) & 0xFFu) - 126) : 0;
      if constexpr (CB) {
        const float inv = __uint_as_float((uint32_t)(127 - e) << 23);
        float hx[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) hx[j] = v[j] * inv;
        // B fragments: pair p of a word holds its codes 2p, 2p+1
        uint2 frag[16 / G::KPW][G::MPW];
#pragma unroll
        for (int wb = 0; wb < 16 / G::KPW; ++wb) {
#pragma unroll
          for (int m = 0; m < G::MPW; ++m) {
            uint32_t bw[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int pr = 2 * m + h;
              bw[h] = h22u(__floats2half2_rn(hx[wb * G::KPW + 2 * pr], hx[wb * G::KPW + 2 * pr + 1]));
            }
            frag[wb][m] = make_uint2(bw[0], bw[1]);
          }
        }
        if (live) {
          const uint32_t sg = k0 / seg_k;
          if (k0 % seg_k == 0)
            sx[n * n_seg + sg] = make_float4(__uint_as_float((uint32_t)(e + 127) << 23), sum, 0.f, 0.f);
#pragma unroll
          for (int wb = 0; wb < 16 / G::KPW; ++wb) {
            const uint32_t gwb = k0 / G::KPW + wb;     // global word-block index
            const uint32_t ch = gwb >> 2, l = gwb & 3;
#pragma unroll
            for (int m = 0; m < G::MPW; ++m) xb[n * tok_stride + (ch * G::MPW + m) * 4 + l] = frag[wb][m];
          }
        }
      } else {
        // uniform grids: x~ = rint(x 2^(14-e)) (|x~| <= 2^14, 15-bit fixed
        // point per segment) split into signed bytes x~ = 256 hi + lo with lo
        // in [-128, 128); hi and lo of token n are the B columns 2n, 2n+1 of
        // the integer MMAs, whose k order follows the code unpacking below
        const int ec = max(e, -112);
        const float up = __uint_as_float((uint32_t)(141 - ec) << 23);
        int hi[16], lo[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int xi = __float2int_rn(v[j] * up);
          lo[j] = (xi << 24) >> 24;
          hi[j] = (xi - lo[j]) >> 8;
        }
        if (live) {
          const uint32_t sg = k0 / seg_k;
          if (k0 % seg_k == 0)
            sx[n * n_seg + sg] = make_float4(__uint_as_float((uint32_t)(113 + ec) << 23), sum, 0.f, 0.f);
          uint2* xh = xb + (2 * n) * 4;       // column 2n (hi); column 2n+1 (lo) follows at +4
          if constexpr (BITS == 4) {
            // 32-code chunk = one MMA; lane l holds codes 8l..8l+7: even codes
            // (low nibbles) in b0, odd codes in b1
            const uint32_t J = k0 >> 5, lb = (k0 & 31) >> 3;
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int* H = hi + 8 * u;
              const int* L = lo + 8 * u;
              xh[J * xcols * 4 + lb + u] = make_uint2(pack_bytes(H[0], H[2], H[4], H[6]), pack_bytes(H[1], H[3], H[5], H[7]));
              xh[J * xcols * 4 + 4 + lb + u] =
                  make_uint2(pack_bytes(L[0], L[2], L[4], L[6]), pack_bytes(L[1], L[3], L[5], L[7]));
            }
          } else if constexpr (BITS == 2) {
            // 64-code chunk = two MMAs; lane l holds codes 16l + 4j + t (crumb t
            // of byte j): MMA m takes crumbs 2m (b0) and 2m+1 (b1)
            const uint32_t l16 = (k0 & 63) >> 4, J0 = (k0 >> 6) * 2;
#pragma unroll
            for (int m = 0; m < 2; ++m) {
              xh[(J0 + m) * xcols * 4 + l16] = make_uint2(pack_bytes(hi[2 * m], hi[4 + 2 * m], hi[8 + 2 * m], hi[12 + 2 * m]),
                                                         pack_bytes(hi[2 * m + 1], hi[5 + 2 * m], hi[9 + 2 * m], hi[13 + 2 * m]));
              xh[(J0 + m) * xcols * 4 + 4 + l16] =
                  make_uint2(pack_bytes(lo[2 * m], lo[4 + 2 * m], lo[8 + 2 * m], lo[12 + 2 * m]),
                             pack_bytes(lo[2 * m + 1], lo[5 + 2 * m], lo[9 + 2 * m], lo[13 + 2 * m]));
            }
          } else {
            // 16-code chunk = half an MMA: even chunks in b0 (k 0..15), odd in b1
            const uint32_t ch = k0 >> 4, J = ch >> 1, h = ch & 1;
            uint32_t* xw = reinterpret_cast<uint32_t*>(xh + J * xcols * 4);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              xw[2 * u + h] = pack_bytes(hi[4 * u], hi[4 * u + 1], hi[4 * u + 2], hi[4 * u + 3]);
              xw[8 + 2 * u + h] = pack_bytes(lo[4 * u], lo[4 * u + 1], lo[4 * u + 2], lo[4 * u + 3]);
            }
          }
        }
      }
    }
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  named_bar_sync(1, kConsumerThreads);
  {
    // epilogue table: bias + sum over the row's outliers, in stored order, of
    // x[:, col] * delta; one thread per (row, token). The activations are read
    // back from the staged B fragments (codebooks: x = x~ 2^e; uniform grids:
    // x = f (256 hi + lo)). Entries of tokens >= mt are never stored.
    const int seg_k = a.seg_chunks * G::KPC;
    const int seg_sh = 31 - __clz(seg_k);
    const __half* o_dh = reinterpret_cast<const __half*>(o_dw) + dl_off;
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(xb);
    for (int it = threadIdx.x; it < n_own_rows * a.mt; it += kConsumerThreads) {
      const int i = it / a.mt, n = it - i * a.mt;
      float c = o_bias[i];
      const int j_end = o_ptr[i + 1] - o_base;
      for (int j = o_ptr[i] - o_base; j < j_end; ++j) {
        const int col = j < kOutCap ? o_col[j] : __ldg(a.q.ocol + o_base + j);
        const float d = __half2float(j < kOutCap ? o_dh[j] : __ldg(a.q.odelta + o_base + j));
        const float f = sx[n * n_seg + (col >> seg_sh)].x;
        float xv;
        if constexpr (CB) {
          const int wb = col / G::KPW, o = col - wb * G::KPW;
          const int p = o >> 1, hi = o & 1;
          const int J = (wb >> 2) * G::MPW + (p >> 1), lw = wb & 3;
          const uint2 u = xb[n * tok_stride + J * 4 + lw];
          const uint32_t hw = (p & 1) ? u.y : u.x;
          xv = __half2float(__ushort_as_half((uint16_t)(hw >> (16 * hi)))) * f;
        } else {
          int J, lw, h, j8;   // MMA, lane, b0/b1, byte of the code's activation (see the staging)
          if constexpr (BITS == 4) {
            const int cc = col & 31;
            J = col >> 5;
            lw = cc >> 3;
            h = cc & 1;
            j8 = (cc & 7) >> 1;
          } else if constexpr (BITS == 2) {
            const int cc = col & 63;
            J = 2 * (col >> 6) + ((cc & 3) >> 1);
            lw = cc >> 4;
            h = cc & 1;
            j8 = (cc & 15) >> 2;
          } else {
            const int ch = col >> 4, cc = col & 15;
            J = ch >> 1;
            lw = cc >> 2;
            h = ch & 1;
            j8 = cc & 3;
          }
          const uint32_t hw = xw[((J * xcols + 2 * n) * 4 + lw) * 2 + h];
          const uint32_t lwd = xw[((J * xcols + 2 * n + 1) * 4 + lw) * 2 + h];
          const int xh = (int)(hw << (24 - 8 * j8)) >> 24, xl = (int)(lwd << (24 - 8 * j8)) >> 24;
          xv = (float)(256 * xh + xl) * f;
        }
        c = fmaf(xv, d, c);
      }
      epi[i * kMaxTok + n] = c;
    }
  }
  named_bar_sync(1, kConsumerThreads);
  if (t0 >= t1) return;

  const int q = lane >> 2, l = lane & 3;   // rows q, q+8; token columns 2l, 2l+1
  const char* lut_lane = lut + lane * (BITS == 2 ? 8 : 4);
  uint32_t rb = t0 / KG, kg = t0 - rb * KG;
  const uint32_t first_rb = rb;
  bool started_here = kg == 0;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};     // (q,2l) (q,2l+1) (q+8,2l) (q+8,2l+1)
  const bool has_b = q < a.mt;
  const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);

  // per-lane constants of the tile loop
  const uint2* xb_lane = xb + q * tok_stride + l;          // B fragment column of this lane's token
  const float4* sx0 = sx + (2 * l) * n_seg;                 // segment stats of tokens 2l, 2l+1
  const float4* sx1 = sx + (2 * l + 1) * n_seg;
  const bool tok0 = 2 * l < a.mt, tok1 = 2 * l + 1 < a.mt;
  const uint32_t slice_g = (uint32_t)(warp * kSlice) >> a.gbytes_shift;   // first group of the slice in the tile
  // integer path: lane (q, l) feeds B column q (token group 0) and 8 + q
  // (group 1, tokens 4..7) and accumulates tokens l and 4 + l
  const bool two = a.mt > 4;
  const bool has_b0 = q < xcols, has_b1 = 8 + q < xcols;
  const uint2* xi_lane0 = xb + q * 4 + l;
  const uint2* xi_lane1 = xb + (8 + q) * 4 + l;
  const bool toka = l < a.mt, tokb = 4 + l < a.mt;
  const float4* sxa = sx + l * n_seg;
  const float4* sxb = sx + (4 + l) * n_seg;

  int& cs = rs;          // consumers: the ring position carries over between layers
  uint32_t& cph = rph;
  TS_PROF(long long pf_wait = 0, pf_math = 0, pf_flush = 0; long long pf_t = clock64();)
  for (uint32_t i = 0; t0 + i < t1; ++i) {
    const int s = cs;
    TS_PROF(long long pf_a = clock64();)
    // warp-uniform: the MMAs below need every lane; after any role's timeout
    // the remaining tiles are skipped without waiting
    bool ok = !__any_sync(0xffffffffu, *s_abort != 0);
    if (ok && !__all_sync(0xffffffffu, mbar_wait_hint(full + s, cph, a.err, 2, a.wait_ns))) {
      ok = false;
      *s_abort = 1;
    }
    if (++cs == S) { cs = 0; cph ^= 1; }
    TS_PROF(long long pf_b = clock64(); pf_wait += pf_b - pf_a;)
    const char* st = stages + s * a.stage_bytes;
    const uint32_t* meta = reinterpret_cast<const uint32_t*>(st + kTileRows * kPitch);
    const uint32_t g0 = kg * (uint32_t)a.gpt;
    const uint32_t row_q = rb * kTileRows + q;
    // metadata slot offsets of rows q, q+8 (element index of the tile's first group)
    const uint32_t moff0 = ((row_q * NGR + g0) & (uint32_t)(E - 1)) + slice_g;
    const uint32_t moff1 = (((row_q + 8) * NGR + g0) & (uint32_t)(E - 1)) + slice_g;
    const uint32_t* mrow0 = meta + q * mrw;
    const uint32_t* mrow1 = meta + (q + 8) * mrw;
    uint32_t sup_lo = 0;
    if constexpr (DQ) sup_lo = dq_div(rb * kTileRows * NGR + g0, a) & ~3u;
    const char* arow0 = st + q * kPitch + warp * kSlice + 4 * l;
    const char* arow1 = arow0 + 8 * kPitch;
    const uint32_t slice_byte0 = kg * (uint32_t)kTileK + warp * kSlice;
    // scale and min of row q + 8r for group `gi` of this warp's slice
    auto group_meta = [&](int r, uint32_t gi, float& sc, float& gm) {
      const uint32_t* mr = r ? mrow1 : mrow0;
      const uint32_t off = (r ? moff1 : moff0) + gi;
      if constexpr (DQ) {
        const uint32_t* sup = meta + 2 * kTileRows * mrw;
        const uint32_t row = row_q + 8 * r;
        const uint32_t sj = dq_div(row * NGR + g0 + slice_g + gi, a) - sup_lo;
        const float2 ms = __half22float2(u2h2(sup[sj]));
        const float2 mg = __half22float2(u2h2(sup[kMaxSupers + sj]));
        const float csv = (float)((mr[off >> 2] >> ((off & 3) * 8)) & 0xFFu);
        const float cgv = (float)((mr[kTileRows * mrw + (off >> 2)] >> ((off & 3) * 8)) & 0xFFu);
        sc = __fadd_rn(__fmul_rn(csv, ms.x), ms.y);
        gm = __fadd_rn(__fmul_rn(cgv, mg.x), mg.y);
      } else {
        sc = h2f((uint16_t)(mr[off >> 1] >> ((off & 1) * 16)));
        gm = h2f((uint16_t)(mr[kTileRows * mrw + (off >> 1)] >> ((off & 1) * 16)));
      }
    };
    const int gseg0 = (int)(slice_byte0 >> 4) / SEG;
    constexpr int NSG = kSlice / 16 / SEG;  // scale segments per warp slice
    if constexpr (CB) {
      const int J_slice = (int)(slice_byte0 >> 4) * G::MPW;
#pragma unroll
      for (int sg = 0; sg < NSG; ++sg) {
        if (!ok || slice_byte0 + sg * SEG * 16 >= (uint32_t)a.q.row_bytes) break;
        // two independent accumulator chains per segment
        float cc[2][4];
#pragma unroll
        for (int u = 0; u < 2; ++u) cc[u][0] = cc[u][1] = cc[u][2] = cc[u][3] = 0.f;
#pragma unroll
        for (int cj = 0; cj < SEG; ++cj) {
          const int cb = (sg * SEG + cj) * 16;
          const uint32_t w0 = *reinterpret_cast<const uint32_t*>(arow0 + cb);
          const uint32_t w1 = *reinterpret_cast<const uint32_t*>(arow1 + cb);
          uint32_t P0[G::PPW], P1[G::PPW];
          expand_cb<BITS>(w0, lut_lane, P0);
          expand_cb<BITS>(w1, lut_lane, P1);
          const int J0 = J_slice + (sg * SEG + cj) * G::MPW;
#pragma unroll
          for (int m = 0; m < G::MPW; ++m) {
            uint2 bf = make_uint2(0u, 0u);
            if (has_b) bf = xb_lane[(J0 + m) * 4];
            mma16816(cc[(cj * G::MPW + m) & 1], P0[2 * m], P1[2 * m], P0[2 * m + 1], P1[2 * m + 1], bf.x, bf.y);
          }
        }
        float c[4];
#pragma unroll
        for (int z = 0; z < 4; ++z) c[z] = cc[0][z] + cc[1][z];
        // close: acc += (s f) (C - Xc) + (g + C_cb s) X for rows q, q+8
        const float4 fx0 = tok0 ? sx0[gseg0 + sg] : zero4;
        const float4 fx1 = tok1 ? sx1[gseg0 + sg] : zero4;
        const uint32_t gi = (uint32_t)(sg * SEG * 16) >> a.gbytes_shift;   // group within the slice
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          float sc, gm;
          group_meta(r, gi, sc, gm);
          const float gp = fmaf(center, sc, gm);
          acc[2 * r] = fmaf(sc * fx0.x, c[2 * r], fmaf(gp, fx0.y, acc[2 * r]));
          acc[2 * r + 1] = fmaf(sc * fx1.x, c[2 * r + 1], fmaf(gp, fx1.y, acc[2 * r + 1]));
        }
      }
    } else {
      // integer path: per segment, s32 sums of code * x~ (hi and lo columns),
      // closed as acc += s f (256 C_hi + C_lo) + g X for rows q, q+8 and
      // tokens l (acc[0], acc[1]) and 4 + l (acc[2], acc[3])
      const int ch_slice = (int)(slice_byte0 >> 4);
      // unpack of chunk `ch` (words w0, w1 of rows q, q+8) into the A operand of MMA m
      auto unpack = [&](uint32_t w0, uint32_t w1, int ch, int m, uint32_t& A0, uint32_t& A1, uint32_t& A2,
                        uint32_t& A3, int& J) {
        if constexpr (BITS == 4) {
          A0 = w0 & 0x0F0F0F0Fu;
          A1 = w1 & 0x0F0F0F0Fu;
          A2 = (w0 >> 4) & 0x0F0F0F0Fu;
          A3 = (w1 >> 4) & 0x0F0F0F0Fu;
          J = ch;
        } else if constexpr (BITS == 2) {
          A0 = (w0 >> (4 * m)) & 0x03030303u;
          A1 = (w1 >> (4 * m)) & 0x03030303u;
          A2 = (w0 >> (4 * m + 2)) & 0x03030303u;
          A3 = (w1 >> (4 * m + 2)) & 0x03030303u;
          J = 2 * ch + m;
        } else {
          const bool odd = ch & 1;
          A0 = odd ? 0u : w0;
          A1 = odd ? 0u : w1;
          A2 = odd ? w0 : 0u;
          A3 = odd ? w1 : 0u;
          J = ch >> 1;
        }
      };
      constexpr int NM = BITS == 2 ? 2 : 1;   // MMAs per chunk
      if (a.mt == 1) {
        // One token: lanes (q, 0) hold each segment's integer sum for rows q,
        // q+8; lane l then closes segments l, l+4, ... (no duplicated scale
        // decode), and the four lanes' partials are added at the flush.
        int va[2][NSG];
#pragma unroll
        for (int sg = 0; sg < NSG; ++sg) {
          va[0][sg] = va[1][sg] = 0;
          if (!ok || slice_byte0 + sg * SEG * 16 >= (uint32_t)a.q.row_bytes) continue;
          int c4[4] = {0, 0, 0, 0};
#pragma unroll
          for (int cj = 0; cj < SEG; ++cj) {
            const int cb = (sg * SEG + cj) * 16;
            const uint32_t w0 = *reinterpret_cast<const uint32_t*>(arow0 + cb);
            const uint32_t w1 = *reinterpret_cast<const uint32_t*>(arow1 + cb);
#pragma unroll
            for (int m = 0; m < NM; ++m) {
              uint32_t A0, A1, A2, A3;
              int J;
              unpack(w0, w1, ch_slice + sg * SEG + cj, m, A0, A1, A2, A3, J);
              const uint2 b0 = has_b0 ? xi_lane0[J * xcols * 4] : make_uint2(0u, 0u);
              imma16832(c4, A0, A1, A2, A3, b0.x, b0.y);
            }
          }
          va[0][sg] = 256 * c4[0] + c4[1];
          va[1][sg] = 256 * c4[2] + c4[3];
        }
#pragma unroll
        for (int s0 = 0; s0 < NSG; s0 += 4) {
          int v0 = 0, v1 = 0;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (s0 + u < NSG) {
              const int t0v = __shfl_sync(0xffffffffu, va[0][s0 + u], lane & ~3);
              const int t1v = __shfl_sync(0xffffffffu, va[1][s0 + u], lane & ~3);
              if (l == u) {
                v0 = t0v;
                v1 = t1v;
              }
            }
          }
          const int sg = s0 + l;
          if (ok && sg < NSG && slice_byte0 + sg * SEG * 16 < (uint32_t)a.q.row_bytes) {
            const float4 fa = sx[gseg0 + sg];
            const uint32_t gi = (uint32_t)(sg * SEG * 16) >> a.gbytes_shift;
            float sc, gm;
            group_meta(0, gi, sc, gm);
            acc[0] = fmaf(sc * fa.x, (float)v0, fmaf(gm, fa.y, acc[0]));
            group_meta(1, gi, sc, gm);
            acc[1] = fmaf(sc * fa.x, (float)v1, fmaf(gm, fa.y, acc[1]));
          }
        }
      } else {
#pragma unroll
      for (int sg = 0; sg < NSG; ++sg) {
        if (!ok || slice_byte0 + sg * SEG * 16 >= (uint32_t)a.q.row_bytes) break;
        int ci[2][2][4];   // [token group][chain][fragment]
#pragma unroll
        for (int g = 0; g < 2; ++g)
#pragma unroll
          for (int u = 0; u < 2; ++u) ci[g][u][0] = ci[g][u][1] = ci[g][u][2] = ci[g][u][3] = 0;
#pragma unroll
        for (int cj = 0; cj < SEG; ++cj) {
          const int cb = (sg * SEG + cj) * 16;
          const uint32_t w0 = *reinterpret_cast<const uint32_t*>(arow0 + cb);
          const uint32_t w1 = *reinterpret_cast<const uint32_t*>(arow1 + cb);
          const int ch = ch_slice + sg * SEG + cj;
#pragma unroll
          for (int m = 0; m < NM; ++m) {
            uint32_t A0, A1, A2, A3;
            int J;
            unpack(w0, w1, ch, m, A0, A1, A2, A3, J);
            const int u = (cj * NM + m) & 1;
            const uint2 b0 = has_b0 ? xi_lane0[J * xcols * 4] : make_uint2(0u, 0u);
            imma16832(ci[0][u], A0, A1, A2, A3, b0.x, b0.y);
            if (two) {
              const uint2 b1 = has_b1 ? xi_lane1[J * xcols * 4] : make_uint2(0u, 0u);
              imma16832(ci[1][u], A0, A1, A2, A3, b1.x, b1.y);
            }
          }
        }
        const float4 fa = toka ? sxa[gseg0 + sg] : zero4;
        const float4 fb = tokb ? sxb[gseg0 + sg] : zero4;
        const uint32_t gi = (uint32_t)(sg * SEG * 16) >> a.gbytes_shift;   // group within the slice
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          float sc, gm;
          group_meta(r, gi, sc, gm);
          const int va = 256 * (ci[0][0][2 * r] + ci[0][1][2 * r]) + (ci[0][0][2 * r + 1] + ci[0][1][2 * r + 1]);
          acc[r] = fmaf(sc * fa.x, (float)va, fmaf(gm, fa.y, acc[r]));
          if (two) {
            const int vb = 256 * (ci[1][0][2 * r] + ci[1][1][2 * r]) + (ci[1][0][2 * r + 1] + ci[1][1][2 * r + 1]);
            acc[2 + r] = fmaf(sc * fb.x, (float)vb, fmaf(gm, fb.y, acc[2 + r]));
          }
        }
      }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + s);
    TS_PROF(long long pf_c = clock64(); pf_math += pf_c - pf_b;)

    const bool last_kg = kg == KG - 1;
    if (last_kg || t0 + i + 1 == t1) {
      // ---- flush row block rb: reduce the 8 warps' k-slices through smem ----
      float* rw = red + warp * kTileRows * kMaxTok;
      if constexpr (CB) {
        rw[q * kMaxTok + 2 * l] = acc[0];
        rw[q * kMaxTok + 2 * l + 1] = acc[1];
        rw[(q + 8) * kMaxTok + 2 * l] = acc[2];
        rw[(q + 8) * kMaxTok + 2 * l + 1] = acc[3];
      } else {
        if (a.mt == 1) {   // the four lanes of a row pair hold partials of token 0
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], 1);
            acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], 2);
          }
        }
        rw[q * kMaxTok + l] = acc[0];
        rw[(q + 8) * kMaxTok + l] = acc[1];
        rw[q * kMaxTok + 4 + l] = acc[2];
        rw[(q + 8) * kMaxTok + 4 + l] = acc[3];
      }
      acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
      named_bar_sync(1, kConsumerThreads);
      const int t = threadIdx.x;                 // t < 128: (row t/8, token t%8)
      const int rr = t >> 3, n = t & 7;
      const int64_t row = (int64_t)rb * kTileRows + rr;
      float tot = 0.f;
      if (t < kTileRows * kMaxTok) {
        for (int w = 0; w < kConsumerWarps; ++w) tot += red[(w * kTileRows + rr) * kMaxTok + n];
        if (started_here) tot += epi[((rb - rb_own0) * kTileRows + rr) * kMaxTok + n];
      }
      if (started_here && last_kg) {
        if (t < kTileRows * kMaxTok && n < a.mt && row < a.q.rows)
          store_f(a.out, a.out_dtype, (a.m0 + n) * a.out_stride + row,
                  a.residual ? tot + __ldcg(a.residual + (a.m0 + n) * a.residual_stride + row) : tot);
      } else {
        const int slot = rb == first_rb ? 0 : 1;
        if (t < kTileRows * kMaxTok)
          a.partials[((size_t)blockIdx.x * 2 + slot) * (kTileRows * kMaxTok) + t] = tot;
        __threadfence();
        named_bar_sync(1, kConsumerThreads);
        if (t == 0) *s_flag = atomicAdd(a.counters + rb, 1);
        named_bar_sync(1, kConsumerThreads);
        const int old = *s_flag;
        const uint64_t u0 = (uint64_t)rb * KG;
        int pieces = 1;
        for (uint32_t cc = 1, prev = cta_of(u0 / Q, UQ, GR); cc < KG; ++cc) {
          const uint32_t w = cta_of((u0 + cc) / Q, UQ, GR);
          pieces += w != prev;
          prev = w;
        }
        if (old == pieces - 1) {
          __threadfence();
          float sum = 0.f;
          for (uint32_t cc = 0, prev = 0xFFFFFFFFu; cc < KG; ++cc) {
            const uint32_t pc = cta_of((u0 + cc) / Q, UQ, GR);
            if (pc == prev) continue;
            prev = pc;
            const uint32_t pfirst = (uint32_t)((UQ * pc / GR * Q) / KG);
            if (t < kTileRows * kMaxTok)
              sum += __ldcg(a.partials + ((size_t)pc * 2 + (rb == pfirst ? 0 : 1)) * (kTileRows * kMaxTok) + t);
          }
          if (t < kTileRows * kMaxTok && n < a.mt && row < a.q.rows)
            store_f(a.out, a.out_dtype, (a.m0 + n) * a.out_stride + row,
                    a.residual ? sum + __ldcg(a.residual + (a.m0 + n) * a.residual_stride + row) : sum);
          if (t == 0) a.counters[rb] = 0;
        }
      }
      named_bar_sync(1, kConsumerThreads);  // `red` and `s_flag` are reused by the next flush
    }
    TS_PROF(pf_flush += clock64() - pf_c;)
    if (last_kg) {
      kg = 0;
      ++rb;
      started_here = true;
    } else {
      ++kg;
    }
  }
  TS_PROF(if (threadIdx.x == 0) {
    unsigned long long* pr = g_gemv_prof[blockIdx.x];   // consumer warp 0, lane 0
    if (layer == 0) pr[1] = (unsigned long long)pf_t;
    pr[2] += pf_wait;
    pr[3] += pf_math;
    pr[4] += pf_flush;
    pr[5] += t1 - t0;
    pr[7] = (unsigned long long)clock64();
  })
}

template <int BITS, bool CB, bool DQ, int SEG, int NL>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) qgemv_kernel(const __grid_constant__ Chain<NL> c) {
  extern __shared__ __align__(128) char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  int* s_flag = reinterpret_cast<int*>(empty + kMaxStages);   // [0] flush arrival, [1] abort
  float* s_rstd = reinterpret_cast<float*>(s_flag + 4);        // [kMaxTok] RMSNorm factors
  char* body = smem + kHeadBytes;
  const Args& a0 = c.L[0];
  TS_PROF(if (threadIdx.x == 0) {
    for (int k = 1; k < 8; ++k) g_gemv_prof[blockIdx.x][k] = 0;
    g_gemv_prof[blockIdx.x][0] = (unsigned long long)clock64();
  })
  const int S = a0.stages;
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(full + i, 1);   // the producer's expect_tx arrival (async-copy arrivals register themselves)
      mbar_init(empty + i, kConsumerWarps);
    }
    s_flag[1] = 0;
    fence_barrier_init();
  }
  __syncthreads();
  const int n = NL == 1 ? 1 : c.n;
  const bool producer = (threadIdx.x >> 5) == kConsumerWarps;
  if (producer) pdl_launch_dependents();
  int rs = 0;
  uint32_t rph = 0, issued = 0;
  for (int L = 0; L < n; ++L) {
    gemv_layer<BITS, CB, DQ, SEG>(c.L[L], body, full, empty, s_flag, s_rstd, rs, rph, issued, L,
                                  NL == 1 ? nullptr : c.sync);
    if (!producer && NL > 1 && L + 1 < n) {
      // every output of this CTA for layer L is stored: count it in
      named_bar_sync(1, kConsumerThreads);
      if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(c.sync + L, 1);
      }
    }
  }
  if (producer) {
    // let the copies still in flight (the last S issues at most) land before
    // this CTA's shared memory goes away: after a timeout the consumers stop
    // waiting for them (in a normal run these phases have completed already)
    for (uint32_t k = issued > (uint32_t)S ? issued - S : 0; k < issued; ++k)
      mbar_wait_hint(full + (k % S), (k / S) & 1, nullptr, 0, a0.wait_ns);
    return;
  }
  if (NL > 1 && n > 1) {
    // the last CTA out zeroes the chain counters for the next launch (no CTA
    // polls them any more once every CTA has counted itself out)
    named_bar_sync(1, kConsumerThreads);
    if (threadIdx.x == 0) {
      __threadfence();
      if (atomicAdd(c.sync + kMaxChain, 1) == (int)gridDim.x - 1) {
        for (int L = 0; L + 1 < n; ++L) c.sync[L] = 0;
        c.sync[kMaxChain] = 0;
        __threadfence();
      }
    }
  }
}

}  // namespace gemv

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

int ilog2(int64_t v) {
  int r = 0;
  while ((int64_t(1) << (r + 1)) <= v) ++r;
  return r;
}

struct Plan {
  uint32_t tiles, kgroups, grid, quantum;
  int n_chunks, seg_chunks, gpt, meta_row_words, stage_bytes, max_owned_rows;
  bool meta_bulk;   // metadata rows are 16-byte multiples: 2-D copies into dense row slots
};

// Metadata of every tile row starts on a 16-byte boundary (and the arrays
// are 16-byte aligned), so a tile's metadata is one 2-D box per array.
static bool meta_bulk_ok(const ts_qweight& w, int gpt) {
  const bool dq = w.dq_scale_codes != nullptr;
  const int step = dq ? 16 : 8;   // elements per 16 bytes of metadata
  bool bulk = w.n_groups % step == 0 && gpt % step == 0;
  if (dq) {
    const int64_t n_sup = (w.rows * w.n_groups + w.dq_group_size - 1) / w.dq_group_size;
    bulk = bulk && n_sup % 4 == 0 && is_aligned(w.dq_scale_codes, 16) && is_aligned(w.dq_gmin_codes, 16) &&
           is_aligned(w.dq_scale_meta, 16) && is_aligned(w.dq_gmin_meta, 16);
  } else {
    bulk = bulk && is_aligned(w.scale, 16) && is_aligned(w.gmin, 16);
  }
  return bulk;
}

int lut_bytes(const ts_qweight& w) { return w.codebook ? (w.bits == 2 ? 256 * 32 * 8 : 256 * 32 * 4) : 0; }

Plan make_plan(const ts_qweight& w) {
  Plan p;
  const int64_t gbytes = (int64_t)w.group_size * w.bits / 8;
  const int E = w.dq_scale_codes ? 4 : 2;
  p.kgroups = (uint32_t)((w.packed_row_bytes + gemv::kTileK - 1) / gemv::kTileK);
  const uint32_t rbs = (uint32_t)((w.rows + gemv::kTileRows - 1) / gemv::kTileRows);
  p.tiles = rbs * p.kgroups;
  p.grid = std::max<uint32_t>(1, std::min<uint32_t>((uint32_t)sm_count() * gemv::kCtasPerSm, p.tiles));
  // Row blocks of several tiles: hand out whole row blocks when that costs at
  // most two tiles of imbalance on the busiest CTA. A row block split between
  // CTAs is finished through global partial sums, a fence and an atomic, whose
  // latency under full HBM load costs more than that.
  p.quantum = 1;
  if (p.kgroups > 1) {
    const uint32_t g_rb = std::min(p.grid, rbs);
    const double avg = (double)p.tiles / p.grid;
    const double max_whole = (double)((rbs + g_rb - 1) / g_rb) * p.kgroups;
    if (max_whole - avg <= 2.0) {
      p.quantum = p.kgroups;
      p.grid = g_rb;
    }
  }
  p.n_chunks = (int)(w.padded_cols * w.bits / 128);
  p.seg_chunks = (int)std::min<int64_t>(4, gbytes / 16);
  p.gpt = (int)(gemv::kTileK / gbytes);
  p.meta_bulk = meta_bulk_ok(w, p.gpt);
  // dense rows of exactly gpt elements for the 2-D copies; otherwise 16-byte
  // slots wide enough for the aligned-down words of a misaligned row
  p.meta_row_words = p.meta_bulk ? p.gpt / E : (int)align_up((size_t)((p.gpt + 2 * (E - 1)) / E), 4);
  size_t meta = (size_t)2 * gemv::kTileRows * p.meta_row_words * 4;
  if (w.dq_scale_codes) meta += (size_t)2 * gemv::kMaxSupers * 4;
  p.stage_bytes = (int)align_up((size_t)gemv::kTileRows * gemv::kPitch + meta, 128);
  const uint32_t per_cta = (p.tiles + p.grid - 1) / p.grid;
  p.max_owned_rows = (int)((per_cta / p.kgroups + 2) * gemv::kTileRows);
  return p;
}

// shared memory besides the stage ring, for `mt` tokens
size_t fixed_smem(const ts_qweight& w, const Plan& p, int mt) {
  const int mpw = 8 / w.bits;
  const size_t n_mma = (size_t)p.n_chunks * mpw;
  const size_t n_seg = (size_t)p.n_chunks / p.seg_chunks;
  return lut_bytes(w) + (size_t)mt * (n_mma * 4 + 4) * 8 + (size_t)mt * n_seg * 16 +
         (size_t)p.max_owned_rows * gemv::kMaxTok * 4 +
         (size_t)gemv::kConsumerWarps * gemv::kTileRows * gemv::kMaxTok * 4 +
         (size_t)(p.max_owned_rows + 4) * 4 + (size_t)gemv::kOutCap * 8 + (size_t)(p.max_owned_rows + 4) * 4 +
         gemv::kHeadBytes + 64;
}

size_t smem_cap() { return (size_t)std::min(max_smem_optin(), 227 * 1024 / gemv::kCtasPerSm - (gemv::kCtasPerSm - 1) * 1024); }

int stages_for(const ts_qweight& w, const Plan& p, int mt) {
  const size_t f = fixed_smem(w, p, mt);
  if (f >= smem_cap()) return 0;
  return (int)std::min<size_t>(gemv::kMaxStages, (smem_cap() - f) / p.stage_bytes);
}

template <int BITS, bool CB, bool DQ, int SEG, int NL>
int launch_one(const gemv::Chain<NL>& c, uint32_t grid, cudaStream_t stream, size_t smem) {
  auto kern = gemv::qgemv_kernel<BITS, CB, DQ, SEG, NL>;
  static thread_local int configured_dev = -1;
  static thread_local size_t configured_smem = 0;
  int dev = 0;
  TS_CUDA_TRY(cudaGetDevice(&dev));
  if (configured_dev != dev || configured_smem < smem) {
    TS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    configured_dev = dev;
    configured_smem = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(gemv::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = NL == 1 ? 1 : 0;
  if (NL > 1) {
    // the layers of a chain wait for one another across CTAs, so every CTA
    // must fit on the device at once (the waits are bounded all the same)
    int per_sm = 0;
    TS_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, gemv::kThreads, smem));
    TS_UNSUPPORTED((int64_t)per_sm * sm_count() >= (int64_t)grid, "qlinear chain: %u CTAs do not fit at once",
                   grid);
  }
  TS_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, c));
  count_launch();
  return TS_OK;
}

template <int BITS, bool CB, bool DQ, int NL>
int launch_seg(int seg, const gemv::Chain<NL>& c, uint32_t grid, cudaStream_t s, size_t smem) {
  if (seg == 1) return launch_one<BITS, CB, DQ, 1, NL>(c, grid, s, smem);
  if (seg == 2) return launch_one<BITS, CB, DQ, 2, NL>(c, grid, s, smem);
  return launch_one<BITS, CB, DQ, 4, NL>(c, grid, s, smem);
}

template <int BITS, int NL>
int launch_bits(bool cb, bool dq, int seg, const gemv::Chain<NL>& c, uint32_t grid, cudaStream_t s, size_t smem) {
  if (cb)
    return dq ? launch_seg<BITS, true, true, NL>(seg, c, grid, s, smem)
              : launch_seg<BITS, true, false, NL>(seg, c, grid, s, smem);
  return dq ? launch_seg<BITS, false, true, NL>(seg, c, grid, s, smem)
            : launch_seg<BITS, false, false, NL>(seg, c, grid, s, smem);
}

template <int NL>
int launch_chain(const ts_qweight& w, int seg, const gemv::Chain<NL>& c, uint32_t grid, cudaStream_t s,
                 size_t smem) {
  const bool cb = w.codebook != nullptr, dq = w.dq_scale_codes != nullptr;
  if (w.bits == 4) return launch_bits<4, NL>(cb, dq, seg, c, grid, s, smem);
  if (w.bits == 2) return launch_bits<2, NL>(cb, dq, seg, c, grid, s, smem);
  return launch_bits<8, NL>(cb, dq, seg, c, grid, s, smem);
}

}  // namespace

// Whether the tensor-core GEMV covers this weight layout: whole 16-byte
// chunks per group (group bytes a power of two in [16, 2048]), a 16-byte row
// pitch, and (double quantization) few enough super-groups per tile.
bool gemv_supported(const ts_qweight& w) {
  const int64_t gbytes = (int64_t)w.group_size * w.bits / 8;
  if (!(w.bits == 2 || w.bits == 4 || w.bits == 8) || gbytes < 16 || gbytes > gemv::kTileK ||
      (gbytes & (gbytes - 1)) != 0)
    return false;
  if (w.rows * w.n_groups >= (int64_t(1) << 31) || w.packed_row_bytes >= (int64_t(1) << 30) ||
      w.packed_row_bytes % 16 != 0 || !is_aligned(w.packed, 16) || w.packed_row_bytes * 8 / w.bits < w.padded_cols)
    return false;
  if (w.dq_scale_codes) {
    const int64_t gpt = gemv::kTileK / gbytes;
    if (15 * w.n_groups + gpt > (int64_t)(gemv::kMaxSupers - 2) * w.dq_group_size) return false;
  }
  return true;
}

// Workspace layout, the same for every weight on a device so that one
// workspace can serve layers of different shapes: the per-CTA partial sums
// first (each slot is written before it is read, so stale values are
// harmless), then the 256-byte error-flag block, then one counter per row
// block (the only part that must start at zero; every call leaves it zeroed).
// Both builds of this file (one and two CTAs per SM) use the same layout,
// sized for the larger grid, because one workspace serves calls of either:
// two partial slots per CTA of a grid of SMs x kLayoutCtasPerSm.
constexpr int kLayoutCtasPerSm = 2;
static_assert(gemv::kCtasPerSm <= kLayoutCtasPerSm, "workspace layout sized for at most two CTAs per SM");
static size_t gemv_partials_bytes() {
  return align_up((size_t)sm_count() * kLayoutCtasPerSm * 2 * gemv::kTileRows * gemv::kMaxTok * sizeof(float), 256);
}

// Byte offset of the wait-timeout flag in the workspace; the row-block
// counters start 256 bytes later.
size_t gemv_error_flag_offset() { return gemv_partials_bytes(); }

size_t gemv_workspace_size(const ts_qweight& w) {
  const int64_t rbs = (w.rows + gemv::kTileRows - 1) / gemv::kTileRows;
  return gemv_partials_bytes() + 256 + align_up((size_t)rbs * sizeof(int), 256);
}

// Largest token count per pass that fits shared memory with >= 2 stages.
int gemv_max_tokens(const ts_qweight& w) {
  const Plan p = make_plan(w);
  for (int mt = gemv::kMaxTok; mt >= 1; --mt)
    if (stages_for(w, p, mt) >= 2) return mt;
  return 0;
}

namespace {

// Kernel arguments of one layer (everything but the pass: m0, mt, stages).
int make_args(const GemvOp& op, const Plan& p, void* workspace, gemv::Args& a) {
  const ts_qweight& w = *op.w;
  a = gemv::Args{};
  a.q = make_qw(w);
  a.x = op.x;
  a.x_dtype = op.x_dtype;
  a.x_stride = op.x_stride;
  a.bias = op.bias;
  a.bias_dtype = op.bias_dtype;
  a.out = op.out;
  a.out_dtype = op.out_dtype;
  a.out_stride = op.out_stride;
  char* ws = reinterpret_cast<char*>(workspace);
  a.partials = reinterpret_cast<float*>(ws);
  a.err = reinterpret_cast<int*>(ws + gemv_partials_bytes());
  a.wait_ns = wait_limit_ns();
  a.gated = op.gated;
  a.act_dtype = op.act_dtype;
  a.norm_w = op.norm_w;
  a.norm_eps = op.norm_eps;
  a.residual = op.residual;
  a.residual_stride = op.residual_stride;
  a.counters = reinterpret_cast<int*>(ws + gemv_partials_bytes() + 256);
  a.tiles = p.tiles;
  a.kgroups = p.kgroups;
  a.grid = p.grid;
  a.quantum = p.quantum;
  a.stage_bytes = p.stage_bytes;
  a.meta_row_words = p.meta_row_words;
  a.n_chunks = p.n_chunks;
  a.seg_chunks = p.seg_chunks;
  a.gpt = p.gpt;
  a.max_owned_rows = p.max_owned_rows;
  a.gbytes_shift = ilog2((int64_t)w.group_size * w.bits / 8);
  a.dq_shift = -1;
  if (w.dq_group_size > 0 && (w.dq_group_size & (w.dq_group_size - 1)) == 0) a.dq_shift = ilog2(w.dq_group_size);
  const bool dq = w.dq_scale_codes != nullptr;
  const int64_t esz = op.x_dtype == TS_F32 ? 4 : 2;
  a.x_vec16 = is_aligned(op.x, 16) && (op.x_stride * esz) % 16 == 0 && (!op.gated || (w.cols * esz) % 16 == 0);
  a.meta_bulk = p.meta_bulk ? 1 : 0;
  if (p.meta_bulk) {
    const CUtensorMapDataType t = dq ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
    const uint64_t eb = dq ? 1 : 2;
    int rc = encode_tmap_2d(&a.smap, dq ? (const void*)w.dq_scale_codes : w.scale, t, (uint64_t)w.n_groups,
                            (uint64_t)w.rows, (uint64_t)w.n_groups * eb, (uint32_t)p.gpt, gemv::kTileRows,
                            CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != TS_OK) return rc;
    rc = encode_tmap_2d(&a.gmap, dq ? (const void*)w.dq_gmin_codes : w.gmin, t, (uint64_t)w.n_groups,
                        (uint64_t)w.rows, (uint64_t)w.n_groups * eb, (uint32_t)p.gpt, gemv::kTileRows,
                        CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != TS_OK) return rc;
  }
  return TS_OK;
}

}  // namespace

int run_gemv(const GemvOp& op, int64_t M, void* workspace, size_t ws_bytes, cudaStream_t stream) {
  const ts_qweight& w = *op.w;
  const int max_mt = gemv_max_tokens(w);
  TS_UNSUPPORTED(max_mt > 0, "qlinear: activations of %lld columns do not fit in shared memory",
                 (long long)w.cols);
  TS_REQUIRE(ws_bytes >= gemv_workspace_size(w), "qlinear: workspace too small (%zu < %zu)", ws_bytes,
             gemv_workspace_size(w));
  const Plan p = make_plan(w);
  gemv::Chain<1> c;
  c.n = 1;
  c.sync = nullptr;
  gemv::Args& a = c.L[0];
  int rc = make_args(op, p, workspace, a);
  if (rc != TS_OK) return rc;
  a.stall = take_test_stall() ? 1 : 0;
  for (int64_t m0 = 0; m0 < M; m0 += max_mt) {
    a.m0 = m0;
    a.mt = (int)std::min<int64_t>(max_mt, M - m0);
    a.stages = stages_for(w, p, a.mt);
    const size_t smem = fixed_smem(w, p, a.mt) + (size_t)a.stages * p.stage_bytes;
    rc = launch_chain<1>(w, p.seg_chunks, c, p.grid, stream, smem);
    if (rc != TS_OK) return rc;
  }
  return TS_OK;
}

// Whether run_gemv_chain takes these layers: one pass each (M tokens), the
// same kernel instantiation and stage layout for all, at most kMaxChain.
bool gemv_chain_ok(const GemvOp* ops, int n, int64_t M) {
  if (n < 1 || n > gemv::kMaxChain || M < 1) return false;
  const ts_qweight& w0 = *ops[0].w;
  const Plan p0 = make_plan(w0);
  for (int i = 0; i < n; ++i) {
    const ts_qweight& w = *ops[i].w;
    if (!gemv_supported(w) || M > gemv_max_tokens(w)) return false;
    if (w.bits != w0.bits || w.group_size != w0.group_size || (w.codebook != nullptr) != (w0.codebook != nullptr) ||
        (w.dq_scale_codes != nullptr) != (w0.dq_scale_codes != nullptr))
      return false;
    const Plan p = make_plan(w);
    if (p.seg_chunks != p0.seg_chunks) return false;
  }
  return true;
}

int run_gemv_chain(const GemvOp* ops, int n, int64_t M, void* workspace, size_t ws_bytes, cudaStream_t stream) {
  TS_UNSUPPORTED(gemv_chain_ok(ops, n, M), "these layers do not form one decode chain");
  gemv::Chain<gemv::kMaxChain> c;
  c.n = n;
  c.sync = reinterpret_cast<int*>(reinterpret_cast<char*>(workspace) + gemv_partials_bytes() + 64);
  size_t fixed = 0;
  uint32_t grid = 1;
  int stages = gemv::kMaxStages;
  int seg = 0, stage_bytes = 0;
  for (int i = 0; i < n; ++i) {
    const ts_qweight& w = *ops[i].w;
    TS_REQUIRE(ws_bytes >= gemv_workspace_size(w), "qlinear chain: workspace too small (%zu < %zu)", ws_bytes,
               gemv_workspace_size(w));
    const Plan p = make_plan(w);
    int rc = make_args(ops[i], p, workspace, c.L[i]);
    if (rc != TS_OK) return rc;
    c.L[i].m0 = 0;
    c.L[i].mt = (int)M;
    c.L[i].stall = 0;
    fixed = std::max(fixed, fixed_smem(w, p, (int)M));
    grid = std::max(grid, p.grid);
    seg = p.seg_chunks;
    stage_bytes = std::max(stage_bytes, p.stage_bytes);   // rows first, then the layer's metadata
  }
  TS_UNSUPPORTED(fixed < smem_cap(), "qlinear chain: shared memory");
  stages = (int)std::min<size_t>(gemv::kMaxStages, (smem_cap() - fixed) / stage_bytes);
  TS_UNSUPPORTED(stages >= 2, "qlinear chain: shared memory for two stages");
  c.L[0].stall = take_test_stall() ? 1 : 0;
  for (int i = 0; i < n; ++i) {
    c.L[i].stages = stages;
    c.L[i].stage_bytes = stage_bytes;
  }
  const size_t smem = fixed + (size_t)stages * stage_bytes;
  return launch_chain<gemv::kMaxChain>(*ops[0].w, seg, c, grid, stream, smem);
}

#ifdef TS_GEMV_PROF
int gemv_prof_read(void* dst) {
  TS_CUDA_TRY(cudaMemcpyFromSymbol(dst, gemv::g_gemv_prof, sizeof(gemv::g_gemv_prof)));
  return TS_OK;
}
#endif

}  // namespace TS_GEMV_NS
}  // namespace ts

#ifdef TS_GEMV_PROF
#define TS_PROF_CAT2(a, b) a##b
#define TS_PROF_CAT(a, b) TS_PROF_CAT2(a, b)
extern "C" __attribute__((visibility("default"))) int TS_PROF_CAT(ts_prof_read_, TS_GEMV_NS)(void* dst) { return ts::TS_GEMV_NS::gemv_prof_read(dst); }
#endif
