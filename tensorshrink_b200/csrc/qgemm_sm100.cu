// Prefill-shaped fused dequant-GEMM on the 5th-generation tensor cores.
//
//   out[M, N] = x[M, K] . W[N, K]^T (+ outliers) (+ bias),  W in the packed
//   GOAP layout (codes + per-group scale/min or their double-quantized form,
//   optional fp32 codebook, CSR outlier tables).
//
// Replaces the reference's M > 64 path (modules.py:898-922: dequantize_weight
// to a dense compute-dtype matrix, triton_kernels.py:1003-1186, then F.linear)
// with one persistent kernel that never writes the dense matrix. A tile is
// 128 weight rows x BT tokens; the MMA computes D[weight row, token] with the
// dequantized weights as the A operand in tensor memory and the activations
// as the B operand in shared memory:
//
//   warp 0      TMA producer: activation tile [BT tokens x 64] (128B swizzle),
//               packed code tile [128 rows x 64 columns], and blocks of group
//               metadata [128 rows x 16 bytes] -> shared memory
//   warp 1      MMA issuer: one thread issues tcgen05.mma M=128 x N=BT x K=16
//               (4 per stage) from TMEM (A) and shared memory (B)
//   warps 2-5   epilogue: tcgen05.ld of the fp32 accumulator (one weight row per
//               thread, 32 tokens per load), + bias, convert, coalesced stores
//   warps 6-21  dequantizers, four groups of four warps taking every fourth
//               stage (a stage's conversion is one long dependent chain per
//               thread, so four groups keep four stages of work in flight):
//               one thread per weight row (= its TMEM lane), 64 columns per
//               stage, unpack codes to the activation dtype in registers,
//               patch the row's outliers in place as fp32(base + delta)
//               rounded once, and store the result into the stage's TMEM
//               columns.
//
// Keeping the dequantized tile out of shared memory leaves shared-memory
// bandwidth to the activation operand alone (the tensor core reads A from
// TMEM), which is what bounds a design that stages both operands there.
// Every wait is bounded in wall-clock time: on timeout the kernel records an
// error flag and all roles unwind to the final barrier, where the TMEM is freed.
#include <algorithm>
#include <cmath>

#include "sm100.cuh"

namespace ts {
namespace qgemm {

constexpr int kBW = 128;        // weight rows per tile = UMMA M = TMEM lanes
constexpr int kBK = 64;         // K per stage = one 128-byte swizzle row of 16-bit values
constexpr int kEpiWarps = 4;
constexpr int kDqGroups = 4;    // dequantizer groups, taking every fourth stage
constexpr int kDqGroupWarps = 4;  // per group: one per TMEM lane quadrant (one thread per stage row)
constexpr int kDqWarps = kDqGroups * kDqGroupWarps;
constexpr int kFirstDqWarp = 2 + kEpiWarps;
constexpr int kThreads = (kFirstDqWarp + kDqWarps) * 32;
constexpr int kTmemCols = 512;
constexpr int kAStageCols = kBK / 2;   // 64 16-bit values per lane = 32 columns
constexpr int kPrefetchStages = 32;    // L2 prefetch distance of the code stream

__device__ int g_err;           // wait-timeout flag, read and cleared by ts_qlinear_status

#ifdef TS_QGEMM_PROF
// Phase cycles of an instrumented build (never the shipped library), per CTA:
// [0] MMA waits on loaded stages, [1] MMA waits on converted stages, [2] MMA
// waits on the drained accumulator, [3] stages issued by the MMA thread,
// [4] dequantizer (group 0, warp lane 0) waits on free TMEM stages, [5] its
// waits on loaded stages, [6] its conversion cycles, [7] its store-wait
// cycles, [8] its metadata waits, [9] producer waits on free stages,
// [10] kernel cycles (MMA thread), [11] epilogue waits on the accumulator.
__device__ unsigned long long g_qgemm_prof[512][12];
#define TS_QPROF(...) __VA_ARGS__
#else
#define TS_QPROF(...)
#endif

struct Args {
  QW q;
  int64_t M;
  const void* bias;
  int bias_dtype;
  void* out;
  int out_dtype;
  int64_t out_stride;
  int tblocks, wblocks, kblocks;   // token blocks, weight-row blocks, stages per tile
  int stages;
  int meta_tma;      // group metadata by TMA blocks (else per-thread loads)
  int meta_groups;   // groups per metadata block (8 fp16 or 16 code bytes = 16 B)
  int gs_shift;      // log2(group_size)
  int dq_shift;      // log2(dq_group_size), or -1 when it is not a power of two
  uint64_t wait_ns;  // limit of every barrier wait
  int stall;         // test hook: the producer issues no copies, so the first waits run out
  int split;         // CTAs take equal ranges of K-stages (tiles split between CTAs)
  float* partials;   // split: [grid][2][128 rows][BT tokens] fp32
  int* counters;     // split: one per tile, zero between calls
  int prefetch_codes;  // L2-prefetch each item's code columns through cmap_wide
  int qcap;          // outlier queue entries per dequantizer thread (0: read the tables in place)
};

// ---- dequantization of 8-column chunks ----------------------------------------
// Output: 4 words of two 16-bit values (columns 2i, 2i+1 in word i), in the
// activation dtype (XT = 1: bf16, XT = 0: fp16).

template <int XT>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if (XT) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// 4-bit uniform codes: (code | magic exponent) is exactly 2^e + code in the
// 16-bit type; subtracting 2^e + 8 gives the centred code c - 8 exactly, and
// one fused multiply-add applies (scale, min + 8 scale), both rounded to the
// activation dtype. Centring keeps the rounded offset near the group's middle
// value instead of its minimum, which roughly halves the rounding error of
// the reconstructed weight in bf16.
template <int XT>
__device__ __forceinline__ uint4 dq4_uniform(uint32_t w, uint32_t s2, uint32_t g2) {
  constexpr uint32_t kMagicByte = XT ? 0x43u : 0x64u;            // 128.0 bf16 / 1024.0 fp16
  constexpr uint32_t kMagic2 = XT ? 0x43084308u : 0x64086408u;   // 136.0 bf16 / 1032.0 fp16
  const uint32_t lo = w & 0x0F0F0F0Fu;                            // codes 0,2,4,6
  const uint32_t hi = (w >> 4) & 0x0F0F0F0Fu;                     // codes 1,3,5,7
  const uint32_t p0 = prmt(lo, hi, 0x5140);                       // bytes c0 c1 c2 c3
  const uint32_t p1 = prmt(lo, hi, 0x7362);                       // bytes c4 c5 c6 c7
  uint32_t o[4] = {prmt(p0, kMagicByte, 0x4140), prmt(p0, kMagicByte, 0x4342), prmt(p1, kMagicByte, 0x4140),
                   prmt(p1, kMagicByte, 0x4342)};
  uint4 r;
  uint32_t* rr = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (XT) {
      const __nv_bfloat162 c = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&o[i]),
                                       *reinterpret_cast<const __nv_bfloat162*>(&kMagic2));
      const __nv_bfloat162 v = __hfma2(c, *reinterpret_cast<const __nv_bfloat162*>(&s2),
                                       *reinterpret_cast<const __nv_bfloat162*>(&g2));
      rr[i] = *reinterpret_cast<const uint32_t*>(&v);
    } else {
      const __half2 c = __hsub2(*reinterpret_cast<const __half2*>(&o[i]),
                                *reinterpret_cast<const __half2*>(&kMagic2));
      const __half2 v = __hfma2(c, *reinterpret_cast<const __half2*>(&s2), *reinterpret_cast<const __half2*>(&g2));
      rr[i] = *reinterpret_cast<const uint32_t*>(&v);
    }
  }
  return r;
}

// 2-bit codes (uniform or codebook) through a 4-entry value table held in two
// registers (entry j = 16-bit value of level j for this row and group): byte
// permutes select each pair of values. w holds 16 codes = 2 chunks.
__device__ __forceinline__ void dq2_lut(uint32_t w, uint32_t L0, uint32_t L1, uint4& c0, uint4& c1) {
  const uint32_t A = (w & 0x33333333u) << 1;       // nibble n: 2 * code(2n)
  const uint32_t B = (w >> 1) & 0x66666666u;       // nibble n: 2 * code(2n+1)
  const uint32_t LE = (A & 0x0F0F0F0Fu) * 0x11u + 0x10101010u;          // selector low bytes, pairs 0,2,4,6
  const uint32_t LO = ((A >> 4) & 0x0F0F0F0Fu) * 0x11u + 0x10101010u;   // pairs 1,3,5,7
  const uint32_t HE = (B & 0x0F0F0F0Fu) * 0x11u + 0x10101010u;
  const uint32_t HO = ((B >> 4) & 0x0F0F0F0Fu) * 0x11u + 0x10101010u;
  const uint32_t s02 = prmt(LE, HE, 0x5140), s46 = prmt(LE, HE, 0x7362);
  const uint32_t s13 = prmt(LO, HO, 0x5140), s57 = prmt(LO, HO, 0x7362);
  c0.x = prmt(L0, L1, s02);
  c0.y = prmt(L0, L1, s13);
  c0.z = prmt(L0, L1, s02 >> 16);
  c0.w = prmt(L0, L1, s13 >> 16);
  c1.x = prmt(L0, L1, s46);
  c1.y = prmt(L0, L1, s57);
  c1.z = prmt(L0, L1, s46 >> 16);
  c1.w = prmt(L0, L1, s57 >> 16);
}

// Generic path (8-bit codes, 4-bit codebook): fp32 value, fp32 fma, one rounding.
template <int BITS, bool CB, int XT>
__device__ __forceinline__ uint4 dq_generic(const uint32_t* cw, const float* cbs, float s, float g) {
  float v[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    uint32_t c;
    if (BITS == 8)
      c = (cw[e >> 2] >> ((e & 3) * 8)) & 0xFFu;
    else
      c = (cw[0] >> (e * 4)) & 0xFu;
    const float cv = CB ? cbs[c] : __int_as_float(0x4B000000 | (int)c) - 8388608.f;
    v[e] = fmaf(cv, s, g);
  }
  return make_uint4(pack2<XT>(v[0], v[1]), pack2<XT>(v[2], v[3]), pack2<XT>(v[4], v[5]), pack2<XT>(v[6], v[7]));
}

// 32 columns (one dequantizer's half of a stage row) -> 16 words of two
// 16-bit values. G = groups in those 32 columns (1, or 2 for 16-column groups),
// a compile-time constant so every per-group register is statically indexed.
template <int BITS, bool CB, int XT, int G>
__device__ __forceinline__ void convert_half(const uint32_t* cw, const float2 (&sg)[2], const float* cbs,
                                             uint32_t (&wv)[16]) {
  if (BITS == 2) {
    uint32_t L0[G], L1[G];
#pragma unroll
    for (int gi = 0; gi < G; ++gi) {
      float lv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) lv[j] = fmaf(CB ? cbs[j] : (float)j, sg[gi].x, sg[gi].y);
      L0[gi] = pack2<XT>(lv[0], lv[1]);
      L1[gi] = pack2<XT>(lv[2], lv[3]);
    }
#pragma unroll
    for (int wi = 0; wi < 2; ++wi) {
      const int gi = wi * G / 2;
      uint4 c0, c1;
      dq2_lut(cw[wi], L0[gi], L1[gi], c0, c1);
      wv[8 * wi + 0] = c0.x; wv[8 * wi + 1] = c0.y; wv[8 * wi + 2] = c0.z; wv[8 * wi + 3] = c0.w;
      wv[8 * wi + 4] = c1.x; wv[8 * wi + 5] = c1.y; wv[8 * wi + 6] = c1.z; wv[8 * wi + 7] = c1.w;
    }
  } else if (BITS == 4 && !CB) {
    uint32_t s2[G], g2[G];
#pragma unroll
    for (int gi = 0; gi < G; ++gi) {
      s2[gi] = pack2<XT>(sg[gi].x, sg[gi].x);
      const float gc = fmaf(8.f, sg[gi].x, sg[gi].y);
      g2[gi] = pack2<XT>(gc, gc);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 c = dq4_uniform<XT>(cw[j], s2[j * G / 4], g2[j * G / 4]);
      wv[4 * j + 0] = c.x; wv[4 * j + 1] = c.y; wv[4 * j + 2] = c.z; wv[4 * j + 3] = c.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 c = dq_generic<BITS, CB, XT>(&cw[j * BITS / 4], cbs, sg[j * G / 4].x, sg[j * G / 4].y);
      wv[4 * j + 0] = c.x; wv[4 * j + 1] = c.y; wv[4 * j + 2] = c.z; wv[4 * j + 3] = c.w;
    }
  }
}

// Replace the 16-bit value at column cc (0..31) of the 16-word half row.
__device__ __forceinline__ void patch_half(uint32_t (&wv)[16], int cc, uint32_t bits16) {
  const int wi = cc >> 1;
  const uint32_t keep = (cc & 1) ? 0x0000FFFFu : 0xFFFF0000u;
  const uint32_t put = (cc & 1) ? (bits16 << 16) : bits16;
#pragma unroll
  for (int i = 0; i < 16; ++i)
    if (i == wi) wv[i] = (wv[i] & keep) | put;
}

// fp32 weight at an outlier position: base reconstruction + stored delta.
template <bool CB>
__device__ __forceinline__ float outlier_value(const QW& q, const float* cbs, int64_t row, int c, int j) {
  const int code = load_code(q, row, c);
  const float v = CB ? cbs[code] : (float)code;
  const float2 g = load_scale_gmin(q, row, c / q.group_size);
  return __fadd_rn(__fmul_rn(v, g.x), g.y) + __half2float(q.odelta[j]);
}

// ---- work items ----------------------------------------------------------------
// A tile is 128 weight rows x BT tokens over the whole K. Without split, CTA b
// takes tiles b, b + grid, ... whole. With split, the tiles' K-stages are laid
// end to end (tile-major) and CTA b takes the contiguous range of units
// [U b / G, U (b + 1) / G): every CTA gets the same number of stages, and a
// tile whose stages span several CTAs is finished by the last of them to
// arrive, from fp32 partial sums in the workspace (pieces added in CTA
// order, so results do not depend on timing).
struct Item {
  int tile, k0, k1;   // stages [k0, k1) of the tile
  int slot;           // partial-sum slot: 0 = the CTA's first item, 1 = any later one
};

struct ItemIter {
  int next, end;
  bool first;
};

__device__ __forceinline__ int split_unit_begin(int units, int cta, int grid) {
  return (int)((int64_t)units * cta / grid);
}

__device__ __forceinline__ ItemIter items_begin(const Args& a, int ntiles) {
  ItemIter it;
  if (a.split) {
    const int U = ntiles * a.kblocks;
    it.next = split_unit_begin(U, blockIdx.x, gridDim.x);
    it.end = split_unit_begin(U, blockIdx.x + 1, gridDim.x);
  } else {
    it.next = blockIdx.x;
    it.end = ntiles;
  }
  it.first = true;
  return it;
}

__device__ __forceinline__ bool items_next(const Args& a, ItemIter& it, Item& x) {
  if (it.next >= it.end) return false;
  if (a.split) {
    x.tile = it.next / a.kblocks;
    x.k0 = it.next - x.tile * a.kblocks;
    x.k1 = min(a.kblocks, x.k0 + (it.end - it.next));
    it.next += x.k1 - x.k0;
  } else {
    x.tile = it.next;
    x.k0 = 0;
    x.k1 = a.kblocks;
    it.next += gridDim.x;
  }
  x.slot = it.first ? 0 : 1;
  it.first = false;
  return true;
}

// ---- the kernel -------------------------------------------------------------
template <int BITS, bool CB, int XT, int BT>
__global__ void __launch_bounds__(kThreads, 1)
    qgemm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap cmap,
                 const __grid_constant__ CUtensorMap smap, const __grid_constant__ CUtensorMap gmap,
                 const __grid_constant__ CUtensorMap cmap_wide, const Args a) {
  constexpr int kXStageBytes = BT * kBK * 2;
  constexpr int kCodeBytes = kBK * BITS / 8;              // per weight row per stage
  constexpr int kCStageBytes = kBW * kCodeBytes;
  constexpr int kMSlotBytes = 2 * kBW * 16;               // {scale, min} x [128 rows][16 B]
  constexpr int kCW = BT >= 32 ? 32 : 16;                 // accumulator columns per TMEM load
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte aligned base by pointer arithmetic on the shared array itself, so
  // the compiler keeps the shared address space (ld.shared, not generic loads)
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int S = a.stages;
  unsigned char* sX = smem;
  unsigned char* sC = sX + (size_t)S * kXStageBytes;
  unsigned char* sM = sC + (size_t)S * kCStageBytes;
  uint64_t* ld_full = reinterpret_cast<uint64_t*>(sM + 2 * kMSlotBytes);
  uint64_t* a_full = ld_full + S;
  uint64_t* empty = a_full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 1;
  uint64_t* m_full = tempty + 1;
  uint64_t* m_empty = m_full + 2;
  uint64_t* mma_drain = m_empty + 2;   // the MMA issuer's final commit
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_drain + 1);
  float* cbs = reinterpret_cast<float*>(tmem_slot + 4);   // codebook copy (<= 256 floats)
  int* epi_flag = reinterpret_cast<int*>(cbs + 256);     // split: counter value seen by the epilogue
  // per-dequantizer-thread outlier queues: [group][entry][128 rows] words of
  // (column - item's first column) | fp16 delta << 16
  uint32_t* oq = reinterpret_cast<uint32_t*>(epi_flag + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const QW& q = a.q;

  if (threadIdx.x == 0) {
    TS_QPROF(for (int z = 0; z < 12; ++z) g_qgemm_prof[blockIdx.x][z] = 0;)
    for (int s = 0; s < S; ++s) {
      mbar_init(ld_full + s, 1);
      mbar_init(a_full + s, kDqGroupWarps);
      mbar_init(empty + s, 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, kEpiWarps * 32);
    mbar_init(mma_drain, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(m_full + i, 1);
      mbar_init(m_empty + i, kDqWarps);
    }
    fence_barrier_init();
    prefetch_tensormap(&xmap);
    prefetch_tensormap(&cmap);
    if (a.meta_tma) {
      prefetch_tensormap(&smap);
      prefetch_tensormap(&gmap);
    }
  }
  if (CB) {
    for (int i = threadIdx.x; i < (1 << BITS); i += blockDim.x) cbs[i] = q.codebook[i];
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;         // columns [0, BT): accumulator; then S A-stages
  const int ntiles = a.tblocks * a.wblocks;
  const int spm = a.meta_groups * q.group_size / kBK;   // stages per metadata block

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0 && !a.stall) {
      uint32_t mit = 0, ph = 0;
      int s = 0;
      bool ok = true;
      uint32_t issued = 0;   // stages issued (ring position = issued % S)
      TS_QPROF(long long q_pw = 0;)
      ItemIter it = items_begin(a, ntiles);
      Item x;
      while (ok && items_next(a, it, x)) {
        const int m0 = (x.tile % a.tblocks) * BT, n0 = (x.tile / a.tblocks) * kBW;
        // Code columns reach L2 ahead of their stages in 256-byte row
        // segments, kPrefetchStages ahead: the per-stage boxes are only 16-64
        // bytes per row, and fetched from DRAM one stage at a time they leave
        // the pipeline waiting on DRAM latency.
        const int c_end = x.k1 * kCodeBytes;
        int c_pf = (x.k0 * kCodeBytes) & ~255;   // next segment to prefetch
        for (int kb = x.k0; kb < x.k1; ++kb) {
          if (a.prefetch_codes) {
            const int c_want = min(c_end, (kb + kPrefetchStages) * kCodeBytes);
            for (; c_pf < c_want; c_pf += 256) tma_prefetch_2d(&cmap_wide, c_pf, n0);
          }
          if (a.meta_tma && (kb == x.k0 || kb % spm == 0)) {
            // the metadata block holding stage kb, once per block per item
            const int ms = mit & 1;
            if (!mbar_wait_hint(m_empty + ms, ((mit >> 1) & 1) ^ 1, &g_err, 17, a.wait_ns)) { ok = false; break; }
            mbar_arrive_expect_tx(m_full + ms, kMSlotBytes);
            unsigned char* slot = sM + (size_t)ms * kMSlotBytes;
            tma_load_2d(slot, &smap, (kb / spm) * a.meta_groups, n0, m_full + ms);
            tma_load_2d(slot + kBW * 16, &gmap, (kb / spm) * a.meta_groups, n0, m_full + ms);
            ++mit;
          }
          TS_QPROF(long long q_p = clock64();)
          if (!mbar_wait_hint(empty + s, ph ^ 1, &g_err, 11, a.wait_ns)) { ok = false; break; }
          TS_QPROF(q_pw += clock64() - q_p;)
          mbar_arrive_expect_tx(ld_full + s, kXStageBytes + kCStageBytes);
          tma_load_2d(sX + (size_t)s * kXStageBytes, &xmap, kb * kBK, m0, ld_full + s);
          tma_load_2d(sC + (size_t)s * kCStageBytes, &cmap, kb * kCodeBytes, n0, ld_full + s);
          ++issued;
          if (++s == S) { s = 0; ph ^= 1; }
        }
      }
      {
        // let the copies in flight land before the CTA exits (after another
        // role's timeout nobody else waits for them; normally they have landed)
        for (uint32_t k = issued > (uint32_t)S ? issued - S : 0; k < issued; ++k)
          mbar_wait_hint(ld_full + (k % S), (k / S) & 1, nullptr, 0, a.wait_ns);
        for (uint32_t k = mit > 2 ? mit - 2 : 0; k < mit; ++k)
          mbar_wait_hint(m_full + (k & 1), (k >> 1) & 1, nullptr, 0, a.wait_ns);
      }
      TS_QPROF(g_qgemm_prof[blockIdx.x][9] = q_pw;)
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // One thread runs the whole loop: tcgen05.mma and tcgen05.commit are
    // single-thread instructions, and keeping warp-wide synchronization out
    // of the loop lets the next stage's MMAs follow its barriers at once
    // (the tensor pipe drains during any gap here).
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(XT, kBW, BT);
      const uint64_t bd0 = umma_desc_sw128(smem_u32(sX));
      uint32_t ph = 0;
      int s = 0;
      bool ok = true;
      int t_local = 0;
      ItemIter it = items_begin(a, ntiles);
      Item x;
      TS_QPROF(long long q_t0 = clock64(); long long pr[4] = {0, 0, 0, 0};)
      while (ok && items_next(a, it, x)) {
        TS_QPROF(long long q_a = clock64();)
        if (!mbar_wait_hint(tempty, (t_local & 1) ^ 1, &g_err, 12, a.wait_ns)) { ok = false; break; }
        TS_QPROF(pr[2] += clock64() - q_a;)
        tc_fence_after();
        for (int kb = x.k0; kb < x.k1; ++kb) {
          TS_QPROF(long long q_b = clock64();)
          if (!mbar_wait_hint(ld_full + s, ph, &g_err, 13, a.wait_ns)) {
            ok = false;
            break;
          }
          TS_QPROF(long long q_c = clock64(); pr[0] += q_c - q_b;)
          if (!mbar_wait_hint(a_full + s, ph, &g_err, 13, a.wait_ns)) {
            ok = false;
            break;
          }
          TS_QPROF(pr[1] += clock64() - q_c; pr[3] += 1;)
          tc_fence_after();
          // stage s: B descriptor start advances by the stage size (16-byte units)
          const uint64_t bd = bd0 + (uint64_t)((s * kXStageBytes) >> 4);
          const uint32_t at = tmem + BT + s * kAStageCols;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)   // K=16: 8 TMEM columns of A, +32 bytes of B (+2 in the address field)
            umma_f16_ts(tmem, at + 8 * k, bd + 2 * k, idesc, (kb != x.k0 || k != 0) ? 1u : 0u);
          umma_commit(empty + s);
          if (++s == S) { s = 0; ph ^= 1; }
        }
        if (ok) umma_commit(tfull);
        ++t_local;
      }
      TS_QPROF(unsigned long long* pg = g_qgemm_prof[blockIdx.x]; pg[10] = clock64() - q_t0;
               for (int z = 0; z < 4; ++z) pg[z] = pr[z];)
      // every MMA issued (also those of an item abandoned after a timeout)
      // has finished before the TMEM is freed
      umma_commit(mma_drain);
      mbar_wait_hint(mma_drain, 0, nullptr, 0, a.wait_ns);
    }
  } else if (warp < kFirstDqWarp) {
    // ---------------- epilogue ----------------
    const int quad = warp & 3;                      // TMEM lanes this warp may read
    const int r = quad * 32 + lane;                 // this thread's row of the tile
    int t_local = 0;
    ItemIter it = items_begin(a, ntiles);
    Item x;
    while (items_next(a, it, x)) {
      const int64_t m0 = (int64_t)(x.tile % a.tblocks) * BT;
      const int wb = x.tile / a.tblocks;
      const int64_t n = (int64_t)wb * kBW + r;      // this thread's weight row
      // every epilogue thread takes the same branch (the split path below syncs them)
      if (!named_bar_and(3, kEpiWarps * 32, mbar_wait_hint(tfull, t_local & 1, &g_err, 14, a.wait_ns))) break;
      ++t_local;
      tc_fence_after();
      const bool nvalid = n < q.rows;
      const bool whole = x.k0 == 0 && x.k1 == a.kblocks;
      const int jn_all = a.M - m0 < BT ? (int)(a.M - m0) : BT;
      float* pp = a.partials + ((size_t)blockIdx.x * 2 + x.slot) * (BT * kBW);
      const float bias = (a.bias && nvalid) ? load_f(a.bias, a.bias_dtype, n) : 0.f;
#pragma unroll 1
      for (int c = 0; c < BT / kCW; ++c) {
        float v[kCW];
        if constexpr (kCW == 32)
          tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + c * kCW, v);
        else
          tmem_ld16(tmem + ((uint32_t)(quad * 32) << 16) + c * kCW, v);
        if (c == BT / kCW - 1) {
          // accumulator fully read: the MMA may start the next item
          tc_fence_before();
          mbar_arrive(tempty);
        }
        if (!whole) {
          // partial sums, [row][token]: each thread's row is contiguous, so
          // both these stores and the final reduction's loads are 16 bytes wide
          float4* dst = reinterpret_cast<float4*>(pp + (size_t)r * BT + c * kCW);
#pragma unroll
          for (int j = 0; j < kCW / 4; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          continue;
        }
        if (!nvalid) continue;
        const int64_t mb = m0 + c * kCW;
        const int jn = a.M - mb < kCW ? (int)(a.M - mb) : kCW;
        if (a.out_dtype == TS_F32) {
          float* op = reinterpret_cast<float*>(a.out) + mb * a.out_stride + n;
#pragma unroll
          for (int j = 0; j < kCW; ++j)
            if (j < jn) op[j * a.out_stride] = v[j] + bias;
        } else if (a.out_dtype == TS_BF16) {
          __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(a.out) + mb * a.out_stride + n;
#pragma unroll
          for (int j = 0; j < kCW; ++j)
            if (j < jn) op[j * a.out_stride] = __float2bfloat16_rn(v[j] + bias);
        } else {
          __half* op = reinterpret_cast<__half*>(a.out) + mb * a.out_stride + n;
#pragma unroll
          for (int j = 0; j < kCW; ++j)
            if (j < jn) op[j * a.out_stride] = __float2half_rn(v[j] + bias);
        }
      }
      if (whole) continue;
      // ---- split tile: the last CTA to arrive adds the pieces and stores ----
      __threadfence();
      named_bar_sync(3, kEpiWarps * 32);
      if (r == 0) *epi_flag = atomicAdd(a.counters + x.tile, 1);
      named_bar_sync(3, kEpiWarps * 32);
      const int U = ntiles * a.kblocks;
      const int G = gridDim.x;
      const int u_lo = x.tile * a.kblocks, u_hi = u_lo + a.kblocks - 1;
      const int c_first = (int)(((int64_t)(u_lo + 1) * G - 1) / U);   // CTA holding unit u_lo
      const int c_last = (int)(((int64_t)(u_hi + 1) * G - 1) / U);
      const int old = *epi_flag;
      named_bar_sync(3, kEpiWarps * 32);                                // epi_flag is reused
      if (old != c_last - c_first) continue;
      __threadfence();
      if (r == 0) a.counters[x.tile] = 0;
      if (!nvalid) continue;
      // 16 tokens at a time: four independent 16-byte loads per piece in
      // flight, pieces added in CTA order
      constexpr int kRT = BT < 16 ? BT : 16;
      for (int j0 = 0; j0 < jn_all; j0 += kRT) {
        float acc[kRT];
#pragma unroll
        for (int u = 0; u < kRT; ++u) acc[u] = 0.f;
        for (int c = c_first; c <= c_last; ++c) {
          const int slot = split_unit_begin(U, c, G) / a.kblocks == x.tile ? 0 : 1;
          const float4* src = reinterpret_cast<const float4*>(
              a.partials + ((size_t)c * 2 + slot) * (BT * kBW) + (size_t)r * BT + j0);
          float4 t[kRT / 4];
#pragma unroll
          for (int u = 0; u < kRT / 4; ++u) t[u] = __ldcg(src + u);
#pragma unroll
          for (int u = 0; u < kRT / 4; ++u) {
            acc[4 * u] += t[u].x;
            acc[4 * u + 1] += t[u].y;
            acc[4 * u + 2] += t[u].z;
            acc[4 * u + 3] += t[u].w;
          }
        }
#pragma unroll
        for (int u = 0; u < kRT; ++u)
          if (j0 + u < jn_all) store_f(a.out, a.out_dtype, (m0 + j0 + u) * a.out_stride + n, acc[u] + bias);
      }
    }
  } else {
    // ---------------- dequantizers ----------------
    const int quad = warp & 3;                             // TMEM lane quadrant of this warp
    const int grp = (warp - kFirstDqWarp) / kDqGroupWarps; // this group converts the item's stages j = grp (mod kDqGroups)
    const int rl = quad * 32 + lane;                      // tile row of this thread = TMEM lane
    const int gs = q.group_size;
    const bool dq = q.dqs_codes != nullptr;
    const int gph = gs >= 32 ? 1 : 32 / gs;               // groups in each 32-column half of the row (1 or 2)
    // Raw metadata of (row, group): 16-bit scale | 16-bit min << 16, or the
    // two double-quant code bytes, loaded by this thread (metadata rows that
    // are not 16-byte multiples).
    auto fetch = [&](int64_t row, int kb, int half, uint32_t (&raw)[2]) {
      if (row >= q.rows) return;
      const int64_t flat = row * q.n_groups + ((kb * kBK + 32 * half) >> a.gs_shift);
#pragma unroll
      for (int gi = 0; gi < 2; ++gi) {
        if (gi < gph) {
          if (dq)
            raw[gi] = (uint32_t)__ldg(q.dqs_codes + flat + gi) | ((uint32_t)__ldg(q.dqg_codes + flat + gi) << 8);
          else
            raw[gi] = (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(q.scale) + flat + gi) |
                      ((uint32_t)__ldg(reinterpret_cast<const unsigned short*>(q.gmin) + flat + gi) << 16);
        }
      }
    };
    auto decode = [&](int64_t row_ng, int kb, int half, const uint32_t (&raw)[2], float2 (&sg)[2]) {
#pragma unroll
      for (int gi = 0; gi < 2; ++gi) {
        if (gi < gph) {
          if (dq) {
            const int64_t flat = row_ng + ((kb * kBK + 32 * half) >> a.gs_shift);
            const int64_t sup = a.dq_shift >= 0 ? (flat + gi) >> a.dq_shift : (flat + gi) / q.dq_gs;
            const float2 ms = __half22float2(q.dqs_meta[sup]);
            const float2 mg = __half22float2(q.dqg_meta[sup]);
            sg[gi].x = __fadd_rn(__fmul_rn((float)(raw[gi] & 0xFF), ms.x), ms.y);
            sg[gi].y = __fadd_rn(__fmul_rn((float)((raw[gi] >> 8) & 0xFF), mg.x), mg.y);
          } else {
            sg[gi].x = h2f((uint16_t)(raw[gi] & 0xFFFF));
            sg[gi].y = h2f((uint16_t)(raw[gi] >> 16));
          }
        }
      }
    };
    // Ring position of the item's first stage (ts, tph) and the metadata
    // block counter (every group waits for and releases every block of an item)
    uint32_t mit = 0, tph = 0;
    int ts = 0;
    bool ok = true;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16) + BT;
    TS_QPROF(long long dqa[5] = {0, 0, 0, 0, 0};)   // waits free / loaded, convert, store wait, metadata
    ItemIter it = items_begin(a, ntiles);
    Item x;
    while (ok && items_next(a, it, x)) {
      const int64_t row = (int64_t)(x.tile / a.tblocks) * kBW + rl;
      const bool valid = row < q.rows;
      const int64_t row_ng = row * q.n_groups;
      const int my_mod = (x.k0 + grp) % kDqGroups;        // stage index (mod kDqGroups) this group converts
      // Outliers of this row inside the item's columns: the entries of this
      // group's stages are gathered at the item's start into this thread's
      // shared-memory queue, sorted by column (so tables in any order within
      // a row work), and the stage loop reads them at shared-memory latency.
      // A row with more entries than the queue holds keeps the smallest
      // columns and refills after the last one consumed. (The host always
      // provides a queue when the weight has outliers.)
      int o_beg = 0, o_end = 0;
      if (valid && q.n_outliers > 0) {
        o_beg = q.orow_ptr[row];
        o_end = q.orow_ptr[row + 1];
      }
      const int col_lo = x.k0 * kBK, col_hi = x.k1 * kBK;
      const int QC = a.qcap;
      uint32_t* oq_t = oq + (size_t)grp * QC * kBW + rl;   // entry e at oq_t[e * kBW]
      int qn = 0, qi = 0;
      bool qmore = false;
      // gather the entries with column > after (relative to col_lo)
      auto refill = [&](int after) {
        qn = 0;
        qi = 0;
        qmore = false;
        for (int j = o_beg; j < o_end; ++j) {
          const int c = q.ocol[j];
          const int cr = c - col_lo;
          if (c < col_lo || c >= col_hi || cr <= after || ((c >> 6) % kDqGroups) != my_mod) continue;
          if (qn == QC) {
            qmore = true;
            if ((int)(oq_t[(QC - 1) * kBW] & 0xFFFFu) < cr) continue;
            --qn;   // drop the largest column; a later refill finds it again
          }
          const uint32_t e = (uint32_t)cr | ((uint32_t)__half_as_ushort(q.odelta[j]) << 16);
          int p = qn;
          while (p > 0 && (int)(oq_t[(p - 1) * kBW] & 0xFFFFu) > cr) {
            oq_t[p * kBW] = oq_t[(p - 1) * kBW];
            --p;
          }
          oq_t[p * kBW] = e;
          ++qn;
        }
      };
      int q_last = -1;   // relative column of the last entry consumed
      // relative column of the next queue entry (INT_MAX: none left), kept
      // in a register so a half without outliers costs one compare
      int nx_c = INT_MAX;
      if (o_end > o_beg) {
        refill(-1);
        if (qn > 0) nx_c = (int)(oq_t[0] & 0xFFFFu);
      }

      const int nst = x.k1 - x.k0;
      for (int b = x.k0 / spm; ok && b * spm < x.k1; ++b) {
        const int kb_lo = max(x.k0, b * spm), kb_hi = min(x.k1, (b + 1) * spm);
        TS_QPROF(long long q_m = clock64();)
        if (a.meta_tma && !mbar_wait_hint(m_full + (mit & 1), (mit >> 1) & 1, &g_err, 18, a.wait_ns)) {
          ok = false;
          break;
        }
        TS_QPROF(dqa[4] += clock64() - q_m;)
        const unsigned char* slot = sM + (size_t)(mit & 1) * kMSlotBytes + rl * 16;
        // first stage of this group in the block: local index j = kb - k0 with j % kDqGroups == grp
        int kb = kb_lo + ((grp - (kb_lo - x.k0)) % kDqGroups + kDqGroups) % kDqGroups;
        // ring slot and phase of stage kb (one division per block; the loop
        // below advances them by kDqGroups stages at a time)
        int cs = ts + (kb - x.k0);
        uint32_t cph = tph;
        {
          const int wr = cs / S;
          cs -= wr * S;
          cph ^= (uint32_t)(wr & 1);
        }
        int kb_in_block = kb - b * spm;
        for (; kb < kb_hi; kb += kDqGroups) {
          uint32_t rawc2[2][2] = {{0, 0}, {0, 0}};   // metadata of each half, decoded when it is converted
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint32_t (&rawc)[2] = rawc2[half];
            if (a.meta_tma) {
              const int ib = ((kb_in_block << 6) + 32 * half) >> a.gs_shift;   // group of the half within the block
#pragma unroll
              for (int gi = 0; gi < 2; ++gi) {
                if (gi < gph) {
                  if (dq)
                    rawc[gi] = (uint32_t)slot[ib + gi] | ((uint32_t)slot[kBW * 16 + ib + gi] << 8);
                  else
                    rawc[gi] = (uint32_t)reinterpret_cast<const uint16_t*>(slot)[ib + gi] |
                               ((uint32_t)reinterpret_cast<const uint16_t*>(slot + kBW * 16)[ib + gi] << 16);
                }
              }
            } else {
              fetch(row, kb, half, rawc);
            }
          }

          TS_QPROF(long long q_d = clock64();)
          if (!mbar_wait_hint(empty + cs, cph ^ 1, &g_err, 15, a.wait_ns)) { ok = false; break; }
          TS_QPROF(long long q_e = clock64(); dqa[0] += q_e - q_d;)
          if (!mbar_wait_hint(ld_full + cs, cph, &g_err, 16, a.wait_ns)) { ok = false; break; }
          TS_QPROF(long long q_f = clock64(); dqa[1] += q_f - q_e;)
          const unsigned char* crow_all = sC + (size_t)cs * kCStageBytes + rl * kCodeBytes;
#pragma unroll 1
          for (int half = 0; half < 2; ++half) {
            const int c0 = kb * kBK + 32 * half;                // first column of this half
            const unsigned char* crow = crow_all + half * (kCodeBytes / 2);
            uint32_t cw[kCodeBytes / 8];
            if (kCodeBytes / 2 >= 16) {
#pragma unroll
              for (int i2 = 0; i2 < kCodeBytes / 32; ++i2) {
                const uint4 u = reinterpret_cast<const uint4*>(crow)[i2];
                cw[4 * i2] = u.x; cw[4 * i2 + 1] = u.y; cw[4 * i2 + 2] = u.z; cw[4 * i2 + 3] = u.w;
              }
            } else {
              const uint2 u = *reinterpret_cast<const uint2*>(crow);
              cw[0] = u.x; cw[kCodeBytes / 8 - 1] = u.y;
            }
            float2 sgh[2];
            const uint32_t rh[2] = {half ? rawc2[1][0] : rawc2[0][0], half ? rawc2[1][1] : rawc2[0][1]};
            if (valid) decode(row_ng, kb, half, rh, sgh);
            uint32_t wv[16];
            if (!valid) {
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) wv[jj] = 0;
            } else if (gph == 1) {
              convert_half<BITS, CB, XT, 1>(cw, sgh, cbs, wv);
            } else {
              convert_half<BITS, CB, XT, 2>(cw, sgh, cbs, wv);
            }
            // outliers in these 32 columns: value = fp32(base) + delta, rounded once
            if (nx_c < c0 - col_lo + 32) {
              {
                while (true) {
                  if (qi == qn) {
                    if (!qmore) { nx_c = INT_MAX; break; }
                    refill(q_last);
                    if (qn == 0) { nx_c = INT_MAX; break; }
                  }
                  const uint32_t e = oq_t[qi * kBW];
                  nx_c = (int)(e & 0xFFFFu);
                  const int cc = (int)(e & 0xFFFFu) + col_lo - c0;
                  if (cc >= 32) break;
                  const uint32_t byte = crow[cc * BITS / 8];
                  const int code = (int)((byte >> ((cc * BITS) & 7)) & ((1u << BITS) - 1));
                  const float2 g = (gph == 2 && cc >= 16) ? sgh[1] : sgh[0];
                  const float v = CB ? cbs[code] : (float)code;
                  const float val = __fadd_rn(__fmul_rn(v, g.x), g.y) + __half2float(__ushort_as_half((unsigned short)(e >> 16)));
                  patch_half(wv, cc, pack2<XT>(val, val) & 0xFFFFu);
                  q_last = (int)(e & 0xFFFFu);
                  ++qi;
                }
              }
            }
            tmem_st16(lane_base + cs * kAStageCols + half * (kAStageCols / 2), wv);
          }
          TS_QPROF(long long q_g = clock64(); dqa[2] += q_g - q_f;)
          tmem_st_wait();
          TS_QPROF(dqa[3] += clock64() - q_g;)
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(a_full + cs);
          kb_in_block += kDqGroups;
          cs += kDqGroups;
          while (cs >= S) {
            cs -= S;
            cph ^= 1u;
          }
        }
        if (!ok) break;
        if (a.meta_tma) {
          // one arrival per warp: 256 arrivals on one barrier word would
          // serialize in the shared-memory atomic unit every block
          __syncwarp();
          if (lane == 0) mbar_arrive(m_empty + (mit & 1));
          ++mit;
        }
      }
      // the next item starts nst stages later in the ring
      const int adv = ts + nst;
      const int wraps = adv / S;
      ts = adv - wraps * S;
      tph ^= (uint32_t)(wraps & 1);
    }
    TS_QPROF(if (warp == kFirstDqWarp && lane == 0) {
      unsigned long long* pg = g_qgemm_prof[blockIdx.x];
      for (int z = 0; z < 4; ++z) pg[4 + z] = dqa[z];
      pg[8] = dqa[4];
    })
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace qgemm

// ---- host -------------------------------------------------------------------

static size_t qgemm_smem(int BT, int bits, int S, int qcap = 0) {
  const size_t stage = (size_t)BT * qgemm::kBK * 2 + (size_t)qgemm::kBW * qgemm::kBK * bits / 8;
  return 1024 + (size_t)S * stage + 2 * (2 * (size_t)qgemm::kBW * 16) + (3 * S + 9) * 8 + 16 + 256 * 4 + 16 +
         (size_t)qgemm::kDqGroups * qgemm::kBW * 4 * qcap;
}

// Outlier queue entries per dequantizer thread: up to kMaxQcap, in the shared
// memory left after S stages (the caller may give up a stage for it).
constexpr int kMaxQcap = 16;
static int qgemm_qcap(int BT, int bits, int S) {
  const size_t base = qgemm_smem(BT, bits, S, 0);
  const size_t lim = (size_t)max_smem_optin();
  if (base >= lim) return 0;
  const size_t per = (size_t)qgemm::kDqGroups * qgemm::kBW * 4;
  return (int)std::min<size_t>(kMaxQcap, (lim - base) / per);
}

static int max_stages(int BT) { return (qgemm::kTmemCols - BT) / qgemm::kAStageCols; }

// Layout conditions of the tensor-core path (everything else uses the GEMV).
static bool qgemm_layout_ok(const ts_qweight& w) {
  if (!(w.bits == 2 || w.bits == 4 || w.bits == 8)) return false;
  const int gs = w.group_size;
  if (gs < 16 || (gs & (gs - 1)) != 0) return false;   // power-of-two groups of at least 16
  const int64_t kb = (w.cols + qgemm::kBK - 1) / qgemm::kBK;
  if (kb * qgemm::kBK > w.padded_cols || kb * qgemm::kBK * w.bits / 8 > w.packed_row_bytes) return false;
  if (w.packed_row_bytes % 16 != 0 || !is_aligned(w.packed, 16)) return false;
  if (w.rows * w.n_groups >= (int64_t(1) << 31) || w.rows >= (int64_t(1) << 31)) return false;
  if (w.cols < 1) return false;
  if (w.cols > 65535) return false;   // outlier queue entries hold 16-bit relative columns
  return max_smem_optin() >= (int)qgemm_smem(256, w.bits, 2);
}

bool qgemm_supported(const ts_qweight& w, const void* x, int64_t x_stride) {
  return qgemm_layout_ok(w) && is_aligned(x, 16) && (x_stride * 2) % 16 == 0;
}

// Tile plan for M tokens: BT tokens per tile (16/32/64 for decode-sized M,
// 128/256 for prefill), and whether CTAs split tiles along K.
struct QgemmPlan {
  int BT, tblocks, wblocks, kblocks, ntiles, grid;
  bool split_wanted;
};

static QgemmPlan qgemm_plan(const ts_qweight& w, int64_t M) {
  QgemmPlan p;
  const int sms = sm_count();
  p.wblocks = (int)((w.rows + qgemm::kBW - 1) / qgemm::kBW);
  p.kblocks = (int)((w.cols + qgemm::kBK - 1) / qgemm::kBK);
  if (M <= 16) p.BT = 16;
  else if (M <= 32) p.BT = 32;
  else if (M <= 64) p.BT = 64;
  else if ((int64_t)((M + 255) / 256) * p.wblocks < sms) p.BT = 128;   // 256 would leave SMs idle
  else p.BT = 256;   // 256-token tiles halve the dequantization per flop
  p.tblocks = (int)((M + p.BT - 1) / p.BT);
  p.ntiles = p.tblocks * p.wblocks;
  // decode-sized M: the few tiles' K-stages are split evenly over the SMs.
  // Prefill keeps whole tiles per CTA: measured, split plans were 4-20%
  // slower there (partial sums and their reduction cost more than the wave
  // imbalance they remove).
  p.split_wanted = p.BT <= 64;
  const int64_t units = (int64_t)p.ntiles * p.kblocks;
  p.grid = (int)std::min<int64_t>(p.split_wanted ? units : p.ntiles, sms);
  return p;
}

static size_t align256(size_t v) { return (v + 255) / 256 * 256; }

static size_t qgemm_partials_bytes(int grid, int BT) { return align256((size_t)grid * 2 * BT * qgemm::kBW * 4); }

// Extra workspace the split plan needs beyond the decode kernel's: its tile
// counters share the zeroed counter area after the error flag, and its
// partial sums sit at the end of the workspace (never over a counter area).
size_t qgemm_workspace_extra(const ts_qweight& w, int64_t M, size_t counters_bytes_gemv) {
  if (!qgemm_layout_ok(w) || M < 1) return 0;
  const QgemmPlan p = qgemm_plan(w, M);
  if (!p.split_wanted) return 0;
  const size_t cnt = align256((size_t)p.ntiles * 4);
  return (cnt > counters_bytes_gemv ? cnt - counters_bytes_gemv : 0) + qgemm_partials_bytes(p.grid, p.BT);
}

template <int BITS, bool CB, int XT, int BT>
static int launch_qgemm(const CUtensorMap* maps, const qgemm::Args& a, int grid, size_t smem, cudaStream_t st) {
  auto k = qgemm::qgemm_kernel<BITS, CB, XT, BT>;
  static thread_local int configured_dev = -1;
  static thread_local size_t configured_smem = 0;
  int dev = 0;
  TS_CUDA_TRY(cudaGetDevice(&dev));
  if (configured_dev != dev || configured_smem < smem) {
    TS_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    configured_dev = dev;
    configured_smem = smem;
  }
  k<<<grid, qgemm::kThreads, smem, st>>>(maps[0], maps[1], maps[2], maps[3], maps[4], a);
  TS_LAUNCH_CHECK();
  return TS_OK;
}

template <int BITS, bool CB, int XT>
static int launch_bt(int BT, const CUtensorMap* maps, const qgemm::Args& a, int grid, size_t smem,
                     cudaStream_t st) {
  switch (BT) {
    case 16: return launch_qgemm<BITS, CB, XT, 16>(maps, a, grid, smem, st);
    case 32: return launch_qgemm<BITS, CB, XT, 32>(maps, a, grid, smem, st);
    case 64: return launch_qgemm<BITS, CB, XT, 64>(maps, a, grid, smem, st);
    case 128: return launch_qgemm<BITS, CB, XT, 128>(maps, a, grid, smem, st);
    default: return launch_qgemm<BITS, CB, XT, 256>(maps, a, grid, smem, st);
  }
}

template <int BITS>
static int launch_bits(bool cb, int xt, int BT, const CUtensorMap* maps, const qgemm::Args& a, int grid,
                       size_t smem, cudaStream_t st) {
  if (cb)
    return xt ? launch_bt<BITS, true, 1>(BT, maps, a, grid, smem, st)
              : launch_bt<BITS, true, 0>(BT, maps, a, grid, smem, st);
  return xt ? launch_bt<BITS, false, 1>(BT, maps, a, grid, smem, st)
            : launch_bt<BITS, false, 0>(BT, maps, a, grid, smem, st);
}

// Whether a call of M tokens runs split with this workspace: the counters
// (from `counters_off`) and the partial sums (at the end) must both fit.
bool qgemm_split_fits(const ts_qweight& w, int64_t M, size_t counters_off, size_t ws_bytes) {
  if (!qgemm_layout_ok(w)) return false;
  const QgemmPlan p = qgemm_plan(w, M);
  if (!p.split_wanted) return false;
  const size_t need = counters_off + align256((size_t)p.ntiles * 4) + qgemm_partials_bytes(p.grid, p.BT);
  return ws_bytes >= need;
}

// The tensor-core path. With `workspace` (counters zeroed from counters_off,
// partial sums at the end) a plan that wants split runs split; without, whole
// tiles per CTA (decode-sized M then needs the workspace: the caller routes
// those calls to the GEMV instead).
int run_qgemm(const ts_qweight& w, const void* x, int x_dtype, int64_t M, int64_t x_stride, const void* bias,
              int bias_dtype, void* out, int out_dtype, int64_t out_stride, void* workspace, size_t counters_off,
              size_t ws_bytes, cudaStream_t stream) {
  TS_UNSUPPORTED(qgemm_supported(w, x, x_stride), "qgemm: layout not supported");
  QgemmPlan p = qgemm_plan(w, M);
  const bool split = p.split_wanted && workspace != nullptr && qgemm_split_fits(w, M, counters_off, ws_bytes);
  const int sms = sm_count();
  if (!split) p.grid = (int)std::min<int64_t>(p.ntiles, sms);
  qgemm::Args a;
  a.q = make_qw(w);
  a.M = M;
  a.bias = bias;
  a.bias_dtype = bias_dtype;
  a.out = out;
  a.out_dtype = out_dtype;
  a.out_stride = out_stride;
  a.wblocks = p.wblocks;
  a.kblocks = p.kblocks;
  a.tblocks = p.tblocks;
  a.split = split ? 1 : 0;
  a.counters = split ? reinterpret_cast<int*>(reinterpret_cast<char*>(workspace) + counters_off) : nullptr;
  a.partials = split ? reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + ws_bytes -
                                                qgemm_partials_bytes(p.grid, p.BT))
                     : nullptr;
  const int BT = p.BT;
  int S = max_stages(BT);
  while (S > 2 && qgemm_smem(BT, w.bits, S) > (size_t)max_smem_optin()) --S;
  // relative outlier columns are 16-bit; a queue of fewer than 4 entries
  // would refill often, so a stage is given up for a longer one
  int qcap = 0;
  if (w.n_outliers > 0) {
    // queue length for a group's share of a row's outliers: mean + 2.5
    // standard deviations (Poisson), so refills (a rescan of the row's table
    // inside the stage loop) stay rare; a stage is given up to reach it
    const double per_group = (double)w.n_outliers / (double)w.rows / qgemm::kDqGroups;
    const int want = std::min(kMaxQcap, std::max(4, (int)std::ceil(per_group + 2.5 * std::sqrt(per_group))));
    qcap = qgemm_qcap(BT, w.bits, S);
    if (qcap < want && S > 3 && qgemm_qcap(BT, w.bits, S - 1) >= want) qcap = qgemm_qcap(BT, w.bits, --S);
    if (qcap < 4 && S > 3) qcap = qgemm_qcap(BT, w.bits, --S);
    while (qcap < 1 && S > 2) qcap = qgemm_qcap(BT, w.bits, --S);
    TS_UNSUPPORTED(qcap >= 1, "qgemm: no shared memory left for the outlier queues");
  }
  a.stages = S;
  a.qcap = qcap;
  const size_t smem = qgemm_smem(BT, w.bits, S, qcap);
  const int grid = p.grid;
  CUtensorMap maps[5];
  int rc = encode_tmap_2d(&maps[0], x, CU_TENSOR_MAP_DATA_TYPE_UINT16, (uint64_t)w.cols, (uint64_t)M,
                          (uint64_t)x_stride * 2, qgemm::kBK, BT, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != TS_OK) return rc;
  rc = encode_tmap_2d(&maps[1], w.packed, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)w.packed_row_bytes,
                      (uint64_t)w.rows, (uint64_t)w.packed_row_bytes, qgemm::kBK * w.bits / 8, qgemm::kBW,
                      CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc != TS_OK) return rc;
  // the same codes with 256-byte-wide boxes, for the L2 prefetch
  a.prefetch_codes = w.packed_row_bytes >= 256 ? 1 : 0;
  maps[4] = maps[1];
  if (a.prefetch_codes) {
    rc = encode_tmap_2d(&maps[4], w.packed, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)w.packed_row_bytes,
                        (uint64_t)w.rows, (uint64_t)w.packed_row_bytes, 256, qgemm::kBW, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != TS_OK) return rc;
  }
  // group metadata blocks of 16 bytes per row: 8 fp16 scales/mins, or 16
  // double-quant code bytes; rows must be 16-byte multiples for the copies
  const bool dq = w.dq_scale_codes != nullptr;
  a.meta_groups = dq ? 16 : 8;
  a.meta_tma = (w.n_groups % a.meta_groups == 0) &&
               (int64_t)a.meta_groups * w.group_size % qgemm::kBK == 0 &&
               (dq ? is_aligned(w.dq_scale_codes, 16) && is_aligned(w.dq_gmin_codes, 16)
                   : is_aligned(w.scale, 16) && is_aligned(w.gmin, 16));
  maps[2] = maps[0];
  maps[3] = maps[0];
  if (a.meta_tma) {
    const CUtensorMapDataType t = dq ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
    const uint64_t eb = dq ? 1 : 2;
    rc = encode_tmap_2d(&maps[2], dq ? (const void*)w.dq_scale_codes : w.scale, t, (uint64_t)w.n_groups,
                        (uint64_t)w.rows, (uint64_t)w.n_groups * eb, a.meta_groups, qgemm::kBW,
                        CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != TS_OK) return rc;
    rc = encode_tmap_2d(&maps[3], dq ? (const void*)w.dq_gmin_codes : w.gmin, t, (uint64_t)w.n_groups,
                        (uint64_t)w.rows, (uint64_t)w.n_groups * eb, a.meta_groups, qgemm::kBW,
                        CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != TS_OK) return rc;
  } else {
    a.meta_groups = w.group_size >= qgemm::kBK ? 1 : qgemm::kBK / w.group_size;   // keeps spm >= 1 (unused)
  }
  a.gs_shift = 0;
  while ((1 << a.gs_shift) < w.group_size) ++a.gs_shift;
  a.wait_ns = wait_limit_ns();
  a.stall = take_test_stall() ? 1 : 0;
  a.dq_shift = -1;
  if (w.dq_group_size > 0 && (w.dq_group_size & (w.dq_group_size - 1)) == 0) {
    a.dq_shift = 0;
    while ((1 << a.dq_shift) < w.dq_group_size) ++a.dq_shift;
  }
  const bool cb = w.codebook != nullptr;
  const int xt = x_dtype == TS_BF16 ? 1 : 0;
  if (w.bits == 2) return launch_bits<2>(cb, xt, BT, maps, a, grid, smem, stream);
  if (w.bits == 4) return launch_bits<4>(cb, xt, BT, maps, a, grid, smem, stream);
  return launch_bits<8>(cb, xt, BT, maps, a, grid, smem, stream);
}

// Wait-timeout flag of the tensor-core kernel on the current device: returns
// its value (0 = no timeout) and zeroes it when `clear` is set.
int qgemm_error_flag(int* code, bool clear, cudaStream_t stream) {
  int v = 0;
  TS_CUDA_TRY(cudaMemcpyFromSymbolAsync(&v, qgemm::g_err, sizeof(int), 0, cudaMemcpyDeviceToHost, stream));
  TS_CUDA_TRY(cudaStreamSynchronize(stream));
  if (clear && v != 0) {
    const int zero = 0;
    TS_CUDA_TRY(cudaMemcpyToSymbolAsync(qgemm::g_err, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream));
    TS_CUDA_TRY(cudaStreamSynchronize(stream));
  }
  *code = v;
  return TS_OK;
}

#ifdef TS_QGEMM_PROF
int qgemm_prof_read(void* dst) {
  TS_CUDA_TRY(cudaMemcpyFromSymbol(dst, qgemm::g_qgemm_prof, sizeof(qgemm::g_qgemm_prof)));
  return TS_OK;
}
#endif

}  // namespace ts

#ifdef TS_QGEMM_PROF
extern "C" __attribute__((visibility("default"))) int ts_prof_read_qgemm(void* dst) { return ts::qgemm_prof_read(dst); }
#endif
