// Prefill-shaped fused dequant-GEMM on the 5th-generation tensor cores.
//
//   out[M, N] = x[M, K] . W[N, K]^T (+ outliers) (+ bias),  W in the packed
//   GOAP layout (codes + per-group scale/min or their double-quantized form,
//   optional fp32 codebook, CSR outlier tables).
//
// Replaces the reference's M > 64 path (modules.py:898-922: dequantize_weight
// to a dense compute-dtype matrix, triton_kernels.py:1003-1186, then F.linear)
// with one persistent kernel that never writes the dense matrix:
//
//   warp 0      TMA producer: x tiles [128 tokens x 64] (128B swizzle), the
//               packed code tile [BN rows x 64 columns], and blocks of group
//               metadata [BN rows x 16 bytes] -> shared memory
//   warp 1      MMA issuer: owns the TMEM accumulators, one thread issues
//               tcgen05.mma M=128 x N=BN x K=16 (4 per stage), commits to barriers
//   warps 2-5   epilogue: tcgen05.ld of the fp32 accumulator (one token per
//               thread), + bias, convert, store
//   warps 6..   dequantizers: one weight row per thread; each stage unpacks that
//               row's 64 codes straight into the tensor-core operand layout
//               (K-major, 128-byte swizzle) in the activation dtype, and patches
//               the row's outliers in place as fp32(base + delta) rounded once,
//               so the sparse correction costs no extra pass and no atomics.
//
// Two TMEM accumulators (2 x BN columns) let the epilogue of tile i overlap the
// main loop of tile i+1. Every wait is bounded in wall-clock time: on timeout
// the kernel records an error flag and all roles unwind to the final barrier,
// where the TMEM is freed.
#include "sm100.cuh"

namespace ts {
namespace qgemm {

constexpr int kBM = 128;        // tokens per tile = UMMA M
constexpr int kBK = 64;         // K per stage = one 128-byte swizzle row of 16-bit values
constexpr int kEpiWarps = 4;
constexpr int kFirstDqWarp = 2 + kEpiWarps;
constexpr int kAStageBytes = kBM * kBK * 2;

__device__ int g_err;           // wait-timeout flag (diagnostic)

__device__ __forceinline__ bool is_aligned_dev(const void* p, int a) {
  return (reinterpret_cast<uintptr_t>(p) & (uintptr_t)(a - 1)) == 0;
}

struct Args {
  QW q;
  int64_t M;
  const void* bias;
  int bias_dtype;
  void* out;
  int out_dtype;
  int64_t out_stride;
  int mblocks, nblocks, kblocks;
  int stages;
  int meta_tma;      // group metadata by TMA blocks (else per-thread loads)
  int meta_groups;   // groups per metadata block (8 fp16 or 16 code bytes = 16 B)
};

template <int BN>
struct Cfg {
  static constexpr int kDqThreads = BN;                       // one weight row per thread
  static constexpr int kThreads = (kFirstDqWarp * 32) + kDqThreads;
  static constexpr int kBStageBytes = BN * kBK * 2;
  static constexpr int kTmemCols = 2 * BN;
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

// One weight row's 64 columns of a stage -> the swizzled operand row `brow`
// (16-byte chunk j stored at chunk position j ^ sw). G = groups per stage,
// a compile-time constant so every per-group register is statically indexed.
template <int BITS, bool CB, int XT, int G>
__device__ __forceinline__ void convert_stage(const uint32_t* cw, const float2 (&sg)[4], const float* cbs,
                                              unsigned char* brow, int sw) {
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
    for (int wi = 0; wi < 4; ++wi) {
      const int gi = wi * G / 4;
      uint4 c0, c1;
      dq2_lut(cw[wi], L0[gi], L1[gi], c0, c1);
      *reinterpret_cast<uint4*>(brow + (((2 * wi) ^ sw) << 4)) = c0;
      *reinterpret_cast<uint4*>(brow + (((2 * wi + 1) ^ sw) << 4)) = c1;
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
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<uint4*>(brow + ((j ^ sw) << 4)) = dq4_uniform<XT>(cw[j], s2[j * G / 8], g2[j * G / 8]);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<uint4*>(brow + ((j ^ sw) << 4)) =
          dq_generic<BITS, CB, XT>(&cw[j * BITS / 4], cbs, sg[j * G / 8].x, sg[j * G / 8].y);
  }
}

// fp32 weight at an outlier position: base reconstruction + stored delta.
template <bool CB>
__device__ __forceinline__ float outlier_value(const QW& q, const float* cbs, int64_t row, int c, int j) {
  const int code = load_code(q, row, c);
  const float v = CB ? cbs[code] : (float)code;
  const float2 g = load_scale_gmin(q, row, c / q.group_size);
  return __fadd_rn(__fmul_rn(v, g.x), g.y) + __half2float(q.odelta[j]);
}

// ---- the kernel -------------------------------------------------------------
template <int BITS, bool CB, int XT, int BN>
__global__ void __launch_bounds__(Cfg<BN>::kThreads, 1)
    qgemm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap cmap,
                 const __grid_constant__ CUtensorMap smap, const __grid_constant__ CUtensorMap gmap,
                 const Args a) {
  using C = Cfg<BN>;
  constexpr int kCodeBytes = kBK * BITS / 8;              // per weight row per stage
  constexpr int kCStageBytes = BN * kCodeBytes;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  unsigned char* sA = smem;
  unsigned char* sB = smem + (size_t)S * kAStageBytes;
  unsigned char* sC = sB + (size_t)S * C::kBStageBytes;    // packed codes, [BN][kCodeBytes] per stage
  unsigned char* sM = sC + (size_t)S * kCStageBytes;     // 2 slots x {scale, min} x [BN][16 B]
  constexpr int kMSlotBytes = 2 * BN * 16;
  uint64_t* ld_full = reinterpret_cast<uint64_t*>(sM + 2 * kMSlotBytes);
  uint64_t* b_full = ld_full + S;
  uint64_t* empty = b_full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* m_full = tempty + 2;
  uint64_t* m_empty = m_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(m_empty + 2);
  float* cbs = reinterpret_cast<float*>(tmem_slot + 4);   // codebook copy (<= 256 floats)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const QW& q = a.q;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(ld_full + s, 1);
      mbar_init(b_full + s, C::kDqThreads);
      mbar_init(empty + s, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(tfull + i, 1);
      mbar_init(tempty + i, kEpiWarps * 32);
      mbar_init(m_full + i, 1);
      mbar_init(m_empty + i, C::kDqThreads);
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
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int ntiles = a.mblocks * a.nblocks;
  const int KB = a.kblocks;
  // stages per metadata block (a block holds meta_groups consecutive groups)
  const int spm = a.meta_groups * q.group_size / kBK;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t it = 0, mit = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const int m0 = (tile % a.mblocks) * kBM, n0 = (tile / a.mblocks) * BN;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % S;
          if (a.meta_tma && kb % spm == 0) {
            const int ms = mit & 1;
            if (!mbar_wait_ns(m_empty + ms, ((mit >> 1) & 1) ^ 1, &g_err, 17)) { ok = false; break; }
            mbar_arrive_expect_tx(m_full + ms, kMSlotBytes);
            unsigned char* slot = sM + (size_t)ms * kMSlotBytes;
            tma_load_2d(slot, &smap, (kb / spm) * a.meta_groups, n0, m_full + ms);
            tma_load_2d(slot + BN * 16, &gmap, (kb / spm) * a.meta_groups, n0, m_full + ms);
            ++mit;
          }
          if (!mbar_wait_ns(empty + s, ((it / S) & 1) ^ 1, &g_err, 11)) { ok = false; break; }
          mbar_arrive_expect_tx(ld_full + s, kAStageBytes + kCStageBytes);
          tma_load_2d(sA + (size_t)s * kAStageBytes, &xmap, kb * kBK, m0, ld_full + s);
          tma_load_2d(sC + (size_t)s * kCStageBytes, &cmap, kb * kCodeBytes, n0, ld_full + s);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = umma_idesc_f16(XT, kBM, BN);
    uint32_t it = 0;
    bool ok = true;
    int t_local = 0;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++t_local) {
      const int acc = t_local & 1;
      if (!mbar_wait_ns(tempty + acc, ((t_local >> 1) & 1) ^ 1, &g_err, 12)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d = tmem + acc * BN;
      for (int kb = 0; kb < KB; ++kb, ++it) {
        const int s = it % S;
        if (!mbar_wait_ns(ld_full + s, (it / S) & 1, &g_err, 13) ||
            !mbar_wait_ns(b_full + s, (it / S) & 1, &g_err, 13)) { ok = false; break; }
        tc_fence_after();
        if (lane == 0) {
          const uint64_t ad = umma_desc_sw128(smem_u32(sA + (size_t)s * kAStageBytes));
          const uint64_t bd = umma_desc_sw128(smem_u32(sB + (size_t)s * C::kBStageBytes));
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)   // +32 bytes along K per step = +2 in the 16-byte address field
            umma_f16(d, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
          umma_commit(empty + s);
        }
        __syncwarp();
      }
      if (lane == 0) umma_commit(tfull + acc);
      __syncwarp();
    }
  } else if (warp < kFirstDqWarp) {
    // ---------------- epilogue ----------------
    const int quad = warp & 3;                      // TMEM lanes this warp may read
    int t_local = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++t_local) {
      const int acc = t_local & 1;
      const int m0 = (tile % a.mblocks) * kBM, n0 = (tile / a.mblocks) * BN;
      if (!mbar_wait_ns(tfull + acc, (t_local >> 1) & 1, &g_err, 14)) break;
      tc_fence_after();
      const int64_t m = m0 + quad * 32 + lane;
      const bool mvalid = m < a.M;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + acc * BN + c * 32, v);
        const int64_t nb = n0 + c * 32;
        if (a.bias) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (nb + i < q.rows) v[i] += load_f(a.bias, a.bias_dtype, nb + i);
        }
        if (mvalid) {
          const int64_t o = m * a.out_stride + nb;
          const bool full_vec = nb + 32 <= q.rows;
          if (a.out_dtype == TS_F32) {
            float* op = reinterpret_cast<float*>(a.out) + o;
            if (full_vec && is_aligned_dev(op, 16)) {
#pragma unroll
              for (int i = 0; i < 32; i += 4)
                *reinterpret_cast<float4*>(op + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
            } else {
              for (int i = 0; i < 32; ++i)
                if (nb + i < q.rows) op[i] = v[i];
            }
          } else {
            uint16_t* op = reinterpret_cast<uint16_t*>(a.out) + o;
            if (full_vec && is_aligned_dev(op, 16)) {
#pragma unroll
              for (int i = 0; i < 32; i += 8) {
                uint4 w;
                if (a.out_dtype == TS_BF16)
                  w = make_uint4(pack2<1>(v[i], v[i + 1]), pack2<1>(v[i + 2], v[i + 3]),
                                 pack2<1>(v[i + 4], v[i + 5]), pack2<1>(v[i + 6], v[i + 7]));
                else
                  w = make_uint4(pack2<0>(v[i], v[i + 1]), pack2<0>(v[i + 2], v[i + 3]),
                                 pack2<0>(v[i + 4], v[i + 5]), pack2<0>(v[i + 6], v[i + 7]));
                *reinterpret_cast<uint4*>(op + i) = w;
              }
            } else {
              for (int i = 0; i < 32; ++i)
                if (nb + i < q.rows) store_f(a.out, a.out_dtype, o + i, v[i]);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(tempty + acc);
    }
  } else {
    // ---------------- dequantizers ----------------
    const int r = threadIdx.x - kFirstDqWarp * 32;      // tile row of this thread
    const int gs = q.group_size;
    const bool dq = q.dqs_codes != nullptr;
    const int groups_per_stage = gs >= kBK ? 1 : kBK / gs;
    // Raw metadata of (row, group): 16-bit scale | 16-bit min << 16, or the
    // two double-quant code bytes. From the TMA'd block in shared memory, or,
    // when the metadata rows are not 16-byte multiples, loaded by this thread
    // two stages ahead so the latency overlaps the stages in between.
    auto fetch = [&](int tile, int kb, uint32_t (&raw)[4]) {
      const int64_t row = (int64_t)(tile / a.mblocks) * BN + r;
      if (tile >= ntiles || row >= q.rows) return;
      const int64_t flat = row * q.n_groups + (int64_t)kb * kBK / gs;
#pragma unroll
      for (int gi = 0; gi < 4; ++gi) {
        if (gi < groups_per_stage) {
          if (dq)
            raw[gi] = (uint32_t)__ldg(q.dqs_codes + flat + gi) | ((uint32_t)__ldg(q.dqg_codes + flat + gi) << 8);
          else
            raw[gi] = (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(q.scale) + flat + gi) |
                      ((uint32_t)__ldg(reinterpret_cast<const unsigned short*>(q.gmin) + flat + gi) << 16);
        }
      }
    };
    auto decode = [&](int64_t row, int kb, const uint32_t (&raw)[4], float2 (&sg)[4]) {
      const int64_t flat = row * q.n_groups + (int64_t)kb * kBK / gs;
#pragma unroll
      for (int gi = 0; gi < 4; ++gi) {
        if (gi < groups_per_stage) {
          if (dq) {
            const int64_t sup = (flat + gi) / q.dq_gs;
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
    uint32_t raw1[4] = {0, 0, 0, 0}, raw2[4] = {0, 0, 0, 0};
    int t2 = blockIdx.x, k2 = 1;                 // position of raw2 (raw1 = the current stage)
    if (k2 == KB) { k2 = 0; t2 += gridDim.x; }
    if (!a.meta_tma) {
      fetch(blockIdx.x, 0, raw1);
      fetch(t2, k2, raw2);
    }
    uint32_t it = 0, mit = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
      const int64_t row = (int64_t)(tile / a.mblocks) * BN + r;
      const bool valid = row < q.rows;
      // Outliers of this row. Column-sorted rows use a cursor whose next
      // (column, delta) is loaded right after the previous patch, so it has
      // landed by the stage that needs it; other rows scan their list.
      int o_beg = 0, o_end = 0;
      bool sorted = true;
      if (valid && q.n_outliers > 0) {
        o_beg = q.orow_ptr[row];
        o_end = q.orow_ptr[row + 1];
        for (int j = o_beg + 1; j < o_end; ++j)
          if (q.ocol[j] < q.ocol[j - 1]) { sorted = false; break; }
      }
      int cur = o_beg;
      int next_col = cur < o_end ? q.ocol[cur] : INT_MAX;
      float next_delta = cur < o_end ? __half2float(q.odelta[cur]) : 0.f;

      for (int kb = 0; kb < KB; ++kb, ++it) {
        const int s = it % S;
        const int k0 = kb * kBK;
        uint32_t rawc[4] = {0, 0, 0, 0};
        if (a.meta_tma) {
          if (kb % spm == 0 &&
              !mbar_wait_ns(m_full + (mit & 1), (mit >> 1) & 1, &g_err, 18)) { ok = false; break; }
          const unsigned char* slot = sM + (size_t)(mit & 1) * kMSlotBytes + r * 16;
          const int ib = (kb % spm) * kBK / gs;             // first group of this stage in the block
#pragma unroll
          for (int gi = 0; gi < 4; ++gi) {
            if (gi < groups_per_stage) {
              if (dq)
                rawc[gi] = (uint32_t)slot[ib + gi] | ((uint32_t)slot[BN * 16 + ib + gi] << 8);
              else
                rawc[gi] = (uint32_t)reinterpret_cast<const uint16_t*>(slot)[ib + gi] |
                           ((uint32_t)reinterpret_cast<const uint16_t*>(slot + BN * 16)[ib + gi] << 16);
            }
          }
          if (kb % spm == spm - 1 || kb == KB - 1) {
            mbar_arrive(m_empty + (mit & 1));
            ++mit;
          }
        } else {
          // rotate the metadata prefetch: raw1 -> current, fetch two ahead
#pragma unroll
          for (int i2 = 0; i2 < 4; ++i2) {
            rawc[i2] = raw1[i2];
            raw1[i2] = raw2[i2];
          }
          if (++k2 == KB) { k2 = 0; t2 += gridDim.x; }
          fetch(t2, k2, raw2);
        }
        float2 sg[4];
        if (valid) decode(row, kb, rawc, sg);

        if (!mbar_wait_ns(empty + s, ((it / S) & 1) ^ 1, &g_err, 15) ||
            !mbar_wait_ns(ld_full + s, (it / S) & 1, &g_err, 16)) { ok = false; break; }
        const unsigned char* crow = sC + (size_t)s * kCStageBytes + r * kCodeBytes;
        uint32_t cw[kCodeBytes / 4];
        {
          const uint4* src = reinterpret_cast<const uint4*>(crow);
#pragma unroll
          for (int i2 = 0; i2 < kCodeBytes / 16; ++i2) {
            const uint4 u = src[i2];
            cw[4 * i2] = u.x; cw[4 * i2 + 1] = u.y; cw[4 * i2 + 2] = u.z; cw[4 * i2 + 3] = u.w;
          }
        }
        unsigned char* brow = sB + (size_t)s * C::kBStageBytes + r * 128;
        const int sw = r & 7;
        if (!valid) {
#pragma unroll
          for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(brow + ((j ^ sw) << 4)) = make_uint4(0, 0, 0, 0);
        } else if (groups_per_stage == 1) {
          convert_stage<BITS, CB, XT, 1>(cw, sg, cbs, brow, sw);
        } else if (groups_per_stage == 2) {
          convert_stage<BITS, CB, XT, 2>(cw, sg, cbs, brow, sw);
        } else {
          convert_stage<BITS, CB, XT, 4>(cw, sg, cbs, brow, sw);
        }
        // outliers in [k0, k0 + 64): value = fp32(base) + delta, rounded once
        if (valid && o_end > o_beg) {
          if (sorted) {
            while (next_col < k0 + kBK) {
              const int cc = next_col - k0;
              const uint32_t byte = crow[cc * BITS / 8];
              const int code = (int)((byte >> ((cc * BITS) & 7)) & ((1u << BITS) - 1));
              const int gi = gs >= kBK ? 0 : cc / gs;
              float2 g = sg[0];
              if (gi == 1) g = sg[1];
              if (gi == 2) g = sg[2];
              if (gi == 3) g = sg[3];
              const float v = CB ? cbs[code] : (float)code;
              const float val = __fadd_rn(__fmul_rn(v, g.x), g.y) + next_delta;
              const uint32_t pv = pack2<XT>(val, val) & 0xFFFFu;
              *reinterpret_cast<uint16_t*>(brow + (((cc >> 3) ^ sw) << 4) + (cc & 7) * 2) = (uint16_t)pv;
              ++cur;
              next_col = cur < o_end ? q.ocol[cur] : INT_MAX;
              next_delta = cur < o_end ? __half2float(q.odelta[cur]) : 0.f;
            }
          } else {
            for (int j = o_beg; j < o_end; ++j) {
              const int c = q.ocol[j];
              if (c < k0 || c >= k0 + kBK) continue;
              const int cc = c - k0;
              const float val = outlier_value<CB>(q, cbs, row, c, j);
              const uint32_t pv = pack2<XT>(val, val) & 0xFFFFu;
              *reinterpret_cast<uint16_t*>(brow + (((cc >> 3) ^ sw) << 4) + (cc & 7) * 2) = (uint16_t)pv;
            }
          }
        }
        fence_proxy_async_smem();
        mbar_arrive(b_full + s);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

}  // namespace qgemm

// ---- host -------------------------------------------------------------------

static size_t qgemm_smem(int BN, int bits, int S) {
  const size_t stage = qgemm::kAStageBytes + (size_t)BN * qgemm::kBK * 2 + (size_t)BN * qgemm::kBK * bits / 8;
  return 1024 + (size_t)S * stage + 2 * (2 * (size_t)BN * 16) + (3 * S + 8) * 8 + 16 + 256 * 4;
}

// Layout conditions of the tensor-core path (everything else uses the GEMV).
bool qgemm_supported(const ts_qweight& w, const void* x, int64_t x_stride) {
  if (!(w.bits == 2 || w.bits == 4 || w.bits == 8)) return false;
  const int gs = w.group_size;
  if (gs % 8 != 0 || !(gs % qgemm::kBK == 0 || qgemm::kBK % gs == 0)) return false;
  if (gs < 16 && w.bits == 2) return false;
  const int64_t kb = (w.cols + qgemm::kBK - 1) / qgemm::kBK;
  if (kb * qgemm::kBK > w.padded_cols || kb * qgemm::kBK * w.bits / 8 > w.packed_row_bytes) return false;
  if (w.packed_row_bytes % 16 != 0 || !is_aligned(w.packed, 16)) return false;
  if (w.rows * w.n_groups >= (int64_t(1) << 31) || w.rows >= (int64_t(1) << 31)) return false;
  if (!is_aligned(x, 16) || (x_stride * 2) % 16 != 0) return false;
  if (w.cols < 1) return false;
  return max_smem_optin() >= (int)qgemm_smem(128, w.bits, 3);
}

template <int BITS, bool CB, int XT, int BN>
static int launch_qgemm(const CUtensorMap* maps, const qgemm::Args& a, int grid, size_t smem, cudaStream_t st) {
  auto k = qgemm::qgemm_kernel<BITS, CB, XT, BN>;
  TS_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  k<<<grid, qgemm::Cfg<BN>::kThreads, smem, st>>>(maps[0], maps[1], maps[2], maps[3], a);
  TS_LAUNCH_CHECK();
  return TS_OK;
}

template <int BITS, bool CB, int XT>
static int launch_bn(int BN, const CUtensorMap* maps, const qgemm::Args& a, int grid, size_t smem,
                     cudaStream_t st) {
  if (BN == 256) return launch_qgemm<BITS, CB, XT, 256>(maps, a, grid, smem, st);
  return launch_qgemm<BITS, CB, XT, 128>(maps, a, grid, smem, st);
}

template <int BITS>
static int launch_bits(bool cb, int xt, int BN, const CUtensorMap* maps, const qgemm::Args& a, int grid,
                       size_t smem, cudaStream_t st) {
  if (cb)
    return xt ? launch_bn<BITS, true, 1>(BN, maps, a, grid, smem, st)
              : launch_bn<BITS, true, 0>(BN, maps, a, grid, smem, st);
  return xt ? launch_bn<BITS, false, 1>(BN, maps, a, grid, smem, st)
            : launch_bn<BITS, false, 0>(BN, maps, a, grid, smem, st);
}

int run_qgemm(const ts_qweight& w, const void* x, int x_dtype, int64_t M, int64_t x_stride, const void* bias,
              int bias_dtype, void* out, int out_dtype, int64_t out_stride, cudaStream_t stream) {
  TS_UNSUPPORTED(qgemm_supported(w, x, x_stride), "qgemm: layout not supported");
  qgemm::Args a;
  a.q = make_qw(w);
  a.M = M;
  a.bias = bias;
  a.bias_dtype = bias_dtype;
  a.out = out;
  a.out_dtype = out_dtype;
  a.out_stride = out_stride;
  a.mblocks = (int)((M + qgemm::kBM - 1) / qgemm::kBM);
  a.kblocks = (int)((w.cols + qgemm::kBK - 1) / qgemm::kBK);
  const int sms = sm_count();
  // 256-row tiles unless that leaves most SMs idle or does not fit
  int BN = 256;
  if ((int64_t)a.mblocks * ((w.rows + 255) / 256) < sms) BN = 128;
  int S = 8;
  while (S > 2 && qgemm_smem(BN, w.bits, S) > (size_t)max_smem_optin()) --S;
  if (S < 3 && BN == 256) {
    BN = 128;
    S = 8;
    while (S > 2 && qgemm_smem(BN, w.bits, S) > (size_t)max_smem_optin()) --S;
  }
  a.nblocks = (int)((w.rows + BN - 1) / BN);
  a.stages = S;
  const size_t smem = qgemm_smem(BN, w.bits, S);
  const int64_t ntiles = (int64_t)a.mblocks * a.nblocks;
  const int grid = (int)std::min<int64_t>(ntiles, sms);
  CUtensorMap maps[4];
  int rc = encode_tmap_2d(&maps[0], x, CU_TENSOR_MAP_DATA_TYPE_UINT16, (uint64_t)w.cols, (uint64_t)M,
                          (uint64_t)x_stride * 2, qgemm::kBK, qgemm::kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != TS_OK) return rc;
  rc = encode_tmap_2d(&maps[1], w.packed, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)w.packed_row_bytes,
                      (uint64_t)w.rows, (uint64_t)w.packed_row_bytes, qgemm::kBK * w.bits / 8, BN,
                      CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc != TS_OK) return rc;
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
                        (uint64_t)w.rows, (uint64_t)w.n_groups * eb, a.meta_groups, BN, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != TS_OK) return rc;
    rc = encode_tmap_2d(&maps[3], dq ? (const void*)w.dq_gmin_codes : w.gmin, t, (uint64_t)w.n_groups,
                        (uint64_t)w.rows, (uint64_t)w.n_groups * eb, a.meta_groups, BN, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != TS_OK) return rc;
  } else {
    a.meta_groups = 1;   // unused; keeps the stages-per-block arithmetic nonzero
    if ((int64_t)w.group_size < qgemm::kBK) a.meta_groups = qgemm::kBK / w.group_size;
  }
  const bool cb = w.codebook != nullptr;
  const int xt = x_dtype == TS_BF16 ? 1 : 0;
  if (w.bits == 2) return launch_bits<2>(cb, xt, BN, maps, a, grid, smem, stream);
  if (w.bits == 4) return launch_bits<4>(cb, xt, BN, maps, a, grid, smem, stream);
  return launch_bits<8>(cb, xt, BN, maps, a, grid, smem, stream);
}

}  // namespace ts
