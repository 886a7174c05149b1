// Decode-step attention for the Llama-shaped decoder: one kernel per layer
// that applies rotary embeddings to the new token's q and k, appends k and v
// to the KV cache at the step's position, and attends over the cache
// (grouped-query: every kv head serves n_q / n_kv query heads).
//
// The unfused step it replaces runs ~20 small torch kernels per layer (rope
// gathers and arithmetic, two index_copy_ into the cache, SDPA with a mask,
// transposes); at batch 1 their launch latency, not their bytes, sets the
// step time.
//
// One CTA per (sequence, kv head), one warp per query head of the group
// (at least four warps, which all help load):
//   1. warp 0 ropes the new k and stores it with v into the cache (the only
//      writer of that cache row); each head warp ropes its q into shared
//      memory (products and sums rounded separately and the results to bf16,
//      as the unfused torch ops compute them);
//   2. the positions below min(attn_len, pos + 1) stream through shared
//      memory in tiles of 64 rows of k and v (16-byte async copies, double
//      buffered); per tile each head warp scores 2 positions per lane (fp32
//      dot products scaled by 1 / sqrt(D)), updates its running max and sum
//      (online softmax) and accumulates p v with lane l owning dims 4l..4l+3;
//   3. the bf16 output row is acc / sum.
#include "sm100.cuh"

namespace ts {
namespace attn {

constexpr int kMaxD = 128;
constexpr int kTile = 64;
constexpr int kPitch = kMaxD + 8;   // bf16 elements per shared row: 16-byte reads across lanes hit distinct banks

__device__ __forceinline__ float bf(const __nv_bfloat16 v) { return __bfloat162float(v); }

__device__ __forceinline__ void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

__global__ void decode_attention_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t qkv_stride, int n_q, int n_kv,
                                        int D, const int64_t* __restrict__ pos_p, const float* __restrict__ cos_t,
                                        const float* __restrict__ sin_t, __nv_bfloat16* k_cache,
                                        __nv_bfloat16* v_cache, int64_t cache_b_stride, int64_t cache_h_stride,
                                        int attn_len, int max_seq, __nv_bfloat16* __restrict__ out,
                                        int64_t out_stride) {
  extern __shared__ __align__(16) char smem_raw[];
  __nv_bfloat16* tiles = reinterpret_cast<__nv_bfloat16*>(smem_raw);   // [2 buf][k, v][kTile][kPitch]
  const int group = n_q / n_kv;
  float* qs = reinterpret_cast<float*>(tiles + 2 * 2 * kTile * kPitch);   // [group][kMaxD]
  float* ps = qs + group * kMaxD;                                          // [group][kTile]
  const int b = blockIdx.x / n_kv, g = blockIdx.x % n_kv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = D / 2;
  const int64_t pos = *pos_p;
  if (pos < 0 || pos >= max_seq) return;   // no cache row for this position (the host checks what it can)
  const int n_ctx = (int)(pos + 1 < (int64_t)attn_len ? pos + 1 : (int64_t)attn_len);   // positions attended
  const __nv_bfloat16* row = qkv + b * qkv_stride;
  const float* cs = cos_t + pos * half;
  const float* sn = sin_t + pos * half;
  __nv_bfloat16* kc = k_cache + b * cache_b_stride + g * cache_h_stride;
  __nv_bfloat16* vc = v_cache + b * cache_b_stride + g * cache_h_stride;

  // 1. rotary embedding of q (head warps) and k (warp 0), cache append
  const bool head = warp < group;
  const int hq = g * group + warp;
  for (int i = lane; i < half; i += 32) {
    const float c = cs[i], s = sn[i];
    if (head) {
      const float x1 = bf(row[hq * D + i]), x2 = bf(row[hq * D + half + i]);
      qs[warp * kMaxD + i] = bf(__float2bfloat16_rn(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s))));
      qs[warp * kMaxD + half + i] = bf(__float2bfloat16_rn(__fadd_rn(__fmul_rn(x1, s), __fmul_rn(x2, c))));
    }
    if (warp == 0) {
      const __nv_bfloat16* kr = row + (int64_t)n_q * D + g * D;
      const __nv_bfloat16* vr = row + (int64_t)(n_q + n_kv) * D + g * D;
      const float k1 = bf(kr[i]), k2 = bf(kr[half + i]);
      kc[pos * D + i] = __float2bfloat16_rn(__fsub_rn(__fmul_rn(k1, c), __fmul_rn(k2, s)));
      kc[pos * D + half + i] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(k1, s), __fmul_rn(k2, c)));
      vc[pos * D + i] = vr[i];
      vc[pos * D + half + i] = vr[half + i];
    }
  }
  __syncthreads();   // the cache row at `pos` (global, written by this CTA) and every q are in place

  // tile loader: rows [t0, t0 + kTile) of k and v into buffer `buf`
  const int chunks = D / 8;   // 16-byte pieces per row
  auto load_tile = [&](int t0, int buf) {
    __nv_bfloat16* kt = tiles + (buf * 2) * kTile * kPitch;
    __nv_bfloat16* vt = kt + kTile * kPitch;
    const int rows = min(kTile, n_ctx - t0);
    for (int i = threadIdx.x; i < rows * chunks; i += blockDim.x) {
      const int r = i / chunks, c = i - r * chunks;
      cp16(kt + r * kPitch + c * 8, kc + (int64_t)(t0 + r) * D + c * 8);
      cp16(vt + r * kPitch + c * 8, vc + (int64_t)(t0 + r) * D + c * 8);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  const float scale = rsqrtf((float)D);
  const float* q = qs + warp * kMaxD;
  float* p = ps + warp * kTile;
  float m = -INFINITY, l = 0.f;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const int d0 = 4 * lane;
  const int n_tiles = (n_ctx + kTile - 1) / kTile;
  load_tile(0, 0);
  for (int t = 0; t < n_tiles; ++t) {
    const int buf = t & 1;
    if (t + 1 < n_tiles) {
      load_tile((t + 1) * kTile, buf ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();   // tile t landed for every thread's copies
    if (head) {
      const __nv_bfloat16* kt = tiles + (buf * 2) * kTile * kPitch;
      const __nv_bfloat16* vt = kt + kTile * kPitch;
      const int rows = min(kTile, n_ctx - t * kTile);
      float sc[2];
      float tmax = -INFINITY;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int r = lane + 32 * u;
        sc[u] = -INFINITY;
        if (r < rows) {
          const uint4* kr = reinterpret_cast<const uint4*>(kt + r * kPitch);
          float a = 0.f;
          for (int c8 = 0; c8 < chunks; ++c8) {
            const uint4 w = kr[c8];
            const float4 qa = *reinterpret_cast<const float4*>(q + c8 * 8);
            const float4 qb = *reinterpret_cast<const float4*>(q + c8 * 8 + 4);
            a = fmaf(qa.x, __uint_as_float(w.x << 16), a);
            a = fmaf(qa.y, __uint_as_float(w.x & 0xFFFF0000u), a);
            a = fmaf(qa.z, __uint_as_float(w.y << 16), a);
            a = fmaf(qa.w, __uint_as_float(w.y & 0xFFFF0000u), a);
            a = fmaf(qb.x, __uint_as_float(w.z << 16), a);
            a = fmaf(qb.y, __uint_as_float(w.z & 0xFFFF0000u), a);
            a = fmaf(qb.z, __uint_as_float(w.w << 16), a);
            a = fmaf(qb.w, __uint_as_float(w.w & 0xFFFF0000u), a);
          }
          sc[u] = a * scale;
          tmax = fmaxf(tmax, sc[u]);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
      const float m_new = fmaxf(m, tmax);
      const float corr = __expf(m - m_new);   // 0 on the first tile (m = -inf)
      float tsum = 0.f;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int r = lane + 32 * u;
        const float e = r < rows ? __expf(sc[u] - m_new) : 0.f;
        p[r] = e;
        tsum += e;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) tsum += __shfl_xor_sync(0xffffffffu, tsum, o);
      l = l * corr + tsum;
      m = m_new;
      __syncwarp();
      if (d0 < D) {
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[e] *= corr;
#pragma unroll 4
        for (int r = 0; r < rows; ++r) {
          const uint2 u = *reinterpret_cast<const uint2*>(vt + r * kPitch + d0);
          const float pr = p[r];
          acc[0] = fmaf(pr, __uint_as_float(u.x << 16), acc[0]);
          acc[1] = fmaf(pr, __uint_as_float(u.x & 0xFFFF0000u), acc[1]);
          acc[2] = fmaf(pr, __uint_as_float(u.y << 16), acc[2]);
          acc[3] = fmaf(pr, __uint_as_float(u.y & 0xFFFF0000u), acc[3]);
        }
      }
      __syncwarp();   // p is rewritten by the next tile
    }
    __syncthreads();  // buffer `buf` is refilled two tiles on
  }
  if (head && d0 < D) {
    const float inv = 1.f / l;
    __nv_bfloat16* o = out + b * out_stride + (int64_t)hq * D + d0;
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = __float2bfloat16_rn(acc[e] * inv);
  }
}

}  // namespace attn
}  // namespace ts

using namespace ts;

extern "C" int ts_decode_attention(const void* qkv, int64_t qkv_row_stride, int batch, int n_q, int n_kv,
                                   int head_dim, const int64_t* pos, const float* rope_cos, const float* rope_sin,
                                   void* k_cache, void* v_cache, int64_t cache_batch_stride,
                                   int64_t cache_head_stride, int attn_len, int max_seq, void* out,
                                   int64_t out_row_stride, void* stream) {
  TS_REQUIRE(qkv && pos && rope_cos && rope_sin && k_cache && v_cache && out, "NULL pointer");
  TS_REQUIRE(batch >= 0 && n_kv > 0 && n_q % n_kv == 0, "bad head counts");
  const int group = n_q / n_kv;
  TS_UNSUPPORTED(group >= 1 && group <= 16, "at most 16 query heads per kv head");
  TS_UNSUPPORTED(head_dim % 8 == 0 && head_dim <= attn::kMaxD && head_dim >= 8, "head_dim must be a multiple of 8, <= 128");
  TS_REQUIRE(attn_len > 0 && attn_len <= max_seq, "attn_len must be in [1, max_seq]");
  const size_t smem = (size_t)2 * 2 * attn::kTile * attn::kPitch * 2 + (size_t)group * (attn::kMaxD + attn::kTile) * 4;
  TS_REQUIRE(is_aligned(k_cache, 16) && is_aligned(v_cache, 16) && cache_head_stride % 8 == 0 &&
                 cache_batch_stride % 8 == 0,
             "KV cache rows must be 16-byte aligned");
  if (batch == 0) return TS_OK;
  auto kern = attn::decode_attention_kernel;
  if (smem > 48 * 1024) TS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  kern<<<batch * n_kv, 32 * std::max(group, 4), smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv), qkv_row_stride, n_q, n_kv, head_dim, pos, rope_cos, rope_sin,
      reinterpret_cast<__nv_bfloat16*>(k_cache), reinterpret_cast<__nv_bfloat16*>(v_cache), cache_batch_stride,
      cache_head_stride, attn_len, max_seq, reinterpret_cast<__nv_bfloat16*>(out), out_row_stride);
  TS_LAUNCH_CHECK();
  return TS_OK;
}
