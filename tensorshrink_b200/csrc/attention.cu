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
// One CTA per (sequence, kv head), one warp per query head of the group:
//   1. warp 0 ropes the new k and stores it with v into the cache (the only
//      writer of that cache row); each warp ropes its q into shared memory
//      (products and sums rounded separately and the results to bf16, as
//      the unfused torch ops compute them);
//   2. lane j scores positions j, j + 32, ... below min(attn_len, pos + 1)
//      (fp32 dot products of the bf16 rows, scaled by 1 / sqrt(D));
//   3. warp-wide max and sum give the softmax; lane l accumulates dims
//      4l .. 4l + 3 of sum_j p_j v_j and writes the bf16 output row.
#include "common.cuh"

namespace ts {
namespace attn {

constexpr int kMaxD = 128;

__device__ __forceinline__ float bf(const __nv_bfloat16 v) { return __bfloat162float(v); }

__global__ void decode_attention_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t qkv_stride, int n_q, int n_kv,
                                        int D, const int64_t* __restrict__ pos_p, const float* __restrict__ cos_t,
                                        const float* __restrict__ sin_t, __nv_bfloat16* k_cache,
                                        __nv_bfloat16* v_cache, int64_t cache_b_stride, int64_t cache_h_stride,
                                        int attn_len, int max_seq, __nv_bfloat16* __restrict__ out,
                                        int64_t out_stride) {
  extern __shared__ float sm[];
  const int group = n_q / n_kv;
  const int b = blockIdx.x / n_kv, g = blockIdx.x % n_kv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = D / 2;
  const int64_t pos = *pos_p;
  if (pos < 0 || pos >= max_seq) return;   // no cache row for this position (the host checks what it can)
  const int n_ctx = (int)(pos + 1 < (int64_t)attn_len ? pos + 1 : (int64_t)attn_len);   // positions attended
  float* qs = sm;                               // [group][D] roped q (bf16-rounded) in fp32
  float* ps = sm + group * kMaxD;               // [group][attn_len] scores, then probabilities
  const __nv_bfloat16* row = qkv + b * qkv_stride;
  const float* cs = cos_t + pos * half;
  const float* sn = sin_t + pos * half;
  __nv_bfloat16* kc = k_cache + b * cache_b_stride + g * cache_h_stride;
  __nv_bfloat16* vc = v_cache + b * cache_b_stride + g * cache_h_stride;

  // 1. rotary embedding of q (every warp, its head) and k (warp 0), cache append
  const int hq = g * group + warp;
  for (int i = lane; i < half; i += 32) {
    const float c = cs[i], s = sn[i];
    const float x1 = bf(row[hq * D + i]), x2 = bf(row[hq * D + half + i]);
    qs[warp * kMaxD + i] = bf(__float2bfloat16_rn(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s))));
    qs[warp * kMaxD + half + i] = bf(__float2bfloat16_rn(__fadd_rn(__fmul_rn(x1, s), __fmul_rn(x2, c))));
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
  __syncthreads();   // the cache row at `pos` and every q are in place

  // 2. scores of this warp's head
  const float scale = rsqrtf((float)D);
  float* p = ps + warp * attn_len;
  const float* q = qs + warp * kMaxD;
  float mx = -INFINITY;
  for (int j = lane; j < n_ctx; j += 32) {
    const uint4* kr = reinterpret_cast<const uint4*>(kc + (int64_t)j * D);
    float acc = 0.f;
    for (int c8 = 0; c8 < D / 8; ++c8) {
      const uint4 u = kr[c8];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        acc = fmaf(q[c8 * 8 + 2 * e], __uint_as_float(w[e] << 16), acc);
        acc = fmaf(q[c8 * 8 + 2 * e + 1], __uint_as_float(w[e] & 0xFFFF0000u), acc);
      }
    }
    acc *= scale;
    p[j] = acc;
    mx = fmaxf(mx, acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
  for (int j = lane; j < n_ctx; j += 32) {
    const float e = __expf(p[j] - mx);
    p[j] = e;
    sum += e;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  __syncwarp();
  const float inv = 1.f / sum;

  // 3. probabilities times values: lane l owns dims 4l .. 4l + 3 (D <= 128)
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const int d0 = 4 * lane;
  if (d0 < D) {
    for (int j = 0; j < n_ctx; ++j) {
      const uint2 u = *reinterpret_cast<const uint2*>(vc + (int64_t)j * D + d0);
      const float pj = p[j];
      acc[0] = fmaf(pj, __uint_as_float(u.x << 16), acc[0]);
      acc[1] = fmaf(pj, __uint_as_float(u.x & 0xFFFF0000u), acc[1]);
      acc[2] = fmaf(pj, __uint_as_float(u.y << 16), acc[2]);
      acc[3] = fmaf(pj, __uint_as_float(u.y & 0xFFFF0000u), acc[3]);
    }
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
  const size_t smem = (size_t)group * (attn::kMaxD + attn_len) * sizeof(float);
  TS_UNSUPPORTED(smem <= 200 * 1024, "attention over %d positions does not fit shared memory", attn_len);
  TS_REQUIRE(is_aligned(k_cache, 16) && is_aligned(v_cache, 16) && cache_head_stride % 8 == 0 &&
                 cache_batch_stride % 8 == 0,
             "KV cache rows must be 16-byte aligned");
  if (batch == 0) return TS_OK;
  auto kern = attn::decode_attention_kernel;
  if (smem > 48 * 1024) TS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  kern<<<batch * n_kv, 32 * group, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv), qkv_row_stride, n_q, n_kv, head_dim, pos, rope_cos, rope_sin,
      reinterpret_cast<__nv_bfloat16*>(k_cache), reinterpret_cast<__nv_bfloat16*>(v_cache), cache_batch_stride,
      cache_head_stride, attn_len, max_seq, reinterpret_cast<__nv_bfloat16*>(out), out_row_stride);
  TS_LAUNCH_CHECK();
  return TS_OK;
}
