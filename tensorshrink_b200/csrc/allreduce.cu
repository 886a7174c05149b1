// One-shot all-reduce of fp32 row-parallel partial sums over NVLink peer
// memory, for the decode-sized exchanges of tensor-parallel QuantLinear
// layers (a few to a few hundred KB per call, where a ring collective is
// latency-bound).
//
// Every rank owns one exchange buffer (cudaMalloc'd here, mapped into the
// other ranks with CUDA IPC): two parities x `world` slots of `cap` floats,
// then two parities x `world` x kMaxBlocks flag words, then an epoch word.
// A call with epoch e (read from the epoch word, so the same launch replays
// correctly inside a CUDA graph) and parity p = e & 1 runs one CTA per chunk
// of the vector:
//   1. the CTA stores its chunk of this rank's partial into slot `rank` of
//      parity p of every rank's buffer (plain peer stores over NVLink);
//   2. fence, then it writes e into its flag word [p][rank][cta] on every rank;
//   3. it waits (bounded) until flag [p][r][cta] == e in its own buffer for
//      every rank r, then sums the world slots of its chunk in rank order
//      (the same order on every rank, so all ranks get identical results),
//      adds the optional residual and writes the output.
// The last CTA to finish advances the epoch word. A parity's slots are
// written again two calls later, by which time every rank has finished
// reading them (it has passed the flags of the call in between). No TMA and
// no multicast: peer memory is touched by plain loads and stores only.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "sm100.cuh"

namespace ts {
namespace ar {

constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 128;
constexpr int kThreads = 512;

struct Args {
  float* peer_buf[kMaxRanks];   // every rank's exchange buffer base (this rank's own included)
  int rank, world;
  int64_t cap;                  // floats per slot
  int64_t n;                    // floats in this call
  const float* in;
  const float* residual;        // or nullptr
  float* out;
  uint64_t wait_ns;
  int* err;
};

__device__ __forceinline__ uint32_t* flags_of(float* base, int64_t cap, int world) {
  return reinterpret_cast<uint32_t*>(base + 2 * (int64_t)world * cap);
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kThreads) oneshot_kernel(const Args a) {
  __shared__ uint32_t s_epoch;
  __shared__ int s_last;
  float* own = a.peer_buf[a.rank];
  uint32_t* own_flags = flags_of(own, a.cap, a.world);
  uint32_t* epoch_word = own_flags + 2 * a.world * kMaxBlocks;
  uint32_t* done_word = epoch_word + 1;
  if (threadIdx.x == 0) s_epoch = *reinterpret_cast<volatile uint32_t*>(epoch_word) + 1;
  __syncthreads();
  const uint32_t e = s_epoch;
  const int p = e & 1;
  const int64_t chunk = ((a.n + gridDim.x - 1) / gridDim.x + 3) & ~(int64_t)3;
  const int64_t c0 = blockIdx.x * chunk, c1 = min(a.n, c0 + chunk);

  // 1. push this rank's chunk to every rank (16-byte stores; chunks are
  //    multiples of 4 floats and the slots 16-byte aligned)
  const bool vec = ((reinterpret_cast<uintptr_t>(a.in) & 15) == 0) && (a.cap % 4 == 0);
  for (int r = 0; r < a.world; ++r) {
    float* dst = a.peer_buf[r] + ((int64_t)p * a.world + a.rank) * a.cap;
    if (vec) {
      const int64_t v1 = c1 & ~(int64_t)3;
      for (int64_t i = c0 + 4 * threadIdx.x; i < v1; i += 4 * blockDim.x)
        *reinterpret_cast<float4*>(dst + i) = *reinterpret_cast<const float4*>(a.in + i);
      for (int64_t i = v1 + threadIdx.x; i < c1; i += blockDim.x) dst[i] = a.in[i];
    } else {
      for (int64_t i = c0 + threadIdx.x; i < c1; i += blockDim.x) dst[i] = a.in[i];
    }
  }
  // 2. publish: the block's stores are ordered before one system-scope
  //    fence by the threads that write the flags
  __syncthreads();
  if (threadIdx.x < a.world) {
    __threadfence_system();
    uint32_t* f = flags_of(a.peer_buf[threadIdx.x], a.cap, a.world) + ((int64_t)p * a.world + a.rank) * kMaxBlocks +
                  blockIdx.x;
    st_release_sys(f, e);
  }
  // 3. wait for every rank's chunk (bounded), then reduce in rank order
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (threadIdx.x < a.world) {
    const uint32_t* f = own_flags + ((int64_t)p * a.world + threadIdx.x) * kMaxBlocks + blockIdx.x;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys(f) != e) {
      if (globaltimer_ns() - t0 > a.wait_ns) {
        atomicExch(a.err, 31);
        s_ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  if (s_ok) {
    for (int64_t i = c0 + threadIdx.x; i < c1; i += blockDim.x) {
      float s = a.residual ? a.residual[i] : 0.f;
      float t = 0.f;
      for (int r = 0; r < a.world; ++r) t += __ldcv(own + ((int64_t)p * a.world + r) * a.cap + i);
      a.out[i] = s + t;
    }
  }
  // the last CTA advances the epoch for the next call
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(done_word, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    *done_word = 0;
    __threadfence();
    *epoch_word = e;
  }
}

}  // namespace ar
}  // namespace ts

using namespace ts;

extern "C" size_t ts_peer_buffer_bytes(int world, int64_t cap) {
  return (size_t)2 * world * cap * sizeof(float) + (size_t)2 * world * ar::kMaxBlocks * 4 + 256;
}

extern "C" int ts_peer_alloc(int world, int64_t cap, void** ptr) {
  TS_REQUIRE(ptr && world >= 1 && world <= ar::kMaxRanks && cap > 0, "bad peer buffer request");
  void* p = nullptr;
  const size_t bytes = ts_peer_buffer_bytes(world, cap);
  TS_CUDA_TRY(cudaMalloc(&p, bytes));
  TS_CUDA_TRY(cudaMemset(p, 0, bytes));
  TS_CUDA_TRY(cudaDeviceSynchronize());
  *ptr = p;
  return TS_OK;
}

extern "C" int ts_peer_free(void* ptr) {
  TS_CUDA_TRY(cudaFree(ptr));
  return TS_OK;
}

extern "C" int ts_ipc_get_handle(void* ptr, void* handle_out /* 64 bytes */) {
  cudaIpcMemHandle_t h;
  TS_CUDA_TRY(cudaIpcGetMemHandle(&h, ptr));
  memcpy(handle_out, &h, sizeof(h));
  return TS_OK;
}

extern "C" int ts_ipc_open(const void* handle /* 64 bytes */, void** ptr) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  TS_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return TS_OK;
}

extern "C" int ts_ipc_close(void* ptr) {
  TS_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
  return TS_OK;
}

extern "C" int ts_allreduce_oneshot(void* const* peer_bufs, int rank, int world, int64_t cap, const float* in,
                                    const float* residual, float* out, int64_t n, int* err_flag, void* stream) {
  TS_REQUIRE(peer_bufs && in && out && err_flag, "NULL pointer");
  TS_REQUIRE(world >= 1 && world <= ar::kMaxRanks && rank >= 0 && rank < world, "bad rank/world");
  TS_REQUIRE(n >= 0 && n <= cap, "all-reduce of %lld floats exceeds the exchange capacity %lld", (long long)n,
             (long long)cap);
  if (n == 0) return TS_OK;
  ar::Args a;
  for (int r = 0; r < ar::kMaxRanks; ++r) a.peer_buf[r] = r < world ? reinterpret_cast<float*>(peer_bufs[r]) : nullptr;
  a.rank = rank;
  a.world = world;
  a.cap = cap;
  a.n = n;
  a.in = in;
  a.residual = residual;
  a.out = out;
  a.wait_ns = wait_limit_ns();
  a.err = err_flag;
  (void)take_test_stall();
  const int blocks = (int)std::min<int64_t>(ar::kMaxBlocks, std::max<int64_t>(1, (n + 2047) / 2048));
  ar::oneshot_kernel<<<blocks, ar::kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  TS_LAUNCH_CHECK();
  return TS_OK;
}
