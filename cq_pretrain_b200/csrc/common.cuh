// Shared helpers for the sm_100a kernels of cq_pretrain_b200.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include <atomic>
#include <cstdint>

namespace cqb {

// Number of kernels this library has launched (read by benchmarks to count native launches).
std::atomic<long long>& launch_counter();
inline void count_launch(int n = 1) { launch_counter().fetch_add(n, std::memory_order_relaxed); }

#define CQB_CHECK_CUDA(expr)                                                                        \
  do {                                                                                              \
    cudaError_t err__ = (expr);                                                                     \
    TORCH_CHECK(err__ == cudaSuccess, "CUDA error ", cudaGetErrorString(err__), " at ", __FILE__, \
                ":", __LINE__);                                                                     \
  } while (0)

#define CQB_LAUNCH_CHECK() CQB_CHECK_CUDA(cudaGetLastError())

inline cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// TMA map over a row-major 2-D bf16 matrix (cols contiguous): 128B-swizzled boxes of
// 64 cols x box_rows rows, out-of-bounds rows and cols read as zero (gemm.cu).
CUtensorMap tma_map_bf16(const at::Tensor& t, int box_rows);

inline int sm_count() {
  static int count = [] {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
  }();
  return count;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// 8 x bf16 <-> 8 x float through one 16-byte vector.
struct alignas(16) Bf16x8 {
  __nv_bfloat162 v[4];
};

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* out) {
  Bf16x8 x = *reinterpret_cast<const Bf16x8*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(x.v[i]);
    out[2 * i] = f.x;
    out[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ void load8(const float* p, float* out) {
  float4 a = *reinterpret_cast<const float4*>(p);
  float4 b = *reinterpret_cast<const float4*>(p + 4);
  out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
  out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* in) {
  Bf16x8 x;
#pragma unroll
  for (int i = 0; i < 4; ++i) x.v[i] = __floats2bfloat162_rn(in[2 * i], in[2 * i + 1]);
  *reinterpret_cast<Bf16x8*>(p) = x;
}

__device__ __forceinline__ void store8(float* p, const float* in) {
  *reinterpret_cast<float4*>(p) = make_float4(in[0], in[1], in[2], in[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(in[4], in[5], in[6], in[7]);
}

__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }

// Graph-safe call epochs of the peer-memory collectives. With a device counter (`ctr` non-null)
// a call's epoch is *ctr + 1, read by thread 0 of every CTA at the start (the previous call of the
// same kind finished in stream order, so the counter is final); the last CTA to finish stores the
// epoch back (`done` counts finished CTAs and is re-zeroed by that CTA). A captured CUDA graph
// therefore advances the epoch on every replay, where a host-chosen epoch would repeat.
__device__ __forceinline__ long long epoch_begin(const long long* ctr, long long host_epoch) {
  return ctr ? *reinterpret_cast<volatile const long long*>(ctr) + 1 : host_epoch;
}
// Called by thread 0 of every CTA after the CTA's last access of the call's buffers and flags.
__device__ __forceinline__ void epoch_end(long long* ctr, unsigned* done, long long epoch) {
  if (!ctr) return;
  __threadfence();
  if (atomicAdd(done, 1u) == gridDim.x * gridDim.y * gridDim.z - 1) {
    *reinterpret_cast<volatile long long*>(ctr) = epoch;
    *reinterpret_cast<volatile unsigned*>(done) = 0u;
    __threadfence();
  }
}

// ---- debug bounds checks ----------------------------------------------------------------------
// Built with -DCQB_DEBUG_BOUNDS (`python -m cq_pretrain_b200.build --debug`), CQB_IN_RANGE(i, n, site)
// tests 0 <= i < n; the first failure of a translation unit is recorded in its status block
// {site, index, bound} and the caller skips the access (no trap: the context stays usable and the
// host reads the block through debug_bounds_status()). Release builds compile the checks away.
#ifdef CQB_DEBUG_BOUNDS
namespace dbg {
static __device__ long long status[3];
__device__ __forceinline__ bool in_range(long long i, long long n, int site) {
  if (i >= 0 && i < n) return true;
  if (atomicCAS(reinterpret_cast<unsigned long long*>(&status[0]), 0ull, (unsigned long long)site) == 0ull) {
    status[1] = i;
    status[2] = n;
  }
  return false;
}
}  // namespace dbg
#define CQB_IN_RANGE(i, n, site) ::cqb::dbg::in_range((long long)(i), (long long)(n), (site))
#define CQB_DEBUG_STATUS_READER(fn)                                                              \
  std::vector<int64_t> fn(bool reset) {                                                          \
    long long h[3] = {0, 0, 0};                                                                  \
    CQB_CHECK_CUDA(cudaMemcpyFromSymbol(h, ::cqb::dbg::status, sizeof(h)));                       \
    if (reset) {                                                                                 \
      long long z[3] = {0, 0, 0};                                                                \
      CQB_CHECK_CUDA(cudaMemcpyToSymbol(::cqb::dbg::status, z, sizeof(z)));                       \
    }                                                                                            \
    return {h[0], h[1], h[2]};                                                                   \
  }
#else
#define CQB_IN_RANGE(i, n, site) true
#endif

}  // namespace cqb
