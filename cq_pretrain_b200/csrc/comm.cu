// Peer-memory plumbing for the in-kernel tensor-parallel collectives (one process per GPU).
//
//  * symmetric buffers: cudaMalloc + CUDA IPC handles exchanged by the host, opened on every
//    peer (NVLink P2P); the same layout on every rank;
//  * epoch flags: a rank publishes "epoch e reached" by a system-scope release store into a
//    slot of every peer's flag area; a waiter acquires its own slots with bounded spins and
//    records a status code (never traps) when the limit expires;
//  * rs_reduce: the reduction half of GEMM->reduce-scatter: sums the tp partial slabs that
//    peers stored into this rank's receive buffer (fp32 accumulate, + bias) into bf16.
#include "common.cuh"
#include "tcgen05.cuh"

#include <cuda_runtime.h>

namespace cqb {

namespace {

__device__ __forceinline__ void st_release_sys(long long* p, long long v) {
  asm volatile("st.release.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ long long ld_acquire_sys(const long long* p) {
  long long v;
  asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Thread t < tp: publish `epoch` into slot `rank` of peer t's flag area; then wait until every
// slot of this rank's own flag area reached `epoch`.
__global__ void signal_wait_kernel(long long* const* peer_flags, long long* my_flags, int rank, int tp,
                                   long long epoch, int wait, int* status) {
  const int t = threadIdx.x;
  if (t < tp) {
    __threadfence_system();
    st_release_sys(peer_flags[t] + rank, epoch);
  }
  if (!wait) return;
  __syncthreads();
  if (t < tp) {
    const unsigned long long start = tc::globaltimer();
    while (ld_acquire_sys(my_flags + t) < epoch) {
      if (tc::globaltimer() - start > tc::kWaitNs) {
        atomicCAS(status, 0, 100 + t);
        break;
      }
    }
  }
  __syncthreads();
}

// out[r, c] = sum_s recv[s][r][c] (+ bias[c]);  recv: [tp][rows][cols] bf16
__global__ void rs_reduce_kernel(const __nv_bfloat16* __restrict__ recv, const __nv_bfloat16* __restrict__ bias,
                                 __nv_bfloat16* __restrict__ out, int tp, int rows, int cols) {
  const size_t vecs = (size_t)rows * cols / 8;
  const size_t slab = (size_t)rows * cols;
  for (size_t v = blockIdx.x * (size_t)blockDim.x + threadIdx.x; v < vecs; v += (size_t)gridDim.x * blockDim.x) {
    const size_t e = v * 8;
    float acc[8], x[8];
    load8(recv + e, acc);
    for (int s = 1; s < tp; ++s) {
      load8(recv + s * slab + e, x);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += x[j];
    }
    if (bias) {
      load8(bias + (e % cols), x);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += x[j];
    }
    store8(out + e, acc);
  }
}

int* comm_status() {
  static int* word = [] {
    int* p = nullptr;
    CQB_CHECK_CUDA(cudaMalloc(&p, sizeof(int)));
    CQB_CHECK_CUDA(cudaMemset(p, 0, sizeof(int)));
    return p;
  }();
  return word;
}

}  // namespace

// ---- symmetric allocation (host) ------------------------------------------------------------
std::vector<at::Tensor> symm_alloc(int64_t bytes) {
  void* p = nullptr;
  CQB_CHECK_CUDA(cudaMalloc(&p, bytes));
  CQB_CHECK_CUDA(cudaMemset(p, 0, bytes));
  cudaIpcMemHandle_t handle;
  CQB_CHECK_CUDA(cudaIpcGetMemHandle(&handle, p));
  auto h = at::empty({(int64_t)sizeof(handle)}, at::TensorOptions().dtype(at::kByte));
  std::memcpy(h.data_ptr(), &handle, sizeof(handle));
  auto ptr = at::empty({1}, at::TensorOptions().dtype(at::kLong));
  ptr[0] = (int64_t)reinterpret_cast<uintptr_t>(p);
  return {ptr, h};
}

int64_t symm_open(at::Tensor handle_bytes) {
  TORCH_CHECK(handle_bytes.numel() == (int64_t)sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t handle;
  std::memcpy(&handle, handle_bytes.cpu().contiguous().data_ptr(), sizeof(handle));
  void* p = nullptr;
  CQB_CHECK_CUDA(cudaIpcOpenMemHandle(&p, handle, cudaIpcMemLazyEnablePeerAccess));
  return (int64_t)reinterpret_cast<uintptr_t>(p);
}

void symm_close(int64_t ptr) { CQB_CHECK_CUDA(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr))); }
void symm_free(int64_t ptr) { CQB_CHECK_CUDA(cudaFree(reinterpret_cast<void*>(ptr))); }

// Wrap `count` elements at byte offset `offset` of a raw device allocation as a tensor view.
at::Tensor symm_view(int64_t base, int64_t offset, std::vector<int64_t> shape, at::ScalarType dtype) {
  auto opts = at::TensorOptions().dtype(dtype).device(at::kCUDA, at::cuda::current_device());
  return at::from_blob(reinterpret_cast<void*>(base + offset), shape, opts);
}

void signal_wait(at::Tensor peer_flag_ptrs, int64_t my_flags, int64_t rank, int64_t tp, int64_t epoch, bool wait) {
  TORCH_CHECK(peer_flag_ptrs.is_cuda() && peer_flag_ptrs.scalar_type() == at::kLong, "peer flag pointers: cuda int64");
  signal_wait_kernel<<<1, 32, 0, stream()>>>(reinterpret_cast<long long* const*>(peer_flag_ptrs.data_ptr()),
                                             reinterpret_cast<long long*>(my_flags), (int)rank, (int)tp, epoch,
                                             wait ? 1 : 0, comm_status());
  CQB_LAUNCH_CHECK();
  count_launch();
}

at::Tensor rs_reduce(at::Tensor recv, c10::optional<at::Tensor> bias, int64_t tp, int64_t rows, int64_t cols) {
  auto out = at::empty({rows, cols}, recv.options());
  const __nv_bfloat16* b = nullptr;
  at::Tensor bb;
  if (bias && bias->defined()) {
    bb = bias->to(at::kBFloat16).contiguous();
    b = (const __nv_bfloat16*)bb.data_ptr();
  }
  const size_t vecs = (size_t)rows * cols / 8;
  const int grid = (int)std::min<size_t>((vecs + 255) / 256, (size_t)sm_count() * 8);
  rs_reduce_kernel<<<std::max(grid, 1), 256, 0, stream()>>>((const __nv_bfloat16*)recv.data_ptr(), b,
                                                           (__nv_bfloat16*)out.data_ptr(), (int)tp, (int)rows, (int)cols);
  CQB_LAUNCH_CHECK();
  count_launch();
  return out;
}

int comm_status_read(bool reset) {
  int v = 0;
  CQB_CHECK_CUDA(cudaMemcpy(&v, comm_status(), sizeof(int), cudaMemcpyDeviceToHost));
  if (reset && v) CQB_CHECK_CUDA(cudaMemset(comm_status(), 0, sizeof(int)));
  return v;
}

}  // namespace cqb
