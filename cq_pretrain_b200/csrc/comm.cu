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


// ---- TP RMSNorm with the cross-rank variance exchanged in-kernel ----------------------------
// Rows of x hold this rank's slice of a full-width vector (heads spread over TP). Per block of
// 64 rows: each warp sums its rows' local squares (fwd) or dy.w.x (bwd); the 64 partials are
// stored into slot `rank` of every peer's receive slab (plain peer stores), a system-scope
// release flag per (block, rank) publishes them, and after acquiring the peers' flags for the
// same block (bounded wait) the block reduces the tp partials and finishes its rows. The grid
// is persistent (<= one CTA per SM) and every rank walks the blocks in the same order.
constexpr int STAT_ROWS = 64;          // rows per block
constexpr int STAT_MAX_TP = 8;

struct TpNormArgs {
  const __nv_bfloat16* x;
  int ld_x;
  const __nv_bfloat16* dy;   // backward only (contiguous [rows, D])
  const float* w;            // [D] fp32
  __nv_bfloat16* y;          // fwd: y; bwd: dx (contiguous [rows, D])
  float* rstd;               // [rows]
  float* dw_partial;         // bwd: [gridDim.x, D]
  int rows, D;
  float inv_total, eps;
  float* const* peer_recv;   // [tp] slab base of each peer (this call's parity): [tp][max_rows] fp32
  float* my_recv;
  long long* const* peer_flags;  // [tp] flag area of each peer: [blocks][STAT_MAX_TP]
  long long* my_flags;
  int rank, tp, max_rows;
  long long epoch;
  int* status;
  // graph-safe epochs (see epoch_begin): device counter, finished-CTA count, odd-parity slabs
  long long* epoch_ctr;
  unsigned* epoch_done;
  float* const* peer_recv_odd;
  float* my_recv_odd;
};

template <bool BWD>
__global__ void __launch_bounds__(256) tp_norm_kernel(TpNormArgs a) {
  __shared__ float part[STAT_ROWS];
  __shared__ float stat[STAT_ROWS];
  __shared__ int failed;
  __shared__ long long s_epoch;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int blocks = (a.rows + STAT_ROWS - 1) / STAT_ROWS;
  float dw_acc[4][8];
  if (BWD) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) dw_acc[i][j] = 0.f;
  }
  if (threadIdx.x == 0) {
    failed = 0;
    s_epoch = epoch_begin(a.epoch_ctr, a.epoch);
  }
  __syncthreads();
  const long long epoch = s_epoch;
  const bool odd = (epoch & 1) && a.peer_recv_odd;
  float* const* peer_recv = odd ? a.peer_recv_odd : a.peer_recv;
  const float* my_recv = odd ? a.my_recv_odd : a.my_recv;
  for (int b = blockIdx.x; b < blocks; b += gridDim.x) {
    // 1) local partials: warp w handles rows 8w..8w+7 of the block
    for (int rr = 0; rr < 8; ++rr) {
      const int lr = warp * 8 + rr, row = b * STAT_ROWS + lr;
      float acc = 0.f;
      if (row < a.rows) {
        for (int c = lane * 8; c < a.D; c += 256) {
          float xv[8];
          load8(a.x + (size_t)row * a.ld_x + c, xv);
          if (BWD) {
            float dv[8], wv[8];
            load8(a.dy + (size_t)row * a.D + c, dv);
            load8(a.w + c, wv);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc += dv[j] * wv[j] * xv[j];
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) acc += xv[j] * xv[j];
          }
        }
      }
      acc = warp_sum(acc);
      if (lane == 0) part[lr] = acc;
    }
    __syncthreads();
    // 2) publish to every peer (including this rank's own slab)
    if (threadIdx.x < STAT_ROWS * a.tp) {
      const int t = threadIdx.x / STAT_ROWS, lr = threadIdx.x % STAT_ROWS;
      peer_recv[t][(size_t)a.rank * a.max_rows + b * STAT_ROWS + lr] = part[lr];
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < a.tp) st_release_sys(a.peer_flags[threadIdx.x] + (size_t)b * STAT_MAX_TP + a.rank, epoch);
    // 3) acquire the peers' partials of this block
    if (threadIdx.x < a.tp) {
      const long long* f = a.my_flags + (size_t)b * STAT_MAX_TP + threadIdx.x;
      const unsigned long long start = tc::globaltimer();
      while (ld_acquire_sys(f) < epoch) {
        if (tc::globaltimer() - start > tc::kWaitNs) {
          atomicCAS(a.status, 0, 200 + threadIdx.x);
          failed = 1;
          break;
        }
      }
    }
    __syncthreads();
    if (failed) break;   // the host reads the status word; outputs of this call are invalid
    if (threadIdx.x < STAT_ROWS) {
      float sum = 0.f;
      for (int t = 0; t < a.tp; ++t) sum += my_recv[(size_t)t * a.max_rows + b * STAT_ROWS + threadIdx.x];
      stat[threadIdx.x] = sum;
    }
    __syncthreads();
    // 4) finish the rows
    for (int rr = 0; rr < 8; ++rr) {
      const int lr = warp * 8 + rr, row = b * STAT_ROWS + lr;
      if (row >= a.rows) continue;
      float r;
      if (!BWD) {
        r = rsqrtf(stat[lr] * a.inv_total + a.eps);
        if (lane == 0) a.rstd[row] = r;
      } else {
        r = a.rstd[row];
      }
      const float g = BWD ? stat[lr] * r * r * r * a.inv_total : 0.f;
      int k = 0;
      for (int c = lane * 8; c < a.D; c += 256, ++k) {
        float xv[8], wv[8], o[8];
        load8(a.x + (size_t)row * a.ld_x + c, xv);
        load8(a.w + c, wv);
        if (!BWD) {
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = xv[j] * r * wv[j];
        } else {
          float dv[8];
          load8(a.dy + (size_t)row * a.D + c, dv);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            o[j] = dv[j] * wv[j] * r - xv[j] * g;
            if (k < 4) dw_acc[k][j] += dv[j] * xv[j] * r;
          }
        }
        store8(a.y + (size_t)row * a.D + c, o);
      }
    }
    __syncthreads();   // part/stat reused by the next block
  }
  if (BWD) {
    // dw partial of this CTA: reduce the 8 warps through shared memory (fixed order)
    __shared__ float red[8][4 * 256];
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int j = 0; j < 8; ++j) red[warp][k * 256 + lane * 8 + j] = dw_acc[k][j];
    __syncthreads();
    for (int c = threadIdx.x; c < a.D; c += blockDim.x) {
      const int k = c / 256, off = c % 256;
      float sum = 0.f;
      for (int wi = 0; wi < 8; ++wi) sum += red[wi][k * 256 + off];
      a.dw_partial[(size_t)blockIdx.x * a.D + c] = sum;
    }
  }
  __syncthreads();   // every thread's peer stores and slab reads of the call are done
  if (threadIdx.x == 0) epoch_end(a.epoch_ctr, a.epoch_done, epoch);
}

__global__ void column_sum_kernel(const float* __restrict__ partial, int rows, int cols, float* __restrict__ out) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float s = 0.f;
  for (int r = 0; r < rows; ++r) s += partial[(size_t)r * cols + c];
  out[c] = s;
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


namespace {

// Vocabulary-parallel cross-entropy statistics, combined over TP in one kernel: per 64-row block
// the LM-head GEMM's per-tile (max, sum exp) partials are merged (one warp per row), this rank's
// (max, sum exp, target logit) triples are stored into slot `rank` of every peer's statistics slab
// (three floats per row), a per-block flag is released to every peer, and after acquiring the
// peers' flags (bounded wait, status 300 + peer) each row's log-sum-exp over the full vocabulary and
// its target logit are formed from the tp triples. Persistent grid, blocks in the same order on
// every rank.
__global__ void __launch_bounds__(256) ce_combine_tp_kernel(const float2* __restrict__ part, int tiles,
                                                            const float* __restrict__ tgt_local, int rows,
                                                            float* __restrict__ lse_out, float* __restrict__ tgt_out,
                                                            float* const* peer_recv_even, const float* my_recv_even,
                                                            long long* const* peer_flags, const long long* my_flags,
                                                            int rank, int tp, int max_rows, long long host_epoch,
                                                            int* status, long long* epoch_ctr, unsigned* epoch_done,
                                                            float* const* peer_recv_odd, const float* my_recv_odd) {
  __shared__ float trip[STAT_ROWS][3];
  __shared__ int failed;
  __shared__ long long s_epoch;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int blocks = (rows + STAT_ROWS - 1) / STAT_ROWS;
  auto merge = [](float& m, float& s, float om, float os) {
    const float nm = fmaxf(m, om);
    if (nm == -INFINITY) return;
    s = s * __expf(m - nm) + os * __expf(om - nm);
    m = nm;
  };
  if (threadIdx.x == 0) {
    failed = 0;
    s_epoch = epoch_begin(epoch_ctr, host_epoch);
  }
  __syncthreads();
  const long long epoch = s_epoch;
  const bool odd = (epoch & 1) && peer_recv_odd;
  float* const* peer_recv = odd ? peer_recv_odd : peer_recv_even;
  const float* my_recv = odd ? my_recv_odd : my_recv_even;
  for (int b = blockIdx.x; b < blocks; b += gridDim.x) {
    for (int rr = 0; rr < STAT_ROWS / 8; ++rr) {
      const int lr = warp * (STAT_ROWS / 8) + rr, row = b * STAT_ROWS + lr;
      float m = -INFINITY, sum = 0.f;
      if (row < rows) {
        for (int t = lane; t < tiles; t += 32) {
          const float2 p = part[(size_t)row * tiles + t];
          merge(m, sum, p.x, p.y);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float om = __shfl_xor_sync(0xffffffffu, m, o), os = __shfl_xor_sync(0xffffffffu, sum, o);
        merge(m, sum, om, os);
      }
      if (lane == 0) {
        trip[lr][0] = m;
        trip[lr][1] = sum;
        trip[lr][2] = row < rows ? tgt_local[row] : 0.f;
      }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < STAT_ROWS * tp; i += blockDim.x) {
      const int t = i / STAT_ROWS, lr = i % STAT_ROWS;
      float* dst = peer_recv[t] + (size_t)rank * max_rows + 3 * (size_t)(b * STAT_ROWS + lr);
      dst[0] = trip[lr][0];
      dst[1] = trip[lr][1];
      dst[2] = trip[lr][2];
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < tp) st_release_sys(peer_flags[threadIdx.x] + (size_t)b * STAT_MAX_TP + rank, epoch);
    if (threadIdx.x < tp) {
      const long long* f = my_flags + (size_t)b * STAT_MAX_TP + threadIdx.x;
      const unsigned long long start = tc::globaltimer();
      while (ld_acquire_sys(f) < epoch) {
        if (tc::globaltimer() - start > tc::kWaitNs) {
          atomicCAS(status, 0, 300 + threadIdx.x);
          failed = 1;
          break;
        }
      }
    }
    __syncthreads();
    if (failed) break;   // the host reads the status word; outputs of this call are invalid
    if (threadIdx.x < STAT_ROWS) {
      const int row = b * STAT_ROWS + threadIdx.x;
      float m = -INFINITY, sum = 0.f, tg = 0.f;
      for (int t = 0; t < tp; ++t) {
        const float* src = my_recv + (size_t)t * max_rows + 3 * (size_t)row;
        merge(m, sum, src[0], src[1]);
        tg += src[2];
      }
      if (row < rows) {
        lse_out[row] = m + __logf(sum);
        tgt_out[row] = tg;
      }
    }
    __syncthreads();   // trip[] is rewritten by the next block
  }
  if (threadIdx.x == 0) epoch_end(epoch_ctr, epoch_done, epoch);
}

}  // namespace

// part: [rows, tiles] float2 from the LM-head GEMM (epilogue 3); tgt_local [rows]; returns the
// full-vocabulary (lse, target logit) per row. The exchange uses three floats per row of the
// statistics slab, so 3 * rows <= max_rows.
std::vector<at::Tensor> ce_combine_tp(at::Tensor part, at::Tensor tgt_local, at::Tensor peer_recv, int64_t my_recv,
                                      at::Tensor peer_flags, int64_t my_flags, int64_t rank, int64_t tp,
                                      int64_t max_rows, int64_t epoch, int64_t epoch_ctr, int64_t epoch_done,
                                      c10::optional<at::Tensor> peer_recv_odd, int64_t my_recv_odd) {
  TORCH_CHECK(part.is_cuda() && part.scalar_type() == at::kFloat && part.dim() == 3 && part.size(2) == 2 &&
                  part.is_contiguous(),
              "part: fp32 [rows, tiles, 2]");
  const int64_t rows = part.size(0);
  TORCH_CHECK(tgt_local.scalar_type() == at::kFloat && tgt_local.numel() == rows && tgt_local.is_contiguous(),
              "tgt_local: fp32 [rows]");
  TORCH_CHECK(tp >= 1 && tp <= STAT_MAX_TP && 3 * rows <= max_rows, "rows exceed the exchange slab");
  auto lse = at::empty({rows}, part.options()), tgt = at::empty({rows}, part.options());
  if (!rows) return {lse, tgt};
  TORCH_CHECK(!epoch_ctr || (epoch_done && my_recv_odd && peer_recv_odd && peer_recv_odd->numel() == tp),
              "ce_combine_tp: device epochs need the done counter and the odd-parity slabs");
  const int grid = std::max(1, std::min((int)((rows + STAT_ROWS - 1) / STAT_ROWS), sm_count()));
  ce_combine_tp_kernel<<<grid, 256, 0, stream()>>>(
      reinterpret_cast<const float2*>(part.data_ptr<float>()), (int)part.size(1), tgt_local.data_ptr<float>(),
      (int)rows, lse.data_ptr<float>(), tgt.data_ptr<float>(), reinterpret_cast<float* const*>(peer_recv.data_ptr()),
      reinterpret_cast<const float*>(my_recv), reinterpret_cast<long long* const*>(peer_flags.data_ptr()),
      reinterpret_cast<const long long*>(my_flags), (int)rank, (int)tp, (int)max_rows, epoch, comm_status(),
      reinterpret_cast<long long*>(epoch_ctr), reinterpret_cast<unsigned*>(epoch_done),
      epoch_ctr ? reinterpret_cast<float* const*>(peer_recv_odd->data_ptr()) : nullptr,
      reinterpret_cast<const float*>(my_recv_odd));
  CQB_LAUNCH_CHECK();
  count_launch();
  return {lse, tgt};
}

namespace {
TpNormArgs tp_norm_args(const at::Tensor& x, const at::Tensor& w, at::Tensor peer_recv, int64_t my_recv,
                        at::Tensor peer_flags, int64_t my_flags, int64_t rank, int64_t tp, int64_t max_rows,
                        int64_t epoch, int64_t total_dim, double eps, int64_t epoch_ctr, int64_t epoch_done,
                        const c10::optional<at::Tensor>& peer_recv_odd, int64_t my_recv_odd) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1 &&
                  x.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
              "x: bf16 [rows, D] with 16-byte aligned rows");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous() && w.numel() == x.size(1), "w: fp32 [D]");
  TORCH_CHECK(x.size(1) % 8 == 0 && x.size(1) <= 1024, "D must be a multiple of 8 and <= 1024");
  TORCH_CHECK(tp >= 1 && tp <= STAT_MAX_TP && x.size(0) <= max_rows, "rows exceed the exchange slab");
  TpNormArgs a{};
  a.x = (const __nv_bfloat16*)x.data_ptr();
  a.ld_x = (int)x.stride(0);
  a.w = w.data_ptr<float>();
  a.rows = (int)x.size(0);
  a.D = (int)x.size(1);
  a.inv_total = 1.f / (float)total_dim;
  a.eps = (float)eps;
  a.peer_recv = reinterpret_cast<float* const*>(peer_recv.data_ptr());
  a.my_recv = reinterpret_cast<float*>(my_recv);
  a.peer_flags = reinterpret_cast<long long* const*>(peer_flags.data_ptr());
  a.my_flags = reinterpret_cast<long long*>(my_flags);
  a.rank = (int)rank;
  a.tp = (int)tp;
  a.max_rows = (int)max_rows;
  a.epoch = epoch;
  a.status = comm_status();
  if (epoch_ctr) {
    TORCH_CHECK(epoch_done && my_recv_odd && peer_recv_odd && peer_recv_odd->numel() == tp,
                "tp_rms: device epochs need the done counter and the odd-parity slabs");
    a.epoch_ctr = reinterpret_cast<long long*>(epoch_ctr);
    a.epoch_done = reinterpret_cast<unsigned*>(epoch_done);
    a.peer_recv_odd = reinterpret_cast<float* const*>(peer_recv_odd->data_ptr());
    a.my_recv_odd = reinterpret_cast<float*>(my_recv_odd);
  }
  return a;
}
int tp_norm_grid(int rows) { return std::max(1, std::min((rows + STAT_ROWS - 1) / STAT_ROWS, sm_count())); }
}  // namespace

// y = x * rsqrt(sum_over_ranks(x^2) / total_dim + eps) * w; returns (y, rstd).
std::vector<at::Tensor> tp_rms_fwd(at::Tensor x, at::Tensor w, at::Tensor peer_recv, int64_t my_recv,
                                   at::Tensor peer_flags, int64_t my_flags, int64_t rank, int64_t tp, int64_t max_rows,
                                   int64_t epoch, int64_t total_dim, double eps, int64_t epoch_ctr,
                                   int64_t epoch_done, c10::optional<at::Tensor> peer_recv_odd, int64_t my_recv_odd) {
  auto a = tp_norm_args(x, w, peer_recv, my_recv, peer_flags, my_flags, rank, tp, max_rows, epoch, total_dim, eps,
                        epoch_ctr, epoch_done, peer_recv_odd, my_recv_odd);
  auto y = at::empty({x.size(0), x.size(1)}, x.options());
  auto rstd = at::empty({x.size(0)}, x.options().dtype(at::kFloat));
  a.y = (__nv_bfloat16*)y.data_ptr();
  a.rstd = rstd.data_ptr<float>();
  if (a.rows) {
    tp_norm_kernel<false><<<tp_norm_grid(a.rows), 256, 0, stream()>>>(a);
    CQB_LAUNCH_CHECK();
    count_launch();
  }
  return {y, rstd};
}

// Backward: returns (dx, dw fp32 [D]); the row dot products dy.w.x are summed over ranks.
std::vector<at::Tensor> tp_rms_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd, at::Tensor peer_recv,
                                   int64_t my_recv, at::Tensor peer_flags, int64_t my_flags, int64_t rank, int64_t tp,
                                   int64_t max_rows, int64_t epoch, int64_t total_dim, int64_t epoch_ctr,
                                   int64_t epoch_done, c10::optional<at::Tensor> peer_recv_odd, int64_t my_recv_odd) {
  auto a = tp_norm_args(x, w, peer_recv, my_recv, peer_flags, my_flags, rank, tp, max_rows, epoch, total_dim, 0.0,
                        epoch_ctr, epoch_done, peer_recv_odd, my_recv_odd);
  auto dyc = dy.contiguous();
  TORCH_CHECK(dyc.scalar_type() == at::kBFloat16 && dyc.sizes() == x.sizes(), "dy like x");
  TORCH_CHECK(rstd.scalar_type() == at::kFloat && rstd.numel() == x.size(0), "rstd: fp32 [rows]");
  auto dx = at::empty({x.size(0), x.size(1)}, x.options());
  auto dw = at::zeros({x.size(1)}, x.options().dtype(at::kFloat));
  if (!a.rows) return {dx, dw};
  const int grid = tp_norm_grid(a.rows);
  auto partial = at::empty({grid, x.size(1)}, dw.options());
  a.dy = (const __nv_bfloat16*)dyc.data_ptr();
  a.y = (__nv_bfloat16*)dx.data_ptr();
  a.rstd = rstd.data_ptr<float>();
  a.dw_partial = partial.data_ptr<float>();
  tp_norm_kernel<true><<<grid, 256, 0, stream()>>>(a);
  CQB_LAUNCH_CHECK();
  column_sum_kernel<<<(a.D + 255) / 256, 256, 0, stream()>>>(partial.data_ptr<float>(), grid, a.D, dw.data_ptr<float>());
  CQB_LAUNCH_CHECK();
  count_launch(2);
  return {dx, dw};
}

int comm_status_read(bool reset) {
  int v = 0;
  CQB_CHECK_CUDA(cudaMemcpy(&v, comm_status(), sizeof(int), cudaMemcpyDeviceToHost));
  if (reset && v) CQB_CHECK_CUDA(cudaMemset(comm_status(), 0, sizeof(int)));
  return v;
}

}  // namespace cqb
