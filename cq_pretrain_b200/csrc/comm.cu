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
// is persistent (every CTA resident at once, sized by the kernel's occupancy) and every rank
// walks the blocks in the same order.
//
// One launch normalises up to two tensors of the same geometry (Wan's q and k: blockIdx.y picks
// the tensor; tensor t uses slab rows [t * 64 * blocks, (t + 1) * 64 * blocks) and flag blocks
// [t * blocks, (t + 1) * blocks)). With `cos` set, the Wan complex-pair RoPE of head size `hd` is
// applied to the normalised row in the forward, and the backward first rotates dy back (the
// rotation by -angle) before the norm backward. Without `exchange` the partials are this rank's
// own (TP = 1): no peer stores, flags or waits.
constexpr int STAT_ROWS = 64;          // rows per block
constexpr int STAT_MAX_TP = 8;

struct TpNormArgs {
  const __nv_bfloat16* x[2];
  int ld_x[2];
  const __nv_bfloat16* dy[2];   // backward only (contiguous [rows, D])
  const float* w[2];            // [D] fp32
  __nv_bfloat16* y[2];          // fwd: y; bwd: dx (contiguous [rows, D])
  float* rstd[2];               // [rows]
  float* dw_partial[2];         // bwd: [gridDim.x, D]
  int rows, D;
  float inv_total, eps;
  const float* cos;             // [rows, hd / 2] (RoPE after the norm) or null
  const float* sin;
  int hd;
  bool exchange;
  float* const* peer_recv;      // [tp] slab base of each peer (even epochs): [tp][max_rows] fp32
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

// (v[2p], v[2p+1]) rotated by sign * angle_p for the four pairs of columns c..c+7 of `row`.
__device__ __forceinline__ void rope_rotate8(float* v, const float* cos_t, const float* sin_t, int hd, int row, int c,
                                             float sign) {
  const int half = hd / 2, i0 = (c % hd) / 2;
  const float4 cv = *reinterpret_cast<const float4*>(cos_t + (size_t)row * half + i0);
  const float4 sv = *reinterpret_cast<const float4*>(sin_t + (size_t)row * half + i0);
  const float cs[4] = {cv.x, cv.y, cv.z, cv.w}, sn[4] = {sign * sv.x, sign * sv.y, sign * sv.z, sign * sv.w};
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const float re = v[2 * p], im = v[2 * p + 1];
    v[2 * p] = re * cs[p] - im * sn[p];
    v[2 * p + 1] = im * cs[p] + re * sn[p];
  }
}

// NCH: 8-column chunks per lane (D <= NCH * 256).
template <bool BWD, int NCH>
__global__ void __launch_bounds__(256) tp_norm_kernel(TpNormArgs a) {
  __shared__ float part[STAT_ROWS];
  __shared__ float stat[STAT_ROWS];
  __shared__ int failed;
  __shared__ long long s_epoch;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.y;
  const int blocks = (a.rows + STAT_ROWS - 1) / STAT_ROWS;
  const __nv_bfloat16* __restrict__ x = a.x[t];
  const __nv_bfloat16* __restrict__ dyp = a.dy[t];
  const float* __restrict__ w = a.w[t];
  const int ld_x = a.ld_x[t];
  const bool rope = a.cos != nullptr;
  float dw_acc[NCH][8];
  if (BWD) {
#pragma unroll
    for (int i = 0; i < NCH; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) dw_acc[i][j] = 0.f;
  }
  if (threadIdx.x == 0) {
    failed = 0;
    s_epoch = a.exchange ? epoch_begin(a.epoch_ctr, a.epoch) : 0;
  }
  __syncthreads();
  const long long epoch = s_epoch;
  const bool odd = (epoch & 1) && a.peer_recv_odd;
  float* const* peer_recv = odd ? a.peer_recv_odd : a.peer_recv;
  const float* my_recv = odd ? a.my_recv_odd : a.my_recv;
  // this tensor's rows in the slabs, padded to whole blocks: the last block of tensor 0 stores
  // partials for all 64 of its rows, which must not land on tensor 1's first rows
  const size_t slab_row0 = (size_t)t * blocks * STAT_ROWS;
  for (int b = blockIdx.x; b < blocks; b += gridDim.x) {
    // 1) local partials: warp w handles rows 8w..8w+7 of the block; the row loop is innermost and
    // unrolled so a lane has the loads of all eight rows in flight (the pass is latency-bound
    // with one row at a time)
    const int row0 = b * STAT_ROWS + warp * 8;
    const int nrow = min(8, a.rows - row0);
    float acc[8];
#pragma unroll
    for (int rr = 0; rr < 8; ++rr) acc[rr] = 0.f;
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      const int c = lane * 8 + k * 256;
      if (c >= a.D) break;
      float wv[8];
      if (BWD) load8(w + c, wv);
#pragma unroll
      for (int rr = 0; rr < 8; ++rr) {
        if (rr < nrow) {
          const int row = row0 + rr;
          float xv[8];
          load8(x + (size_t)row * ld_x + c, xv);
          if (BWD) {
            float dv[8];
            load8(dyp + (size_t)row * a.D + c, dv);
            if (rope) rope_rotate8(dv, a.cos, a.sin, a.hd, row, c, -1.f);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[rr] += dv[j] * wv[j] * xv[j];
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[rr] += xv[j] * xv[j];
          }
        }
      }
    }
#pragma unroll
    for (int rr = 0; rr < 8; ++rr) {
      const float v = warp_sum(acc[rr]);
      if (lane == 0) part[warp * 8 + rr] = v;
    }
    __syncthreads();
    if (a.exchange) {
      // 2) publish to every peer (including this rank's own slab)
      if (threadIdx.x < STAT_ROWS * a.tp) {
        const int p = threadIdx.x / STAT_ROWS, lr = threadIdx.x % STAT_ROWS;
        peer_recv[p][(size_t)a.rank * a.max_rows + slab_row0 + b * STAT_ROWS + lr] = part[lr];
      }
      __threadfence_system();
      __syncthreads();
      const size_t fb = (size_t)t * blocks + b;   // flag block
      if (threadIdx.x < a.tp) st_release_sys(a.peer_flags[threadIdx.x] + fb * STAT_MAX_TP + a.rank, epoch);
      // 3) acquire the peers' partials of this block
      if (threadIdx.x < a.tp) {
        const long long* f = a.my_flags + fb * STAT_MAX_TP + threadIdx.x;
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
        for (int p = 0; p < a.tp; ++p)
          sum += my_recv[(size_t)p * a.max_rows + slab_row0 + b * STAT_ROWS + threadIdx.x];
        stat[threadIdx.x] = sum;
      }
    } else if (threadIdx.x < STAT_ROWS) {
      stat[threadIdx.x] = part[threadIdx.x];
    }
    __syncthreads();
    // 4) finish the rows (chunk outer, the warp's rows inner and unrolled, as in 1)
    float rr_r[8], rr_g[8];
#pragma unroll
    for (int rr = 0; rr < 8; ++rr) {
      const int lr = warp * 8 + rr;
      rr_r[rr] = rr_g[rr] = 0.f;
      if (rr < nrow) {
        if (!BWD) {
          rr_r[rr] = rsqrtf(stat[lr] * a.inv_total + a.eps);
          if (lane == 0) a.rstd[t][row0 + rr] = rr_r[rr];
        } else {
          rr_r[rr] = a.rstd[t][row0 + rr];
          rr_g[rr] = stat[lr] * rr_r[rr] * rr_r[rr] * rr_r[rr] * a.inv_total;
        }
      }
    }
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      const int c = lane * 8 + k * 256;
      if (c >= a.D) break;
      float wv[8];
      load8(w + c, wv);
#pragma unroll
      for (int rr = 0; rr < 8; ++rr) {
        if (rr < nrow) {
          const int row = row0 + rr;
          const float r = rr_r[rr];
          float xv[8], o[8];
          load8(x + (size_t)row * ld_x + c, xv);
          if (!BWD) {
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = xv[j] * r * wv[j];
            if (rope) rope_rotate8(o, a.cos, a.sin, a.hd, row, c, 1.f);
          } else {
            float dv[8];
            load8(dyp + (size_t)row * a.D + c, dv);
            if (rope) rope_rotate8(dv, a.cos, a.sin, a.hd, row, c, -1.f);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              o[j] = dv[j] * wv[j] * r - xv[j] * rr_g[rr];
              dw_acc[k][j] += dv[j] * xv[j] * r;
            }
          }
          store8(a.y[t] + (size_t)row * a.D + c, o);
        }
      }
    }
    __syncthreads();   // part/stat reused by the next block
  }
  if (BWD) {
    // dw partial of this CTA: reduce the 8 warps through shared memory (fixed order), one
    // 256-column chunk at a time
    __shared__ float red[8][256];
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      if (k * 256 >= a.D) break;
#pragma unroll
      for (int j = 0; j < 8; ++j) red[warp][lane * 8 + j] = dw_acc[k][j];
      __syncthreads();
      const int c = k * 256 + threadIdx.x;
      if (c < a.D) {
        float sum = 0.f;
        for (int wi = 0; wi < 8; ++wi) sum += red[wi][threadIdx.x];
        a.dw_partial[t][(size_t)blockIdx.x * a.D + c] = sum;
      }
      __syncthreads();
    }
  }
  __syncthreads();   // every thread's peer stores and slab reads of the call are done
  if (threadIdx.x == 0 && a.exchange) epoch_end(a.epoch_ctr, a.epoch_done, epoch);
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
// statistics slab for every row of its whole 64-row blocks, so 3 * rows rounded up to 64 <= max_rows.
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
  TORCH_CHECK(tp >= 1 && tp <= STAT_MAX_TP && 3 * ((rows + STAT_ROWS - 1) / STAT_ROWS * STAT_ROWS) <= max_rows,
              "rows exceed the exchange slab (whole 64-row blocks)");
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
void check_norm_input(const at::Tensor& x, const at::Tensor& w) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1 &&
                  x.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
              "x: bf16 [rows, D] with 16-byte aligned rows");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous() && w.numel() == x.size(1), "w: fp32 [D]");
  TORCH_CHECK(x.size(1) % 8 == 0 && x.size(1) <= 2048, "D must be a multiple of 8 and <= 2048");
}

// xs / ws: one or two tensors of the same geometry (the launch's blockIdx.y).
TpNormArgs norm_args(const std::vector<at::Tensor>& xs, const std::vector<at::Tensor>& ws, int64_t total_dim,
                     double eps) {
  TpNormArgs a{};
  for (size_t t = 0; t < xs.size(); ++t) {
    check_norm_input(xs[t], ws[t]);
    TORCH_CHECK(xs[t].sizes() == xs[0].sizes(), "normalised tensors must share one geometry");
    a.x[t] = (const __nv_bfloat16*)xs[t].data_ptr();
    a.ld_x[t] = (int)xs[t].stride(0);
    a.w[t] = ws[t].data_ptr<float>();
  }
  a.rows = (int)xs[0].size(0);
  a.D = (int)xs[0].size(1);
  a.inv_total = 1.f / (float)total_dim;
  a.eps = (float)eps;
  a.status = comm_status();
  return a;
}

// The peer exchange (TP > 1): slabs of both parities, flag areas, the device epoch counter.
void set_exchange(TpNormArgs& a, int ntens, const c10::optional<at::Tensor>& peer_recv, int64_t my_recv,
                  const c10::optional<at::Tensor>& peer_flags, int64_t my_flags, int64_t rank, int64_t tp,
                  int64_t max_rows, int64_t epoch, int64_t epoch_ctr, int64_t epoch_done,
                  const c10::optional<at::Tensor>& peer_recv_odd, int64_t my_recv_odd) {
  if (!peer_recv) return;
  TORCH_CHECK(peer_flags && my_recv && my_flags, "the row-statistic exchange needs slabs and flags");
  const int64_t padded = (int64_t)(a.rows + STAT_ROWS - 1) / STAT_ROWS * STAT_ROWS;
  TORCH_CHECK(tp >= 1 && tp <= STAT_MAX_TP && ntens * padded <= max_rows, "rows exceed the exchange slab");
  TORCH_CHECK(peer_recv->is_cuda() && peer_recv->numel() == tp && peer_flags->numel() == tp,
              "peer arrays: cuda int64 [tp]");
  a.exchange = true;
  a.peer_recv = reinterpret_cast<float* const*>(peer_recv->data_ptr());
  a.my_recv = reinterpret_cast<float*>(my_recv);
  a.peer_flags = reinterpret_cast<long long* const*>(peer_flags->data_ptr());
  a.my_flags = reinterpret_cast<long long*>(my_flags);
  a.rank = (int)rank;
  a.tp = (int)tp;
  a.max_rows = (int)max_rows;
  a.epoch = epoch;
  if (epoch_ctr) {
    TORCH_CHECK(epoch_done && my_recv_odd && peer_recv_odd && peer_recv_odd->numel() == tp,
                "tp_rms: device epochs need the done counter and the odd-parity slabs");
    a.epoch_ctr = reinterpret_cast<long long*>(epoch_ctr);
    a.epoch_done = reinterpret_cast<unsigned*>(epoch_done);
    a.peer_recv_odd = reinterpret_cast<float* const*>(peer_recv_odd->data_ptr());
    a.my_recv_odd = reinterpret_cast<float*>(my_recv_odd);
  }
}

void set_rope(TpNormArgs& a, const c10::optional<at::Tensor>& cos_t, const c10::optional<at::Tensor>& sin_t,
              int64_t head_dim) {
  if (!cos_t) return;
  TORCH_CHECK(sin_t && head_dim % 8 == 0 && head_dim > 0 && a.D % head_dim == 0,
              "rope: head_dim a multiple of 8 dividing D");
  TORCH_CHECK(cos_t->scalar_type() == at::kFloat && cos_t->is_contiguous() && sin_t->scalar_type() == at::kFloat &&
                  sin_t->is_contiguous() && cos_t->dim() == 2 && cos_t->size(0) == a.rows &&
                  cos_t->size(1) == head_dim / 2 && sin_t->sizes() == cos_t->sizes(),
              "rope: cos / sin fp32 [rows, head_dim / 2]");
  a.cos = cos_t->data_ptr<float>();
  a.sin = sin_t->data_ptr<float>();
  a.hd = (int)head_dim;
}

// Persistent grid of one tensor's CTAs: every CTA of the launch (ntens tensors) must be resident at
// once, because a block's exchange waits for the peers' CTAs of the same block; the per-SM limit
// comes from the kernel instance's occupancy (registers differ between the variants).
template <bool BWD, int NCH>
int tp_norm_grid(int rows, int ntens) {
  static const int per_sm = [] {
    int n = 0;
    CQB_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, tp_norm_kernel<BWD, NCH>, 256, 0));
    return std::max(1, n);
  }();
  const int blocks = (rows + STAT_ROWS - 1) / STAT_ROWS;
  return std::max(1, std::min(blocks, per_sm * sm_count() / ntens));
}

// Forward of one or two tensors: returns (y per tensor, rstd [ntens, rows]).
std::vector<at::Tensor> norm_fwd(TpNormArgs& a, int ntens, const at::TensorOptions& opts) {
  auto rstd = at::empty({ntens, a.rows}, opts.dtype(at::kFloat));
  std::vector<at::Tensor> out;
  for (int t = 0; t < ntens; ++t) {
    out.push_back(at::empty({a.rows, a.D}, opts));
    a.y[t] = (__nv_bfloat16*)out.back().data_ptr();
    a.rstd[t] = rstd.data_ptr<float>() + (size_t)t * a.rows;
  }
  if (a.rows) {
    if (a.D <= 1024)
      tp_norm_kernel<false, 4><<<dim3(tp_norm_grid<false, 4>(a.rows, ntens), ntens), 256, 0, stream()>>>(a);
    else
      tp_norm_kernel<false, 8><<<dim3(tp_norm_grid<false, 8>(a.rows, ntens), ntens), 256, 0, stream()>>>(a);
    CQB_LAUNCH_CHECK();
    count_launch();
  }
  out.push_back(rstd);
  return out;
}

// Backward: returns (dx per tensor, dw fp32 [D] per tensor).
std::vector<at::Tensor> norm_bwd(TpNormArgs& a, int ntens, const std::vector<at::Tensor>& dys, const at::Tensor& rstd,
                                 const at::TensorOptions& opts) {
  TORCH_CHECK(rstd.scalar_type() == at::kFloat && rstd.is_contiguous() && rstd.numel() == (int64_t)ntens * a.rows,
              "rstd: fp32 [ntens, rows]");
  std::vector<at::Tensor> dx, dw, keep;
  const int grid = a.D <= 1024 ? tp_norm_grid<true, 4>(a.rows, ntens) : tp_norm_grid<true, 8>(a.rows, ntens);
  for (int t = 0; t < ntens; ++t) {
    auto dyc = dys[t].contiguous();
    TORCH_CHECK(dyc.scalar_type() == at::kBFloat16 && dyc.numel() == (int64_t)a.rows * a.D, "dy like x");
    keep.push_back(dyc);
    dx.push_back(at::empty({a.rows, a.D}, opts));
    dw.push_back(at::zeros({a.D}, opts.dtype(at::kFloat)));
    a.dy[t] = (const __nv_bfloat16*)dyc.data_ptr();
    a.y[t] = (__nv_bfloat16*)dx.back().data_ptr();
    a.rstd[t] = const_cast<float*>(rstd.data_ptr<float>()) + (size_t)t * a.rows;
  }
  if (a.rows) {
    auto partial = at::empty({ntens, grid, a.D}, opts.dtype(at::kFloat));
    for (int t = 0; t < ntens; ++t) a.dw_partial[t] = partial.data_ptr<float>() + (size_t)t * grid * a.D;
    if (a.D <= 1024)
      tp_norm_kernel<true, 4><<<dim3(grid, ntens), 256, 0, stream()>>>(a);
    else
      tp_norm_kernel<true, 8><<<dim3(grid, ntens), 256, 0, stream()>>>(a);
    CQB_LAUNCH_CHECK();
    for (int t = 0; t < ntens; ++t) {
      column_sum_kernel<<<(a.D + 255) / 256, 256, 0, stream()>>>(a.dw_partial[t], grid, a.D, dw[t].data_ptr<float>());
      CQB_LAUNCH_CHECK();
    }
    count_launch(1 + ntens);
  }
  for (auto& t : dw) dx.push_back(t);
  return dx;
}
}  // namespace

// y = x * rsqrt(sum_over_ranks(x^2) / total_dim + eps) * w; returns (y, rstd).
std::vector<at::Tensor> tp_rms_fwd(at::Tensor x, at::Tensor w, at::Tensor peer_recv, int64_t my_recv,
                                   at::Tensor peer_flags, int64_t my_flags, int64_t rank, int64_t tp, int64_t max_rows,
                                   int64_t epoch, int64_t total_dim, double eps, int64_t epoch_ctr,
                                   int64_t epoch_done, c10::optional<at::Tensor> peer_recv_odd, int64_t my_recv_odd) {
  auto a = norm_args({x}, {w}, total_dim, eps);
  set_exchange(a, 1, peer_recv, my_recv, peer_flags, my_flags, rank, tp, max_rows, epoch, epoch_ctr, epoch_done,
               peer_recv_odd, my_recv_odd);
  auto out = norm_fwd(a, 1, x.options());
  return {out[0], out[1].view({-1})};
}

// Backward: returns (dx, dw fp32 [D]); the row dot products dy.w.x are summed over ranks.
std::vector<at::Tensor> tp_rms_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd, at::Tensor peer_recv,
                                   int64_t my_recv, at::Tensor peer_flags, int64_t my_flags, int64_t rank, int64_t tp,
                                   int64_t max_rows, int64_t epoch, int64_t total_dim, int64_t epoch_ctr,
                                   int64_t epoch_done, c10::optional<at::Tensor> peer_recv_odd, int64_t my_recv_odd) {
  auto a = norm_args({x}, {w}, total_dim, 0.0);
  set_exchange(a, 1, peer_recv, my_recv, peer_flags, my_flags, rank, tp, max_rows, epoch, epoch_ctr, epoch_done,
               peer_recv_odd, my_recv_odd);
  TORCH_CHECK(dy.sizes() == x.sizes(), "dy like x");
  return norm_bwd(a, 1, {dy}, rstd.contiguous(), x.options());
}

// Wan self-attention q / k: full-width RMSNorm of both (the per-row sums exchanged over the TP
// group when `peer_recv` is given) followed by the complex-pair RoPE (when `cos` is given), one
// launch. Returns (q_out, k_out, rstd [2, rows]).
std::vector<at::Tensor> qk_norm_rope_fwd(at::Tensor q, at::Tensor k, at::Tensor wq, at::Tensor wk,
                                         c10::optional<at::Tensor> cos_t, c10::optional<at::Tensor> sin_t,
                                         int64_t head_dim, int64_t total_dim, double eps,
                                         c10::optional<at::Tensor> peer_recv, int64_t my_recv,
                                         c10::optional<at::Tensor> peer_flags, int64_t my_flags, int64_t rank,
                                         int64_t tp, int64_t max_rows, int64_t epoch_ctr, int64_t epoch_done,
                                         c10::optional<at::Tensor> peer_recv_odd, int64_t my_recv_odd) {
  auto a = norm_args({q, k}, {wq, wk}, total_dim, eps);
  set_rope(a, cos_t, sin_t, head_dim);
  set_exchange(a, 2, peer_recv, my_recv, peer_flags, my_flags, rank, tp, max_rows, 0, epoch_ctr, epoch_done,
               peer_recv_odd, my_recv_odd);
  return norm_fwd(a, 2, q.options());
}

// Backward of qk_norm_rope_fwd: (dq, dk, dwq, dwk) from the gradients of its two outputs.
std::vector<at::Tensor> qk_norm_rope_bwd(at::Tensor dyq, at::Tensor dyk, at::Tensor q, at::Tensor k, at::Tensor wq,
                                         at::Tensor wk, at::Tensor rstd, c10::optional<at::Tensor> cos_t,
                                         c10::optional<at::Tensor> sin_t, int64_t head_dim, int64_t total_dim,
                                         c10::optional<at::Tensor> peer_recv, int64_t my_recv,
                                         c10::optional<at::Tensor> peer_flags, int64_t my_flags, int64_t rank,
                                         int64_t tp, int64_t max_rows, int64_t epoch_ctr, int64_t epoch_done,
                                         c10::optional<at::Tensor> peer_recv_odd, int64_t my_recv_odd) {
  auto a = norm_args({q, k}, {wq, wk}, total_dim, 0.0);
  set_rope(a, cos_t, sin_t, head_dim);
  set_exchange(a, 2, peer_recv, my_recv, peer_flags, my_flags, rank, tp, max_rows, 0, epoch_ctr, epoch_done,
               peer_recv_odd, my_recv_odd);
  return norm_bwd(a, 2, {dyq, dyk}, rstd.contiguous(), q.options());
}

int comm_status_read(bool reset) {
  int v = 0;
  CQB_CHECK_CUDA(cudaMemcpy(&v, comm_status(), sizeof(int), cudaMemcpyDeviceToHost));
  if (reset && v) CQB_CHECK_CUDA(cudaMemset(comm_status(), 0, sizeof(int)));
  return v;
}

}  // namespace cqb
