// Row gathers of the CQ event streams and their atomic-free backward.
//
// gather: out[i] = src0[idx[i]] if idx[i] < n0, src1[idx[i] - n0] if idx[i] < n0 + n1, else 0
//   (a sentinel index reads zeros, so callers never append a zero row, and two sources --
//   e.g. content and query conv outputs -- need no concatenation).
// backward: with the host-built inverse levels inv[l][j] = l-th output row that read source row
//   j (or m = rows of the output when there is none), d_src[j] = sum_l grad[inv[l][j]]; a warp per
//   source row sums the levels in fp32 and writes the gradient once (deterministic).
#include "common.cuh"

namespace cqb {

namespace {

template <typename T>
__global__ void gather_rows_kernel(const T* __restrict__ src0, long n0, long ld0, const T* __restrict__ src1, long n1,
                                   long ld1, const long* __restrict__ idx, T* __restrict__ out, long m, int width) {
  const int vecs = width * (int)sizeof(T) / 16;
  const long warp = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  for (long i = warp; i < m; i += ((long)gridDim.x * blockDim.x) >> 5) {
    const long s = idx[i];
    const uint4* from = nullptr;
    if (!CQB_IN_RANGE(s, n0 + n1 + 1, 1)) {   // valid: a source row or the zero sentinel n0 + n1
    } else if (s < n0) from = reinterpret_cast<const uint4*>(src0 + s * ld0);
    else if (s < n0 + n1) from = reinterpret_cast<const uint4*>(src1 + (s - n0) * ld1);
    uint4* to = reinterpret_cast<uint4*>(out + i * width);
    for (int v = lane; v < vecs; v += 32) to[v] = from ? __ldg(from + v) : make_uint4(0, 0, 0, 0);
  }
}

__device__ __forceinline__ void load_any(const __nv_bfloat16* p, float* v) { load8(p, v); }
__device__ __forceinline__ void load_any(const float* p, float* v) { load8(p, v); }

template <typename T>
__global__ void gather_rows_bwd_kernel(const T* __restrict__ grad, long m, const long* __restrict__ inv, int levels,
                                       long inv_stride, T* __restrict__ out0, long n0, T* __restrict__ out1, long total,
                                       int width) {
  const long warp = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  for (long j = warp; j < total; j += ((long)gridDim.x * blockDim.x) >> 5) {
    T* dst = j < n0 ? out0 + j * width : out1 + (j - n0) * width;
    for (int c = lane * 8; c < width; c += 256) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int l = 0; l < levels; ++l) {
        const long r = inv[(long)l * inv_stride + j];
        if (!CQB_IN_RANGE(r, m + 1, 2) || r >= m) continue;   // r == m: no reader at this level
        float v[8];
        load_any(grad + r * width + c, v);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] += v[q];
      }
      store8(dst + c, acc);
    }
  }
}

// Embedding backward in two deterministic passes (no atomics). `order` lists the token positions
// sorted by id; the sorted list is cut into segments of at most SEG positions that never span two
// ids. Pass 1: one warp per segment sums its rows into partial[seg] (fp32). Pass 2: one warp per
// (id, 256-column slice) adds the id's segment partials in order into out[id]. A repeated id
// (e.g. the mask token of every query row) is thus summed by many warps instead of one.
template <typename T>
__global__ void segment_sum_kernel(const T* __restrict__ grad, const long* __restrict__ order,
                                   const long* __restrict__ seg_start, long segments, long positions,
                                   float* __restrict__ partial, int width) {
  const long warp = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  for (long sg = warp; sg < segments; sg += ((long)gridDim.x * blockDim.x) >> 5) {
    const long k0 = seg_start[sg], k1 = seg_start[sg + 1];
    for (int c = lane * 8; c < width; c += 256) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (long k = k0; k < k1; ++k) {
        const long row = order[k];
        if (!CQB_IN_RANGE(row, positions, 4)) continue;
        float v[8];
        load_any(grad + row * width + c, v);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] += v[q];
      }
      store8(partial + sg * width + c, acc);
    }
  }
}

__global__ void run_accumulate_kernel(const float* __restrict__ partial, const long* __restrict__ run_seg,
                                      const long* __restrict__ ids, long runs, long rows_out,
                                      float* __restrict__ out, int width) {
  const int slices = (width + 255) / 256;
  const long warp = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  for (long w = warp; w < runs * slices; w += ((long)gridDim.x * blockDim.x) >> 5) {
    const long r = w / slices;
    const int c = (int)(w % slices) * 256 + lane * 8;
    const long id = ids[r];
    if (c >= width || id >= rows_out || !CQB_IN_RANGE(id, rows_out, 3)) continue;   // >= rows_out: other shards
    float acc[8];
    load8(out + id * width + c, acc);
    for (long sg = run_seg[r]; sg < run_seg[r + 1]; ++sg) {
      float v[8];
      load8(partial + sg * width + c, v);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += v[q];
    }
    store8(out + id * width + c, acc);
  }
}

int gather_grid(long rows) {
  return (int)std::max<long>(1, std::min<long>((rows * 32 + 255) / 256, (long)sm_count() * 16));
}

}  // namespace

namespace {
// Rows of a source: contiguous inside a row, any row stride (e.g. a column slice of a projection).
long row_stride(const at::Tensor& t, long width) {
  TORCH_CHECK(t.is_cuda() && t.dim() >= 1, "gather_rows: CUDA source");
  if (t.size(0) <= 1) return width;
  auto row = t[0];
  TORCH_CHECK(row.is_contiguous() && row.numel() == width, "gather_rows: each source row must be contiguous");
  return t.stride(0);
}
}  // namespace

// src1 may be undefined (one source). Rows are [width] elements with a row stride; the row bytes,
// the row stride in bytes and the base addresses must be multiples of 16.
at::Tensor gather_rows(at::Tensor src0, c10::optional<at::Tensor> src1_opt, at::Tensor idx) {
  TORCH_CHECK(idx.scalar_type() == at::kLong && idx.is_contiguous(), "gather_rows: int64 index");
  const long n0 = src0.size(0);
  const long width = n0 ? src0.numel() / n0 : 0;
  const long ld0 = row_stride(src0, width);
  at::Tensor src1;
  long n1 = 0, ld1 = width;
  if (src1_opt && src1_opt->defined()) {
    src1 = *src1_opt;
    TORCH_CHECK(src1.scalar_type() == src0.scalar_type() && src1.numel() == src1.size(0) * width,
                "gather_rows: second source must match the first's row shape and dtype");
    n1 = src1.size(0);
    ld1 = row_stride(src1, width);
  }
  const long es = src0.element_size();
  TORCH_CHECK(width * es % 16 == 0 && ld0 * es % 16 == 0 && ld1 * es % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(src0.data_ptr()) % 16 == 0 &&
                  (!n1 || reinterpret_cast<uintptr_t>(src1.data_ptr()) % 16 == 0),
              "gather_rows: rows, strides and bases must be 16-byte aligned");
  auto shape = src0.sizes().vec();
  const long m = idx.numel();
  shape[0] = m;
  auto out = at::empty(shape, src0.options().memory_format(at::MemoryFormat::Contiguous));
  if (!m) return out;
  const int grid = gather_grid(m);
  if (src0.scalar_type() == at::kBFloat16)
    gather_rows_kernel<__nv_bfloat16><<<grid, 256, 0, stream()>>>(
        (const __nv_bfloat16*)src0.data_ptr(), n0, ld0, n1 ? (const __nv_bfloat16*)src1.data_ptr() : nullptr, n1, ld1,
        (const long*)idx.data_ptr(), (__nv_bfloat16*)out.data_ptr(), m, (int)width);
  else if (src0.scalar_type() == at::kFloat)
    gather_rows_kernel<float><<<grid, 256, 0, stream()>>>(src0.data_ptr<float>(), n0, ld0,
                                                          n1 ? src1.data_ptr<float>() : nullptr, n1, ld1,
                                                          (const long*)idx.data_ptr(), out.data_ptr<float>(), m,
                                                          (int)width);
  else
    TORCH_CHECK(false, "gather_rows: bf16 or fp32");
  CQB_LAUNCH_CHECK();
  count_launch();
  return out;
}

// grad [m, ...]; inv [levels, n_src] int64 (values in [0, m], m = none); returns the gradients of the
// first n0 source rows and (n1 > 0) of the next n1 rows; source rows past n0 + n1 (sentinels) are
// dropped.
std::vector<at::Tensor> gather_rows_bwd(at::Tensor grad, at::Tensor inv, int64_t n0, int64_t n1) {
  TORCH_CHECK(grad.is_cuda() && grad.is_contiguous(), "gather_rows_bwd: contiguous grad");
  TORCH_CHECK(inv.scalar_type() == at::kLong && inv.is_contiguous() && inv.dim() == 2, "inv: int64 [levels, n_src]");
  const long m = grad.size(0);
  const int width = (int)(grad.numel() / std::max<long>(m, 1));
  TORCH_CHECK(width % 8 == 0, "gather_rows_bwd: row width must be a multiple of 8 elements");
  const long n_src = inv.size(1);
  TORCH_CHECK(n0 + n1 <= n_src, "inverse map smaller than the sources");
  auto s0 = grad.sizes().vec();
  s0[0] = n0;
  auto out0 = at::empty(s0, grad.options());
  at::Tensor out1;
  if (n1) {
    auto s1 = grad.sizes().vec();
    s1[0] = n1;
    out1 = at::empty(s1, grad.options());
  }
  const int levels = (int)inv.size(0);
  if (!levels || !m) {
    out0.zero_();
    if (n1) out1.zero_();
    return n1 ? std::vector<at::Tensor>{out0, out1} : std::vector<at::Tensor>{out0};
  }
  const int grid = gather_grid(n0 + n1);
  if (grad.scalar_type() == at::kBFloat16)
    gather_rows_bwd_kernel<__nv_bfloat16><<<grid, 256, 0, stream()>>>(
        (const __nv_bfloat16*)grad.data_ptr(), m, (const long*)inv.data_ptr(), levels, n_src,
        (__nv_bfloat16*)out0.data_ptr(), n0, n1 ? (__nv_bfloat16*)out1.data_ptr() : nullptr, n0 + n1, width);
  else if (grad.scalar_type() == at::kFloat)
    gather_rows_bwd_kernel<float><<<grid, 256, 0, stream()>>>(grad.data_ptr<float>(), m, (const long*)inv.data_ptr(),
                                                              levels, n_src, out0.data_ptr<float>(), n0,
                                                              n1 ? out1.data_ptr<float>() : nullptr, n0 + n1, width);
  else
    TORCH_CHECK(false, "gather_rows_bwd: bf16 or fp32");
  CQB_LAUNCH_CHECK();
  count_launch();
  return n1 ? std::vector<at::Tensor>{out0, out1} : std::vector<at::Tensor>{out0};
}

// out fp32 [rows_out, width] += per-id sums of grad rows: order (positions sorted by id),
// seg_start [segments + 1] (segment boundaries in `order`), run_seg [runs + 1] (first segment of
// every id), ids [runs] (see segment_sum_kernel / run_accumulate_kernel).
void rows_accumulate(at::Tensor grad, at::Tensor order, at::Tensor seg_start, at::Tensor run_seg, at::Tensor ids,
                     at::Tensor out) {
  TORCH_CHECK(grad.is_cuda() && grad.dim() == 2 && grad.is_contiguous() && grad.size(1) % 8 == 0,
              "rows_accumulate: contiguous [m, width] grad, width a multiple of 8");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous() && out.dim() == 2 && out.size(1) == grad.size(1),
              "rows_accumulate: fp32 [rows, width] output");
  for (auto* t : {&order, &seg_start, &run_seg, &ids})
    TORCH_CHECK(t->scalar_type() == at::kLong && t->is_contiguous() && t->is_cuda(), "rows_accumulate: int64 indices");
  const long runs = ids.numel(), segments = seg_start.numel() - 1;
  TORCH_CHECK(run_seg.numel() == runs + 1 && segments >= 0, "rows_accumulate: segment tables");
  if (!runs) return;
  const int width = (int)grad.size(1);
  auto partial = at::empty({std::max<long>(segments, 1), width}, out.options());
  if (grad.scalar_type() == at::kBFloat16)
    segment_sum_kernel<__nv_bfloat16><<<gather_grid(segments), 256, 0, stream()>>>(
        (const __nv_bfloat16*)grad.data_ptr(), order.data_ptr<int64_t>(), seg_start.data_ptr<int64_t>(), segments,
        grad.size(0), partial.data_ptr<float>(), width);
  else
    segment_sum_kernel<float><<<gather_grid(segments), 256, 0, stream()>>>(
        grad.data_ptr<float>(), order.data_ptr<int64_t>(), seg_start.data_ptr<int64_t>(), segments, grad.size(0),
        partial.data_ptr<float>(), width);
  CQB_LAUNCH_CHECK();
  const long work = runs * ((width + 255) / 256);
  run_accumulate_kernel<<<gather_grid(work), 256, 0, stream()>>>(partial.data_ptr<float>(), run_seg.data_ptr<int64_t>(),
                                                               ids.data_ptr<int64_t>(), runs, out.size(0),
                                                               out.data_ptr<float>(), width);
  CQB_LAUNCH_CHECK();
  count_launch(2);
}

#ifdef CQB_DEBUG_BOUNDS
CQB_DEBUG_STATUS_READER(debug_status_gather)
#endif

}  // namespace cqb
