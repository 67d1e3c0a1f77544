// Causal depthwise short convolution + SiLU over packed documents (GDN q/k/v mixing), and the
// GDN chunk-layout gathers.
//
//  conv:   y[t, c] = silu( sum_i w[c, i] * x[t - (K-1) + i, c] ),  taps before the row's
//          document start read zero (pos[t] = index of row t inside its document);
//  bwd:    g = dy * silu'(pre);  dx[t, c] = sum_s w[c, K-1-s] g[t+s, c] (same document);
//          dw[c, i] = sum_t g[t, c] x[t-(K-1)+i, c]  (per-block partials, summed in a fixed order).
//  chunks: rows of [E, H, D] events are gathered into the zero-padded chunk layout
//          [Nc, H, 64, D], optionally L2-normalised on the way (rsqrt norms saved), and
//          scattered back (with the L2-norm backward fused).
#include "noalloc.h"
#include "common.cuh"

#include <cstdio>
#include <mutex>

namespace cqb {

namespace {

// Block (32, 8): x -> 8-channel vector (256 channels per block), y -> row group of ROWS rows.
// Taps come from a register window of the previous 3 rows, so every x row is read once per
// thread (plus a 3-row halo); the transposed fp32 weight wT [4, C] is read once per thread.
constexpr int CONV_K = 4;
constexpr int CONV_ROWS = 32;
constexpr int CONV_GROUPS = 8;

struct ConvTaps {
  float w[CONV_K][8];
  __device__ __forceinline__ void load(const float* __restrict__ wT, int c, int C) {
#pragma unroll
    for (int i = 0; i < CONV_K; ++i) load8(wT + (size_t)i * C + c, w[i]);
  }
  // sum_i w_i x[t - (K-1) + i] over the taps inside the document (p = row index in document)
  __device__ __forceinline__ void apply(float* acc, const float (*win)[8], const float* cur, int p) const {
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = w[CONV_K - 1][j] * cur[j];
#pragma unroll
    for (int back = 1; back < CONV_K; ++back)
      if (back <= p)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += w[CONV_K - 1 - back][j] * win[CONV_K - 1 - back][j];
  }
};

__device__ __forceinline__ void load_row_or_zero(const __nv_bfloat16* x, long row, int C, int c, float* out) {
  if (row >= 0) {
    load8(x + (size_t)row * C + c, out);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) out[j] = 0.f;
  }
}

__global__ void __launch_bounds__(256) conv_fwd_kernel(const __nv_bfloat16* __restrict__ x,
                                                       const float* __restrict__ wT, const int* __restrict__ pos,
                                                       __nv_bfloat16* __restrict__ y, int n, int C) {
  const int v = blockIdx.x * 32 + threadIdx.x;
  if (v >= C / 8) return;
  const int c = v * 8;
  const int t0 = (blockIdx.y * CONV_GROUPS + threadIdx.y) * CONV_ROWS;
  const int t1 = min(n, t0 + CONV_ROWS);
  if (t0 >= t1) return;
  ConvTaps taps;
  taps.load(wT, c, C);
  float win[CONV_K - 1][8];  // rows t-3, t-2, t-1
#pragma unroll
  for (int b = 0; b < CONV_K - 1; ++b) load_row_or_zero(x, (long)t0 - (CONV_K - 1) + b, C, c, win[b]);
#pragma unroll 4
  for (int t = t0; t < t1; ++t) {
    float cur[8], acc[8];
    load8(x + (size_t)t * C + c, cur);
    taps.apply(acc, win, cur, pos[t]);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = silu(acc[j]);
    store8(y + (size_t)t * C + c, acc);
#pragma unroll
    for (int b = 0; b < CONV_K - 2; ++b)
#pragma unroll
      for (int j = 0; j < 8; ++j) win[b][j] = win[b + 1][j];
#pragma unroll
    for (int j = 0; j < 8; ++j) win[CONV_K - 2][j] = cur[j];
  }
}

// Fused backward. Row u: pre_u (recomputed), g_u = dy_u silu'(pre_u); dw partials use rows of the
// thread's own range; dx_t = sum_s w_{K-1-s} g_{t+s} (same document) is emitted K-1 rows behind
// u, so the thread recomputes g for a (K-1)-row halo past its range. Per-block dw partials are
// reduced over the 8 row groups in shared memory and written to partial[blockIdx.y, C, K].
__global__ void __launch_bounds__(256) conv_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                                       const __nv_bfloat16* __restrict__ x,
                                                       const float* __restrict__ wT, const int* __restrict__ pos,
                                                       __nv_bfloat16* __restrict__ dx, float* __restrict__ partial,
                                                       int n, int C) {
  __shared__ float red[CONV_GROUPS][CONV_K * 8][33];
  const int v = blockIdx.x * 32 + threadIdx.x;
  const bool active = v < C / 8;
  const int c = v * 8;
  const int t0 = (blockIdx.y * CONV_GROUPS + threadIdx.y) * CONV_ROWS;
  const int t1 = min(n, t0 + CONV_ROWS);
  float part[CONV_K][8];
#pragma unroll
  for (int i = 0; i < CONV_K; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) part[i][j] = 0.f;
  if (active && t0 < t1) {
    ConvTaps taps;
    taps.load(wT, c, C);
    float xw[CONV_K - 1][8], gw[CONV_K - 1][8];
    int pw[CONV_K - 1];
#pragma unroll
    for (int b = 0; b < CONV_K - 1; ++b) {
      load_row_or_zero(x, (long)t0 - (CONV_K - 1) + b, C, c, xw[b]);
      pw[b] = -1;
#pragma unroll
      for (int j = 0; j < 8; ++j) gw[b][j] = 0.f;
    }
    const int u_end = t1 + CONV_K - 1;
#pragma unroll 2
    for (int u = t0; u < u_end; ++u) {
      float cur[8], g[8];
      int p = -1;
      if (u < n) {
        p = pos[u];
        load8(x + (size_t)u * C + c, cur);
        float pre[8], d[8];
        taps.apply(pre, xw, cur, p);
        load8(dy + (size_t)u * C + c, d);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float sg = 1.f / (1.f + __expf(-pre[j]));
          g[j] = d[j] * sg * (1.f + pre[j] * (1.f - sg));
        }
        if (u < t1) {
#pragma unroll
          for (int j = 0; j < 8; ++j) part[CONV_K - 1][j] += g[j] * cur[j];
#pragma unroll
          for (int back = 1; back < CONV_K; ++back)
            if (back <= p)
#pragma unroll
              for (int j = 0; j < 8; ++j) part[CONV_K - 1 - back][j] += g[j] * xw[CONV_K - 1 - back][j];
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) cur[j] = g[j] = 0.f;
      }
      const int t = u - (CONV_K - 1);
      if (t >= t0) {
        // s = 0 is row t itself; s = 1..K-1 are gw[s] (rows t+1..t+K-2) and g (row u = t+K-1)
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = taps.w[CONV_K - 1][j] * gw[0][j];
#pragma unroll
        for (int s = 1; s < CONV_K - 1; ++s)
          if (pw[s] >= s)
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] += taps.w[CONV_K - 1 - s][j] * gw[s][j];
        if (p >= CONV_K - 1)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] += taps.w[0][j] * g[j];
        store8(dx + (size_t)t * C + c, acc);
      }
#pragma unroll
      for (int b = 0; b < CONV_K - 2; ++b) {
        pw[b] = pw[b + 1];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          xw[b][j] = xw[b + 1][j];
          gw[b][j] = gw[b + 1][j];
        }
      }
      pw[CONV_K - 2] = p;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        xw[CONV_K - 2][j] = cur[j];
        gw[CONV_K - 2][j] = g[j];
      }
    }
  }
#pragma unroll
  for (int i = 0; i < CONV_K; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) red[threadIdx.y][j * CONV_K + i][threadIdx.x] = part[i][j];
  __syncthreads();
  // 256 threads write the block's 32 vectors x 8 channels x K taps = 1024 values
  const int tid = threadIdx.y * 32 + threadIdx.x;
  for (int e = tid; e < 32 * 8 * CONV_K; e += 256) {
    const int lane = e / (8 * CONV_K), r = e % (8 * CONV_K);
    const int vv = blockIdx.x * 32 + lane;
    if (vv >= C / 8) continue;
    float sum = 0.f;
#pragma unroll
    for (int gi = 0; gi < CONV_GROUPS; ++gi) sum += red[gi][r][lane];
    partial[((size_t)blockIdx.y * C + vv * 8) * CONV_K + r] = sum;
  }
}

// dw[e] = sum_b partial[b, e]  (fixed order: deterministic)
__global__ void sum_rows_kernel(const float* __restrict__ partial, float* __restrict__ out, int rows, int width) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= width) return;
  float s = 0.f;
  for (int b = 0; b < rows; ++b) s += partial[(size_t)b * width + e];
  out[e] = s;
}


// ---- query-side short conv (GDN read-only query events) -------------------------------------
// A query event's conv input is its own projected row plus the last K-1 content inputs of its
// document (or zeros): out[i, c] = silu(raw[qs[i], c] w[c, K-1] + sum_j hist_j(i)[c] w[c, j]),
// hist_j(i) = updates[qh[i, j]] (qh == nc: zero row). Only the first `size` (q) channels of
// the raw/updates rows are read (row strides ld_raw / ld_upd).
constexpr int QROWS = 16;   // queries per thread in the backward row pass

__global__ void __launch_bounds__(256) qconv_fwd_kernel(const __nv_bfloat16* __restrict__ raw, int ld_raw,
                                                        const __nv_bfloat16* __restrict__ upd, int ld_upd,
                                                        const long* __restrict__ qs, const long* __restrict__ qh,
                                                        long nc, const float* __restrict__ wT,
                                                        __nv_bfloat16* __restrict__ out, int nq, int size) {
  const int vecs = size / 8;
  const size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (idx >= (size_t)nq * vecs) return;
  const int i = (int)(idx / vecs), c = (int)(idx % vecs) * 8;
  float acc[8], x[8], w[8];
  load8(raw + (size_t)qs[i] * ld_raw + c, x);
  load8(wT + (size_t)(CONV_K - 1) * size + c, w);
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = x[j] * w[j];
#pragma unroll
  for (int t = 0; t < CONV_K - 1; ++t) {
    const long r = qh[(size_t)i * (CONV_K - 1) + t];
    if (r == nc) continue;
    load8(upd + (size_t)r * ld_upd + c, x);
    load8(wT + (size_t)t * size + c, w);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] += x[j] * w[j];
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = silu(acc[j]);
  store8(out + (size_t)i * size + c, acc);
}

// g = dy silu'(pre) -> gbuf (fp32); d_raw[qs[i]] = g w[K-1] (skipped when d_raw is null); per-block
// dw partials.
__global__ void __launch_bounds__(256) qconv_bwd_rows_kernel(
    const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ raw, int ld_raw,
    const __nv_bfloat16* __restrict__ upd, int ld_upd, const long* __restrict__ qs, const long* __restrict__ qh,
    long nc, const float* __restrict__ wT, float* __restrict__ gbuf, __nv_bfloat16* __restrict__ d_raw, int ld_draw,
    float* __restrict__ partial, int nq, int size) {
  __shared__ float red[CONV_GROUPS][CONV_K * 8][33];
  const int v = blockIdx.x * 32 + threadIdx.x;
  const bool active = v < size / 8;
  const int c = v * 8;
  const int i0 = (blockIdx.y * CONV_GROUPS + threadIdx.y) * QROWS;
  float part[CONV_K][8];
#pragma unroll
  for (int t = 0; t < CONV_K; ++t)
#pragma unroll
    for (int j = 0; j < 8; ++j) part[t][j] = 0.f;
  if (active) {
    float w[CONV_K][8];
#pragma unroll
    for (int t = 0; t < CONV_K; ++t) load8(wT + (size_t)t * size + c, w[t]);
    for (int i = i0; i < min(nq, i0 + QROWS); ++i) {
      float x[CONV_K][8], pre[8], d[8], g[8];
      load8(raw + (size_t)qs[i] * ld_raw + c, x[CONV_K - 1]);
#pragma unroll
      for (int j = 0; j < 8; ++j) pre[j] = x[CONV_K - 1][j] * w[CONV_K - 1][j];
#pragma unroll
      for (int t = 0; t < CONV_K - 1; ++t) {
        const long r = qh[(size_t)i * (CONV_K - 1) + t];
        if (r == nc) {
#pragma unroll
          for (int j = 0; j < 8; ++j) x[t][j] = 0.f;
        } else {
          load8(upd + (size_t)r * ld_upd + c, x[t]);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) pre[j] += x[t][j] * w[t][j];
      }
      load8(dy + (size_t)i * size + c, d);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float sg = 1.f / (1.f + __expf(-pre[j]));
        g[j] = d[j] * sg * (1.f + pre[j] * (1.f - sg));
      }
      store8(gbuf + (size_t)i * size + c, g);
      if (d_raw) {
        float dr[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) dr[j] = g[j] * w[CONV_K - 1][j];
        store8(d_raw + (size_t)qs[i] * ld_draw + c, dr);
      }
#pragma unroll
      for (int t = 0; t < CONV_K; ++t)
#pragma unroll
        for (int j = 0; j < 8; ++j) part[t][j] += g[j] * x[t][j];
    }
  }
#pragma unroll
  for (int t = 0; t < CONV_K; ++t)
#pragma unroll
    for (int j = 0; j < 8; ++j) red[threadIdx.y][j * CONV_K + t][threadIdx.x] = part[t][j];
  __syncthreads();
  const int tid = threadIdx.y * 32 + threadIdx.x;
  for (int e = tid; e < 32 * 8 * CONV_K; e += 256) {
    const int lane = e / (8 * CONV_K), r = e % (8 * CONV_K);
    const int vv = blockIdx.x * 32 + lane;
    if (vv >= size / 8) continue;
    float sum = 0.f;
#pragma unroll
    for (int gi = 0; gi < CONV_GROUPS; ++gi) sum += red[gi][r][lane];
    partial[((size_t)blockIdx.y * size + vv * 8) * CONV_K + r] = sum;
  }
}

// d_upd[rows[k]] (+)= sum over entries e of row k: gbuf[e / (K-1)] * w[e % (K-1)] (one block per
// row; `accumulate` adds to the row already there, e.g. the causal conv's input gradient).
__global__ void __launch_bounds__(256) qconv_bwd_hist_kernel(const float* __restrict__ gbuf,
                                                             const float* __restrict__ wT,
                                                             const int* __restrict__ rows,
                                                             const int* __restrict__ offsets,
                                                             const int* __restrict__ entries,
                                                             __nv_bfloat16* __restrict__ d_upd, int ld_upd, int size,
                                                             int accumulate) {
  const int k = blockIdx.x;
  const int e0 = offsets[k], e1 = offsets[k + 1];
  for (int c = threadIdx.x * 8; c < size; c += blockDim.x * 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (accumulate) load8(d_upd + (size_t)rows[k] * ld_upd + c, acc);
    for (int e = e0; e < e1; ++e) {
      const int ent = entries[e];
      const int i = ent / (CONV_K - 1), t = ent % (CONV_K - 1);
      float g[8], w[8];
      load8(gbuf + (size_t)i * size + c, g);
      load8(wT + (size_t)t * size + c, w);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += g[j] * w[j];
    }
    store8(d_upd + (size_t)rows[k] * ld_upd + c, acc);
  }
}

// d_raw[qs[i], :size] = gbuf[i] * w[:, K-1]: the query's own-projection gradient, written after the
// content rows of d_raw (which leave every query row zero).
__global__ void __launch_bounds__(256) qconv_raw_grad_kernel(const float* __restrict__ gbuf,
                                                             const float* __restrict__ wlast,
                                                             const long* __restrict__ qs,
                                                             __nv_bfloat16* __restrict__ d_raw, int ld_draw, int nq,
                                                             int size) {
  const long v = blockIdx.x * (long)blockDim.x + threadIdx.x;
  const int per_row = size / 8;
  if (v >= (long)nq * per_row) return;
  const int i = (int)(v / per_row), c = (int)(v % per_row) * 8;
  float g[8], w[8];
  load8(gbuf + (size_t)i * size + c, g);
  load8(wlast + c, w);
#pragma unroll
  for (int j = 0; j < 8; ++j) g[j] *= w[j];
  store8(d_raw + (size_t)qs[i] * ld_draw + c, g);
}

// out[n, h, c, :] = normalise?(x[idx[n*64 + c], h, :]) (zero when idx < 0); r[e, h] = rsqrt norm.
// 16 lanes per (slot, head) row, 8 elements (one 16-byte vector) per lane, two rows per warp; the
// row reductions are width-16 shuffles, so every lane of a warp takes part (rows past the end too).
template <int D>
__global__ void chunk_gather_kernel(const __nv_bfloat16* __restrict__ x, const long* __restrict__ idx,
                                    __nv_bfloat16* __restrict__ out, float* __restrict__ rnorm, int slots, int H,
                                    float scale, int normalize, long events) {
  static_assert(D == 16 * 8, "16 lanes x 8 elements per row");
  const long row = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 4;
  const int sub = threadIdx.x & 15;
  const bool valid = row < (long)slots * H;
  const int slot = valid ? (int)(row / H) : 0, h = valid ? (int)(row % H) : 0;
  long e = valid ? idx[slot] : -1;
  if (e >= 0 && !CQB_IN_RANGE(e, events, 11)) e = -1;    // -1 marks a padding slot
  float v[8];
  if (e >= 0) {
    load8(x + ((size_t)e * H + h) * D + sub * 8, v);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = 0.f;
  }
  if (normalize) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += v[j] * v[j];
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o, 16);
    const float r = rsqrtf(ss + 1e-6f);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] *= r * scale;
    if (sub == 0 && e >= 0) rnorm[(size_t)e * H + h] = r;
  }
  if (valid) {
    const int chunk = slot / 64, c = slot % 64;
    store8(out + (((size_t)chunk * H + h) * 64 + c) * D + sub * 8, v);
  }
}

// dx[e, h, :] = L2-norm backward of dy_chunks[slot(e)] (fp32) or a plain copy when !normalize
// (same 16-lanes-per-row layout as the gather).
template <int D, typename T>
__global__ void chunk_scatter_kernel(const T* __restrict__ dyc, const long* __restrict__ slot_of,
                                     const __nv_bfloat16* __restrict__ x, const float* __restrict__ rnorm,
                                     __nv_bfloat16* __restrict__ dx, int events, int H, float scale, int normalize,
                                     long slots) {
  static_assert(D == 16 * 8, "16 lanes x 8 elements per row");
  const long row = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 4;
  const int sub = threadIdx.x & 15;
  const bool valid = row < (long)events * H;
  const int e = valid ? (int)(row / H) : 0, h = valid ? (int)(row % H) : 0;
  float g[8];
  if (valid && CQB_IN_RANGE(slot_of[e], slots, 12)) {
    const long slot = slot_of[e];
    const int chunk = (int)(slot / 64), c = (int)(slot % 64);
    load8(dyc + (((size_t)chunk * H + h) * 64 + c) * D + sub * 8, g);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) g[j] = 0.f;
  }
  if (normalize) {
    float xv[8], dot = 0.f;
    float r = 0.f;
    if (valid) {
      r = rnorm[(size_t)e * H + h];
      load8(x + ((size_t)e * H + h) * D + sub * 8, xv);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) xv[j] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) dot += xv[j] * g[j];
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o, 16);
#pragma unroll
    for (int j = 0; j < 8; ++j) g[j] = scale * (r * g[j] - r * r * r * xv[j] * dot);
  }
  if (valid) store8(dx + ((size_t)e * H + h) * D + sub * 8, g);
}

int blocks_for(size_t threads, int per = 256) { return (int)((threads + per - 1) / per); }

}  // namespace

dim3 conv_grid(int n, int C) {
  return dim3((C / 8 + 31) / 32, (n + CONV_ROWS * CONV_GROUPS - 1) / (CONV_ROWS * CONV_GROUPS));
}

void check_conv(const at::Tensor& x, const at::Tensor& w, const at::Tensor& pos) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2 &&
                  x.size(1) % 8 == 0,
              "x: contiguous bf16 [n, C], C % 8 == 0");
  TORCH_CHECK(w.dim() == 2 && w.size(0) == x.size(1) && w.size(1) == CONV_K, "w: [C, 4] (only kernel size 4)");
  TORCH_CHECK(pos.scalar_type() == at::kInt && pos.is_contiguous() && pos.numel() == x.size(0), "pos: int32 [n]");
}

at::Tensor conv_fwd(at::Tensor x, at::Tensor w, at::Tensor pos) {
  check_conv(x, w, pos);
  const int n = x.size(0), C = x.size(1);
  auto wT = w.to(at::kFloat).t().contiguous();
  auto y = at::empty_like(x);
  if (!n) return y;
  conv_fwd_kernel<<<conv_grid(n, C), dim3(32, CONV_GROUPS), 0, stream()>>>(
      (const __nv_bfloat16*)x.data_ptr(), wT.data_ptr<float>(), pos.data_ptr<int>(), (__nv_bfloat16*)y.data_ptr(), n,
      C);
  CQB_LAUNCH_CHECK();
  count_launch();
  return y;
}

std::vector<at::Tensor> conv_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor pos) {
  check_conv(x, w, pos);
  TORCH_CHECK(dy.scalar_type() == at::kBFloat16 && dy.is_contiguous() && dy.sizes() == x.sizes(), "dy: like x");
  const int n = x.size(0), C = x.size(1);
  auto wT = w.to(at::kFloat).t().contiguous();
  auto dx = at::empty_like(x);
  auto dw = at::empty({C, CONV_K}, x.options().dtype(at::kFloat));
  if (!n) return {dx, dw.zero_()};
  const dim3 grid = conv_grid(n, C);
  auto partial = at::empty({(long)grid.y, C, CONV_K}, x.options().dtype(at::kFloat));
  conv_bwd_kernel<<<grid, dim3(32, CONV_GROUPS), 0, stream()>>>(
      (const __nv_bfloat16*)dy.data_ptr(), (const __nv_bfloat16*)x.data_ptr(), wT.data_ptr<float>(),
      pos.data_ptr<int>(), (__nv_bfloat16*)dx.data_ptr(), partial.data_ptr<float>(), n, C);
  CQB_LAUNCH_CHECK();
  sum_rows_kernel<<<(C * CONV_K + 255) / 256, 256, 0, stream()>>>(partial.data_ptr<float>(), dw.data_ptr<float>(),
                                                                  grid.y, C * CONV_K);
  CQB_LAUNCH_CHECK();
  count_launch(2);
  return {dx, dw};
}


namespace {
void check_qconv(const at::Tensor& raw, const at::Tensor& upd, const at::Tensor& w, const at::Tensor& qs,
                 const at::Tensor& qh) {
  for (const auto* t : {&raw, &upd})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->dim() == 2 && t->stride(1) == 1 &&
                    t->stride(0) % 8 == 0,
                "raw/updates: bf16 row-major, row stride a multiple of 8");
  TORCH_CHECK(w.dim() == 2 && w.size(1) == CONV_K && w.size(0) % 8 == 0, "w: [size, 4], size % 8 == 0");
  TORCH_CHECK(raw.size(1) >= w.size(0) && upd.size(1) >= w.size(0), "rows narrower than the conv channels");
  TORCH_CHECK(qs.scalar_type() == at::kLong && qh.scalar_type() == at::kLong && qh.is_contiguous() &&
                  qh.dim() == 2 && qh.size(1) == CONV_K - 1 && qh.size(0) == qs.numel(),
              "query_source int64 [nq], query_history int64 [nq, 3]");
}
}  // namespace

// Query conv forward: [nq, size] bf16.
at::Tensor qconv_fwd(at::Tensor raw, at::Tensor updates, at::Tensor w, at::Tensor qs, at::Tensor qh) {
  check_qconv(raw, updates, w, qs, qh);
  const int nq = qs.numel(), size = w.size(0);
  auto wT = w.to(at::kFloat).t().contiguous();
  auto qsc = qs.contiguous();
  auto out = at::empty({nq, size}, raw.options());
  if (!nq) return out;
  qconv_fwd_kernel<<<blocks_for((size_t)nq * size / 8), 256, 0, stream()>>>(
      (const __nv_bfloat16*)raw.data_ptr(), (int)raw.stride(0), (const __nv_bfloat16*)updates.data_ptr(),
      (int)updates.stride(0), (const long*)qsc.data_ptr(), (const long*)qh.data_ptr(), (long)updates.size(0),
      wT.data_ptr<float>(), (__nv_bfloat16*)out.data_ptr(), nq, size);
  CQB_LAUNCH_CHECK();
  count_launch();
  return out;
}

// Query conv backward: (d_raw like raw, d_updates like updates: zero outside the rows/channels the
// queries read; dw [size, 4] fp32).
std::vector<at::Tensor> qconv_bwd(at::Tensor dy, at::Tensor raw, at::Tensor updates, at::Tensor w, at::Tensor qs,
                                  at::Tensor qh, at::Tensor hist_rows, at::Tensor hist_offsets,
                                  at::Tensor hist_entries) {
  check_qconv(raw, updates, w, qs, qh);
  TORCH_CHECK(hist_rows.scalar_type() == at::kInt && hist_offsets.scalar_type() == at::kInt &&
                  hist_entries.scalar_type() == at::kInt && hist_offsets.numel() == hist_rows.numel() + 1,
              "history CSR: int32 rows [U], offsets [U+1], entries [E]");
  const int nq = qs.numel(), size = w.size(0);
  auto dyc = dy.contiguous();
  TORCH_CHECK(dyc.scalar_type() == at::kBFloat16 && dyc.numel() == (int64_t)nq * size, "dy: bf16 [nq, size]");
  auto wT = w.to(at::kFloat).t().contiguous();
  auto qsc = qs.contiguous();
  auto d_raw = at::zeros({raw.size(0), raw.size(1)}, raw.options());
  auto d_upd = at::zeros({updates.size(0), updates.size(1)}, updates.options());
  auto dw = at::zeros({size, CONV_K}, raw.options().dtype(at::kFloat));
  if (!nq) return {d_raw, d_upd, dw};
  auto gbuf = at::empty({nq, size}, raw.options().dtype(at::kFloat));
  const dim3 grid((size / 8 + 31) / 32, (nq + QROWS * CONV_GROUPS - 1) / (QROWS * CONV_GROUPS));
  auto partial = at::empty({(long)grid.y, size, CONV_K}, dw.options());
  qconv_bwd_rows_kernel<<<grid, dim3(32, CONV_GROUPS), 0, stream()>>>(
      (const __nv_bfloat16*)dyc.data_ptr(), (const __nv_bfloat16*)raw.data_ptr(), (int)raw.stride(0),
      (const __nv_bfloat16*)updates.data_ptr(), (int)updates.stride(0), (const long*)qsc.data_ptr(),
      (const long*)qh.data_ptr(), (long)updates.size(0), wT.data_ptr<float>(), gbuf.data_ptr<float>(),
      (__nv_bfloat16*)d_raw.data_ptr(), (int)d_raw.stride(0), partial.data_ptr<float>(), nq, size);
  CQB_LAUNCH_CHECK();
  sum_rows_kernel<<<(size * CONV_K + 255) / 256, 256, 0, stream()>>>(partial.data_ptr<float>(), dw.data_ptr<float>(),
                                                                     grid.y, size * CONV_K);
  CQB_LAUNCH_CHECK();
  const int U = hist_rows.numel();
  if (U)
    qconv_bwd_hist_kernel<<<U, 256, 0, stream()>>>(gbuf.data_ptr<float>(), wT.data_ptr<float>(),
                                                   hist_rows.data_ptr<int>(), hist_offsets.data_ptr<int>(),
                                                   hist_entries.data_ptr<int>(), (__nv_bfloat16*)d_upd.data_ptr(),
                                                   (int)d_upd.stride(0), size, 0);
  CQB_LAUNCH_CHECK();
  count_launch(3);
  return {d_raw, d_upd, dw};
}

// Query conv backward into existing buffers: adds the history gradient into `d_upd` (the causal
// conv's input gradient, bf16 [nc, >= size]) and returns (dw [size, 4] fp32, g [nq, size] fp32); the
// own-projection gradient goes to d_raw later through qconv_raw_grad(g, w, qs, d_raw).
std::vector<at::Tensor> qconv_bwd_into(at::Tensor dy, at::Tensor raw, at::Tensor updates, at::Tensor w,
                                       at::Tensor qs, at::Tensor qh, at::Tensor hist_rows, at::Tensor hist_offsets,
                                       at::Tensor hist_entries, at::Tensor d_upd) {
  check_qconv(raw, updates, w, qs, qh);
  TORCH_CHECK(hist_rows.scalar_type() == at::kInt && hist_offsets.scalar_type() == at::kInt &&
                  hist_entries.scalar_type() == at::kInt && hist_offsets.numel() == hist_rows.numel() + 1,
              "history CSR: int32 rows [U], offsets [U+1], entries [E]");
  const int nq = qs.numel(), size = w.size(0);
  TORCH_CHECK(d_upd.is_cuda() && d_upd.scalar_type() == at::kBFloat16 && d_upd.dim() == 2 &&
                  d_upd.size(0) == updates.size(0) && d_upd.size(1) >= size && d_upd.stride(1) == 1 &&
                  d_upd.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(d_upd.data_ptr()) % 16 == 0,
              "d_upd: bf16 [nc, >= size] with 16-byte aligned rows");
  auto dyc = dy.contiguous();
  TORCH_CHECK(dyc.scalar_type() == at::kBFloat16 && dyc.numel() == (int64_t)nq * size, "dy: bf16 [nq, size]");
  auto wT = w.to(at::kFloat).t().contiguous();
  auto qsc = qs.contiguous();
  auto dw = at::zeros({size, CONV_K}, raw.options().dtype(at::kFloat));
  auto gbuf = at::empty({nq, size}, raw.options().dtype(at::kFloat));
  if (!nq) return {dw, gbuf};
  const dim3 grid((size / 8 + 31) / 32, (nq + QROWS * CONV_GROUPS - 1) / (QROWS * CONV_GROUPS));
  auto partial = at::empty({(long)grid.y, size, CONV_K}, dw.options());
  qconv_bwd_rows_kernel<<<grid, dim3(32, CONV_GROUPS), 0, stream()>>>(
      (const __nv_bfloat16*)dyc.data_ptr(), (const __nv_bfloat16*)raw.data_ptr(), (int)raw.stride(0),
      (const __nv_bfloat16*)updates.data_ptr(), (int)updates.stride(0), (const long*)qsc.data_ptr(),
      (const long*)qh.data_ptr(), (long)updates.size(0), wT.data_ptr<float>(), gbuf.data_ptr<float>(), nullptr, 0,
      partial.data_ptr<float>(), nq, size);
  CQB_LAUNCH_CHECK();
  sum_rows_kernel<<<(size * CONV_K + 255) / 256, 256, 0, stream()>>>(partial.data_ptr<float>(), dw.data_ptr<float>(),
                                                                     grid.y, size * CONV_K);
  CQB_LAUNCH_CHECK();
  const int U = hist_rows.numel();
  if (U)
    qconv_bwd_hist_kernel<<<U, 256, 0, stream()>>>(gbuf.data_ptr<float>(), wT.data_ptr<float>(),
                                                   hist_rows.data_ptr<int>(), hist_offsets.data_ptr<int>(),
                                                   hist_entries.data_ptr<int>(), (__nv_bfloat16*)d_upd.data_ptr(),
                                                   (int)d_upd.stride(0), size, 1);
  CQB_LAUNCH_CHECK();
  count_launch(U ? 3 : 2);
  return {dw, gbuf};
}

// d_raw[qs[i], :size] = g[i] * w[:, K-1] (see qconv_bwd_into).
void qconv_raw_grad(at::Tensor g, at::Tensor w, at::Tensor qs, at::Tensor d_raw) {
  const int nq = qs.numel(), size = w.size(0);
  TORCH_CHECK(g.scalar_type() == at::kFloat && g.is_contiguous() && g.numel() == (int64_t)nq * size,
              "g: fp32 [nq, size]");
  TORCH_CHECK(w.dim() == 2 && w.size(1) == CONV_K && size % 8 == 0, "w: [size, 4], size a multiple of 8");
  TORCH_CHECK(qs.scalar_type() == at::kLong, "qs: int64");
  TORCH_CHECK(d_raw.scalar_type() == at::kBFloat16 && d_raw.dim() == 2 && d_raw.size(1) >= size &&
                  d_raw.stride(1) == 1 && d_raw.stride(0) % 8 == 0 &&
                  reinterpret_cast<uintptr_t>(d_raw.data_ptr()) % 16 == 0,
              "d_raw: bf16 [rows, >= size] with 16-byte aligned rows");
  if (!nq) return;
  auto wlast = w.select(1, CONV_K - 1).to(at::kFloat).contiguous();
  auto qsc = qs.contiguous();
  const long vectors = (long)nq * (size / 8);
  qconv_raw_grad_kernel<<<(unsigned)((vectors + 255) / 256), 256, 0, stream()>>>(
      g.data_ptr<float>(), wlast.data_ptr<float>(), (const long*)qsc.data_ptr(), (__nv_bfloat16*)d_raw.data_ptr(),
      (int)d_raw.stride(0), nq, size);
  CQB_LAUNCH_CHECK();
  count_launch();
}

std::vector<at::Tensor> chunk_gather(at::Tensor x, at::Tensor idx, int64_t chunks, bool normalize, double scale) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 3 && x.size(2) == 128,
              "x: bf16 [E, H, 128]");
  TORCH_CHECK(idx.scalar_type() == at::kLong && idx.numel() == chunks * 64, "idx: int64 [chunks * 64]");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "x: 16-byte aligned base");
  const int E = x.size(0), H = x.size(1);
  const int slots = idx.numel();
  auto out = at::empty({chunks, H, 64, 128}, x.options());
  auto r = at::empty({E, H}, x.options().dtype(at::kFloat));
  if (!slots) return {out, r};
  const size_t threads = (size_t)slots * H * 16;
  chunk_gather_kernel<128><<<blocks_for(threads), 256, 0, stream()>>>(
      (const __nv_bfloat16*)x.data_ptr(), (const long*)idx.data_ptr(), (__nv_bfloat16*)out.data_ptr(),
      r.data_ptr<float>(), slots, H, (float)scale, normalize ? 1 : 0, (long)x.size(0));
  CQB_LAUNCH_CHECK();
  count_launch();
  return {out, r};
}

at::Tensor chunk_scatter(at::Tensor dyc, at::Tensor slot_of, at::Tensor x, at::Tensor rnorm, bool normalize,
                         double scale) {
  TORCH_CHECK((dyc.scalar_type() == at::kFloat || dyc.scalar_type() == at::kBFloat16) && dyc.is_contiguous() &&
                  dyc.dim() == 4 && dyc.size(2) == 64 && dyc.size(3) == 128,
              "chunks: fp32/bf16 [Nc, H, 64, 128]");
  TORCH_CHECK(slot_of.scalar_type() == at::kLong, "slot_of: int64");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(dyc.data_ptr()) % 16 == 0 &&
                  (!normalize || reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0),
              "chunks / x: 16-byte aligned bases");
  if (normalize)
    TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && rnorm.scalar_type() == at::kFloat,
                "normalize needs bf16 x and fp32 rnorm");
  const int E = slot_of.numel(), H = dyc.size(1);
  auto dx = at::empty({E, H, 128}, dyc.options().dtype(at::kBFloat16));
  if (!E) return dx;
  const size_t threads = (size_t)E * H * 16;
  const long* so = (const long*)slot_of.data_ptr();
  const __nv_bfloat16* xp = normalize ? (const __nv_bfloat16*)x.data_ptr() : nullptr;
  const float* rp = normalize ? rnorm.data_ptr<float>() : nullptr;
  if (dyc.scalar_type() == at::kFloat)
    chunk_scatter_kernel<128, float><<<blocks_for(threads), 256, 0, stream()>>>(
        dyc.data_ptr<float>(), so, xp, rp, (__nv_bfloat16*)dx.data_ptr(), E, H, (float)scale, normalize ? 1 : 0,
        (long)dyc.size(0) * 64);
  else
    chunk_scatter_kernel<128, __nv_bfloat16><<<blocks_for(threads), 256, 0, stream()>>>(
        (const __nv_bfloat16*)dyc.data_ptr(), so, xp, rp, (__nv_bfloat16*)dx.data_ptr(), E, H, (float)scale,
        normalize ? 1 : 0, (long)dyc.size(0) * 64);
  CQB_LAUNCH_CHECK();
  count_launch();
  return dx;
}

#ifdef CQB_DEBUG_BOUNDS
CQB_DEBUG_STATUS_READER(debug_status_conv)
#endif

}  // namespace cqb

// ==== Allocation-free causal-conv backward (C ABI, declared in noalloc.h) =====================
//
// This entry point has no counterpart in the reference framework. It serves callers that must
// not allocate device memory while they run the backward pass of the short convolution:
//   * hooks that run inside a caching allocator or memory pool (they cannot re-enter the
//     allocator they belong to);
//   * C or C++ hosts that drive the kernels without PyTorch and so have no tensor allocator;
//   * steps whose device memory was reserved once up front, where a late cudaMalloc could fail
//     or fragment the reserved pool.
// It launches the same two kernels as the tensor entry point `conv_bwd` (fused backward per row
// group, then a fixed-order sum of the per-block weight-gradient partials). The partials live in
// a file-scope device array instead of a fresh allocation, and the caller passes every buffer,
// including the transposed fp32 weight.
//
// Contract:
//   * Size limit: ceil(n / 256) * C * 4 floats of partials must fit in the scratch array of
//     2,097,152 floats (8 MiB; for C = 6144 that is n <= 21,760 rows). Larger inputs are rejected
//     with CQB_NOALLOC_TOO_LARGE; cqb_noalloc_last_error() returns the message.
//   * Every GPU that loads this library holds the 8 MiB array until the process exits.
//   * Set-up: the first call on a device (or cqb_conv_bwd_noalloc_init() with that device
//     current) looks up the array's device address with cudaGetSymbolAddress. Make that first
//     call before any stream capture begins.
//   * All calls on a device share the array, and it keeps the last call's contents. Calls that
//     overlap on the GPU (different streams, or threads without ordering) race on it: serialise
//     them on one stream or order them with events. Each call overwrites every partial it
//     reads, so nothing has to start at zero; for n == 0 the weight gradient is cleared with
//     cudaMemsetAsync.
//   * No cudaMalloc, cudaFree or allocating library routine is called.

static __device__ __align__(256) float g_conv_noalloc_scratch[size_t(2) * 1024 * 1024];

namespace {

constexpr size_t kNoAllocScratchFloats = size_t(2) * 1024 * 1024;
constexpr int kMaxDevices = 64;
float* g_scratch_ptr[kMaxDevices] = {};   // device address of the scratch array, per device
std::mutex g_scratch_mu;
thread_local char g_noalloc_error[256] = "";

int noalloc_fail(int code, const char* fmt, long a = 0, long b = 0) {
  snprintf(g_noalloc_error, sizeof(g_noalloc_error), fmt, a, b);
  return code;
}

}  // namespace

extern "C" {

// Message of the last failed call on this host thread.
__attribute__((visibility("default"))) const char* cqb_noalloc_last_error(void) { return g_noalloc_error; }

// Capacity of the scratch array in floats.
__attribute__((visibility("default"))) size_t cqb_conv_bwd_noalloc_scratch_floats(void) {
  return kNoAllocScratchFloats;
}

// Looks up the scratch address for the current device (idempotent). Call before stream capture.
__attribute__((visibility("default"))) int cqb_conv_bwd_noalloc_init(void) {
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return noalloc_fail(CQB_NOALLOC_CUDA_ERROR, "cudaGetDevice failed (error %ld)", (long)err);
  if (device < 0 || device >= kMaxDevices)
    return noalloc_fail(CQB_NOALLOC_BAD_ARGUMENT, "device %ld is outside the supported range [0, %ld)", device,
                        kMaxDevices);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[device] != nullptr) return CQB_NOALLOC_OK;
  float* ptr = nullptr;
  err = cudaGetSymbolAddress((void**)&ptr, g_conv_noalloc_scratch);
  if (err != cudaSuccess || ptr == nullptr)
    return noalloc_fail(CQB_NOALLOC_CUDA_ERROR, "cudaGetSymbolAddress of the conv scratch failed (error %ld)",
                        (long)err);
  g_scratch_ptr[device] = ptr;
  return CQB_NOALLOC_OK;
}

// Backward of y = silu(causal_conv(x, w)) per document.
//   dy, x, dx: bf16 [n, C] row-major, 16-byte aligned;  wT: fp32 [4, C] (tap-major: the transpose
//   of the [C, 4] weight), 16-byte aligned;  pos: int32 [n], index of each row inside its
//   document;  dw: fp32 [C, 4] output.  C must be a positive multiple of 8.
// Returns CQB_NOALLOC_OK or an error code (message in cqb_noalloc_last_error()).
__attribute__((visibility("default"))) int cqb_conv_bwd_noalloc(const void* dy, const void* x, const float* wT,
                                                                 const int* pos, void* dx, float* dw, long n, long C,
                                                                 cudaStream_t stream) {
  if (n < 0 || C <= 0 || C % 8 != 0 || C > (1L << 24) || n > (1L << 30))
    return noalloc_fail(CQB_NOALLOC_BAD_ARGUMENT, "need n >= 0 and C a positive multiple of 8 (n=%ld, C=%ld)", n, C);
  if (!dw || (n > 0 && (!dy || !x || !wT || !pos || !dx)))
    return noalloc_fail(CQB_NOALLOC_BAD_ARGUMENT, "null buffer pointer");
  auto misaligned = [](const void* p, uintptr_t bytes) { return reinterpret_cast<uintptr_t>(p) % bytes != 0; };
  if (misaligned(dy, 16) || misaligned(x, 16) || misaligned(dx, 16) || misaligned(wT, 16) || misaligned(pos, 4) ||
      misaligned(dw, 4))
    return noalloc_fail(CQB_NOALLOC_BAD_ARGUMENT, "dy, x, dx and wT must be 16-byte aligned, pos and dw 4-byte");
  const int rc = cqb_conv_bwd_noalloc_init();
  if (rc != CQB_NOALLOC_OK) return rc;
  if (n == 0) {
    const cudaError_t err = cudaMemsetAsync(dw, 0, sizeof(float) * C * cqb::CONV_K, stream);
    return err == cudaSuccess ? CQB_NOALLOC_OK
                              : noalloc_fail(CQB_NOALLOC_CUDA_ERROR, "cudaMemsetAsync failed (error %ld)", (long)err);
  }
  const dim3 grid = cqb::conv_grid((int)n, (int)C);
  const size_t need = (size_t)grid.y * C * cqb::CONV_K;
  if (need > kNoAllocScratchFloats)
    return noalloc_fail(CQB_NOALLOC_TOO_LARGE,
                        "input too large for the static scratch: it needs %ld floats (ceil(n / 256) * C * 4), "
                        "the limit is %ld",
                        (long)need, (long)kNoAllocScratchFloats);
  if (grid.y > 65535u || grid.x > 2147483647u)
    return noalloc_fail(CQB_NOALLOC_TOO_LARGE, "input too large for one launch: %ld row blocks (limit %ld)",
                        (long)grid.y, 65535L);
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return noalloc_fail(CQB_NOALLOC_CUDA_ERROR, "cudaGetDevice failed (error %ld)", (long)err);
  float* scratch = g_scratch_ptr[device];
  // Do not launch over (or clear) an error the caller left pending: report it instead.
  err = cudaPeekAtLastError();
  if (err != cudaSuccess)
    return noalloc_fail(CQB_NOALLOC_CUDA_ERROR, "an earlier CUDA error is pending (error %ld); nothing was launched",
                        (long)err);
  cqb::conv_bwd_kernel<<<grid, dim3(32, cqb::CONV_GROUPS), 0, stream>>>(
      (const __nv_bfloat16*)dy, (const __nv_bfloat16*)x, wT, pos, (__nv_bfloat16*)dx, scratch, (int)n, (int)C);
  err = cudaGetLastError();
  if (err != cudaSuccess)
    return noalloc_fail(CQB_NOALLOC_CUDA_ERROR, "launch of the conv backward failed (error %ld)", (long)err);
  cqb::sum_rows_kernel<<<(unsigned)((C * cqb::CONV_K + 255) / 256), 256, 0, stream>>>(scratch, dw, (int)grid.y,
                                                                                       (int)(C * cqb::CONV_K));
  err = cudaGetLastError();
  if (err != cudaSuccess)
    return noalloc_fail(CQB_NOALLOC_CUDA_ERROR, "launch of the partial sum failed (error %ld)", (long)err);
  cqb::count_launch(2);
  return CQB_NOALLOC_OK;
}

}  // extern "C"
