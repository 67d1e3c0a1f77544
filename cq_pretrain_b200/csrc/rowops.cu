// Row-wise normalisation / activation kernels (memory-bound; one warp per row, fp32 statistics).
//
//  rms_norm      y = x * rsqrt(mean x^2 + eps) * (1 + w)                  (Qwen3.5 offset RMSNorm)
//  gated_norm    y = bf16(x * rsqrt(mean x^2 + eps)) * w * silu(z)          (GDN output norm)
//  ln_modulate   y = LN(x) * (1 + scale[idx[r]]) + shift[idx[r]]            (Wan adaLN, fp32 math)
//  gated_add     y = x + gate[idx[r]] * branch                              (Wan fp32 gated residual)
//  swiglu        y = silu(x[:, :F]) * x[:, F:]
//
// Backward kernels reduce weight / modulation gradients per warp over contiguous rows in
// registers, then per block in shared memory, then with one fp32 atomicAdd per block and column.
#include "common.cuh"

namespace cqb {

namespace {

constexpr int kWarps = 8;  // rows per 256-thread block in forward kernels

template <typename T>
__device__ __forceinline__ void load_vec(const T* p, float* out) { load8(p, out); }

// With `add` (may be null): the normalised row is s = x + add, and s is also written to `sum`
// (a residual add fused into the norm that follows it).
template <int NV, typename T, typename WT>
__global__ void __launch_bounds__(256) rms_fwd_kernel(const T* __restrict__ x, const WT* __restrict__ w,
                                                     T* __restrict__ y, float* __restrict__ rstd, int rows, int width,
                                                     float eps, const T* __restrict__ add, T* __restrict__ sum) {
  const int row = blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* xr = x + (size_t)row * width;
  float v[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < width) {
      load_vec(xr + c, v[i]);
      if (add != nullptr) {
        float a[8];
        load_vec(add + (size_t)row * width + c, a);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] += a[j];
        store8(sum + (size_t)row * width + c, v[i]);
        if (sizeof(T) == 2) {   // normalise the bf16-rounded sum that the residual stream carries on
#pragma unroll
          for (int j = 0; j < 8; ++j) v[i][j] = __bfloat162float(__float2bfloat16(v[i][j]));
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / width + eps);
  T* yr = y + (size_t)row * width;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < width) {
      float wv[8], o[8];
      load_vec(w + c, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[i][j] * r * (1.f + wv[j]);
      store8(yr + c, o);
    }
  }
  if (lane == 0) rstd[row] = r;
}

// dx = r * (g - xhat * mean(g * xhat)) (+ dres), g = dy * (1 + w);  dw += dy * xhat. dres (may be
// null) is the gradient the same x receives through a residual connection, summed in here.
// Row-parallel form of the backward: one warp per row (x and dy stay in registers between the two
// passes), RB_WARPS rows per block; the block's weight-gradient rows are summed in a fixed order
// and written to partial[block], and rms_dw_reduce_kernel sums the partials over blocks in a fixed
// order (deterministic, no atomics).
constexpr int RB_WARPS = 4;

template <int NV, typename T, typename WT>
__global__ void __launch_bounds__(RB_WARPS * 32) rms_bwd_rows_kernel(
    const T* __restrict__ dy, const T* __restrict__ x, const WT* __restrict__ w, const float* __restrict__ rstd,
    const T* __restrict__ dres, T* __restrict__ dx, float* __restrict__ partial, int rows, int width) {
  static_assert(sizeof(T) == 2, "bf16 rows (kept packed in registers between the passes)");
  extern __shared__ float part[];   // [RB_WARPS][width]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * RB_WARPS + warp;
  float* mine = part + warp * width;
  if (row < rows) {
    const float r = rstd[row];
    const T* xr = x + (size_t)row * width;
    const T* gr = dy + (size_t)row * width;
    uint4 xraw[NV], graw[NV], rraw[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {   // every load of the row in flight at once
      const int c = (i * 32 + lane) * 8;
      if (c < width) {
        xraw[i] = *reinterpret_cast<const uint4*>(xr + c);
        graw[i] = *reinterpret_cast<const uint4*>(gr + c);
        if (dres) rraw[i] = *reinterpret_cast<const uint4*>(dres + (size_t)row * width + c);
      }
    }
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < width) {
        float wv[8], xv[8], gv[8];
        load_vec(w + c, wv);
        load8(reinterpret_cast<const __nv_bfloat16*>(&xraw[i]), xv);
        load8(reinterpret_cast<const __nv_bfloat16*>(&graw[i]), gv);
        float pw[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float xh = xv[j] * r;
          dot += gv[j] * (1.f + wv[j]) * xh;
          pw[j] = gv[j] * xh;
        }
        *reinterpret_cast<float4*>(mine + c) = make_float4(pw[0], pw[1], pw[2], pw[3]);
        *reinterpret_cast<float4*>(mine + c + 4) = make_float4(pw[4], pw[5], pw[6], pw[7]);
      }
    }
    dot = warp_sum(dot) / width;
    T* dr = dx + (size_t)row * width;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < width) {
        float wv[8], xv[8], gv[8], o[8];
        load_vec(w + c, wv);
        load8(reinterpret_cast<const __nv_bfloat16*>(&xraw[i]), xv);
        load8(reinterpret_cast<const __nv_bfloat16*>(&graw[i]), gv);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = r * (gv[j] * (1.f + wv[j]) - xv[j] * r * dot);
        if (dres) {
          float rv[8];
          load8(reinterpret_cast<const __nv_bfloat16*>(&rraw[i]), rv);
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] += rv[j];
        }
        store8(dr + c, o);
      }
    }
  } else {
    for (int c = lane; c < width; c += 32) mine[c] = 0.f;
  }
  __syncthreads();
  for (int c = threadIdx.x; c < width; c += blockDim.x) {
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < RB_WARPS; ++k) acc += part[k * width + c];
    partial[(size_t)blockIdx.x * width + c] = acc;
  }
}

// Gated-norm backward at width 128 (a GDN head): one row per half-warp (16 lanes x 8 columns),
// 16 rows per 256-thread block per step, a fixed grid striding over the rows; every thread keeps its
// 8 columns' weight-gradient sums in registers, the block adds its 16 half-warps in order into
// partial[block] (then the two-stage deterministic reduction below).
constexpr int GB_BLOCKS_PER_SM = 4;

// z row r lives at z + (r / heads) * z_stride + (r % heads) * 128 (the gate columns of a token's
// projection row, read in place); x, dy, dx, dz are contiguous [rows, 128].
__device__ __forceinline__ size_t gate_offset(int row, int heads, long z_stride) {
  return (size_t)(row / heads) * z_stride + (size_t)(row % heads) * 128;
}

template <typename T, typename WT>
__global__ void __launch_bounds__(256) gated_fwd_rows_kernel(const T* __restrict__ x, const T* __restrict__ z,
                                                             const WT* __restrict__ w, T* __restrict__ y,
                                                             float* __restrict__ rstd, int rows, int heads,
                                                             long z_stride, float eps) {
  constexpr int W = 128;
  const int hw = threadIdx.x >> 4, l = threadIdx.x & 15, c = l * 8;
  const int row = blockIdx.x * 16 + hw;
  const bool live = row < rows;
  float xv[8], zv[8], wv[8];
  if (live) {
    load_vec(x + (size_t)row * W + c, xv);
    load_vec(z + gate_offset(row, heads, z_stride) + c, zv);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) xv[j] = zv[j] = 0.f;
  }
  load_vec(w + c, wv);
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) ss += xv[j] * xv[j];
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o, 16);
  const float r = rsqrtf(ss / W + eps);
  if (live) {
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float n = __bfloat162float(__float2bfloat16(xv[j] * r));
      o[j] = n * wv[j] * silu(zv[j]);
    }
    store8(y + (size_t)row * W + c, o);
    if (l == 0) rstd[row] = r;
  }
}

template <typename T, typename WT>
__global__ void __launch_bounds__(256) gated_bwd_rows_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                                                             const T* __restrict__ z, const WT* __restrict__ w,
                                                             const float* __restrict__ rstd, T* __restrict__ dx,
                                                             T* __restrict__ dz, float* __restrict__ partial, int rows,
                                                             int heads, long z_stride) {
  constexpr int W = 128;
  __shared__ float red[16][W];
  const int hw = threadIdx.x >> 4, l = threadIdx.x & 15, c = l * 8;
  float wv[8], acc[8];
  load_vec(w + c, wv);
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  const int warp_row0 = blockIdx.x * 16 + (hw & ~1);   // both half-warps of a warp run the same steps
  for (int base = warp_row0; base < rows; base += gridDim.x * 16) {
    const int row = base + (hw & 1);
    const bool live = row < rows;
    float xv[8], gv[8], zv[8];
    float r = 0.f;
    const size_t off = (size_t)(live ? row : 0) * W + c;
    if (live) {
      load_vec(x + off, xv);
      load_vec(dy + off, gv);
      load_vec(z + gate_offset(row, heads, z_stride) + c, zv);
      r = rstd[row];
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) xv[j] = gv[j] = zv[j] = 0.f;
    }
    float dot = 0.f, dzo[8], sv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float n = xv[j] * r;
      const float sg = 1.f / (1.f + __expf(-zv[j]));
      sv[j] = zv[j] * sg;
      acc[j] += gv[j] * n * sv[j];
      dot += gv[j] * wv[j] * sv[j] * n;
      dzo[j] = gv[j] * n * wv[j] * sg * (1.f + zv[j] * (1.f - sg));
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o, 16);
    dot /= W;
    if (live) {
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = r * (gv[j] * wv[j] * sv[j] - xv[j] * r * dot);
      store8(dz + off, dzo);
      store8(dx + off, o);
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) red[hw][c + j] = acc[j];
  __syncthreads();
  if (threadIdx.x < W) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) t += red[k][threadIdx.x];
    partial[(size_t)blockIdx.x * W + threadIdx.x] = t;
  }
}

// Deterministic sum of partial[blocks][width] over blocks in two launches. Stage 1: block
// (column group cx of 32 columns, slice sy of RD_SLICES) has warp w sum the partial rows
// g, g + G, g + 2G, ... with g = sy * 8 + w and G = 8 * RD_SLICES (coalesced 128-byte rows), then
// the 8 warp sums are added in warp order into stage[sy][col]. Stage 2 adds the slices in order.
constexpr int RD_SLICES = 16;

__global__ void __launch_bounds__(256) rms_dw_reduce_kernel(const float* __restrict__ partial, int blocks, int width,
                                                           float* __restrict__ stage) {
  __shared__ float sums[8][33];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x * 32 + lane;
  const int g0 = blockIdx.y * 8 + warp, step = 8 * RD_SLICES;
  float acc = 0.f;
  if (c < width) {
    int b = g0;
    for (; b + 3 * step < blocks; b += 4 * step) {   // four independent loads in flight
      const float a0 = partial[(size_t)b * width + c], a1 = partial[(size_t)(b + step) * width + c];
      const float a2 = partial[(size_t)(b + 2 * step) * width + c], a3 = partial[(size_t)(b + 3 * step) * width + c];
      acc += a0;
      acc += a1;
      acc += a2;
      acc += a3;
    }
    for (; b < blocks; b += step) acc += partial[(size_t)b * width + c];
  }
  sums[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && c < width) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += sums[w][lane];
    stage[(size_t)blockIdx.y * width + c] = t;
  }
}

__global__ void __launch_bounds__(256) rms_dw_final_kernel(const float* __restrict__ stage, int width,
                                                          float* __restrict__ dw) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= width) return;
  float t = 0.f;
#pragma unroll
  for (int sy = 0; sy < RD_SLICES; ++sy) t += stage[(size_t)sy * width + c];
  dw[c] = t;
}

template <int NV, typename T, typename WT>
__global__ void __launch_bounds__(512) rms_bwd_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                                                     const WT* __restrict__ w, const float* __restrict__ rstd,
                                                     const T* __restrict__ dres, T* __restrict__ dx,
                                                     float* __restrict__ dw, int rows, int width) {
  extern __shared__ float smem[];  // [width]
  const int warps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int c = threadIdx.x; c < width; c += blockDim.x) smem[c] = 0.f;
  __syncthreads();
  float acc[NV][8];
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  const int total = gridDim.x * warps;
  const int per = (rows + total - 1) / total;
  const int gw = blockIdx.x * warps + warp;
  const int r0 = gw * per, r1 = min(rows, r0 + per);
  for (int row = r0; row < r1; ++row) {
    const float r = rstd[row];
    const T* xr = x + (size_t)row * width;
    const T* gr = dy + (size_t)row * width;
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < width) {
        float xv[8], gv[8], wv[8];
        load_vec(xr + c, xv);
        load_vec(gr + c, gv);
        load_vec(w + c, wv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float xh = xv[j] * r;
          acc[i][j] += gv[j] * xh;
          dot += gv[j] * (1.f + wv[j]) * xh;
        }
      }
    }
    dot = warp_sum(dot) / width;
    T* dr = dx + (size_t)row * width;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < width) {
        float xv[8], gv[8], wv[8], o[8];
        load_vec(xr + c, xv);
        load_vec(gr + c, gv);
        load_vec(w + c, wv);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = r * (gv[j] * (1.f + wv[j]) - xv[j] * r * dot);
        if (dres) {
          float rv[8];
          load_vec(dres + (size_t)row * width + c, rv);
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] += rv[j];
        }
        store8(dr + c, o);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < width)
#pragma unroll
      for (int j = 0; j < 8; ++j) atomicAdd(&smem[c + j], acc[i][j]);
  }
  __syncthreads();
  for (int c = threadIdx.x; c < width; c += blockDim.x) atomicAdd(&dw[c], smem[c]);
}

template <int NV, typename T, typename WT>
__global__ void __launch_bounds__(256) gated_fwd_kernel(const T* __restrict__ x, const T* __restrict__ z,
                                                       const WT* __restrict__ w, T* __restrict__ y,
                                                       float* __restrict__ rstd, int rows, int width, float eps) {
  const int row = blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* xr = x + (size_t)row * width;
  float v[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < width) {
      load_vec(xr + c, v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / width + eps);
  const T* zr = z + (size_t)row * width;
  T* yr = y + (size_t)row * width;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < width) {
      float wv[8], zv[8], o[8];
      load_vec(w + c, wv);
      load_vec(zr + c, zv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float n = __bfloat162float(__float2bfloat16(v[i][j] * r));
        o[j] = n * wv[j] * silu(zv[j]);
      }
      store8(yr + c, o);
    }
  }
  if (lane == 0) rstd[row] = r;
}

// n = x r; dn = dy w silu(z); dx = r (dn - n mean(dn n)); dz = dy n w silu'(z); dw += dy n silu(z)
template <int NV, typename T, typename WT>
__global__ void __launch_bounds__(512) gated_bwd_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                                                       const T* __restrict__ z, const WT* __restrict__ w,
                                                       const float* __restrict__ rstd, T* __restrict__ dx,
                                                       T* __restrict__ dz, float* __restrict__ dw, int rows, int width) {
  extern __shared__ float smem[];
  const int warps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int c = threadIdx.x; c < width; c += blockDim.x) smem[c] = 0.f;
  __syncthreads();
  float acc[NV][8];
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  const int total = gridDim.x * warps;
  const int per = (rows + total - 1) / total;
  const int gw = blockIdx.x * warps + warp;
  const int r0 = gw * per, r1 = min(rows, r0 + per);
  for (int row = r0; row < r1; ++row) {
    const float r = rstd[row];
    const size_t off = (size_t)row * width;
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < width) {
        float xv[8], gv[8], wv[8], zv[8], dzo[8];
        load_vec(x + off + c, xv);
        load_vec(dy + off + c, gv);
        load_vec(w + c, wv);
        load_vec(z + off + c, zv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float n = xv[j] * r;
          const float sg = 1.f / (1.f + __expf(-zv[j]));
          const float s = zv[j] * sg;
          acc[i][j] += gv[j] * n * s;
          dot += gv[j] * wv[j] * s * n;
          dzo[j] = gv[j] * n * wv[j] * sg * (1.f + zv[j] * (1.f - sg));
        }
        store8(dz + off + c, dzo);
      }
    }
    dot = warp_sum(dot) / width;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < width) {
        float xv[8], gv[8], wv[8], zv[8], o[8];
        load_vec(x + off + c, xv);
        load_vec(dy + off + c, gv);
        load_vec(w + c, wv);
        load_vec(z + off + c, zv);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = r * (gv[j] * wv[j] * silu(zv[j]) - xv[j] * r * dot);
        store8(dx + off + c, o);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < width)
#pragma unroll
      for (int j = 0; j < 8; ++j) atomicAdd(&smem[c + j], acc[i][j]);
  }
  __syncthreads();
  for (int c = threadIdx.x; c < width; c += blockDim.x) atomicAdd(&dw[c], smem[c]);
}

template <int NV, typename T>
__global__ void __launch_bounds__(256) lnmod_fwd_kernel(const T* __restrict__ x, const float* __restrict__ scale,
                                                       const float* __restrict__ shift, const int* __restrict__ idx,
                                                       __nv_bfloat16* __restrict__ y, float* __restrict__ mean_out,
                                                       float* __restrict__ rstd_out, int rows, int width, float eps) {
  const int row = blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* xr = x + (size_t)row * width;
  float v[NV][8];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < width) {
      load_vec(xr + c, v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) s += v[i][j];
    }
  }
  const float mu = warp_sum(s) / width;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < width)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = v[i][j] - mu;
        ss += d * d;
      }
  }
  const float r = rsqrtf(warp_sum(ss) / width + eps);
  const size_t m = (size_t)idx[row] * width;
  __nv_bfloat16* yr = y + (size_t)row * width;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < width) {
      float sc[8], sh[8], o[8];
      load8(scale + m + c, sc);
      load8(shift + m + c, sh);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = (v[i][j] - mu) * r * (1.f + sc[j]) + sh[j];
      store8(yr + c, o);
    }
  }
  if (lane == 0) {
    mean_out[row] = mu;
    rstd_out[row] = r;
  }
}

template <typename BT>
__global__ void gated_add_fwd_kernel(const float* __restrict__ x, const BT* __restrict__ branch,
                                     const float* __restrict__ gate, const int* __restrict__ idx,
                                     float* __restrict__ y, int rows, int width) {
  const size_t vecs = (size_t)rows * width / 8;
  for (size_t v = blockIdx.x * (size_t)blockDim.x + threadIdx.x; v < vecs; v += (size_t)gridDim.x * blockDim.x) {
    const size_t e = v * 8;
    const int row = (int)(e / width), c = (int)(e % width);
    float xv[8], bv[8], gv[8], o[8];
    load8(x + e, xv);
    load_vec(branch + e, bv);
    load8(gate + (size_t)idx[row] * width + c, gv);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = xv[j] + gv[j] * bv[j];
    store8(y + e, o);
  }
}


// ---- per-sample column sums of the modulation backward -------------------------------------
// dscale[m, c] = sum_{rows of sample m} dy * xhat (MODE 0, with dshift = sum dy) or
// dgate[m, c] = sum dy * branch (MODE 1). Block (32, 8): x -> 8 columns, y -> a run of MOD_RB
// rows; each thread accumulates its rows (flushing on a sample change) and adds its totals with
// one atomic per column, so a [2048, 1536] input uses ~1500 blocks instead of a few long warps.
constexpr int MOD_RB = 16;

template <int MODE, typename AT>
__global__ void __launch_bounds__(256) mod_colsum_kernel(const float* __restrict__ dy32,
                                                         const __nv_bfloat16* __restrict__ dy16,
                                                         const AT* __restrict__ a, const int* __restrict__ idx,
                                                         const float* __restrict__ mean,
                                                         const float* __restrict__ rstd, float* __restrict__ out_a,
                                                         float* __restrict__ out_b, int rows, int width) {
  const int c = (blockIdx.x * 32 + threadIdx.x) * 8;
  if (c >= width) return;
  const int r0 = (blockIdx.y * 8 + threadIdx.y) * MOD_RB;
  const int r1 = min(rows, r0 + MOD_RB);
  if (r0 >= r1) return;
  float sa[8] = {0, 0, 0, 0, 0, 0, 0, 0}, sb[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int cur = idx[r0];
  auto flush = [&](int m) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      atomicAdd(out_a + (size_t)m * width + c + j, sa[j]);
      if (MODE == 0) atomicAdd(out_b + (size_t)m * width + c + j, sb[j]);
      sa[j] = sb[j] = 0.f;
    }
  };
  for (int row = r0; row < r1; ++row) {
    const int m = idx[row];
    if (m != cur) {
      flush(cur);
      cur = m;
    }
    float g[8], av[8];
    if (dy32) load8(dy32 + (size_t)row * width + c, g);
    else load8(dy16 + (size_t)row * width + c, g);
    load_vec(a + (size_t)row * width + c, av);
    if (MODE == 0) {
      const float mu = mean[row], r = rstd[row];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        sa[j] += g[j] * (av[j] - mu) * r;
        sb[j] += g[j];
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) sa[j] += g[j] * av[j];
    }
  }
  flush(cur);
}

// dx of the modulated LayerNorm, one warp per row (grid-stride).
template <int NV, typename T>
__global__ void __launch_bounds__(256) lnmod_dx_kernel(const __nv_bfloat16* __restrict__ dy, const T* __restrict__ x,
                                                      const float* __restrict__ scale, const int* __restrict__ idx,
                                                      const float* __restrict__ mean, const float* __restrict__ rstd,
                                                      T* __restrict__ dx, int rows, int width) {
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * kWarps + (threadIdx.x >> 5); row < rows; row += gridDim.x * kWarps) {
    const int m = idx[row];
    const float mu = mean[row], r = rstd[row];
    const size_t off = (size_t)row * width, mo = (size_t)m * width;
    float xv[NV][8], gv[NV][8], sc[NV][8];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < width) {
        load_vec(x + off + c, xv[i]);
        load8(dy + off + c, gv[i]);
        load8(scale + mo + c, sc[i]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float dn = gv[i][j] * (1.f + sc[i][j]);
          s1 += dn;
          s2 += dn * (xv[i][j] - mu) * r;
        }
      }
    }
    s1 = warp_sum(s1) / width;
    s2 = warp_sum(s2) / width;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < width) {
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float xh = (xv[i][j] - mu) * r;
          o[j] = r * (gv[i][j] * (1.f + sc[i][j]) - s1 - xh * s2);
        }
        store8(dx + off + c, o);
      }
    }
  }
}

// dbranch = dy * gate[sample]
template <typename BT>
__global__ void gated_add_dbranch_kernel(const float* __restrict__ dy, const float* __restrict__ gate,
                                         const int* __restrict__ idx, BT* __restrict__ dbranch, int rows, int width) {
  const size_t vecs = (size_t)rows * width / 8;
  for (size_t v = blockIdx.x * (size_t)blockDim.x + threadIdx.x; v < vecs; v += (size_t)gridDim.x * blockDim.x) {
    const size_t e = v * 8;
    const int row = (int)(e / width), c = (int)(e % width);
    float g[8], gt[8], o[8];
    load8(dy + e, g);
    load8(gate + (size_t)idx[row] * width + c, gt);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = g[j] * gt[j];
    store8(dbranch + e, o);
  }
}


// Column sums of a bf16 / fp32 matrix (bias gradients) without an fp32 copy: block (32, 8)
// reduces 8 x BIAS_RB rows of 256 columns into partial[blockIdx.y]; a second pass adds the
// partials in a fixed order (deterministic).
constexpr int BIAS_RB = 32;

template <typename T>
__global__ void __launch_bounds__(256) colsum_partial_kernel(const T* __restrict__ x, int rows, int cols,
                                                             float* __restrict__ partial) {
  __shared__ float red[8][256 + 8];
  const int c = (blockIdx.x * 32 + threadIdx.x) * 8;
  const int r0 = (blockIdx.y * 8 + threadIdx.y) * BIAS_RB;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (c < cols)
    for (int r = r0; r < min(rows, r0 + BIAS_RB); ++r) {
      float v[8];
      load_vec(x + (size_t)r * cols + c, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += v[j];
    }
#pragma unroll
  for (int j = 0; j < 8; ++j) red[threadIdx.y][threadIdx.x * 8 + j] = acc[j];
  __syncthreads();
  const int t = threadIdx.y * 32 + threadIdx.x;   // 256 threads -> 256 columns of the block
  const int col = blockIdx.x * 256 + t;
  if (col < cols) {
    float sum = 0.f;
#pragma unroll
    for (int y = 0; y < 8; ++y) sum += red[y][t];
    partial[(size_t)blockIdx.y * cols + col] = sum;
  }
}

__global__ void colsum_finish_kernel(const float* __restrict__ partial, int parts, int cols, float* __restrict__ out) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float s = 0.f;
  for (int p = 0; p < parts; ++p) s += partial[(size_t)p * cols + c];
  out[c] = s;
}


// Complex-pair rotary embedding: (x[2i], x[2i+1]) of every head rotated by angle_i of the row
// (cos/sin [rows, half]); the backward is the rotation by -angle (sign = -1).
template <typename T>
__global__ void rope_pairs_kernel(const T* __restrict__ x, const float* __restrict__ cos_t,
                                  const float* __restrict__ sin_t, T* __restrict__ y, int rows, int heads, int hd,
                                  float sign) {
  const int half = hd / 2;
  const size_t pairs4 = (size_t)rows * heads * half / 4;     // 4 pairs = 8 elements per thread
  for (size_t v = blockIdx.x * (size_t)blockDim.x + threadIdx.x; v < pairs4; v += (size_t)gridDim.x * blockDim.x) {
    const size_t e = v * 8;                                 // element offset
    const size_t row = e / ((size_t)heads * hd);
    const int i0 = (int)((e % hd) / 2);                     // first pair index within the head
    float xv[8], o[8], c[4], s[4];
    load_vec(x + e, xv);
    const float4 cv = *reinterpret_cast<const float4*>(cos_t + row * half + i0);
    const float4 sv = *reinterpret_cast<const float4*>(sin_t + row * half + i0);
    c[0] = cv.x; c[1] = cv.y; c[2] = cv.z; c[3] = cv.w;
    s[0] = sign * sv.x; s[1] = sign * sv.y; s[2] = sign * sv.z; s[3] = sign * sv.w;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const float re = xv[2 * p], im = xv[2 * p + 1];
      o[2 * p] = re * c[p] - im * s[p];
      o[2 * p + 1] = im * c[p] + re * s[p];
    }
    store8(y + e, o);
  }
}

__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y, int rows,
                                  int half) {
  const size_t vecs = (size_t)rows * half / 8;
  for (size_t v = blockIdx.x * (size_t)blockDim.x + threadIdx.x; v < vecs; v += (size_t)gridDim.x * blockDim.x) {
    const size_t e = v * 8;
    const size_t row = e / half, c = e % half;
    float g[8], u[8], o[8];
    load8(x + row * 2 * half + c, g);
    load8(x + row * 2 * half + half + c, u);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = silu(g[j]) * u[j];
    store8(y + e, o);
  }
}

__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                  __nv_bfloat16* __restrict__ dx, int rows, int half) {
  const size_t vecs = (size_t)rows * half / 8;
  for (size_t v = blockIdx.x * (size_t)blockDim.x + threadIdx.x; v < vecs; v += (size_t)gridDim.x * blockDim.x) {
    const size_t e = v * 8;
    const size_t row = e / half, c = e % half;
    float g[8], u[8], d[8], dg[8], du[8];
    load8(x + row * 2 * half + c, g);
    load8(x + row * 2 * half + half + c, u);
    load8(dy + e, d);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float sg = 1.f / (1.f + __expf(-g[j]));
      du[j] = d[j] * g[j] * sg;
      dg[j] = d[j] * u[j] * sg * (1.f + g[j] * (1.f - sg));
    }
    store8(dx + row * 2 * half + c, dg);
    store8(dx + row * 2 * half + half + c, du);
  }
}

int grid_for(size_t vecs) {
  const size_t blocks = (vecs + 255) / 256;
  return (int)std::min<size_t>(blocks, (size_t)sm_count() * 16);
}

#define NV_DISPATCH(width, ...)                                          \
  [&] {                                                                  \
    const int nv__ = ((width) + 255) / 256;                              \
    if (nv__ <= 1) { constexpr int NV = 1; __VA_ARGS__(); }              \
    else if (nv__ <= 2) { constexpr int NV = 2; __VA_ARGS__(); }         \
    else if (nv__ <= 4) { constexpr int NV = 4; __VA_ARGS__(); }         \
    else if (nv__ <= 6) { constexpr int NV = 6; __VA_ARGS__(); }         \
    else if (nv__ <= 8) { constexpr int NV = 8; __VA_ARGS__(); }         \
    else TORCH_CHECK(false, "row width above 2048 is not supported"); \
  }()

void check_rows(const at::Tensor& x) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous(), "expected a contiguous 2-D CUDA tensor");
  TORCH_CHECK(x.size(1) % 8 == 0, "row width must be a multiple of 8");
}

}  // namespace

// Returns (y, rstd), or with `add` (same shape as x) (y, rstd, x + add) where y normalises x + add.
std::vector<at::Tensor> rms_norm_fwd(at::Tensor x, at::Tensor w, double eps, c10::optional<at::Tensor> add) {
  check_rows(x);
  const int rows = x.size(0), width = x.size(1);
  auto y = at::empty_like(x);
  auto rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  at::Tensor a, sum;
  if (add && add->defined()) {
    a = add->contiguous();
    TORCH_CHECK(a.sizes() == x.sizes() && a.scalar_type() == x.scalar_type(), "rms_norm_fwd: add must match x");
    sum = at::empty_like(x);
  }
  if (!rows) return a.defined() ? std::vector<at::Tensor>{y, rstd, sum} : std::vector<at::Tensor>{y, rstd};
  auto wc = w.contiguous();
  const int blocks = (rows + kWarps - 1) / kWarps;
  AT_DISPATCH_SWITCH(x.scalar_type(), "rms_norm_fwd", AT_DISPATCH_CASE(at::kBFloat16, [&] {
                       using T = __nv_bfloat16;
                       NV_DISPATCH(width, [&] {
                         const T* ap = a.defined() ? (const T*)a.data_ptr() : nullptr;
                         T* sp = a.defined() ? (T*)sum.data_ptr() : nullptr;
                         if (wc.scalar_type() == at::kFloat)
                           rms_fwd_kernel<NV, T, float><<<blocks, 256, 0, stream()>>>(
                               (const T*)x.data_ptr(), wc.data_ptr<float>(), (T*)y.data_ptr(), rstd.data_ptr<float>(),
                               rows, width, (float)eps, ap, sp);
                         else
                           rms_fwd_kernel<NV, T, T><<<blocks, 256, 0, stream()>>>(
                               (const T*)x.data_ptr(), (const T*)wc.data_ptr(), (T*)y.data_ptr(), rstd.data_ptr<float>(),
                               rows, width, (float)eps, ap, sp);
                       });
                     }) AT_DISPATCH_CASE(at::kFloat, [&] {
                       using T = float;
                       NV_DISPATCH(width, [&] {
                         auto wf = wc.to(at::kFloat);
                         rms_fwd_kernel<NV, T, float><<<blocks, 256, 0, stream()>>>(
                             x.data_ptr<float>(), wf.data_ptr<float>(), y.data_ptr<float>(), rstd.data_ptr<float>(), rows,
                             width, (float)eps, a.defined() ? a.data_ptr<float>() : nullptr,
                             a.defined() ? sum.data_ptr<float>() : nullptr);
                       });
                     }));
  CQB_LAUNCH_CHECK();
  count_launch();
  if (a.defined()) return {y, rstd, sum};
  return {y, rstd};
}

static int bwd_grid(int rows) { return std::max(1, std::min(sm_count(), (rows + 15) / 16)); }

std::vector<at::Tensor> rms_norm_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd,
                                     c10::optional<at::Tensor> dres_opt) {
  check_rows(x);
  at::Tensor dres;
  if (dres_opt && dres_opt->defined()) {
    dres = dres_opt->contiguous();
    TORCH_CHECK(dres.sizes() == x.sizes() && dres.scalar_type() == x.scalar_type(), "dres must match x");
  }
  const int rows = x.size(0), width = x.size(1);
  auto dx = at::empty_like(x);
  auto dw = at::zeros({width}, x.options().dtype(at::kFloat));
  if (!rows) return {dx, dw};
  auto wc = w.contiguous();
  const int grid = bwd_grid(rows);
  const size_t sm = width * sizeof(float);
  AT_DISPATCH_SWITCH(x.scalar_type(), "rms_norm_bwd", AT_DISPATCH_CASE(at::kBFloat16, [&] {
                       using T = __nv_bfloat16;
                       // bf16 rows: warp per row + deterministic two-stage weight gradient
                       const int blocks = (rows + RB_WARPS - 1) / RB_WARPS;
                       auto partial = at::empty({blocks, width}, x.options().dtype(at::kFloat));
                       const size_t psm = (size_t)RB_WARPS * width * sizeof(float);
                       NV_DISPATCH(width, [&] {
                         if (wc.scalar_type() == at::kFloat)
                           rms_bwd_rows_kernel<NV, T, float><<<blocks, RB_WARPS * 32, psm, stream()>>>(
                               (const T*)dy.data_ptr(), (const T*)x.data_ptr(), wc.data_ptr<float>(),
                               rstd.data_ptr<float>(), dres.defined() ? (const T*)dres.data_ptr() : nullptr,
                               (T*)dx.data_ptr(), partial.data_ptr<float>(), rows, width);
                         else
                           rms_bwd_rows_kernel<NV, T, T><<<blocks, RB_WARPS * 32, psm, stream()>>>(
                               (const T*)dy.data_ptr(), (const T*)x.data_ptr(), (const T*)wc.data_ptr(),
                               rstd.data_ptr<float>(), dres.defined() ? (const T*)dres.data_ptr() : nullptr,
                               (T*)dx.data_ptr(), partial.data_ptr<float>(), rows, width);
                       });
                       CQB_LAUNCH_CHECK();
                       auto stage = at::empty({RD_SLICES, width}, x.options().dtype(at::kFloat));
                       rms_dw_reduce_kernel<<<dim3((width + 31) / 32, RD_SLICES), 256, 0, stream()>>>(
                           partial.data_ptr<float>(), blocks, width, stage.data_ptr<float>());
                       CQB_LAUNCH_CHECK();
                       rms_dw_final_kernel<<<(width + 255) / 256, 256, 0, stream()>>>(stage.data_ptr<float>(), width,
                                                                                     dw.data_ptr<float>());
                       count_launch(2);
                     }) AT_DISPATCH_CASE(at::kFloat, [&] {
                       NV_DISPATCH(width, [&] {
                         auto wf = wc.to(at::kFloat);
                         rms_bwd_kernel<NV, float, float><<<grid, 512, sm, stream()>>>(
                             dy.data_ptr<float>(), x.data_ptr<float>(), wf.data_ptr<float>(), rstd.data_ptr<float>(),
                             dres.defined() ? dres.data_ptr<float>() : nullptr, dx.data_ptr<float>(),
                             dw.data_ptr<float>(), rows, width);
                       });
                     }));
  CQB_LAUNCH_CHECK();
  count_launch();
  return {dx, dw};
}

// z for the width-128 row kernels: contiguous [rows, 128], or [tokens, heads, 128] with unit inner
// strides and any token stride (the gate slice of a projection output, read in place).
static bool gate_layout(const at::Tensor& z, int rows, int width, int& heads, long& z_stride) {
  if (width != 128 || z.scalar_type() != at::kBFloat16) return false;
  if (z.dim() == 2 && z.is_contiguous() && z.size(0) == rows && z.size(1) == 128) {
    heads = 1;
    z_stride = 128;
    return true;
  }
  if (z.dim() == 3 && z.size(2) == 128 && z.stride(2) == 1 && z.stride(1) == 128 && z.size(0) * z.size(1) == rows &&
      z.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(z.data_ptr()) % 16 == 0) {
    heads = (int)z.size(1);
    z_stride = (long)z.stride(0);
    return true;
  }
  return false;
}

// x [rows, width] contiguous; z as x, or for width 128 [tokens, heads, 128] read in place.
std::vector<at::Tensor> gated_norm_fwd(at::Tensor x, at::Tensor z, at::Tensor w, double eps) {
  check_rows(x);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && z.scalar_type() == at::kBFloat16, "gated norm expects bf16");
  const int rows = x.size(0), width = x.size(1);
  auto y = at::empty_like(x);
  auto rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  if (!rows) return {y, rstd};
  auto wf = w.to(at::kFloat).contiguous();
  using T = __nv_bfloat16;
  int heads = 1;
  long zs = width;
  if (gate_layout(z, rows, width, heads, zs)) {
    gated_fwd_rows_kernel<T, float><<<(rows + 15) / 16, 256, 0, stream()>>>(
        (const T*)x.data_ptr(), (const T*)z.data_ptr(), wf.data_ptr<float>(), (T*)y.data_ptr(), rstd.data_ptr<float>(),
        rows, heads, zs, (float)eps);
    CQB_LAUNCH_CHECK();
    count_launch();
    return {y, rstd};
  }
  auto zc = z.reshape({rows, width}).contiguous();
  const int blocks = (rows + kWarps - 1) / kWarps;
  NV_DISPATCH(width, [&] {
    gated_fwd_kernel<NV, T, float><<<blocks, 256, 0, stream()>>>((const T*)x.data_ptr(), (const T*)zc.data_ptr(),
                                                                 wf.data_ptr<float>(), (T*)y.data_ptr(),
                                                                 rstd.data_ptr<float>(), rows, width, (float)eps);
  });
  CQB_LAUNCH_CHECK();
  count_launch();
  return {y, rstd};
}

// dz comes back contiguous [rows, width] whatever z's layout.
std::vector<at::Tensor> gated_norm_bwd(at::Tensor dy, at::Tensor x, at::Tensor z, at::Tensor w, at::Tensor rstd) {
  const int rows = x.size(0), width = x.size(1);
  auto dx = at::empty_like(x);
  auto dz = at::empty({rows, width}, x.options());
  auto dw = at::zeros({width}, x.options().dtype(at::kFloat));
  if (!rows) return {dx, dz, dw};
  auto wf = w.to(at::kFloat).contiguous();
  using T = __nv_bfloat16;
  int heads = 1;
  long zs = width;
  if (x.is_contiguous() && dy.is_contiguous() && gate_layout(z, rows, width, heads, zs)) {
    // GDN head rows: half-warp rows and a deterministic two-stage weight gradient
    const int blocks = std::max(1, std::min(sm_count() * GB_BLOCKS_PER_SM, (rows + 15) / 16));
    auto partial = at::empty({blocks, width}, x.options().dtype(at::kFloat));
    gated_bwd_rows_kernel<T, float><<<blocks, 256, 0, stream()>>>(
        (const T*)dy.data_ptr(), (const T*)x.data_ptr(), (const T*)z.data_ptr(), wf.data_ptr<float>(),
        rstd.data_ptr<float>(), (T*)dx.data_ptr(), (T*)dz.data_ptr(), partial.data_ptr<float>(), rows, heads, zs);
    CQB_LAUNCH_CHECK();
    auto stage = at::empty({RD_SLICES, width}, x.options().dtype(at::kFloat));
    rms_dw_reduce_kernel<<<dim3((width + 31) / 32, RD_SLICES), 256, 0, stream()>>>(partial.data_ptr<float>(), blocks,
                                                                                  width, stage.data_ptr<float>());
    CQB_LAUNCH_CHECK();
    rms_dw_final_kernel<<<1, 256, 0, stream()>>>(stage.data_ptr<float>(), width, dw.data_ptr<float>());
    CQB_LAUNCH_CHECK();
    count_launch(3);
    return {dx, dz, dw};
  }
  const int grid = bwd_grid(rows);
  auto zc = z.reshape({rows, width}).contiguous();
  NV_DISPATCH(width, [&] {
    gated_bwd_kernel<NV, T, float><<<grid, 512, width * sizeof(float), stream()>>>(
        (const T*)dy.data_ptr(), (const T*)x.data_ptr(), (const T*)zc.data_ptr(), wf.data_ptr<float>(),
        rstd.data_ptr<float>(), (T*)dx.data_ptr(), (T*)dz.data_ptr(), dw.data_ptr<float>(), rows, width);
  });
  CQB_LAUNCH_CHECK();
  count_launch();
  return {dx, dz, dw};
}

std::vector<at::Tensor> ln_modulate_fwd(at::Tensor x, at::Tensor scale, at::Tensor shift, at::Tensor idx, double eps) {
  check_rows(x);
  TORCH_CHECK(scale.scalar_type() == at::kFloat && shift.scalar_type() == at::kFloat, "modulation must be fp32");
  const int rows = x.size(0), width = x.size(1);
  auto y = at::empty({rows, width}, x.options().dtype(at::kBFloat16));
  auto mean = at::empty({rows}, x.options().dtype(at::kFloat));
  auto rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  if (!rows) return {y, mean, rstd};
  const int blocks = (rows + kWarps - 1) / kWarps;
  AT_DISPATCH_SWITCH(x.scalar_type(), "ln_modulate_fwd", AT_DISPATCH_CASE(at::kBFloat16, [&] {
                       using T = __nv_bfloat16;
                       NV_DISPATCH(width, [&] {
                         lnmod_fwd_kernel<NV, T><<<blocks, 256, 0, stream()>>>(
                             (const T*)x.data_ptr(), scale.data_ptr<float>(), shift.data_ptr<float>(),
                             idx.data_ptr<int>(), (__nv_bfloat16*)y.data_ptr(), mean.data_ptr<float>(),
                             rstd.data_ptr<float>(), rows, width, (float)eps);
                       });
                     }) AT_DISPATCH_CASE(at::kFloat, [&] {
                       NV_DISPATCH(width, [&] {
                         lnmod_fwd_kernel<NV, float><<<blocks, 256, 0, stream()>>>(
                             x.data_ptr<float>(), scale.data_ptr<float>(), shift.data_ptr<float>(), idx.data_ptr<int>(),
                             (__nv_bfloat16*)y.data_ptr(), mean.data_ptr<float>(), rstd.data_ptr<float>(), rows, width,
                             (float)eps);
                       });
                     }));
  CQB_LAUNCH_CHECK();
  count_launch();
  return {y, mean, rstd};
}

std::vector<at::Tensor> ln_modulate_bwd(at::Tensor dy, at::Tensor x, at::Tensor scale, at::Tensor idx, at::Tensor mean,
                                        at::Tensor rstd) {
  const int rows = x.size(0), width = x.size(1);
  auto dx = at::empty_like(x);
  auto dscale = at::zeros_like(scale);
  auto dshift = at::zeros_like(scale);
  if (!rows) return {dx, dscale, dshift};
  auto dyc = dy.to(at::kBFloat16).contiguous();
  const int row_blocks = std::min((rows + kWarps - 1) / kWarps, sm_count() * 16);
  const dim3 cgrid((width / 8 + 31) / 32, (rows + 8 * MOD_RB - 1) / (8 * MOD_RB));
  AT_DISPATCH_SWITCH(x.scalar_type(), "ln_modulate_bwd", AT_DISPATCH_CASE(at::kBFloat16, [&] {
                       using T = __nv_bfloat16;
                       NV_DISPATCH(width, [&] {
                         lnmod_dx_kernel<NV, T><<<row_blocks, 256, 0, stream()>>>(
                             (const __nv_bfloat16*)dyc.data_ptr(), (const T*)x.data_ptr(), scale.data_ptr<float>(),
                             idx.data_ptr<int>(), mean.data_ptr<float>(), rstd.data_ptr<float>(), (T*)dx.data_ptr(),
                             rows, width);
                       });
                       mod_colsum_kernel<0, T><<<cgrid, dim3(32, 8), 0, stream()>>>(
                           nullptr, (const __nv_bfloat16*)dyc.data_ptr(), (const T*)x.data_ptr(), idx.data_ptr<int>(),
                           mean.data_ptr<float>(), rstd.data_ptr<float>(), dscale.data_ptr<float>(),
                           dshift.data_ptr<float>(), rows, width);
                     }) AT_DISPATCH_CASE(at::kFloat, [&] {
                       NV_DISPATCH(width, [&] {
                         lnmod_dx_kernel<NV, float><<<row_blocks, 256, 0, stream()>>>(
                             (const __nv_bfloat16*)dyc.data_ptr(), x.data_ptr<float>(), scale.data_ptr<float>(),
                             idx.data_ptr<int>(), mean.data_ptr<float>(), rstd.data_ptr<float>(), dx.data_ptr<float>(),
                             rows, width);
                       });
                       mod_colsum_kernel<0, float><<<cgrid, dim3(32, 8), 0, stream()>>>(
                           nullptr, (const __nv_bfloat16*)dyc.data_ptr(), x.data_ptr<float>(), idx.data_ptr<int>(),
                           mean.data_ptr<float>(), rstd.data_ptr<float>(), dscale.data_ptr<float>(),
                           dshift.data_ptr<float>(), rows, width);
                     }));
  CQB_LAUNCH_CHECK();
  count_launch(2);
  return {dx, dscale, dshift};
}

at::Tensor gated_add_fwd(at::Tensor x, at::Tensor branch, at::Tensor gate, at::Tensor idx) {
  TORCH_CHECK(x.scalar_type() == at::kFloat && gate.scalar_type() == at::kFloat, "gated add expects fp32 x and gate");
  const int rows = x.size(0), width = x.size(1);
  auto y = at::empty_like(x);
  if (!rows) return y;
  auto b = branch.contiguous();
  const int grid = grid_for((size_t)rows * width / 8);
  if (b.scalar_type() == at::kBFloat16)
    gated_add_fwd_kernel<__nv_bfloat16><<<grid, 256, 0, stream()>>>(
        x.data_ptr<float>(), (const __nv_bfloat16*)b.data_ptr(), gate.data_ptr<float>(), idx.data_ptr<int>(),
        y.data_ptr<float>(), rows, width);
  else
    gated_add_fwd_kernel<float><<<grid, 256, 0, stream()>>>(x.data_ptr<float>(), b.to(at::kFloat).data_ptr<float>(),
                                                            gate.data_ptr<float>(), idx.data_ptr<int>(),
                                                            y.data_ptr<float>(), rows, width);
  CQB_LAUNCH_CHECK();
  count_launch();
  return y;
}

std::vector<at::Tensor> gated_add_bwd(at::Tensor dy, at::Tensor branch, at::Tensor gate, at::Tensor idx) {
  const int rows = dy.size(0), width = dy.size(1);
  auto dgate = at::zeros_like(gate);
  auto dbranch = at::empty_like(branch);
  if (!rows) return {dbranch, dgate};
  auto dyc = dy.to(at::kFloat).contiguous();
  const int grid = grid_for((size_t)rows * width / 8);
  const dim3 cgrid((width / 8 + 31) / 32, (rows + 8 * MOD_RB - 1) / (8 * MOD_RB));
  if (branch.scalar_type() == at::kBFloat16) {
    auto b = branch.contiguous();
    gated_add_dbranch_kernel<__nv_bfloat16><<<grid, 256, 0, stream()>>>(
        dyc.data_ptr<float>(), gate.data_ptr<float>(), idx.data_ptr<int>(), (__nv_bfloat16*)dbranch.data_ptr(), rows,
        width);
    mod_colsum_kernel<1, __nv_bfloat16><<<cgrid, dim3(32, 8), 0, stream()>>>(
        dyc.data_ptr<float>(), nullptr, (const __nv_bfloat16*)b.data_ptr(), idx.data_ptr<int>(), nullptr, nullptr,
        dgate.data_ptr<float>(), nullptr, rows, width);
  } else {
    auto b = branch.to(at::kFloat).contiguous();
    gated_add_dbranch_kernel<float><<<grid, 256, 0, stream()>>>(dyc.data_ptr<float>(), gate.data_ptr<float>(),
                                                                idx.data_ptr<int>(), dbranch.data_ptr<float>(), rows,
                                                                width);
    mod_colsum_kernel<1, float><<<cgrid, dim3(32, 8), 0, stream()>>>(dyc.data_ptr<float>(), nullptr,
                                                                     b.data_ptr<float>(), idx.data_ptr<int>(), nullptr,
                                                                     nullptr, dgate.data_ptr<float>(), nullptr, rows,
                                                                     width);
  }
  CQB_LAUNCH_CHECK();
  count_launch(2);
  return {dbranch, dgate};
}

at::Tensor swiglu_fwd(at::Tensor x) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.is_contiguous(), "swiglu expects bf16 2-D");
  const int rows = x.size(0), half = x.size(1) / 2;
  TORCH_CHECK(half % 8 == 0, "swiglu half width must be a multiple of 8");
  auto y = at::empty({rows, half}, x.options());
  if (!rows) return y;
  swiglu_fwd_kernel<<<grid_for((size_t)rows * half / 8), 256, 0, stream()>>>(
      (const __nv_bfloat16*)x.data_ptr(), (__nv_bfloat16*)y.data_ptr(), rows, half);
  CQB_LAUNCH_CHECK();
  count_launch();
  return y;
}

at::Tensor swiglu_bwd(at::Tensor dy, at::Tensor x) {
  const int rows = x.size(0), half = x.size(1) / 2;
  auto dx = at::empty_like(x);
  if (!rows) return dx;
  auto d = dy.contiguous();
  swiglu_bwd_kernel<<<grid_for((size_t)rows * half / 8), 256, 0, stream()>>>(
      (const __nv_bfloat16*)d.data_ptr(), (const __nv_bfloat16*)x.data_ptr(), (__nv_bfloat16*)dx.data_ptr(), rows,
      half);
  CQB_LAUNCH_CHECK();
  count_launch();
  return dx;
}


// fp32 [cols] = sum over rows of x (bf16 or fp32 [rows, cols], cols % 8 == 0).
at::Tensor column_sum(at::Tensor x) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.size(1) % 8 == 0, "column_sum: 2-D, cols % 8 == 0");
  auto xc = x.contiguous();
  const int rows = xc.size(0), cols = xc.size(1);
  auto out = at::empty({cols}, xc.options().dtype(at::kFloat));
  if (!rows) return out.zero_();
  const dim3 grid((cols / 8 + 31) / 32, (rows + 8 * BIAS_RB - 1) / (8 * BIAS_RB));
  auto partial = at::empty({(long)grid.y, cols}, out.options());
  if (xc.scalar_type() == at::kBFloat16)
    colsum_partial_kernel<__nv_bfloat16><<<grid, dim3(32, 8), 0, stream()>>>(
        (const __nv_bfloat16*)xc.data_ptr(), rows, cols, partial.data_ptr<float>());
  else
    colsum_partial_kernel<float><<<grid, dim3(32, 8), 0, stream()>>>(xc.to(at::kFloat).data_ptr<float>(), rows, cols,
                                                                      partial.data_ptr<float>());
  colsum_finish_kernel<<<(cols + 255) / 256, 256, 0, stream()>>>(partial.data_ptr<float>(), grid.y, cols,
                                                                 out.data_ptr<float>());
  CQB_LAUNCH_CHECK();
  count_launch(2);
  return out;
}


// x [rows, heads, hd] (bf16/fp32, contiguous, hd % 8 == 0), cos/sin fp32 [rows, hd/2].
at::Tensor rope_pairs(at::Tensor x, at::Tensor cos_t, at::Tensor sin_t, bool inverse) {
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && x.dim() == 3 && x.size(2) % 8 == 0, "rope_pairs: x [rows, H, hd]");
  auto c = cos_t.to(at::kFloat).contiguous(), sn = sin_t.to(at::kFloat).contiguous();
  TORCH_CHECK(c.dim() == 2 && c.size(0) == x.size(0) && c.size(1) == x.size(2) / 2 && sn.sizes() == c.sizes(),
              "rope_pairs: cos/sin [rows, hd/2]");
  auto y = at::empty_like(x);
  const int rows = x.size(0), heads = x.size(1), hd = x.size(2);
  if (!rows) return y;
  const int grid = grid_for((size_t)rows * heads * hd / 8);
  const float sign = inverse ? -1.f : 1.f;
  if (x.scalar_type() == at::kBFloat16)
    rope_pairs_kernel<__nv_bfloat16><<<grid, 256, 0, stream()>>>((const __nv_bfloat16*)x.data_ptr(), c.data_ptr<float>(),
                                                                sn.data_ptr<float>(), (__nv_bfloat16*)y.data_ptr(),
                                                                rows, heads, hd, sign);
  else
    rope_pairs_kernel<float><<<grid, 256, 0, stream()>>>(x.data_ptr<float>(), c.data_ptr<float>(), sn.data_ptr<float>(),
                                                         y.data_ptr<float>(), rows, heads, hd, sign);
  CQB_LAUNCH_CHECK();
  count_launch();
  return y;
}

}  // namespace cqb
