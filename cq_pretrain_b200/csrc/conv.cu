// Causal depthwise short convolution + SiLU over packed documents (GDN q/k/v mixing), and the
// GDN chunk-layout gathers.
//
//  conv:   y[t, c] = silu( sum_i w[c, i] * x[t - (K-1) + i, c] ),  taps before the row's
//          document start read zero (pos[t] = index of row t inside its document);
//  bwd:    g = dy * silu'(pre);  dx[t, c] = sum_s w[c, K-1-s] g[t+s, c] (same document);
//          dw[c, i] = sum_t g[t, c] x[t-(K-1)+i, c]  (per-thread partials, one atomic each).
//  chunks: rows of [E, H, D] events are gathered into the zero-padded chunk layout
//          [Nc, H, 64, D], optionally L2-normalised on the way (rsqrt norms saved), and
//          scattered back (with the L2-norm backward fused).
#include "common.cuh"

namespace cqb {

namespace {

template <int K>
__global__ void conv_fwd_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w,
                                const int* __restrict__ pos, __nv_bfloat16* __restrict__ y, int n, int C) {
  const int vecs = C / 8;
  const size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (idx >= (size_t)n * vecs) return;
  const int t = (int)(idx / vecs), c = (int)(idx % vecs) * 8;
  const int p = pos[t];
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < K; ++i) {
    const int back = K - 1 - i;
    if (back <= p) {
      float xv[8];
      load8(x + (size_t)(t - back) * C + c, xv);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += w[(c + j) * K + i] * xv[j];
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = silu(acc[j]);
  store8(y + (size_t)t * C + c, acc);
}

template <int K>
__global__ void conv_grad_pre_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                     const float* __restrict__ w, const int* __restrict__ pos, float* __restrict__ g,
                                     int n, int C) {
  const int vecs = C / 8;
  const size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (idx >= (size_t)n * vecs) return;
  const int t = (int)(idx / vecs), c = (int)(idx % vecs) * 8;
  const int p = pos[t];
  float pre[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < K; ++i) {
    const int back = K - 1 - i;
    if (back <= p) {
      float xv[8];
      load8(x + (size_t)(t - back) * C + c, xv);
#pragma unroll
      for (int j = 0; j < 8; ++j) pre[j] += w[(c + j) * K + i] * xv[j];
    }
  }
  float d[8], o[8];
  load8(dy + (size_t)t * C + c, d);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float sg = 1.f / (1.f + __expf(-pre[j]));
    o[j] = d[j] * sg * (1.f + pre[j] * (1.f - sg));
  }
  store8(g + (size_t)t * C + c, o);
}

// One thread: 8 channels x ROWS consecutive rows; dw partials in registers.
template <int K, int ROWS>
__global__ void conv_bwd_kernel(const float* __restrict__ g, const __nv_bfloat16* __restrict__ x,
                                const float* __restrict__ w, const int* __restrict__ pos,
                                __nv_bfloat16* __restrict__ dx, float* __restrict__ dw, int n, int C) {
  const int vecs = C / 8;
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= vecs) return;
  const int c = v * 8;
  const int t0 = blockIdx.y * ROWS, t1 = min(n, t0 + ROWS);
  float wl[K][8];
#pragma unroll
  for (int i = 0; i < K; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) wl[i][j] = w[(c + j) * K + i];
  float part[K][8];
#pragma unroll
  for (int i = 0; i < K; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) part[i][j] = 0.f;
  for (int t = t0; t < t1; ++t) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int s = 0; s < K; ++s) {
      const int tt = t + s;
      if (tt < n && pos[tt] >= s) {
        float gv[8];
        load8(g + (size_t)tt * C + c, gv);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += wl[K - 1 - s][j] * gv[j];
      }
    }
    store8(dx + (size_t)t * C + c, acc);
    float gt[8];
    load8(g + (size_t)t * C + c, gt);
    const int p = pos[t];
#pragma unroll
    for (int i = 0; i < K; ++i) {
      const int back = K - 1 - i;
      if (back <= p) {
        float xv[8];
        load8(x + (size_t)(t - back) * C + c, xv);
#pragma unroll
        for (int j = 0; j < 8; ++j) part[i][j] += gt[j] * xv[j];
      }
    }
  }
#pragma unroll
  for (int i = 0; i < K; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) atomicAdd(dw + (c + j) * K + i, part[i][j]);
}

// out[n, h, c, :] = normalise?(x[idx[n*64 + c], h, :]) (zero when idx < 0); r[e, h] = rsqrt norm.
template <int D>
__global__ void chunk_gather_kernel(const __nv_bfloat16* __restrict__ x, const long* __restrict__ idx,
                                    __nv_bfloat16* __restrict__ out, float* __restrict__ rnorm, int slots, int H,
                                    float scale, int normalize) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= slots * H) return;
  const int slot = warp / H, h = warp % H;
  const int chunk = slot / 64, c = slot % 64;
  const long e = idx[slot];
  constexpr int PER = D / 32;  // elements per lane (4 for D=128)
  float v[PER];
  if (e >= 0) {
    const __nv_bfloat16* src = x + ((size_t)e * H + h) * D + lane * PER;
#pragma unroll
    for (int j = 0; j < PER; ++j) v[j] = __bfloat162float(src[j]);
  } else {
#pragma unroll
    for (int j = 0; j < PER; ++j) v[j] = 0.f;
  }
  if (normalize) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) ss += v[j] * v[j];
    ss = warp_sum(ss);
    const float r = rsqrtf(ss + 1e-6f);
#pragma unroll
    for (int j = 0; j < PER; ++j) v[j] *= r * scale;
    if (lane == 0 && e >= 0) rnorm[(size_t)e * H + h] = r;
  }
  __nv_bfloat16* dst = out + (((size_t)chunk * H + h) * 64 + c) * D + lane * PER;
#pragma unroll
  for (int j = 0; j < PER; ++j) dst[j] = __float2bfloat16(v[j]);
}

// dx[e, h, :] = L2-norm backward of dy_chunks[slot(e)] (fp32) or a plain copy when !normalize.
__device__ __forceinline__ float as_float(float v) { return v; }
__device__ __forceinline__ float as_float(__nv_bfloat16 v) { return __bfloat162float(v); }

template <int D, typename T>
__global__ void chunk_scatter_kernel(const T* __restrict__ dyc, const long* __restrict__ slot_of,
                                     const __nv_bfloat16* __restrict__ x, const float* __restrict__ rnorm,
                                     __nv_bfloat16* __restrict__ dx, int events, int H, float scale, int normalize) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= events * H) return;
  const int e = warp / H, h = warp % H;
  const long slot = slot_of[e];
  const int chunk = (int)(slot / 64), c = (int)(slot % 64);
  constexpr int PER = D / 32;
  const T* src = dyc + (((size_t)chunk * H + h) * 64 + c) * D + lane * PER;
  float g[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) g[j] = as_float(src[j]);
  __nv_bfloat16* dst = dx + ((size_t)e * H + h) * D + lane * PER;
  if (normalize) {
    const float r = rnorm[(size_t)e * H + h];
    const __nv_bfloat16* xs = x + ((size_t)e * H + h) * D + lane * PER;
    float xv[PER], dot = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      xv[j] = __bfloat162float(xs[j]);
      dot += xv[j] * g[j];
    }
    dot = warp_sum(dot);
#pragma unroll
    for (int j = 0; j < PER; ++j) dst[j] = __float2bfloat16(scale * (r * g[j] - r * r * r * xv[j] * dot));
  } else {
#pragma unroll
    for (int j = 0; j < PER; ++j) dst[j] = __float2bfloat16(g[j]);
  }
}

int blocks_for(size_t threads, int per = 256) { return (int)((threads + per - 1) / per); }

}  // namespace

at::Tensor conv_fwd(at::Tensor x, at::Tensor w, at::Tensor pos) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2 && x.size(1) % 8 == 0,
              "x: contiguous bf16 [n, C], C % 8 == 0");
  TORCH_CHECK(pos.scalar_type() == at::kInt && pos.numel() == x.size(0), "pos: int32 [n]");
  const int n = x.size(0), C = x.size(1), K = w.size(1);
  auto wf = w.to(at::kFloat).contiguous();
  auto y = at::empty_like(x);
  if (!n) return y;
  TORCH_CHECK(K == 4, "only kernel size 4 is compiled");
  conv_fwd_kernel<4><<<blocks_for((size_t)n * C / 8), 256, 0, stream()>>>(
      (const __nv_bfloat16*)x.data_ptr(), wf.data_ptr<float>(), pos.data_ptr<int>(), (__nv_bfloat16*)y.data_ptr(), n, C);
  CQB_LAUNCH_CHECK();
  count_launch();
  return y;
}

std::vector<at::Tensor> conv_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor pos) {
  const int n = x.size(0), C = x.size(1), K = w.size(1);
  auto wf = w.to(at::kFloat).contiguous();
  auto dx = at::empty_like(x);
  auto dw = at::zeros({C, K}, x.options().dtype(at::kFloat));
  if (!n) return {dx, dw};
  TORCH_CHECK(K == 4, "only kernel size 4 is compiled");
  auto g = at::empty({n, C}, x.options().dtype(at::kFloat));
  auto d = dy.contiguous();
  conv_grad_pre_kernel<4><<<blocks_for((size_t)n * C / 8), 256, 0, stream()>>>(
      (const __nv_bfloat16*)d.data_ptr(), (const __nv_bfloat16*)x.data_ptr(), wf.data_ptr<float>(),
      pos.data_ptr<int>(), g.data_ptr<float>(), n, C);
  constexpr int ROWS = 64;
  dim3 grid((C / 8 + 127) / 128, (n + ROWS - 1) / ROWS);
  conv_bwd_kernel<4, ROWS><<<grid, 128, 0, stream()>>>(g.data_ptr<float>(), (const __nv_bfloat16*)x.data_ptr(),
                                                     wf.data_ptr<float>(), pos.data_ptr<int>(),
                                                     (__nv_bfloat16*)dx.data_ptr(), dw.data_ptr<float>(), n, C);
  CQB_LAUNCH_CHECK();
  count_launch(2);
  return {dx, dw};
}

std::vector<at::Tensor> chunk_gather(at::Tensor x, at::Tensor idx, int64_t chunks, bool normalize, double scale) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 3 && x.size(2) == 128,
              "x: bf16 [E, H, 128]");
  TORCH_CHECK(idx.scalar_type() == at::kLong && idx.numel() == chunks * 64, "idx: int64 [chunks * 64]");
  const int E = x.size(0), H = x.size(1);
  const int slots = idx.numel();
  auto out = at::empty({chunks, H, 64, 128}, x.options());
  auto r = at::empty({E, H}, x.options().dtype(at::kFloat));
  if (!slots) return {out, r};
  const size_t threads = (size_t)slots * H * 32;
  chunk_gather_kernel<128><<<blocks_for(threads), 256, 0, stream()>>>(
      (const __nv_bfloat16*)x.data_ptr(), (const long*)idx.data_ptr(), (__nv_bfloat16*)out.data_ptr(),
      r.data_ptr<float>(), slots, H, (float)scale, normalize ? 1 : 0);
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
  if (normalize)
    TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && rnorm.scalar_type() == at::kFloat,
                "normalize needs bf16 x and fp32 rnorm");
  const int E = slot_of.numel(), H = dyc.size(1);
  auto dx = at::empty({E, H, 128}, dyc.options().dtype(at::kBFloat16));
  if (!E) return dx;
  const size_t threads = (size_t)E * H * 32;
  const long* so = (const long*)slot_of.data_ptr();
  const __nv_bfloat16* xp = normalize ? (const __nv_bfloat16*)x.data_ptr() : nullptr;
  const float* rp = normalize ? rnorm.data_ptr<float>() : nullptr;
  if (dyc.scalar_type() == at::kFloat)
    chunk_scatter_kernel<128, float><<<blocks_for(threads), 256, 0, stream()>>>(
        dyc.data_ptr<float>(), so, xp, rp, (__nv_bfloat16*)dx.data_ptr(), E, H, (float)scale, normalize ? 1 : 0);
  else
    chunk_scatter_kernel<128, __nv_bfloat16><<<blocks_for(threads), 256, 0, stream()>>>(
        (const __nv_bfloat16*)dyc.data_ptr(), so, xp, rp, (__nv_bfloat16*)dx.data_ptr(), E, H, (float)scale,
        normalize ? 1 : 0);
  CQB_LAUNCH_CHECK();
  count_launch();
  return dx;
}

}  // namespace cqb
