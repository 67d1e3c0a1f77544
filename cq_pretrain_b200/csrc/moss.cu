// Pointwise ops of the MOSS-Image-Base renderer, forward and backward, for sm_100a
// (reference models/moss_kernels.py:11-130, where they are Triton kernels):
//   situ(h, g)          = (4 tanh(g / 4) sigmoid(g)) * (25 tanh(h / 25))
//   affine(h, s, t)     = h (1 + s) + t
//   gated_add(h, b, g)  = h + b g
// Operands are [rows, width] with a row stride each (strided column slices of a fused QKV or
// FFN projection are read in place) and a contiguous width; outputs and gradients are dense.
// Arithmetic is fp32; each output is rounded once to the activation dtype. One thread handles
// eight consecutive elements (16-byte vectors of bf16).
#include "common.cuh"

namespace cqb {

namespace {

enum MossKind { kSitu = 0, kAffine = 1, kGatedAdd = 2 };

struct Operand {
  const void* p;
  long ld;  // row stride in elements
};

template <typename T>
__device__ __forceinline__ void load_row8(const Operand& o, long r, int c, float* v) {
  load8(reinterpret_cast<const T*>(o.p) + r * o.ld + c, v);
}

__device__ __forceinline__ void situ_terms(float h, float g, float& act, float& sq, float& th, float& tg, float& sg) {
  tg = tanhf(g * 0.25f);
  th = tanhf(h * 0.04f);
  sg = 1.f / (1.f + __expf(-g));
  act = 4.f * tg * sg;  // gate factor
  sq = 25.f * th;       // soft-clipped hidden
}

template <typename T, int KIND>
__global__ void moss_fwd_kernel(Operand a, Operand b, Operand c, T* __restrict__ y, long rows, int width) {
  const int vpr = width / 8;
  const long total = rows * vpr;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long r = i / vpr;
    const int col = (int)(i % vpr) * 8;
    float va[8], vb[8], vc[8], out[8];
    load_row8<T>(a, r, col, va);
    load_row8<T>(b, r, col, vb);
    if (KIND != kSitu) load_row8<T>(c, r, col, vc);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (KIND == kSitu) {
        float act, sq, th, tg, sg;
        situ_terms(va[j], vb[j], act, sq, th, tg, sg);
        out[j] = act * sq;
      } else if (KIND == kAffine) {
        out[j] = va[j] * (1.f + vb[j]) + vc[j];
      } else {
        out[j] = va[j] + vb[j] * vc[j];
      }
    }
    store8(y + r * width + col, out);
  }
}

// Gradients: situ -> (dh, dg); affine -> (dh, ds) (dt = dy); gated_add -> (db, dg) (dh = dy).
template <typename T, int KIND>
__global__ void moss_bwd_kernel(Operand a, Operand b, Operand c, Operand dy, T* __restrict__ d0, T* __restrict__ d1,
                                long rows, int width) {
  const int vpr = width / 8;
  const long total = rows * vpr;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long r = i / vpr;
    const int col = (int)(i % vpr) * 8;
    float g[8], va[8], vb[8], o0[8], o1[8];
    load_row8<T>(dy, r, col, g);
    if (KIND == kGatedAdd) {
      load_row8<T>(b, r, col, va);  // branch
      load_row8<T>(c, r, col, vb);  // gate
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        o0[j] = g[j] * vb[j];
        o1[j] = g[j] * va[j];
      }
    } else {
      load_row8<T>(a, r, col, va);
      load_row8<T>(b, r, col, vb);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (KIND == kSitu) {
          float act, sq, th, tg, sg;
          situ_terms(va[j], vb[j], act, sq, th, tg, sg);
          o0[j] = g[j] * act * (1.f - th * th);
          o1[j] = g[j] * sq * ((1.f - tg * tg) * sg + 4.f * tg * sg * (1.f - sg));
        } else {
          o0[j] = g[j] * (1.f + vb[j]);
          o1[j] = g[j] * va[j];
        }
      }
    }
    store8(d0 + r * width + col, o0);
    store8(d1 + r * width + col, o1);
  }
}

Operand operand(const at::Tensor& t, const at::Tensor& like) {
  TORCH_CHECK(t.is_cuda() && t.dim() == 2 && t.size(0) == like.size(0) && t.size(1) == like.size(1) &&
                  t.scalar_type() == like.scalar_type() && t.stride(1) == 1,
              "moss pointwise: operands must be [rows, width] with a contiguous width and one dtype");
  TORCH_CHECK(t.size(0) <= 1 || (t.stride(0) * t.element_size()) % 16 == 0, "moss pointwise: row stride alignment");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, "moss pointwise: base alignment");
  return Operand{t.data_ptr(), t.size(0) > 1 ? t.stride(0) : t.size(1)};
}

int grid_for(long vectors) { return (int)std::max<long>(1, std::min<long>((vectors + 255) / 256, (long)sm_count() * 8)); }

#define MOSS_DISPATCH(kind, T, ...)                                                 \
  [&] {                                                                             \
    if (kind == kSitu) { constexpr int K = kSitu; __VA_ARGS__(); }                  \
    else if (kind == kAffine) { constexpr int K = kAffine; __VA_ARGS__(); }         \
    else { constexpr int K = kGatedAdd; __VA_ARGS__(); }                            \
  }()

}  // namespace

// kind: 0 situ(a=hidden, b=gate), 1 affine(a=hidden, b=scale, c=shift), 2 gated_add(a=hidden,
// b=branch, c=gate). c is ignored for situ.
at::Tensor moss_pointwise_fwd(int64_t kind, at::Tensor a, at::Tensor b, at::Tensor c) {
  TORCH_CHECK(kind >= 0 && kind <= 2, "moss pointwise kind");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 || a.scalar_type() == at::kFloat, "moss pointwise: bf16 or fp32");
  TORCH_CHECK(a.dim() == 2 && a.size(1) % 8 == 0, "moss pointwise: width must be a multiple of 8");
  const Operand oa = operand(a, a), ob = operand(b, a), oc = kind == kSitu ? oa : operand(c, a);
  auto y = at::empty({a.size(0), a.size(1)}, a.options());
  const long rows = a.size(0);
  const int width = (int)a.size(1);
  if (rows == 0) return y;
  const int grid = grid_for(rows * (width / 8));
  MOSS_DISPATCH(kind, T, [&] {
    if (a.scalar_type() == at::kBFloat16)
      moss_fwd_kernel<__nv_bfloat16, K><<<grid, 256, 0, stream()>>>(oa, ob, oc, (__nv_bfloat16*)y.data_ptr(), rows, width);
    else
      moss_fwd_kernel<float, K><<<grid, 256, 0, stream()>>>(oa, ob, oc, y.data_ptr<float>(), rows, width);
  });
  CQB_LAUNCH_CHECK();
  count_launch();
  return y;
}

// Returns the two computed gradients (situ: dh, dg; affine: dh, dscale; gated_add: dbranch, dgate).
std::vector<at::Tensor> moss_pointwise_bwd(int64_t kind, at::Tensor dy, at::Tensor a, at::Tensor b, at::Tensor c) {
  TORCH_CHECK(kind >= 0 && kind <= 2, "moss pointwise kind");
  TORCH_CHECK(a.dim() == 2 && a.size(1) % 8 == 0, "moss pointwise: width must be a multiple of 8");
  const Operand og = operand(dy, a), oa = operand(a, a), ob = operand(b, a),
                oc = kind == kSitu ? oa : operand(c, a);
  auto d0 = at::empty({a.size(0), a.size(1)}, a.options());
  auto d1 = at::empty({a.size(0), a.size(1)}, a.options());
  const long rows = a.size(0);
  const int width = (int)a.size(1);
  if (rows == 0) return {d0, d1};
  const int grid = grid_for(rows * (width / 8));
  MOSS_DISPATCH(kind, T, [&] {
    if (a.scalar_type() == at::kBFloat16)
      moss_bwd_kernel<__nv_bfloat16, K><<<grid, 256, 0, stream()>>>(oa, ob, oc, og, (__nv_bfloat16*)d0.data_ptr(),
                                                                    (__nv_bfloat16*)d1.data_ptr(), rows, width);
    else
      moss_bwd_kernel<float, K><<<grid, 256, 0, stream()>>>(oa, ob, oc, og, d0.data_ptr<float>(), d1.data_ptr<float>(),
                                                           rows, width);
  });
  CQB_LAUNCH_CHECK();
  count_launch();
  return {d0, d1};
}

}  // namespace cqb
