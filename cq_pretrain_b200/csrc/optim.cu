// Multi-tensor optimizer kernels for the ZeRO-1 distributed optimizer: one launch updates every
// owned shard (AdamW with decoupled weight decay, gradient scaling by a device-resident clip
// coefficient, and the write of the updated parameter in its training dtype), and one launch
// pair computes the global squared gradient norm in a fixed reduction order.
//
// Tensors are described by a device table; work is split into fixed 16K-element chunks that a
// persistent grid walks (148 SMs x 8 blocks at most), so thousands of shards cost one launch.
#include "common.cuh"

#include <mutex>
#include <unordered_map>

namespace cqb {

namespace {

constexpr int OPT_CHUNK = 16384;
constexpr int OPT_THREADS = 256;

struct AdamTensor {
  float* p;
  const float* g;
  float* m;
  float* v;
  const uint8_t* decay;
  void* out;      // parameter in its training dtype (bf16 or fp32); may be null
  float* ema;     // EMA shadow of the master (fp32), lerped toward the updated master; may be null
  long n;
  int out_bf16;
  int vec;        // every pointer is 16-byte aligned (8-byte for the bf16 output)
};

struct Chunk {
  int tensor;
  int pad;
  long start;
};

struct AdamScalars {
  float lr, b1, b2, eps, wd, bc1, bc2;
  float ema_w;    // 1 - EMA decay
};

__device__ __forceinline__ void adam_one(float& p, float g, float& m, float& v, uint8_t decay, float gs,
                                         const AdamScalars& a) {
  g *= gs;
  m = a.b1 * m + (1.f - a.b1) * g;
  v = a.b2 * v + (1.f - a.b2) * g * g;
  const float update = (m / a.bc1) / (sqrtf(v / a.bc2) + a.eps);
  p = p * (1.f - a.lr * a.wd * (float)decay) - a.lr * update;
}

__global__ void __launch_bounds__(OPT_THREADS) adamw_kernel(const AdamTensor* __restrict__ tensors,
                                                             const Chunk* __restrict__ chunks, int num_chunks,
                                                             const float* __restrict__ gscale, AdamScalars a) {
  const float gs = *gscale;
  for (int ci = blockIdx.x; ci < num_chunks; ci += gridDim.x) {
    const Chunk ch = chunks[ci];
    const AdamTensor t = tensors[ch.tensor];
    const long end = min(t.n, ch.start + (long)OPT_CHUNK);
    if (t.vec) {
      for (long i = ch.start + 4 * threadIdx.x; i < end; i += 4 * OPT_THREADS) {
        if (i + 4 <= end) {
          float4 p = *reinterpret_cast<const float4*>(t.p + i);
          const float4 g = __ldcs(reinterpret_cast<const float4*>(t.g + i));
          float4 m = *reinterpret_cast<const float4*>(t.m + i);
          float4 v = *reinterpret_cast<const float4*>(t.v + i);
          const uchar4 d = *reinterpret_cast<const uchar4*>(t.decay + i);
          adam_one(p.x, g.x, m.x, v.x, d.x, gs, a);
          adam_one(p.y, g.y, m.y, v.y, d.y, gs, a);
          adam_one(p.z, g.z, m.z, v.z, d.z, gs, a);
          adam_one(p.w, g.w, m.w, v.w, d.w, gs, a);
          *reinterpret_cast<float4*>(t.p + i) = p;
          *reinterpret_cast<float4*>(t.m + i) = m;
          *reinterpret_cast<float4*>(t.v + i) = v;
          if (t.ema) {
            float4 e = *reinterpret_cast<const float4*>(t.ema + i);
            e.x += a.ema_w * (p.x - e.x);
            e.y += a.ema_w * (p.y - e.y);
            e.z += a.ema_w * (p.z - e.z);
            e.w += a.ema_w * (p.w - e.w);
            *reinterpret_cast<float4*>(t.ema + i) = e;
          }
          if (t.out) {
            if (t.out_bf16) {
              __nv_bfloat162 lo = __floats2bfloat162_rn(p.x, p.y), hi = __floats2bfloat162_rn(p.z, p.w);
              uint2 packed;
              packed.x = *reinterpret_cast<uint32_t*>(&lo);
              packed.y = *reinterpret_cast<uint32_t*>(&hi);
              *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(t.out) + i) = packed;
            } else {
              *reinterpret_cast<float4*>(static_cast<float*>(t.out) + i) = p;
            }
          }
        } else {
          for (long j = i; j < end; ++j) {
            float p = t.p[j], m = t.m[j], v = t.v[j];
            adam_one(p, t.g[j], m, v, t.decay[j], gs, a);
            t.p[j] = p; t.m[j] = m; t.v[j] = v;
            if (t.ema) t.ema[j] += a.ema_w * (p - t.ema[j]);
            if (t.out) {
              if (t.out_bf16) static_cast<__nv_bfloat16*>(t.out)[j] = __float2bfloat16(p);
              else static_cast<float*>(t.out)[j] = p;
            }
          }
        }
      }
    } else {
      for (long j = ch.start + threadIdx.x; j < end; j += OPT_THREADS) {
        float p = t.p[j], m = t.m[j], v = t.v[j];
        adam_one(p, t.g[j], m, v, t.decay[j], gs, a);
        t.p[j] = p; t.m[j] = m; t.v[j] = v;
        if (t.ema) t.ema[j] += a.ema_w * (p - t.ema[j]);
        if (t.out) {
          if (t.out_bf16) static_cast<__nv_bfloat16*>(t.out)[j] = __float2bfloat16(p);
          else static_cast<float*>(t.out)[j] = p;
        }
      }
    }
  }
}

struct SumTensor {
  const float* x;
  long n;
  int vec;
  int pad;
};

// partial[block] = sum of squares over the chunks this block visits (fixed assignment).
__global__ void __launch_bounds__(OPT_THREADS) sumsq_kernel(const SumTensor* __restrict__ tensors,
                                                             const Chunk* __restrict__ chunks, int num_chunks,
                                                             float* __restrict__ partial) {
  float acc = 0.f;
  for (int ci = blockIdx.x; ci < num_chunks; ci += gridDim.x) {
    const Chunk ch = chunks[ci];
    const SumTensor t = tensors[ch.tensor];
    const long end = min(t.n, ch.start + (long)OPT_CHUNK);
    if (t.vec && ch.start + OPT_CHUNK <= t.n) {
      for (long i = ch.start + 4 * threadIdx.x; i < end; i += 4 * OPT_THREADS) {
        const float4 g = __ldcs(reinterpret_cast<const float4*>(t.x + i));
        acc += g.x * g.x + g.y * g.y + g.z * g.z + g.w * g.w;
      }
    } else {
      for (long j = ch.start + threadIdx.x; j < end; j += OPT_THREADS) acc += t.x[j] * t.x[j];
    }
  }
  __shared__ float red[OPT_THREADS / 32];
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float s = threadIdx.x < OPT_THREADS / 32 ? red[threadIdx.x] : 0.f;
    s = warp_sum(s);
    if (threadIdx.x == 0) partial[blockIdx.x] = s;
  }
}

__global__ void sum_partials_kernel(const float* __restrict__ partial, int count, float* __restrict__ out) {
  float acc = 0.f;
  for (int i = threadIdx.x; i < count; i += 32) acc += partial[i];
  acc = warp_sum(acc);
  if (threadIdx.x == 0) *out = acc;
}

bool aligned(const void* p, int bytes) { return p == nullptr || reinterpret_cast<uintptr_t>(p) % bytes == 0; }

// Device copies of the tensor + chunk tables, cached by the tensor table's bytes (the
// optimizer's shards never move, so after the first step nothing is uploaded again).
struct TableCache {
  std::mutex mu;
  std::unordered_map<std::string, std::pair<at::Tensor, int>> entries;
};

TableCache& table_cache() {
  static TableCache cache;
  return cache;
}

void add_chunks(std::vector<Chunk>& chunks, int index, long n) {
  for (long s = 0; s < n; s += OPT_CHUNK) chunks.push_back(Chunk{index, 0, s});
}

// Returns (device table = [tensors..., chunks...], number of chunks).
template <typename T>
std::pair<at::Tensor, int> device_table(const std::vector<T>& tensors, const at::Device& device) {
  // keyed by the descriptor bytes, tagged with the descriptor size so the two table kinds never mix
  std::string key(sizeof(T) * tensors.size(), '\0');
  std::memcpy(key.data(), tensors.data(), key.size());
  const std::string tagged = std::to_string(sizeof(T)) + ":" + key;
  auto& cache = table_cache();
  std::lock_guard<std::mutex> lock(cache.mu);
  auto it = cache.entries.find(tagged);
  if (it != cache.entries.end()) return it->second;
  std::vector<Chunk> chunks;
  for (size_t i = 0; i < tensors.size(); ++i) add_chunks(chunks, (int)i, tensors[i].n);
  const size_t bytes = key.size() + sizeof(Chunk) * chunks.size();
  auto host = at::empty({(long)std::max<size_t>(bytes, 1)}, at::TensorOptions().dtype(at::kByte));
  std::memcpy(host.data_ptr(), key.data(), key.size());
  if (!chunks.empty())
    std::memcpy(static_cast<char*>(host.data_ptr()) + key.size(), chunks.data(), sizeof(Chunk) * chunks.size());
  if (cache.entries.size() > 16) cache.entries.clear();
  auto entry = std::make_pair(host.to(device), (int)chunks.size());
  cache.entries.emplace(tagged, entry);
  return entry;
}

int grid_for(size_t chunks) { return (int)std::max<size_t>(1, std::min<size_t>(chunks, (size_t)sm_count() * 8)); }

}  // namespace

// ema: empty, or one fp32 tensor per master (numel 0 = no EMA for that tensor), lerped toward the
// updated master with weight ema_weight (= 1 - decay) in the same pass.
void adamw_step(std::vector<at::Tensor> masters, std::vector<at::Tensor> grads, std::vector<at::Tensor> exp_avg,
                std::vector<at::Tensor> exp_avg_sq, std::vector<at::Tensor> decay, std::vector<at::Tensor> params,
                at::Tensor gscale, double lr, double b1, double b2, double eps, double wd, double bc1, double bc2,
                std::vector<at::Tensor> ema, double ema_weight) {
  const size_t count = masters.size();
  TORCH_CHECK(grads.size() == count && exp_avg.size() == count && exp_avg_sq.size() == count &&
                  decay.size() == count && (params.empty() || params.size() == count) &&
                  (ema.empty() || ema.size() == count),
              "adamw_step: list lengths differ");
  TORCH_CHECK(gscale.scalar_type() == at::kFloat && gscale.numel() == 1 && gscale.is_cuda(), "gscale: fp32 scalar");
  std::vector<AdamTensor> tensors;
  for (size_t i = 0; i < count; ++i) {
    const long n = masters[i].numel();
    for (const auto* t : {&masters[i], &grads[i], &exp_avg[i], &exp_avg_sq[i]})
      TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == n && t->is_cuda(),
                  "adamw_step: fp32 contiguous CUDA tensors of equal size");
    TORCH_CHECK(decay[i].scalar_type() == at::kByte && decay[i].numel() == n && decay[i].is_contiguous(),
                "adamw_step: decay mask uint8");
    void* out = nullptr;
    int out_bf16 = 0;
    if (!params.empty()) {
      TORCH_CHECK(params[i].numel() == n && params[i].is_contiguous() &&
                      (params[i].scalar_type() == at::kBFloat16 || params[i].scalar_type() == at::kFloat),
                  "adamw_step: parameter output bf16/fp32 contiguous");
      out = params[i].data_ptr();
      out_bf16 = params[i].scalar_type() == at::kBFloat16;
    }
    float* shadow = nullptr;
    if (!ema.empty() && ema[i].numel()) {
      TORCH_CHECK(ema[i].scalar_type() == at::kFloat && ema[i].is_contiguous() && ema[i].numel() == n,
                  "adamw_step: EMA shadow fp32 contiguous like the master");
      shadow = ema[i].data_ptr<float>();
    }
    AdamTensor t{masters[i].data_ptr<float>(), grads[i].data_ptr<float>(), exp_avg[i].data_ptr<float>(),
                 exp_avg_sq[i].data_ptr<float>(), decay[i].data_ptr<uint8_t>(), out, shadow, n, out_bf16, 0};
    t.vec = aligned(t.p, 16) && aligned(t.g, 16) && aligned(t.m, 16) && aligned(t.v, 16) && aligned(t.decay, 4) &&
            aligned(out, out_bf16 ? 8 : 16) && aligned(shadow, 16);
    tensors.push_back(t);
  }
  if (tensors.empty()) return;
  auto [table, num_chunks] = device_table(tensors, masters[0].device());
  if (!num_chunks) return;
  const auto* dt = reinterpret_cast<const AdamTensor*>(table.data_ptr());
  const auto* dc = reinterpret_cast<const Chunk*>(static_cast<const char*>(table.data_ptr()) +
                                                  sizeof(AdamTensor) * tensors.size());
  AdamScalars a{(float)lr, (float)b1, (float)b2, (float)eps, (float)wd, (float)bc1, (float)bc2, (float)ema_weight};
  adamw_kernel<<<grid_for(num_chunks), OPT_THREADS, 0, stream()>>>(dt, dc, num_chunks, gscale.data_ptr<float>(), a);
  CQB_LAUNCH_CHECK();
  count_launch();
}

at::Tensor sum_squares(std::vector<at::Tensor> xs) {
  std::vector<SumTensor> tensors;
  TORCH_CHECK(!xs.empty(), "sum_squares: no tensors");
  for (size_t i = 0; i < xs.size(); ++i) {
    TORCH_CHECK(xs[i].scalar_type() == at::kFloat && xs[i].is_contiguous() && xs[i].is_cuda(),
                "sum_squares: fp32 contiguous CUDA tensors");
    SumTensor t{xs[i].data_ptr<float>(), xs[i].numel(), aligned(xs[i].data_ptr(), 16) ? 1 : 0, 0};
    tensors.push_back(t);
  }
  auto out = at::zeros({}, xs[0].options());
  auto [table, num_chunks] = device_table(tensors, xs[0].device());
  if (!num_chunks) return out;
  const auto* dt = reinterpret_cast<const SumTensor*>(table.data_ptr());
  const auto* dc = reinterpret_cast<const Chunk*>(static_cast<const char*>(table.data_ptr()) +
                                                  sizeof(SumTensor) * tensors.size());
  const int grid = grid_for(num_chunks);
  auto partial = at::empty({grid}, xs[0].options());
  sumsq_kernel<<<grid, OPT_THREADS, 0, stream()>>>(dt, dc, num_chunks, partial.data_ptr<float>());
  CQB_LAUNCH_CHECK();
  sum_partials_kernel<<<1, 32, 0, stream()>>>(partial.data_ptr<float>(), grid, out.data_ptr<float>());
  CQB_LAUNCH_CHECK();
  count_launch(2);
  return out;
}

}  // namespace cqb
