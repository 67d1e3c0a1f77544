// Persistent tcgen05 GEMM for sm_100a: D[M,N] = sum_k A[m,k] B[n,k] with bf16 operands and fp32
// accumulation in tensor memory.
//
//  * 128 x 256 x 64 tiles; 4-stage TMA ring (48 KB per stage) with 128-byte swizzle;
//  * warp 0 issues TMA loads, warp 1 allocates TMEM and issues tcgen05.mma (one thread),
//    warps 2-5 drain the accumulator with tcgen05.ld and run the epilogue;
//  * two TMEM accumulators (2 x 256 fp32 columns) so the epilogue of tile i overlaps the MMAs
//    of tile i+1;
//  * operands may be K-major (contraction dim contiguous) or MN-major (output dim
//    contiguous), so y = x W^T, dX = dY W and dW += dY^T X all run without transposes;
//  * epilogues: bf16 store (+ bias), or fp32 read-add-write into an existing fp32 matrix
//    (the FP32 main_grad accumulation of weight gradients).
//
// Waits are bounded (tcgen05.cuh); on expiry the kernel records an error code, stops issuing,
// waits for its outstanding TMA transactions (bounded), frees TMEM and exits.
#include "common.cuh"
#include "tcgen05.cuh"

#include <mutex>
#include <unordered_map>

namespace cqb {

namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_BOX = 32;                                   // 32 x 32 output box per warp store
constexpr int STAGING_BYTES = 4 /*warps*/ * 2 /*buffers*/ * EPI_BOX * EPI_BOX * 4;  // sized for fp32
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + STAGING_BYTES + 1024 /*align*/ + 256 /*barriers*/;
constexpr int THREADS = 192;

int* status_word() {
  static int* word = [] {
    int* p = nullptr;
    CQB_CHECK_CUDA(cudaMalloc(&p, sizeof(int)));
    CQB_CHECK_CUDA(cudaMemset(p, 0, sizeof(int)));
    return p;
  }();
  return word;
}

struct GemmArgs {
  int M, N, K;
  void* out;          // bf16 [M, ldo] or fp32 [M, ldo]
  int ldo;
  const __nv_bfloat16* bias;  // [N] or null
};

template <bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const __grid_constant__ CUtensorMap map_out, GemmArgs args, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging = smem + STAGES * STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(staging + STAGING_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_m = (args.M + BM - 1) / BM, tiles_n = (args.N + BN - 1) / BN;
  const int tiles = tiles_m * tiles_n;
  const int kblocks = (args.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&tfull[b], 1);
      tc::mbar_init(&tempty[b], 4);
    }
    tc::mbar_init(drain, 1);
    *abort_flag = 0;
    tc::fence_mbar_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, 2 * BN);
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tc::prefetch_map(&map_a);
      tc::prefetch_map(&map_b);
      int stage = 0;
      uint32_t phase = 0;
      int armed[STAGES];  // parity of the last armed phase of each stage, -1 = never armed
#pragma unroll
      for (int s = 0; s < STAGES; ++s) armed[s] = -1;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int m0 = (t % tiles_m) * BM, n0 = (t / tiles_m) * BN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!tc::mbar_wait(&empty[stage], phase ^ 1, status, abort_flag, 1)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          tc::mbar_expect_tx(&full[stage], STAGE_BYTES);
          const int k0 = kb * BK;
          if (A_MN) {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tc::tma_load_2d(sa + j * (BK * 128), &map_a, &full[stage], m0 + j * 64, k0);
          } else {
            tc::tma_load_2d(sa, &map_a, &full[stage], k0, m0);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tc::tma_load_2d(sb + j * (BK * 128), &map_b, &full[stage], n0 + j * 64, k0);
          } else {
            tc::tma_load_2d(sb, &map_b, &full[stage], k0, n0);
          }
          armed[stage] = (int)phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Drain: every armed stage's transaction must land before the CTA's smem is released.
        for (int s = 0; s < STAGES; ++s) {
          if (armed[s] < 0) continue;
          const unsigned long long t0 = tc::globaltimer();
          while (!tc::mbar_try_wait(&full[s], (uint32_t)armed[s]) && tc::globaltimer() - t0 < tc::kWaitNs) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++local) {
        const int buf = local & 1;
        const uint32_t use = (local >> 1) & 1;
        if (!tc::mbar_wait(&tempty[buf], use ^ 1, status, abort_flag, 2)) break;
        tc::fence_after();
        const uint32_t d = tmem + buf * BN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!tc::mbar_wait(&full[stage], phase, status, abort_flag, 3)) {
            ok = false;
            break;
          }
          tc::fence_after();
          const uint32_t sa = tc::smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? tc::smem_desc(sa + k * 2048, BK * 128, 1024) : tc::smem_desc(sa + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? tc::smem_desc(sb + k * 2048, BK * 128, 1024) : tc::smem_desc(sb + k * 32, 16, 1024);
            tc::mma_bf16(d, ad, bd, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          tc::mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) tc::mma_commit(&tfull[buf]);
      }
      // Let every issued MMA retire before TMEM is released (matters only on the abort path).
      tc::mma_commit(drain);
      const unsigned long long t0 = tc::globaltimer();
      while (!tc::mbar_try_wait(drain, 0) && tc::globaltimer() - t0 < tc::kWaitNs) {
      }
    }
  } else {
    // Epilogue warps 2..5 -> TMEM lane quarter (warp % 4). Each warp owns 32 rows of the tile:
    // TMEM -> registers (tcgen05.ld) -> dense 32x32 smem box -> TMA store (bf16) or TMA
    // reduce-add (fp32 accumulate), double-buffered per warp so the next tcgen05.ld overlaps
    // the previous bulk copy.
    const int quarter = warp & 3;
    constexpr int ESIZE = EPI == 0 ? 2 : 4;
    uint8_t* my_stage = staging + quarter * 2 * EPI_BOX * EPI_BOX * 4;
    int local = 0, chunk = 0;
    if (lane == 0) tc::prefetch_map(&map_out);
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++local) {
      const int buf = local & 1;
      const uint32_t use = (local >> 1) & 1;
      if (!tc::mbar_wait(&tfull[buf], use, status, abort_flag, 4)) break;
      tc::fence_after();
      const int m0 = (t % tiles_m) * BM, n0 = (t / tiles_m) * BN;
      const uint32_t base = tmem + buf * BN + ((uint32_t)(quarter * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < BN; c += EPI_BOX, ++chunk) {
        float v[32];
        tc::tmem_ld32(base + c, v);
        const int col0 = n0 + c;
        if (col0 >= args.N) continue;  // whole box outside the matrix (uniform across the warp)
        uint8_t* box = my_stage + (chunk & 1) * EPI_BOX * EPI_BOX * 4;
        if (lane == 0) tc::bulk_wait_read1();  // the store that last used this buffer finished reading
        __syncwarp();
        if (EPI == 0) {
          __nv_bfloat16* row = reinterpret_cast<__nv_bfloat16*>(box) + lane * EPI_BOX;
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            float o[8];
#pragma unroll
            for (int q = 0; q < 8; ++q)
              o[q] = v[j + q] + ((args.bias && col0 + j + q < args.N) ? __bfloat162float(args.bias[col0 + j + q]) : 0.f);
            store8(row + j, o);
          }
        } else {
          float* row = reinterpret_cast<float*>(box) + lane * EPI_BOX;
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(row + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        }
        tc::fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          if (EPI == 0)
            tc::tma_store_2d(&map_out, box, col0, m0 + quarter * 32);
          else
            tc::tma_reduce_add_2d(&map_out, box, col0, m0 + quarter * 32);
          tc::bulk_commit();
        }
        (void)ESIZE;
      }
      tc::fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&tempty[buf]);
    }
    if (lane == 0) tc::bulk_wait_all();
    __syncwarp();
  }
  __syncthreads();
  if (warp == 1) {
    tc::fence_after();
    tc::tmem_dealloc(tmem, 2 * BN);
  }
}

// ---- host side ----------------------------------------------------------------------------
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
  static EncodeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    CQB_CHECK_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    TORCH_CHECK(p != nullptr && q == cudaDriverEntryPointSuccess, "cuTensorMapEncodeTiled unavailable");
    return reinterpret_cast<EncodeFn>(p);
  }();
  return fn;
}

// 2-D bf16 row-major matrix [rows, cols] (cols contiguous), 128B-swizzled boxes of
// (64 cols x box_rows rows).
CUtensorMap make_map(const at::Tensor& t, int box_rows) {
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, "TMA operand must be row-major 2-D");
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, "TMA operand must be bf16");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((t.stride(0) * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)t.size(1), (cuuint64_t)t.size(0)};
  cuuint64_t strides[1] = {(cuuint64_t)t.stride(0) * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, t.data_ptr(), dims, strides, box, elem,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return map;
}

// Output map: dense 32x32 boxes (no swizzle) over a row-major [rows, cols] bf16 or fp32 matrix.
CUtensorMap make_out_map(const at::Tensor& t) {
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, "output must be row-major 2-D");
  const bool f32 = t.scalar_type() == at::kFloat;
  TORCH_CHECK(f32 || t.scalar_type() == at::kBFloat16, "output must be bf16 or fp32");
  const int esize = f32 ? 4 : 2;
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0 && (t.stride(0) * esize) % 16 == 0,
              "output base / row stride must be 16-byte aligned");
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)t.size(1), (cuuint64_t)t.size(0)};
  cuuint64_t strides[1] = {(cuuint64_t)t.stride(0) * esize};
  cuuint32_t box[2] = {(cuuint32_t)EPI_BOX, (cuuint32_t)EPI_BOX};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = encode_fn()(&map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                           t.data_ptr(), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (output) failed: ", (int)r);
  return map;
}

template <bool A_MN, bool B_MN, int EPI>
void launch(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo, GemmArgs args) {
  auto kernel = gemm_kernel<A_MN, B_MN, EPI>;
  static std::once_flag once;
  std::call_once(once, [&] {
    CQB_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
  });
  const int tiles = ((args.M + BM - 1) / BM) * ((args.N + BN - 1) / BN);
  const int grid = std::max(1, std::min(tiles, sm_count()));
  kernel<<<grid, THREADS, SMEM_BYTES, stream()>>>(ma, mb, mo, args, status_word());
  CQB_LAUNCH_CHECK();
  count_launch();
}

// Inner (contiguous) TMA extents must be multiples of 8 elements (16 bytes); outer extents are free.
void check_dims(int64_t m, int64_t n, int64_t k, bool k_inner = true) {
  TORCH_CHECK(m > 0 && n > 0 && k > 0, "empty GEMM");
  TORCH_CHECK(n % 16 == 0, "GEMM N must be a multiple of 16");
  TORCH_CHECK(!k_inner || k % 16 == 0, "GEMM K must be a multiple of 16");
}

}  // namespace

// y[M,N] = x[M,K] w[N,K]^T (+ bias)
at::Tensor gemm_nt(at::Tensor x, at::Tensor w, c10::optional<at::Tensor> bias) {
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K, "gemm_nt: inner dims differ");
  check_dims(M, N, K);
  auto y = at::empty({M, N}, x.options());
  auto ma = make_map(x, BM);
  auto mb = make_map(w, BN);
  at::Tensor b;
  if (bias && bias->defined()) b = bias->to(at::kBFloat16).contiguous();
  GemmArgs args{(int)M, (int)N, (int)K, y.data_ptr(), (int)N,
                b.defined() ? reinterpret_cast<const __nv_bfloat16*>(b.data_ptr()) : nullptr};
  launch<false, false, 0>(ma, mb, make_out_map(y), args);
  return y;
}

// y[M,N] = a[M,K] b[K,N]   (b row-major: output dim contiguous -> MN-major B operand)
at::Tensor gemm_nn(at::Tensor a, at::Tensor b) {
  const int64_t M = a.size(0), K = a.size(1), N = b.size(1);
  TORCH_CHECK(b.size(0) == K, "gemm_nn: inner dims differ");
  check_dims(M, N, K);
  auto y = at::empty({M, N}, a.options());
  auto ma = make_map(a, BM);
  auto mb = make_map(b, BK);
  GemmArgs args{(int)M, (int)N, (int)K, y.data_ptr(), (int)N, nullptr};
  launch<false, true, 0>(ma, mb, make_out_map(y), args);
  return y;
}

// out[N,K] (fp32) += a[M,N]^T b[M,K]   (contraction over rows: both operands MN-major)
void gemm_tn_acc(at::Tensor a, at::Tensor b, at::Tensor out) {
  const int64_t M = a.size(0), N = a.size(1), K = b.size(1);
  TORCH_CHECK(b.size(0) == M, "gemm_tn_acc: row counts differ");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() == N * K, "out must be fp32 [N,K]");
  TORCH_CHECK(N % 16 == 0, "gemm_tn_acc: N must be a multiple of 16");
  check_dims(N, K, M, /*k_inner=*/false);
  auto ma = make_map(a, BK);
  auto mb = make_map(b, BK);
  GemmArgs args{(int)N, (int)K, (int)M, out.data_ptr(), (int)K, nullptr};
  launch<true, true, 1>(ma, mb, make_out_map(out.view({N, K})), args);
}

int gemm_status(bool reset) {
  int v = 0;
  CQB_CHECK_CUDA(cudaMemcpy(&v, status_word(), sizeof(int), cudaMemcpyDeviceToHost));
  if (reset && v) CQB_CHECK_CUDA(cudaMemset(status_word(), 0, sizeof(int)));
  return v;
}

}  // namespace cqb
