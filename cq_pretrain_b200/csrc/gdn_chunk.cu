// Chunk-local work of the chunked gated delta rule: one CTA per (chunk, head), 8 warps,
// bf16 tensor-core tiles (mma.sync m16n8k16, fp32 accumulate) in shared memory.
//
// Per chunk of C = 64 events (key/value dim 128), with b = cumsum(g) inside the chunk,
// E_ij = exp(b_i - b_j):
//   A  = tril(beta_i E_ij k_i.k_j, -1)          T = (I + A)^-1   (column substitution, fp32)
//   W  = T diag(beta e^b) K                     U = T diag(beta) V
//   P  = tril(Q K^T * E)                        Qd = diag(e^b) Q     Kt = diag(e^{b_C - b}) K
//   gamma = e^{b_C}
// These are the inputs of the per-document state recurrence (gdn.cu). The same algebra is the
// chunked form used by the reference's GDN backends (ops/gated_delta_net.py:143-214).
#include "common.cuh"
#include "mma_sync.cuh"
#include "tcgen05.cuh"

namespace cqb {

// Status word of the tcgen05 GDN kernels (gdn_chunk.cu and gdn.cu): the first expired bounded
// wait records its code here.
int* gdn_status_word() {
  static int* word = [] {
    int* p = nullptr;
    CQB_CHECK_CUDA(cudaMalloc(&p, sizeof(int)));
    CQB_CHECK_CUDA(cudaMemset(p, 0, sizeof(int)));
    return p;
  }();
  return word;
}

namespace {

using namespace ws;

constexpr int CH = 64, DH = 128, THREADS_C = 256;
constexpr int LD = DH + 8;     // bf16 row of a 128-wide tile (272 bytes: rows stay 16-byte aligned)
constexpr int LD64 = CH + 8;   // bf16 row of a 64-wide tile
constexpr int LDF = CH + 1;    // fp32 row of a 64x64 matrix
constexpr int TILE = CH * LD;  // elements of one 64x128 bf16 tile

struct PrepArgs {
  const __nv_bfloat16* Q;  // [Nc*H, 64, 128] normalised, scaled queries
  const __nv_bfloat16* K;  // [Nc*H, 64, 128] normalised keys
  const __nv_bfloat16* V;  // [Nc*H, 64, 128]
  const float* G;          // [Nc*H, 64] log decay
  const float* B;          // [Nc*H, 64] beta
  __nv_bfloat16* W;
  __nv_bfloat16* U;
  __nv_bfloat16* P;        // [Nc*H, 64, 64]
  __nv_bfloat16* Qd;
  __nv_bfloat16* Kt;
  float* gamma;            // [Nc*H]
};

__device__ __forceinline__ void load_tile_async(__nv_bfloat16* dst, const __nv_bfloat16* src, int tid) {
  for (int i = tid; i < CH * DH / 8; i += THREADS_C) {
    const int r = i >> 4, c = (i & 15) * 8;
    cp_async16(dst + r * LD + c, src + r * DH + c);
  }
}

// smem tile (row-major, ld LD) -> global [64][128] with 16-byte vectors, rows scaled by rs[] if given
__device__ __forceinline__ void store_tile(__nv_bfloat16* dst, const __nv_bfloat16* src, const float* rs, int tid,
                                           int first, int stride) {
  for (int i = tid - first; i < CH * DH / 8; i += stride) {
    if (i < 0) continue;
    const int r = i >> 4, c = (i & 15) * 8;
    float v[8];
    load8(src + r * LD + c, v);
    if (rs) {
      const float s = rs[r];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] *= s;
    }
    store8(dst + r * DH + c, v);
  }
}

// Inclusive cumsum of g (64 values) by warp 0; fills b, e^b, e^{b_C - b}; returns b_C on lane 0.
__device__ __forceinline__ float chunk_decay(const float* g, float* b, float* eb, float* kdec, int lane) {
  const float g0 = g[2 * lane], g1 = g[2 * lane + 1];
  float s = g0 + g1;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const float v = __shfl_up_sync(0xffffffffu, s, off);
    if (lane >= off) s += v;
  }
  const float excl = s - (g0 + g1);
  const float b0 = excl + g0, b1 = excl + g0 + g1;
  const float bc = __shfl_sync(0xffffffffu, s, 31);
  b[2 * lane] = b0;
  b[2 * lane + 1] = b1;
  eb[2 * lane] = __expf(b0);
  eb[2 * lane + 1] = __expf(b1);
  kdec[2 * lane] = __expf(bc - b0);
  kdec[2 * lane + 1] = __expf(bc - b1);
  return bc;
}

// T = (I + A)^-1 for strictly lower-triangular A (fp32, ld LDF), by 16x16 blocks; every thread of
// the CTA calls it (it synchronises). Step 1: warps 0-3 invert the diagonal blocks D_k = I + A_kk
// by forward substitution (lane c owns column c, unrolled over rows) while warps 4-7 clear the
// upper blocks. Step 2, block rows bi = 1..3 in turn: Y_j = sum_{k=j}^{bi-1} A_{bi,k} T_{k,j},
// then T_{bi,j} = -D_bi^-1 Y_j; two warps share each block (8 rows each, 4 columns per lane).
// `scratch` holds 3 x 16 x 17 floats.
__device__ void unit_lower_inverse(const float* A, float* T, float* scratch, int warp, int lane) {
  if (warp < 4) {
    const int k0 = 16 * warp, c = lane & 15;
    float x[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < r; ++j) s += A[(k0 + r) * LDF + k0 + j] * x[j];
      x[r] = r < c ? 0.f : (r == c ? 1.f : -s);
    }
    if (lane < 16)
#pragma unroll
      for (int r = 0; r < 16; ++r) T[(k0 + r) * LDF + k0 + c] = x[r];
  } else {
    for (int e = (warp - 4) * 32 + lane; e < 6 * 256; e += 128) {
      const int blk = e >> 8, w = e & 255;   // upper blocks (0,1) (0,2) (0,3) (1,2) (1,3) (2,3)
      const int bi = blk < 3 ? 0 : (blk < 5 ? 1 : 2);
      const int bj = blk < 3 ? blk + 1 : (blk < 5 ? blk - 1 : 3);
      T[(16 * bi + (w >> 4)) * LDF + 16 * bj + (w & 15)] = 0.f;
    }
  }
  __syncthreads();
  const int bj = warp >> 1, r = 8 * (warp & 1) + (lane >> 2), c0 = 4 * (lane & 3);
  for (int bi = 1; bi < 4; ++bi) {
    const bool active = bj < bi;
    if (active) {
      float y[4] = {0.f, 0.f, 0.f, 0.f};
      for (int k = bj; k < bi; ++k) {
#pragma unroll 4
        for (int m = 0; m < 16; ++m) {
          const float av = A[(16 * bi + r) * LDF + 16 * k + m];
          const float* tr = T + (16 * k + m) * LDF + 16 * bj + c0;
#pragma unroll
          for (int q = 0; q < 4; ++q) y[q] += av * tr[q];
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) scratch[(bj * 16 + r) * 17 + c0 + q] = y[q];
    }
    __syncthreads();
    if (active) {
      float t[4] = {0.f, 0.f, 0.f, 0.f};
      for (int m = 0; m <= r; ++m) {
        const float dv = T[(16 * bi + r) * LDF + 16 * bi + m];
#pragma unroll
        for (int q = 0; q < 4; ++q) t[q] += dv * scratch[(bj * 16 + m) * 17 + c0 + q];
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) T[(16 * bi + r) * LDF + 16 * bj + c0 + q] = -t[q];
    }
    __syncthreads();
  }
}

// ---- warp-tile products: acc[NT][4] (rows rs..rs+15, n-tiles c0 + 8j) += A x B over kdim ----
// A row-major [m][k] (lda), B row-major [k][n] (ldb)
template <int NT>
__device__ __forceinline__ void mm_ab(float (*acc)[4], const __nv_bfloat16* A, int lda, const __nv_bfloat16* B,
                                      int ldb, int rs, int c0, int kdim, int lane) {
#pragma unroll 2
  for (int k0 = 0; k0 < kdim; k0 += 16) {
    uint32_t a[4];
    frag_a(a, A, rs, k0, lda, lane);
#pragma unroll
    for (int j = 0; j < NT; j += 2) {
      uint32_t b[4];
      frag_b2(b, B, k0, c0 + 8 * j, ldb, lane);
      mma16816(acc[j], a, b[0], b[1]);
      mma16816(acc[j + 1], a, b[2], b[3]);
    }
  }
}
// A row-major [m][k], B = X^T with X row-major [n][k]
template <int NT>
__device__ __forceinline__ void mm_abt(float (*acc)[4], const __nv_bfloat16* A, int lda, const __nv_bfloat16* X,
                                       int ldx, int rs, int c0, int kdim, int lane) {
#pragma unroll 2
  for (int k0 = 0; k0 < kdim; k0 += 16) {
    uint32_t a[4];
    frag_a(a, A, rs, k0, lda, lane);
#pragma unroll
    for (int j = 0; j < NT; j += 2) {
      uint32_t b[4];
      frag_bt2(b, X, k0, c0 + 8 * j, ldx, lane);
      mma16816(acc[j], a, b[0], b[1]);
      mma16816(acc[j + 1], a, b[2], b[3]);
    }
  }
}
// A = X^T with X row-major [k][m], B row-major [k][n]
template <int NT>
__device__ __forceinline__ void mm_atb(float (*acc)[4], const __nv_bfloat16* X, int ldx, const __nv_bfloat16* B,
                                       int ldb, int rs, int c0, int kdim, int lane) {
#pragma unroll 2
  for (int k0 = 0; k0 < kdim; k0 += 16) {
    uint32_t a[4];
    frag_at(a, X, rs, k0, ldx, lane);
#pragma unroll
    for (int j = 0; j < NT; j += 2) {
      uint32_t b[4];
      frag_b2(b, B, k0, c0 + 8 * j, ldb, lane);
      mma16816(acc[j], a, b[0], b[1]);
      mma16816(acc[j + 1], a, b[2], b[3]);
    }
  }
}

template <int NT>
__device__ __forceinline__ void zero_acc(float (*acc)[4]) {
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
}

// Element e of n-tile j sits at row rs + g + 8 (e >> 1), column c0 + 8 j + 2 t + (e & 1).
__device__ __forceinline__ int acc_row(int rs, int lane, int e) { return rs + (lane >> 2) + 8 * (e >> 1); }
__device__ __forceinline__ int acc_col(int c0, int j, int lane, int e) { return c0 + 8 * j + 2 * (lane & 3) + (e & 1); }

// Sum over the 4 lanes of a quad (same rows) / over the 8 lanes sharing t (same columns).
__device__ __forceinline__ float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  return v + __shfl_xor_sync(0xffffffffu, v, 2);
}
__device__ __forceinline__ float column_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 8);
  return v + __shfl_xor_sync(0xffffffffu, v, 16);
}

// Row sums (rows g, g+8 of the strip) of an accumulator-layout value added into dst[] (shared).
template <int NT, typename F>
__device__ __forceinline__ void add_row_sums(float* dst, int rs, int lane, F value) {
  float lo = 0.f, hi = 0.f;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    lo += value(j, 0) + value(j, 1);
    hi += value(j, 2) + value(j, 3);
  }
  lo = quad_sum(lo);
  hi = quad_sum(hi);
  if ((lane & 3) == 0) {
    atomicAdd(dst + rs + (lane >> 2), lo);
    atomicAdd(dst + rs + (lane >> 2) + 8, hi);
  }
}

__device__ __forceinline__ void store_acc_f32(float* dst, int ld, const float (*acc)[4], int rs, int c0, int nt,
                                              int lane) {
  for (int j = 0; j < nt; ++j) {
    const int col = c0 + 8 * j + 2 * (lane & 3);
    const int r = rs + (lane >> 2);
    *reinterpret_cast<float2*>(dst + (size_t)r * ld + col) = make_float2(acc[j][0], acc[j][1]);
    *reinterpret_cast<float2*>(dst + (size_t)(r + 8) * ld + col) = make_float2(acc[j][2], acc[j][3]);
  }
}

__device__ __forceinline__ void store_acc_bf16_tile(__nv_bfloat16* dst, int ld, const float (*acc)[4], int rs, int c0,
                                                    int nt, int lane, float scale = 1.f) {
  for (int j = 0; j < nt; ++j) {
    const int col = c0 + 8 * j + 2 * (lane & 3);
    const int r = rs + (lane >> 2);
    *reinterpret_cast<__nv_bfloat162*>(dst + r * ld + col) =
        __floats2bfloat162_rn(scale * acc[j][0], scale * acc[j][1]);
    *reinterpret_cast<__nv_bfloat162*>(dst + (r + 8) * ld + col) =
        __floats2bfloat162_rn(scale * acc[j][2], scale * acc[j][3]);
  }
}

__device__ __forceinline__ float bf(const __nv_bfloat16* p) { return __bfloat162float(*p); }

constexpr size_t PREP_SMEM = (size_t)3 * TILE * 2 + 2 * CH * LDF * 4 + 2 * CH * LD64 * 2 + 5 * CH * 4 + 3 * 16 * 17 * 4;

__global__ void __launch_bounds__(THREADS_C, 2) gdn_prep_kernel(PrepArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  __nv_bfloat16* sK = sQ + TILE;
  __nv_bfloat16* sV = sK + TILE;
  float* sA = reinterpret_cast<float*>(sV + TILE);
  float* sT = sA + CH * LDF;
  __nv_bfloat16* sTw = reinterpret_cast<__nv_bfloat16*>(sT + CH * LDF);
  __nv_bfloat16* sTv = sTw + CH * LD64;
  float* sb = reinterpret_cast<float*>(sTv + CH * LD64);
  float* seb = sb + CH;
  float* skd = seb + CH;
  float* sbeta = skd + CH;
  float* sg = sbeta + CH;
  float* sY = sg + CH;   // inverse scratch, 3 x 16 x 17

  const int cta = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const size_t tile_off = (size_t)cta * CH * DH;
  load_tile_async(sQ, a.Q + tile_off, tid);
  load_tile_async(sK, a.K + tile_off, tid);
  load_tile_async(sV, a.V + tile_off, tid);
  cp_commit();
  if (tid < CH) {
    sg[tid] = a.G[(size_t)cta * CH + tid];
    sbeta[tid] = a.B[(size_t)cta * CH + tid];
  }
  __syncthreads();
  if (warp == 0) {
    const float bc = chunk_decay(sg, sb, seb, skd, lane);
    if (lane == 0) a.gamma[cta] = __expf(bc);
  }
  cp_wait_all();
  __syncthreads();

  // KK = K K^T and QK = Q K^T: warp -> rows rs..rs+15, cols cb..cb+31
  const int rs = 16 * (warp & 3), cb = 32 * (warp >> 2);
  {
    float kk[4][4], qk[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) kk[j][e] = qk[j][e] = 0.f;
#pragma unroll
    for (int k0 = 0; k0 < DH; k0 += 16) {
      uint32_t ak[4], aq[4];
      frag_a(ak, sK, rs, k0, LD, lane);
      frag_a(aq, sQ, rs, k0, LD, lane);
#pragma unroll
      for (int j = 0; j < 4; j += 2) {
        uint32_t bk[4];
        frag_bt2(bk, sK, k0, cb + 8 * j, LD, lane);
        mma16816(kk[j], ak, bk[0], bk[1]);
        mma16816(kk[j + 1], ak, bk[2], bk[3]);
        mma16816(qk[j], aq, bk[0], bk[1]);
        mma16816(qk[j + 1], aq, bk[2], bk[3]);
      }
    }
    __nv_bfloat16* P = a.P + (size_t)cta * CH * CH;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int i = rs + gq + 8 * half;
        const int c0 = cb + 8 * j + 2 * tq;
        float av[2], pv[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int col = c0 + e;
          const float ev = col <= i ? __expf(sb[i] - sb[col]) : 0.f;
          av[e] = col < i ? sbeta[i] * kk[j][2 * half + e] * ev : 0.f;
          pv[e] = qk[j][2 * half + e] * ev;
        }
        sA[i * LDF + c0] = av[0];
        sA[i * LDF + c0 + 1] = av[1];
        *reinterpret_cast<__nv_bfloat162*>(P + i * CH + c0) = __floats2bfloat162_rn(pv[0], pv[1]);
      }
    }
  }
  // Qd = e^b Q and Kt = e^{b_C - b} K (the decay vectors are ready since the first barrier)
  store_tile(a.Qd + tile_off, sQ, seb, tid, 0, THREADS_C);
  store_tile(a.Kt + tile_off, sK, skd, tid, 0, THREADS_C);
  __syncthreads();
  unit_lower_inverse(sA, sT, sY, warp, lane);
  for (int e = tid; e < CH * CH; e += THREADS_C) {
    const int i = e >> 6, j = e & 63;
    const float t = sT[i * LDF + j];
    sTw[i * LD64 + j] = __float2bfloat16(t * sbeta[j] * seb[j]);
    sTv[i * LD64 + j] = __float2bfloat16(t * sbeta[j]);
  }
  __syncthreads();
  // W = Tw K, U = Tv V: warp -> rows rs..rs+15, cols cw..cw+63
  const int cw = 64 * (warp >> 2);
  float w[8][4], u[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) w[j][e] = u[j][e] = 0.f;
#pragma unroll
  for (int k0 = 0; k0 < CH; k0 += 16) {
    uint32_t aw[4], av[4];
    frag_a(aw, sTw, rs, k0, LD64, lane);
    frag_a(av, sTv, rs, k0, LD64, lane);
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      uint32_t bk[4], bv[4];
      frag_b2(bk, sK, k0, cw + 8 * j, LD, lane);
      frag_b2(bv, sV, k0, cw + 8 * j, LD, lane);
      mma16816(w[j], aw, bk[0], bk[1]);
      mma16816(w[j + 1], aw, bk[2], bk[3]);
      mma16816(u[j], av, bv[0], bv[1]);
      mma16816(u[j + 1], av, bv[2], bv[3]);
    }
  }
  __syncthreads();  // every read of sK / sV is done: stage W in sQ, U in sK
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int col = cw + 8 * j + 2 * tq;
    *reinterpret_cast<__nv_bfloat162*>(sQ + (rs + gq) * LD + col) = __floats2bfloat162_rn(w[j][0], w[j][1]);
    *reinterpret_cast<__nv_bfloat162*>(sQ + (rs + gq + 8) * LD + col) = __floats2bfloat162_rn(w[j][2], w[j][3]);
    *reinterpret_cast<__nv_bfloat162*>(sK + (rs + gq) * LD + col) = __floats2bfloat162_rn(u[j][0], u[j][1]);
    *reinterpret_cast<__nv_bfloat162*>(sK + (rs + gq + 8) * LD + col) = __floats2bfloat162_rn(u[j][2], u[j][3]);
  }
  __syncthreads();
  store_tile(a.W + tile_off, sQ, nullptr, tid, 0, THREADS_C);
  store_tile(a.U + tile_off, sK, nullptr, tid, 0, THREADS_C);
}

// ---- fused chunk backward -------------------------------------------------------------------
//
// Given dO, the entering state S and the gradient dS of the leaving state (both fp32 from the
// recurrence kernels), one CTA computes the chunk's dQ, dK, dV (fp32) and dG, dBeta:
//   Delta = U - W S          dDelta = P^T dO + Kt dS      (= dU)
//   dW = -dDelta S^T         dQd = dO S^T        dP = dO Delta^T       dKt = Delta dS^T
//   dT = dU Vb^T + dW Kw^T   dVb = T^T dU        dKw = T^T dW          dA = -T^T dT T^T
// and the chain through e^b, E, beta and b = cumsum(g) (dg_i = sum_{j >= i} db_j).
struct BwdArgs {
  const __nv_bfloat16* Q;
  const __nv_bfloat16* K;
  const __nv_bfloat16* V;
  const __nv_bfloat16* dO;  // [Nc*H, 64, 128]
  const float* G;
  const float* B;
  const float* S;           // [Nc*H, 128, 128] state entering the chunk
  const float* dS;          // [Nc*H, 128, 128] gradient of the state leaving the chunk
  float* dQ;                // [Nc*H, 64, 128]
  float* dK;
  float* dV;
  float* dG;                // [Nc*H, 64]
  float* dB;
  const float* dgamma;      // tcgen05 kernel: <S, dS> per (chunk, head), from the backward recurrence
};

constexpr int LDS = DH + 8;                       // bf16 row of the 128x128 state tiles
constexpr int STILE = DH * LDS;
constexpr size_t OFF_Q = 0, OFF_K = OFF_Q + TILE * 2, OFF_V = OFF_K + TILE * 2, OFF_DO = OFF_V + TILE * 2;
constexpr size_t OFF_W = OFF_DO + TILE * 2, OFF_U = OFF_W + TILE * 2, OFF_DD = OFF_U + TILE * 2;
constexpr size_t OFF_S = OFF_DD + TILE * 2, OFF_DS = OFF_S + STILE * 2;
constexpr size_t OFF_T = OFF_DS + STILE * 2, OFF_TB = OFF_T + CH * LDF * 4, OFF_P = OFF_TB + CH * LD64 * 2;
constexpr size_t OFF_VEC = OFF_P + CH * LD64 * 2;
constexpr size_t BWD_SMEM = OFF_VEC + 7 * CH * 4 + 16;
static_assert(BWD_SMEM <= 232448, "chunk backward exceeds the shared memory of one CTA");
static_assert(CH * LDF * 4 <= STILE * 2 && 2 * CH * LD64 * 2 + 3 * 16 * 17 * 4 <= STILE * 2,
              "phase-0 scratch must fit in the state tiles");

__global__ void __launch_bounds__(THREADS_C, 1) gdn_chunk_bwd_kernel(BwdArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem_raw + OFF_Q);
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(smem_raw + OFF_K);
  __nv_bfloat16* sV = reinterpret_cast<__nv_bfloat16*>(smem_raw + OFF_V);
  __nv_bfloat16* sdO = reinterpret_cast<__nv_bfloat16*>(smem_raw + OFF_DO);
  __nv_bfloat16* sW = reinterpret_cast<__nv_bfloat16*>(smem_raw + OFF_W);    // W, later dW
  __nv_bfloat16* sU = reinterpret_cast<__nv_bfloat16*>(smem_raw + OFF_U);    // U, later Delta
  __nv_bfloat16* sdD = reinterpret_cast<__nv_bfloat16*>(smem_raw + OFF_DD);  // dDelta = dU
  __nv_bfloat16* sS = reinterpret_cast<__nv_bfloat16*>(smem_raw + OFF_S);
  __nv_bfloat16* sdS = reinterpret_cast<__nv_bfloat16*>(smem_raw + OFF_DS);
  float* sA = reinterpret_cast<float*>(smem_raw + OFF_S);                     // phase 0 (aliases sS)
  __nv_bfloat16* sTw = reinterpret_cast<__nv_bfloat16*>(smem_raw + OFF_DS);  // phase 0 (aliases sdS)
  __nv_bfloat16* sTv = sTw + CH * LD64;
  float* sdT = reinterpret_cast<float*>(smem_raw + OFF_S);                    // late phases (aliases sS)
  float* sX = reinterpret_cast<float*>(smem_raw + OFF_DS);                    // late phases (aliases sdS)
  float* sT = reinterpret_cast<float*>(smem_raw + OFF_T);
  __nv_bfloat16* sTb = reinterpret_cast<__nv_bfloat16*>(smem_raw + OFF_TB);  // bf16 T, later M
  __nv_bfloat16* sP = reinterpret_cast<__nv_bfloat16*>(smem_raw + OFF_P);    // P, later dP * E
  float* sb = reinterpret_cast<float*>(smem_raw + OFF_VEC);
  float* seb = sb + CH;
  float* skd = seb + CH;
  float* sbeta = skd + CH;
  float* sg = sbeta + CH;
  float* sdb = sg + CH;
  float* sdbeta = sdb + CH;
  float* sscal = sdbeta + CH;   // [0] = dgamma, [1] = d b_C from Kt

  const int cta = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const size_t toff = (size_t)cta * CH * DH;
  load_tile_async(sQ, a.Q + toff, tid);
  load_tile_async(sK, a.K + toff, tid);
  load_tile_async(sV, a.V + toff, tid);
  load_tile_async(sdO, a.dO + toff, tid);
  cp_commit();
  if (tid < CH) {
    sg[tid] = a.G[(size_t)cta * CH + tid];
    sbeta[tid] = a.B[(size_t)cta * CH + tid];
    sdb[tid] = 0.f;
    sdbeta[tid] = 0.f;
  }
  if (tid < 2) sscal[tid] = 0.f;
  __syncthreads();
  float bc = 0.f;
  if (warp == 0) bc = chunk_decay(sg, sb, seb, skd, lane);
  cp_wait_all();
  __syncthreads();
  bc = sb[CH - 1];
  const int rs = 16 * (warp & 3), cb = 32 * (warp >> 2), cw = 64 * (warp >> 2);

  // ---- phase 0: recompute A (-> sA), P (-> sP), T, W, U ----
  {
    float kk[4][4], qk[4][4];
    zero_acc<4>(kk);
    zero_acc<4>(qk);
    mm_abt<4>(kk, sK, LD, sK, LD, rs, cb, DH, lane);
    mm_abt<4>(qk, sQ, LD, sK, LD, rs, cb, DH, lane);
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = acc_row(rs, lane, e), c = acc_col(cb, j, lane, e);
        const float ev = c <= i ? __expf(sb[i] - sb[c]) : 0.f;
        sA[i * LDF + c] = c < i ? sbeta[i] * kk[j][e] * ev : 0.f;
        sP[i * LD64 + c] = __float2bfloat16(qk[j][e] * ev);
      }
  }
  __syncthreads();
  unit_lower_inverse(sA, sT, reinterpret_cast<float*>(sTv + CH * LD64), warp, lane);
  for (int e = tid; e < CH * CH; e += THREADS_C) {
    const int i = e >> 6, j = e & 63;
    const float t = sT[i * LDF + j];
    sTb[i * LD64 + j] = __float2bfloat16(t);
    sTw[i * LD64 + j] = __float2bfloat16(t * sbeta[j] * seb[j]);
    sTv[i * LD64 + j] = __float2bfloat16(t * sbeta[j]);
  }
  __syncthreads();
  {
    float w[8][4], u[8][4];
    zero_acc<8>(w);
    zero_acc<8>(u);
    mm_ab<8>(w, sTw, LD64, sK, LD, rs, cw, CH, lane);
    mm_ab<8>(u, sTv, LD64, sV, LD, rs, cw, CH, lane);
    store_acc_bf16_tile(sW, LD, w, rs, cw, 8, lane);
    store_acc_bf16_tile(sU, LD, u, rs, cw, 8, lane);
  }
  __syncthreads();  // Tw / Tv / A are dead: the state tiles may be loaded over them

  // ---- phase 1: S, dS -> bf16 tiles; dgamma = <S, dS> ----
  {
    const float4* gS = reinterpret_cast<const float4*>(a.S + (size_t)cta * DH * DH);
    const float4* gdS = reinterpret_cast<const float4*>(a.dS + (size_t)cta * DH * DH);
    float dg = 0.f;
#pragma unroll 4
    for (int i = tid; i < DH * DH / 4; i += THREADS_C) {
      const float4 x = __ldcs(gS + i), y = __ldcs(gdS + i);
      dg += x.x * y.x + x.y * y.y + x.z * y.z + x.w * y.w;
      const int r = i >> 5, c = (i & 31) * 4;
      __nv_bfloat162* ps = reinterpret_cast<__nv_bfloat162*>(sS + r * LDS + c);
      __nv_bfloat162* pd = reinterpret_cast<__nv_bfloat162*>(sdS + r * LDS + c);
      ps[0] = __floats2bfloat162_rn(x.x, x.y);
      ps[1] = __floats2bfloat162_rn(x.z, x.w);
      pd[0] = __floats2bfloat162_rn(y.x, y.y);
      pd[1] = __floats2bfloat162_rn(y.z, y.w);
    }
    dg = warp_sum(dg);
    if (lane == 0) atomicAdd(sscal, dg);
  }
  __syncthreads();

  // ---- phase 2: Delta (-> sU), dDelta (-> sdD), dQ from dQd ----
  float dq[8][4];
  {
    float x[8][4];
    zero_acc<8>(x);
    mm_ab<8>(x, sW, LD, sS, LDS, rs, cw, DH, lane);   // W S
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = acc_row(rs, lane, e), c = acc_col(cw, j, lane, e);
        x[j][e] = bf(sU + i * LD + c) - x[j][e];
      }
    store_acc_bf16_tile(sU, LD, x, rs, cw, 8, lane);   // each thread rewrites only what it read
    float y[8][4];
    zero_acc<8>(x);
    zero_acc<8>(y);
    mm_atb<8>(x, sP, LD64, sdO, LD, rs, cw, CH, lane);  // P^T dO
    mm_ab<8>(y, sK, LD, sdS, LDS, rs, cw, DH, lane);     // K dS
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) x[j][e] += skd[acc_row(rs, lane, e)] * y[j][e];
    store_acc_bf16_tile(sdD, LD, x, rs, cw, 8, lane);
    zero_acc<8>(dq);
    mm_abt<8>(dq, sdO, LD, sS, LDS, rs, cw, DH, lane);  // dQd = dO S^T
    add_row_sums<8>(sdb, rs, lane, [&](int j, int e) {
      const int i = acc_row(rs, lane, e), c = acc_col(cw, j, lane, e);
      return seb[i] * dq[j][e] * bf(sQ + i * LD + c);
    });
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) dq[j][e] *= seb[acc_row(rs, lane, e)];
  }
  __syncthreads();

  // ---- phase 3: dW (-> sW), dK from dKt, dP * E (-> sP) with its b-gradient ----
  float dk[8][4];
  {
    float x[8][4];
    zero_acc<8>(x);
    mm_abt<8>(x, sdD, LD, sS, LDS, rs, cw, DH, lane);   // dDelta S^T
    store_acc_bf16_tile(sW, LD, x, rs, cw, 8, lane, -1.f);
    zero_acc<8>(dk);
    mm_abt<8>(dk, sU, LD, sdS, LDS, rs, cw, DH, lane);  // dKt = Delta dS^T
    float rkt_lo = 0.f, rkt_hi = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = acc_row(rs, lane, e), c = acc_col(cw, j, lane, e);
        const float v = skd[i] * dk[j][e];
        (e < 2 ? rkt_lo : rkt_hi) += v * bf(sK + i * LD + c);
        dk[j][e] = v;
      }
    rkt_lo = quad_sum(rkt_lo);
    rkt_hi = quad_sum(rkt_hi);
    if ((lane & 3) == 0) {
      atomicAdd(sdb + rs + (lane >> 2), -rkt_lo);
      atomicAdd(sdb + rs + (lane >> 2) + 8, -rkt_hi);
    }
    float tot = (lane & 3) == 0 ? rkt_lo + rkt_hi : 0.f;
    tot = warp_sum(tot);
    if (lane == 0) atomicAdd(sscal + 1, tot);

    float dp[4][4], qk[4][4];
    zero_acc<4>(dp);
    zero_acc<4>(qk);
    mm_abt<4>(dp, sdO, LD, sU, LD, rs, cb, DH, lane);   // dP = dO Delta^T
    mm_abt<4>(qk, sQ, LD, sK, LD, rs, cb, DH, lane);
    float row_lo = 0.f, row_hi = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float col[2] = {0.f, 0.f};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = acc_row(rs, lane, e), c = acc_col(cb, j, lane, e);
        const float ev = c <= i ? __expf(sb[i] - sb[c]) : 0.f;
        const float dpm = dp[j][e] * ev;
        const float t = dpm * qk[j][e];
        (e < 2 ? row_lo : row_hi) += t;
        col[e & 1] += t;
        sP[i * LD64 + c] = __float2bfloat16(dpm);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float v = column_sum(col[h]);
        if ((lane >> 2) == 0) atomicAdd(sdb + cb + 8 * j + 2 * (lane & 3) + h, -v);
      }
    }
    row_lo = quad_sum(row_lo);
    row_hi = quad_sum(row_hi);
    if ((lane & 3) == 0) {
      atomicAdd(sdb + rs + (lane >> 2), row_lo);
      atomicAdd(sdb + rs + (lane >> 2) + 8, row_hi);
    }
  }
  __syncthreads();

  // ---- phase 4: dQ += dPm K (store), dK += dPm^T Q, dT (-> sdT), dV (store), dK from dKw ----
  mm_ab<8>(dq, sP, LD64, sK, LD, rs, cw, CH, lane);
  store_acc_f32(a.dQ + toff, DH, dq, rs, cw, 8, lane);
  mm_atb<8>(dk, sP, LD64, sQ, LD, rs, cw, CH, lane);
  {
    float t1[4][4], t2[4][4];
    zero_acc<4>(t1);
    zero_acc<4>(t2);
    mm_abt<4>(t1, sdD, LD, sV, LD, rs, cb, DH, lane);   // dU V^T
    mm_abt<4>(t2, sW, LD, sK, LD, rs, cb, DH, lane);    // dW K^T
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = acc_row(rs, lane, e), c = acc_col(cb, j, lane, e);
        sdT[i * LDF + c] = sbeta[c] * (t1[j][e] + seb[c] * t2[j][e]);
      }
  }
  {
    float x[8][4];
    zero_acc<8>(x);
    mm_atb<8>(x, sTb, LD64, sdD, LD, rs, cw, CH, lane);  // dVb = T^T dU
    add_row_sums<8>(sdbeta, rs, lane, [&](int j, int e) {
      return x[j][e] * bf(sV + acc_row(rs, lane, e) * LD + acc_col(cw, j, lane, e));
    });
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) x[j][e] *= sbeta[acc_row(rs, lane, e)];
    store_acc_f32(a.dV + toff, DH, x, rs, cw, 8, lane);
    zero_acc<8>(x);
    mm_atb<8>(x, sTb, LD64, sW, LD, rs, cw, CH, lane);   // dKw = T^T dW
    float sw_lo = 0.f, sw_hi = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = acc_row(rs, lane, e), c = acc_col(cw, j, lane, e);
        (e < 2 ? sw_lo : sw_hi) += x[j][e] * bf(sK + i * LD + c);
        dk[j][e] += x[j][e] * sbeta[i] * seb[i];
      }
    sw_lo = quad_sum(sw_lo);
    sw_hi = quad_sum(sw_hi);
    if ((lane & 3) == 0) {
      const int i0 = rs + (lane >> 2), i1 = i0 + 8;
      atomicAdd(sdbeta + i0, sw_lo * seb[i0]);
      atomicAdd(sdbeta + i1, sw_hi * seb[i1]);
      atomicAdd(sdb + i0, sw_lo * seb[i0] * sbeta[i0]);
      atomicAdd(sdb + i1, sw_hi * seb[i1] * sbeta[i1]);
    }
  }
  __syncthreads();

  // ---- phase 5: dA = -T^T (dT T^T), fp32 on CUDA cores, 4x4 outputs per thread. T is lower
  // triangular, so X[i][j] sums k <= j and dA[i][j] sums k >= i; each warp shares its bound. ----
  {
    const int i0 = 4 * (tid & 15), j0 = 4 * (tid >> 4);
    float x[4][4] = {};
    for (int k = 0; k < j0 + 4; ++k) {   // X = dT T^T: X[i][j] = sum_k dT[i][k] T[j][k]
      float l[4], r[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        l[q] = sdT[(i0 + q) * LDF + k];
        r[q] = sT[(j0 + q) * LDF + k];
      }
#pragma unroll
      for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int q = 0; q < 4; ++q) x[p][q] += l[p] * r[q];
    }
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
      for (int q = 0; q < 4; ++q) sX[(i0 + p) * LDF + j0 + q] = x[p][q];
  }
  __syncthreads();
  {
    const int i0 = 4 * (tid >> 4), j0 = 4 * (tid & 15);
    float x[4][4] = {};
    for (int k = i0; k < CH; ++k) {   // dA[i][j] = -sum_k T[k][i] X[k][j]
      float l[4], r[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        l[q] = sT[k * LDF + i0 + q];
        r[q] = sX[k * LDF + j0 + q];
      }
#pragma unroll
      for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int q = 0; q < 4; ++q) x[p][q] -= l[p] * r[q];
    }
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
      for (int q = 0; q < 4; ++q) sdT[(i0 + p) * LDF + j0 + q] = x[p][q];   // dT is dead: reuse for dA
  }
  __syncthreads();

  // ---- phase 6: dA through A = beta_i KK E (strict lower): beta, b and M = dKK + dKK^T (-> sTb) ----
  {
    float kk[4][4];
    zero_acc<4>(kk);
    mm_abt<4>(kk, sK, LD, sK, LD, rs, cb, DH, lane);
    float row_lo = 0.f, row_hi = 0.f, rb_lo = 0.f, rb_hi = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float col[2] = {0.f, 0.f};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = acc_row(rs, lane, e), c = acc_col(cb, j, lane, e);
        float m = 0.f;
        if (c < i) {
          const float ev = __expf(sb[i] - sb[c]);
          const float da = sdT[i * LDF + c];
          const float kke = kk[j][e] * ev;
          const float ta = da * sbeta[i] * kke;
          (e < 2 ? rb_lo : rb_hi) += da * kke;
          (e < 2 ? row_lo : row_hi) += ta;
          col[e & 1] += ta;
          m = da * ev * sbeta[i];
          sTb[c * LD64 + i] = __float2bfloat16(m);   // upper mirror
        } else if (c == i) {
          sTb[i * LD64 + i] = __float2bfloat16(0.f);
        }
        if (c <= i) sTb[i * LD64 + c] = __float2bfloat16(m);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float v = column_sum(col[h]);
        if ((lane >> 2) == 0) atomicAdd(sdb + cb + 8 * j + 2 * (lane & 3) + h, -v);
      }
    }
    row_lo = quad_sum(row_lo);
    row_hi = quad_sum(row_hi);
    rb_lo = quad_sum(rb_lo);
    rb_hi = quad_sum(rb_hi);
    if ((lane & 3) == 0) {
      const int i0 = rs + (lane >> 2);
      atomicAdd(sdb + i0, row_lo);
      atomicAdd(sdb + i0 + 8, row_hi);
      atomicAdd(sdbeta + i0, rb_lo);
      atomicAdd(sdbeta + i0 + 8, rb_hi);
    }
  }
  __syncthreads();

  // ---- phase 7: dK += M K (store); dG = reverse cumsum(db) with db_C += d b_C; dBeta ----
  mm_ab<8>(dk, sTb, LD64, sK, LD, rs, cw, CH, lane);
  store_acc_f32(a.dK + toff, DH, dk, rs, cw, 8, lane);
  if (warp == 0) {
    const float gamma = __expf(bc);
    float d0 = sdb[2 * lane], d1 = sdb[2 * lane + 1];
    if (lane == 31) d1 += sscal[1] + sscal[0] * gamma;
    // reverse inclusive scan: dg_i = sum_{j >= i} db_j
    float s = d0 + d1;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const float v = __shfl_down_sync(0xffffffffu, s, off);
      if (lane + off < 32) s += v;
    }
    const float after = s - (d0 + d1);   // sum over pairs to the right
    a.dG[(size_t)cta * CH + 2 * lane + 1] = after + d1;
    a.dG[(size_t)cta * CH + 2 * lane] = after + d1 + d0;
    a.dB[(size_t)cta * CH + 2 * lane] = sdbeta[2 * lane];
    a.dB[(size_t)cta * CH + 2 * lane + 1] = sdbeta[2 * lane + 1];
  }
}

// ---- tcgen05 chunk preparation ------------------------------------------------------------------
//
// Same outputs as gdn_prep_kernel. One CTA per (chunk, head), 256 threads, two CTAs per SM (about
// 102 KB of shared memory and 256 TMEM columns each). Thread 0 loads K, Q and V with TMA (128-byte
// swizzle, K and Q stacked as one 128-row tile) and issues the tensor-core products; all eight warps
// run the element-wise steps on TMEM rows (warp w reads lanes 32 (w % 4) ..+31, and warps w and
// w + 4 split the columns):
//   1. G = [K; Q] K^T: one M = 128 product (rows 0-63 K K^T, rows 64-127 Q K^T; N = 64, K = 128)
//      -> the masked, decayed A = tril(beta K K^T E, -1) (fp32, shared) and P = tril(Q K^T E) (bf16)
//   2. T = (I + A)^-1 on the CUDA cores (fp32), then Tw = T diag(beta e^b), Tv = T diag(beta) as
//      bf16 K-major tiles
//   3. W^T = K^T Tw^T and U^T = V^T Tv^T (M = 128 key / value dims, N = 64 events, K = 64): K and V
//      are read as the MN-major A operand, so no transposed copy is made; the rows leave through a
//      row-major staging tile in [event][dim] order.
// Qd = e^b Q and Kt = e^{b_C - b} K are written from the swizzled tiles while product 1 runs. Every
// wait is bounded (status codes 41-43); on expiry the CTA stops issuing, waits (bounded) for what
// it has in flight, frees its TMEM and returns.
constexpr int TC_THREADS = 256;
constexpr uint32_t TC_ATOM_KQ = 128 * 128;           // one 64-column atom of the stacked [K; Q] tile
constexpr uint32_t TC_KQ = 0;                        // [2 atoms][128 rows][128 B]
constexpr uint32_t TC_ATOM_V = 64 * 128;
constexpr uint32_t TC_V = TC_KQ + 2 * TC_ATOM_KQ;    // [2 atoms][64 rows][128 B]
constexpr uint32_t TC_TW = TC_V + 2 * TC_ATOM_V;     // [64 rows][128 B]
constexpr uint32_t TC_TV = TC_TW + 64 * 128;
constexpr uint32_t TC_A = TC_TV + 64 * 128;          // fp32 [64][LDF]
constexpr uint32_t TC_T = TC_A + CH * LDF * 4;
constexpr uint32_t TC_Y = TC_T + CH * LDF * 4;       // inverse scratch, 3 x 16 x 17 floats
constexpr uint32_t TC_VEC = TC_Y + 3 * 16 * 17 * 4;  // b, e^b, e^{b_C - b}, beta, g
constexpr uint32_t TC_BAR = (TC_VEC + 5 * CH * 4 + 7) & ~7u;
constexpr uint32_t TC_SMEM = TC_BAR + 64 + 1024;     // + slack to align the base to 1024 bytes
constexpr int TC_TMEM_COLS = 256;                    // G: 0-63, W^T: 64-127, U^T: 128-191
constexpr int TC_OUT_LD = DH + 8;                    // bf16 row of the W / U staging tiles
static_assert(2 * CH * TC_OUT_LD * 2 <= TC_TW, "W / U staging must fit in the K, Q, V tiles");
static_assert(2 * TC_SMEM <= 232448, "two preparation CTAs must fit on one SM");

__global__ void __launch_bounds__(TC_THREADS, 2)
    gdn_prep_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                       const __grid_constant__ CUtensorMap map_v, PrepArgs a, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_tc[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_tc) + 1023) & ~uintptr_t(1023));
  uint8_t* kq = smem + TC_KQ;
  uint8_t* sv = smem + TC_V;
  uint8_t* tw = smem + TC_TW;
  uint8_t* tv = smem + TC_TV;
  float* sA = reinterpret_cast<float*>(smem + TC_A);
  float* sT = reinterpret_cast<float*>(smem + TC_T);
  float* sY = reinterpret_cast<float*>(smem + TC_Y);
  float* sb = reinterpret_cast<float*>(smem + TC_VEC);
  float* seb = sb + CH;
  float* skd = seb + CH;
  float* sbeta = skd + CH;
  float* sg = sbeta + CH;
  uint64_t* load_bar = reinterpret_cast<uint64_t*>(smem + TC_BAR);
  uint64_t* mma_bar = load_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(load_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int unit = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const size_t tile_off = (size_t)unit * CH * DH;
  if (tid == 0) {
    tc::mbar_init(load_bar, 1);
    tc::mbar_init(mma_bar, 1);
    *abort_flag = 0;
    tc::fence_mbar_init();
  }
  if (warp == 0) tc::tmem_alloc(tmem_slot, TC_TMEM_COLS);
  if (tid < CH) {
    sg[tid] = a.G[(size_t)unit * CH + tid];
    sbeta[tid] = a.B[(size_t)unit * CH + tid];
  }
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) {
    tc::prefetch_map(&map_q);
    tc::prefetch_map(&map_k);
    tc::prefetch_map(&map_v);
    tc::mbar_expect_tx(load_bar, 3 * CH * DH * 2);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      tc::tma_load_2d(kq + h * TC_ATOM_KQ, &map_k, load_bar, h * 64, unit * CH);
      tc::tma_load_2d(kq + h * TC_ATOM_KQ + CH * 128, &map_q, load_bar, h * 64, unit * CH);
      tc::tma_load_2d(sv + h * TC_ATOM_V, &map_v, load_bar, h * 64, unit * CH);
    }
  }
  if (warp == 1) {
    const float bc = chunk_decay(sg, sb, seb, skd, lane);
    if (lane == 0) a.gamma[unit] = __expf(bc);
  }
  bool load_seen = tc::mbar_wait(load_bar, 0, status, abort_flag, 41);
  bool ok = __syncthreads_and(load_seen);   // also publishes the decay vectors
  bool mma1 = false, mma2 = false;
  if (ok && tid == 0) {
    tc::fence_after();
    constexpr uint32_t idesc = tc::idesc_bf16(128, 64, false, false);
    const uint32_t base = tc::smem_u32(kq);
#pragma unroll
    for (int k = 0; k < DH / 16; ++k) {
      const uint32_t off = (k >> 2) * TC_ATOM_KQ + (k & 3) * 32;
      tc::mma_bf16(tmem, tc::smem_desc(base + off, 16, 1024), tc::smem_desc(base + off, 16, 1024), idesc, k > 0);
    }
    tc::mma_commit(mma_bar);
  }
  mma1 = ok;
  if (ok) {   // Qd = e^b Q (Q: rows 64-127 of the stacked tile), Kt = e^{b_C - b} K
    for (int e = tid; e < 2 * CH * 16; e += TC_THREADS) {
      const int kt = e >= CH * 16, r = (e >> 4) & (CH - 1), ch = e & 15;
      const uint8_t* src = kq + (ch >> 3) * TC_ATOM_KQ + (kt ? 0 : CH * 128) + r * 128 + (((ch & 7) ^ (r & 7)) << 4);
      float v[8];
      load8(reinterpret_cast<const __nv_bfloat16*>(src), v);
      const float sc = kt ? skd[r] : seb[r];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] *= sc;
      store8((kt ? a.Kt : a.Qd) + tile_off + r * DH + ch * 8, v);
    }
  }
  bool seen1 = !mma1 || tc::mbar_wait(mma_bar, 0, status, abort_flag, 42);
  ok = __syncthreads_and(ok && seen1);
  tc::fence_after();
  const int quad = warp & 3, half = warp >> 2, row = 32 * quad + lane;
  const uint32_t lane_base = tmem + ((uint32_t)(32 * quad) << 16);
  if (ok) {
    float v[32];
    tc::tmem_ld32(lane_base + 32 * half, v);
    if (row < CH) {   // A row i
      const float bi = sb[row], be = sbeta[row];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const int j = 32 * half + c;
        sA[row * LDF + j] = j < row ? be * v[c] * __expf(bi - sb[j]) : 0.f;
      }
    } else {          // P row i
      const int i = row - CH;
      const float bi = sb[i];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const int j = 32 * half + c;
        v[c] = j <= i ? v[c] * __expf(bi - sb[j]) : 0.f;
      }
      __nv_bfloat16* dst = a.P + ((size_t)unit * CH + i) * CH + 32 * half;
#pragma unroll
      for (int q = 0; q < 4; ++q) store8(dst + 8 * q, v + 8 * q);
    }
  }
  __syncthreads();
  unit_lower_inverse(sA, sT, sY, warp, lane);
  for (int e = tid; e < CH * 8; e += TC_THREADS) {   // Tw, Tv: row i, 16-byte chunk ch (8 columns)
    const int i = e >> 3, ch = e & 7;
    float w8[8], v8[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int j = 8 * ch + q;
      const float t = sT[i * LDF + j] * sbeta[j];
      v8[q] = t;
      w8[q] = t * seb[j];
    }
    const uint32_t off = i * 128 + ((ch ^ (i & 7)) << 4);
    store8(reinterpret_cast<__nv_bfloat16*>(tw + off), w8);
    store8(reinterpret_cast<__nv_bfloat16*>(tv + off), v8);
  }
  tc::fence_proxy_async();
  __syncthreads();
  if (ok && tid == 0) {
    tc::fence_after();
    constexpr uint32_t idesc = tc::idesc_bf16(128, 64, true, false);   // A = K^T / V^T, MN-major
    const uint32_t kb = tc::smem_u32(kq), vb = tc::smem_u32(sv), wb = tc::smem_u32(tw), ub = tc::smem_u32(tv);
#pragma unroll
    for (int k = 0; k < CH / 16; ++k) {
      tc::mma_bf16(tmem + 64, tc::smem_desc(kb + k * 2048, TC_ATOM_KQ, 1024), tc::smem_desc(wb + k * 32, 16, 1024),
                   idesc, k > 0);
      tc::mma_bf16(tmem + 128, tc::smem_desc(vb + k * 2048, TC_ATOM_V, 1024), tc::smem_desc(ub + k * 32, 16, 1024),
                   idesc, k > 0);
    }
    tc::mma_commit(mma_bar);
  }
  mma2 = ok;
  bool seen2 = !mma2 || tc::mbar_wait(mma_bar, 1, status, abort_flag, 43);
  ok = __syncthreads_and(ok && seen2);
  tc::fence_after();
  __nv_bfloat16* stw = reinterpret_cast<__nv_bfloat16*>(smem + TC_KQ);   // the products have retired
  __nv_bfloat16* stu = stw + CH * TC_OUT_LD;
  if (ok) {
    float v[32];
    tc::tmem_ld32(lane_base + 64 + 32 * half, v);
#pragma unroll
    for (int c = 0; c < 32; ++c) stw[(32 * half + c) * TC_OUT_LD + row] = __float2bfloat16(v[c]);
    tc::tmem_ld32(lane_base + 128 + 32 * half, v);
#pragma unroll
    for (int c = 0; c < 32; ++c) stu[(32 * half + c) * TC_OUT_LD + row] = __float2bfloat16(v[c]);
  }
  __syncthreads();
  if (ok) {
    for (int e = tid; e < 2 * CH * 16; e += TC_THREADS) {
      const int second = e >= CH * 16, r = (e >> 4) & (CH - 1), ch = e & 15;
      const __nv_bfloat16* src = (second ? stu : stw) + r * TC_OUT_LD + ch * 8;
      *reinterpret_cast<uint4*>((second ? a.U : a.W) + tile_off + r * DH + ch * 8) =
          *reinterpret_cast<const uint4*>(src);
    }
  }
  if (tid == 0) {   // nothing issued by this CTA is still in flight when it retires (bounded)
    const unsigned long long t0 = tc::globaltimer();
    if (!load_seen)
      while (!tc::mbar_try_wait(load_bar, 0) && tc::globaltimer() - t0 < tc::kWaitNs) {
      }
    if (mma1 && !seen1)
      while (!tc::mbar_try_wait(mma_bar, 0) && tc::globaltimer() - t0 < tc::kWaitNs) {
      }
    if (mma2 && !seen2)
      while (!tc::mbar_try_wait(mma_bar, 1) && tc::globaltimer() - t0 < tc::kWaitNs) {
      }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, TC_TMEM_COLS);
}

// ---- tcgen05 fused chunk backward ------------------------------------------------------------
//
// Same math and outputs as gdn_chunk_bwd_kernel (see its comment), one CTA per (chunk, head), 256
// threads, one CTA per SM, all 512 TMEM columns. Every matrix product is a tcgen05.mma issued by
// thread 0 with M = 128. Products whose result feeds another product as a [dim][event] operand
// are computed transposed (M = the 128-wide key / value dim, N = 64 events: W^T, U^T, Delta^T,
// dDelta^T); products whose epilogue reduces over the feature dim per event keep the event as M,
// with the upper 64 rows of the A operand reading the next 8 KB of shared memory (their TMEM
// lanes 64-127 are never read). Operand transposes are MN-major descriptors, never copies.
// [Q; K] is one stacked 128-row TMA tile, so G = [Q; K] K^T gives Q K^T in lanes 0-63 (read by
// the threads that own the same event rows of dP) and K K^T in lanes 64-127 (the A path).
// TMEM columns: G 0-63 (kept to the end), then per group:
//   P2  W^T 64-127, U^T 128-191
//   P3  S^T W^T 192-255, dO^T P 256-319, dS^T K^T 320-383, dQ (natural) 384-511
//   P4a dW 64-191, dK (natural, accumulated to the end) 192-319, dP 320-383
//   P4b T1 = dDelta V^T 64-127, T2 = dW K^T 128-191, dQ += dPm K, dK += dPm^T Q
//   P4c dVb = T^T dDelta 64-191, dKw = T^T dW 384-511
//   P7  dK += M K
// The fp32 T, dT and dA (the triangular inverse and dA = -T^T dT T^T) stay on the CUDA cores as
// in the mma.sync kernel. Bounded waits, status codes 61-68.
namespace cb {
constexpr uint32_t ATOM_KQ = 128 * 128;          // one 64-column atom of a 128-row tile
constexpr uint32_t ATOM64 = 64 * 128;            // one 64-column atom of a 64-row tile
constexpr uint32_t KQ = 0;                       // [Q; K]: Q rows 0-63, K rows 64-127 of each atom
constexpr uint32_t K_OFF = 64 * 128;
constexpr uint32_t V = KQ + 2 * ATOM_KQ;
constexpr uint32_t DO = V + 2 * ATOM64;
constexpr uint32_t SB = DO + 2 * ATOM64;         // bf16 S [2 atoms (v)][128 rows (d)]; later fp32 dT
constexpr uint32_t DSB = SB + 2 * ATOM_KQ;       // bf16 dS; later fp32 X
constexpr uint32_t W = DSB + 2 * ATOM_KQ;        // W [i][d], later dW
constexpr uint32_t DL = W + 2 * ATOM64;          // Delta^T [128 rows (v)][64 events]
constexpr uint32_t P = DL + ATOM_KQ;             // P [i][j], later dPm
constexpr uint32_t TB = P + ATOM64;              // bf16 T [i][j], later M
constexpr uint32_t R1 = TB + ATOM64;             // fp32 A, then Tw | Tv, then dDelta^T [128 rows (v)][64]
constexpr uint32_t R1_BYTES = 17408;
constexpr uint32_t TF = R1 + R1_BYTES;           // fp32 T [64][LDF]
constexpr uint32_t VEC = TF + 17408;             // b, eb, kd, beta, g, db, dbeta (64 each), scal[4], inverse scratch
constexpr uint32_t BAR = VEC + 5120;
constexpr uint32_t SMEM = BAR + 64 + 1024;
static_assert(CH * LDF * 4 <= R1_BYTES && 2 * ATOM64 <= R1_BYTES && ATOM_KQ <= R1_BYTES, "R1 region");
static_assert(CH * LDF * 4 <= 17408 && CH * LDF * 4 <= 2 * ATOM_KQ, "fp32 T / dT / X tiles");
static_assert(7 * CH * 4 + 16 + 3 * 16 * 17 * 4 <= 5120, "vectors and inverse scratch");
static_assert(SMEM <= 232448, "chunk backward exceeds one CTA's shared memory");
}  // namespace cb

// bf16 element (row, col) of a 128-byte-swizzled tile whose 64-column atoms are `atom` bytes apart.
__device__ __forceinline__ uint32_t swz(uint32_t row, uint32_t col, uint32_t atom) {
  return (col >> 6) * atom + row * 128 + (((((col & 63) >> 3) ^ row) & 7) << 4) + (col & 7) * 2;
}
__device__ __forceinline__ float ldsb(const uint8_t* base, uint32_t off) {
  return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(base + off));
}
__device__ __forceinline__ void stsb(uint8_t* base, uint32_t off, float v) {
  *reinterpret_cast<__nv_bfloat16*>(base + off) = __float2bfloat16(v);
}

__global__ void __launch_bounds__(TC_THREADS, 1)
    gdn_chunk_bwd_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                            const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_do,
                            const __grid_constant__ CUtensorMap map_s, const __grid_constant__ CUtensorMap map_ds,
                            BwdArgs a, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_tc[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_tc) + 1023) & ~uintptr_t(1023));
  uint8_t* kq = sm + cb::KQ;
  uint8_t* sv = sm + cb::V;
  uint8_t* sdo = sm + cb::DO;
  uint8_t* ssb = sm + cb::SB;
  uint8_t* sdsb = sm + cb::DSB;
  uint8_t* sw = sm + cb::W;
  uint8_t* sdl = sm + cb::DL;
  uint8_t* sp = sm + cb::P;
  uint8_t* stb = sm + cb::TB;
  uint8_t* r1 = sm + cb::R1;
  float* sA = reinterpret_cast<float*>(r1);
  float* sT = reinterpret_cast<float*>(sm + cb::TF);
  float* sdT = reinterpret_cast<float*>(ssb);
  float* sX = reinterpret_cast<float*>(sdsb);
  float* sb = reinterpret_cast<float*>(sm + cb::VEC);
  float* seb = sb + CH;
  float* skd = seb + CH;
  float* sbeta = skd + CH;
  float* sg = sbeta + CH;
  float* sdb = sg + CH;
  float* sdbeta = sdb + CH;
  float* sscal = sdbeta + CH;    // [0] dgamma = <S, dS>, [1] d b_C from Kt
  float* sinv = sscal + 4;       // triangular-inverse scratch, 3 x 16 x 17
  uint64_t* load_bar = reinterpret_cast<uint64_t*>(sm + cb::BAR);
  uint64_t* mma_bar = load_bar + 1;
  uint64_t* state_bar = load_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(load_bar + 3);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int unit = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, hf = warp >> 2, row = 32 * quad + lane;
  const size_t toff = (size_t)unit * CH * DH;
  if (tid == 0) {
    tc::mbar_init(load_bar, 1);
    tc::mbar_init(mma_bar, 1);
    tc::mbar_init(state_bar, 1);
    *abort_flag = 0;
    tc::fence_mbar_init();
  }
  if (warp == 0) tc::tmem_alloc(tmem_slot, 512);
  if (tid < CH) {
    sg[tid] = a.G[(size_t)unit * CH + tid];
    sbeta[tid] = a.B[(size_t)unit * CH + tid];
    sdb[tid] = 0.f;
    sdbeta[tid] = 0.f;
  }
  if (tid == 0) {
    sscal[0] = a.dgamma[unit];
    sscal[1] = 0.f;
  }
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lb = tmem + ((uint32_t)(32 * quad) << 16);   // this warp's TMEM lane quadrant
  if (tid == 0) {
    tc::prefetch_map(&map_q);
    tc::prefetch_map(&map_k);
    tc::prefetch_map(&map_v);
    tc::prefetch_map(&map_do);
    tc::prefetch_map(&map_s);
    tc::prefetch_map(&map_ds);
    tc::mbar_expect_tx(load_bar, 4 * CH * DH * 2);
#pragma unroll
    for (int x = 0; x < 2; ++x) {
      tc::tma_load_2d(kq + x * cb::ATOM_KQ, &map_q, load_bar, 64 * x, unit * CH);
      tc::tma_load_2d(kq + x * cb::ATOM_KQ + cb::K_OFF, &map_k, load_bar, 64 * x, unit * CH);
      tc::tma_load_2d(sv + x * cb::ATOM64, &map_v, load_bar, 64 * x, unit * CH);
      tc::tma_load_2d(sdo + x * cb::ATOM64, &map_do, load_bar, 64 * x, unit * CH);
    }
    // the bf16 states [2 atoms (v)][128 rows (d)] land while the first products run
    tc::mbar_expect_tx(state_bar, 2 * DH * DH * 2);
#pragma unroll
    for (int x = 0; x < 2; ++x) {
      tc::tma_load_2d(ssb + x * cb::ATOM_KQ, &map_s, state_bar, 64 * x, unit * DH);
      tc::tma_load_2d(sdsb + x * cb::ATOM_KQ, &map_ds, state_bar, 64 * x, unit * DH);
    }
  }
  if (warp == 1) chunk_decay(sg, sb, seb, skd, lane);
  const bool loaded = tc::mbar_wait(load_bar, 0, status, abort_flag, 61);
  bool ok = __syncthreads_and(loaded);   // also publishes the decay vectors
  bool states_seen = false;
  uint32_t phase = 0;
  bool pending = false;
  auto commit_wait = [&](int code) {
    if (tid == 0 && ok) {
      tc::mma_commit(mma_bar);
      pending = true;
    }
    const bool seen = !ok || tc::mbar_wait(mma_bar, phase & 1, status, abort_flag, code);
    ok = __syncthreads_and(ok && seen);
    if (ok) pending = false;
    ++phase;
    tc::fence_after();
  };
  const uint32_t kq_a = tc::smem_u32(kq), v_a = tc::smem_u32(sv), do_a = tc::smem_u32(sdo);
  const uint32_t sb_a = tc::smem_u32(ssb), dsb_a = tc::smem_u32(sdsb), w_a = tc::smem_u32(sw);
  const uint32_t dl_a = tc::smem_u32(sdl), p_a = tc::smem_u32(sp), tb_a = tc::smem_u32(stb), r1_a = tc::smem_u32(r1);
  const uint32_t k_a = kq_a + cb::K_OFF;
  // K-major / MN-major descriptors of the k-th 16-wide K step
  auto kmaj = [](uint32_t base, uint32_t atom, int k) { return tc::smem_desc(base + (k >> 2) * atom + (k & 3) * 32, 16, 1024); };
  auto mnmaj = [](uint32_t base, uint32_t lbo, int k) { return tc::smem_desc(base + k * 2048, lbo, 1024); };

  // ---- P1: G = [Q; K] K^T -> P (rows 0-63) and A (rows 64-127) ----
  if (ok && tid == 0) {
    tc::fence_after();
    constexpr uint32_t id = tc::idesc_bf16(128, 64, false, false);
#pragma unroll
    for (int k = 0; k < DH / 16; ++k) tc::mma_bf16(tmem, kmaj(kq_a, cb::ATOM_KQ, k), kmaj(k_a, cb::ATOM_KQ, k), id, k > 0);
  }
  commit_wait(62);
  if (ok) {
    float x[32];
    tc::tmem_ld32(lb + 32 * hf, x);
    const int i = row & 63;
    const float bi = sb[i];
    if (row >= CH) {   // K K^T row i -> A
      const float be = sbeta[i];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const int j = 32 * hf + c;
        sA[i * LDF + j] = j < i ? be * x[c] * __expf(bi - sb[j]) : 0.f;
      }
    } else {           // Q K^T row i -> P (bf16 [i][j])
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        float p[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int j = 32 * hf + 8 * c8 + q;
          p[q] = j <= i ? x[8 * c8 + q] * __expf(bi - sb[j]) : 0.f;
        }
        store8(reinterpret_cast<__nv_bfloat16*>(sp + swz(i, 32 * hf + 8 * c8, cb::ATOM64)), p);
      }
    }
  }
  __syncthreads();
  unit_lower_inverse(sA, sT, sinv, warp, lane);
  // T (bf16), Tw = T diag(beta e^b), Tv = T diag(beta): [i][j] tiles (Tw, Tv over the dead A)
  for (int e = tid; e < CH * 8; e += TC_THREADS) {
    const int i = e >> 3, c8 = (e & 7) * 8;
    float t[8], tw8[8], tv8[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int j = c8 + q;
      t[q] = sT[i * LDF + j];
      tv8[q] = t[q] * sbeta[j];
      tw8[q] = tv8[q] * seb[j];
    }
    const uint32_t off = swz(i, c8, cb::ATOM64);
    store8(reinterpret_cast<__nv_bfloat16*>(stb + off), t);
    store8(reinterpret_cast<__nv_bfloat16*>(r1 + off), tw8);
    store8(reinterpret_cast<__nv_bfloat16*>(r1 + cb::ATOM64 + off), tv8);
  }
  tc::fence_proxy_async();
  __syncthreads();

  // ---- P2: W^T = K^T Tw^T, U^T = V^T Tv^T (K, V as MN-major A) ----
  if (ok && tid == 0) {
    tc::fence_after();
    constexpr uint32_t id = tc::idesc_bf16(128, 64, true, false);
#pragma unroll
    for (int k = 0; k < CH / 16; ++k) {
      tc::mma_bf16(tmem + 64, mnmaj(k_a, cb::ATOM_KQ, k), kmaj(r1_a, cb::ATOM64, k), id, k > 0);
      tc::mma_bf16(tmem + 128, mnmaj(v_a, cb::ATOM64, k), kmaj(r1_a + cb::ATOM64, cb::ATOM64, k), id, k > 0);
    }
  }
  commit_wait(63);
  if (ok) {   // W [i][d] from W^T row d = row (events 32 hf ..)
    float x[32];
    tc::tmem_ld32(lb + 64 + 32 * hf, x);
#pragma unroll
    for (int c = 0; c < 32; ++c) stsb(sw, swz(32 * hf + c, row, cb::ATOM64), x[c]);
  }
  tc::fence_proxy_async();
  tc::fence_before();
  __syncthreads();

  // ---- P3: S^T W^T, dO^T P, dS^T K^T (transposed, lanes = v) and dQd = dO S^T (lanes = i) ----
  if (ok && tid == 0) states_seen = tc::mbar_wait(state_bar, 0, status, abort_flag, 69);
  ok = __syncthreads_and(ok && (tid != 0 || states_seen));
  if (ok && tid == 0) {
    tc::fence_after();
    constexpr uint32_t id_t = tc::idesc_bf16(128, 64, true, false);
    constexpr uint32_t id_op = tc::idesc_bf16(128, 64, true, true);
    constexpr uint32_t id_n = tc::idesc_bf16(128, 128, false, false);
#pragma unroll
    for (int k = 0; k < DH / 16; ++k) {
      tc::mma_bf16(tmem + 192, mnmaj(sb_a, cb::ATOM_KQ, k), kmaj(w_a, cb::ATOM64, k), id_t, k > 0);
      tc::mma_bf16(tmem + 320, mnmaj(dsb_a, cb::ATOM_KQ, k), kmaj(k_a, cb::ATOM_KQ, k), id_t, k > 0);
      tc::mma_bf16(tmem + 384, kmaj(do_a, cb::ATOM64, k), kmaj(sb_a, cb::ATOM_KQ, k), id_n, k > 0);
    }
#pragma unroll
    for (int k = 0; k < CH / 16; ++k)
      tc::mma_bf16(tmem + 256, mnmaj(do_a, cb::ATOM64, k), mnmaj(p_a, cb::ATOM64, k), id_op, k > 0);
  }
  commit_wait(64);
  if (ok) {
    // Delta^T = U^T - S^T W^T and dDelta^T = dO^T P + kd dS^T K^T, rows v = row, events 32 hf ..
    float u[32], x[32], y[32], z[32];
    tc::tmem_ld32(lb + 128 + 32 * hf, u);
    tc::tmem_ld32(lb + 192 + 32 * hf, x);
    tc::tmem_ld32(lb + 256 + 32 * hf, y);
    tc::tmem_ld32(lb + 320 + 32 * hf, z);
#pragma unroll
    for (int c8 = 0; c8 < 4; ++c8) {
      float dl[8], dd[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int c = 8 * c8 + q, i = 32 * hf + c;
        dl[q] = u[c] - x[c];
        dd[q] = y[c] + skd[i] * z[c];
      }
      const uint32_t off = row * 128 + ((((4 * hf + c8) ^ row) & 7) << 4);
      store8(reinterpret_cast<__nv_bfloat16*>(sdl + off), dl);
      store8(reinterpret_cast<__nv_bfloat16*>(r1 + off), dd);
    }
    if (row < CH) {   // dQd row i: db_i += e^b_i sum_d dQd Q, then dQ = e^b_i dQd (kept in TMEM)
      const int i = row;
      float part = 0.f;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int col = 64 * hf + 32 * h2;
        tc::tmem_ld32(lb + 384 + col, x);
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          part += x[c] * ldsb(kq, swz(i, col + c, cb::ATOM_KQ));
          x[c] *= seb[i];
        }
        tc::tmem_st32(lb + 384 + col, x);
      }
      atomicAdd(sdb + i, seb[i] * part);
    }
  }
  tc::fence_proxy_async();
  tc::fence_before();
  __syncthreads();

  // ---- P4a: dW = -dDelta S^T, dKt = Delta dS^T, dP = dO Delta^T (lanes = i) ----
  if (ok && tid == 0) {
    tc::fence_after();
    constexpr uint32_t id_n = tc::idesc_bf16(128, 128, true, false);
    constexpr uint32_t id_p = tc::idesc_bf16(128, 64, false, true);
#pragma unroll
    for (int k = 0; k < DH / 16; ++k) {
      tc::mma_bf16(tmem + 64, mnmaj(r1_a, cb::ATOM_KQ, k), kmaj(sb_a, cb::ATOM_KQ, k), id_n, k > 0);
      tc::mma_bf16(tmem + 192, mnmaj(dl_a, cb::ATOM_KQ, k), kmaj(dsb_a, cb::ATOM_KQ, k), id_n, k > 0);
      tc::mma_bf16(tmem + 320, kmaj(do_a, cb::ATOM64, k), mnmaj(dl_a, cb::ATOM_KQ, k), id_p, k > 0);
    }
  }
  commit_wait(65);
  if (ok && row < CH) {
    const int i = row;
    float x[32];
    // dW row i (negated) -> bf16 tile over W
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const int col = 64 * hf + 32 * h2;
      tc::tmem_ld32(lb + 64 + col, x);
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        float w8[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) w8[q] = -x[8 * c8 + q];
        store8(reinterpret_cast<__nv_bfloat16*>(sw + swz(i, col + 8 * c8, cb::ATOM64)), w8);
      }
    }
    // dK = e^{b_C - b_i} dKt (TMEM); d b from Kt = e^{b_C - b} K
    float rkt = 0.f;
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const int col = 64 * hf + 32 * h2;
      tc::tmem_ld32(lb + 192 + col, x);
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        x[c] *= skd[i];
        rkt += x[c] * ldsb(kq + cb::K_OFF, swz(i, col + c, cb::ATOM_KQ));
      }
      tc::tmem_st32(lb + 192 + col, x);
    }
    atomicAdd(sdb + i, -rkt);
    atomicAdd(sscal + 1, rkt);
    // dP row i, events 32 hf ..: dPm = dP E (j <= i) -> bf16 over P; t = dPm (Q K^T)
    float qk[32];
    tc::tmem_ld32(lb + 320 + 32 * hf, x);
    tc::tmem_ld32(lb + 32 * hf, qk);
    const float bi = sb[i];
    float rsum = 0.f;
#pragma unroll
    for (int c8 = 0; c8 < 4; ++c8) {
      float m8[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int c = 8 * c8 + q, j = 32 * hf + c;
        const float dpm = j <= i ? x[c] * __expf(bi - sb[j]) : 0.f;
        m8[q] = dpm;
        const float t = dpm * qk[c];
        rsum += t;
        x[c] = t;   // column contribution
      }
      store8(reinterpret_cast<__nv_bfloat16*>(sp + swz(i, 32 * hf + 8 * c8, cb::ATOM64)), m8);
    }
    atomicAdd(sdb + i, rsum);
#pragma unroll
    for (int c = 0; c < 32; ++c) {   // column sums over the rows of this warp
      const float v = warp_sum(x[c]);
      if (lane == 0) atomicAdd(sdb + 32 * hf + c, -v);
    }
  }
  tc::fence_proxy_async();
  tc::fence_before();
  __syncthreads();

  // ---- P4b: T1 = dDelta V^T, T2 = dW K^T; dQ += dPm K; dK += dPm^T Q ----
  if (ok && tid == 0) {
    tc::fence_after();
    constexpr uint32_t id_t1 = tc::idesc_bf16(128, 64, true, false);
    constexpr uint32_t id_t2 = tc::idesc_bf16(128, 64, false, false);
    constexpr uint32_t id_q = tc::idesc_bf16(128, 128, false, true);
    constexpr uint32_t id_k = tc::idesc_bf16(128, 128, true, true);
#pragma unroll
    for (int k = 0; k < DH / 16; ++k) {
      tc::mma_bf16(tmem + 64, mnmaj(r1_a, cb::ATOM_KQ, k), kmaj(v_a, cb::ATOM64, k), id_t1, k > 0);
      tc::mma_bf16(tmem + 128, kmaj(w_a, cb::ATOM64, k), kmaj(k_a, cb::ATOM_KQ, k), id_t2, k > 0);
    }
#pragma unroll
    for (int k = 0; k < CH / 16; ++k) {
      tc::mma_bf16(tmem + 384, kmaj(p_a, cb::ATOM64, k), mnmaj(k_a, cb::ATOM_KQ, k), id_q, 1u);
      tc::mma_bf16(tmem + 192, mnmaj(p_a, cb::ATOM64, k), mnmaj(kq_a, cb::ATOM_KQ, k), id_k, 1u);
    }
  }
  commit_wait(66);
  if (ok && row < CH) {
    const int i = row;
    float x[32], y[32];
    tc::tmem_ld32(lb + 64 + 32 * hf, x);
    tc::tmem_ld32(lb + 128 + 32 * hf, y);
#pragma unroll
    for (int c = 0; c < 32; ++c) {
      const int j = 32 * hf + c;
      sdT[i * LDF + j] = sbeta[j] * (x[c] + seb[j] * y[c]);
    }
    float* dq = a.dQ + toff + (size_t)i * DH;
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const int col = 64 * hf + 32 * h2;
      tc::tmem_ld32(lb + 384 + col, x);
#pragma unroll
      for (int q = 0; q < 32; q += 4) *reinterpret_cast<float4*>(dq + col + q) = make_float4(x[q], x[q + 1], x[q + 2], x[q + 3]);
    }
  }
  tc::fence_before();
  __syncthreads();

  // ---- P4c: dVb = T^T dDelta, dKw = T^T dW (lanes = j) ----
  if (ok && tid == 0) {
    tc::fence_after();
    constexpr uint32_t id_v = tc::idesc_bf16(128, 128, true, false);
    constexpr uint32_t id_w = tc::idesc_bf16(128, 128, true, true);
#pragma unroll
    for (int k = 0; k < CH / 16; ++k) {
      tc::mma_bf16(tmem + 64, mnmaj(tb_a, cb::ATOM64, k), tc::smem_desc(r1_a + k * 32, 16, 1024), id_v, k > 0);
      tc::mma_bf16(tmem + 384, mnmaj(tb_a, cb::ATOM64, k), mnmaj(w_a, cb::ATOM64, k), id_w, k > 0);
    }
  }
  commit_wait(67);
  if (ok && row < CH) {
    const int j = row;
    float x[32];
    float* dv = a.dV + toff + (size_t)j * DH;
    float dbt = 0.f, swk = 0.f;
    const float bj = sbeta[j], ej = seb[j];
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const int col = 64 * hf + 32 * h2;
      tc::tmem_ld32(lb + 64 + col, x);
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        dbt += x[c] * ldsb(sv, swz(j, col + c, cb::ATOM64));
        x[c] *= bj;
      }
#pragma unroll
      for (int q = 0; q < 32; q += 4) *reinterpret_cast<float4*>(dv + col + q) = make_float4(x[q], x[q + 1], x[q + 2], x[q + 3]);
      float y[32];
      tc::tmem_ld32(lb + 384 + col, x);
      tc::tmem_ld32(lb + 192 + col, y);
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        swk += x[c] * ldsb(kq + cb::K_OFF, swz(j, col + c, cb::ATOM_KQ));
        y[c] += x[c] * bj * ej;
      }
      tc::tmem_st32(lb + 192 + col, y);
    }
    atomicAdd(sdbeta + j, dbt + swk * ej);
    atomicAdd(sdb + j, swk * ej * bj);
  }
  tc::fence_before();
  __syncthreads();

  // ---- P5: dA = -T^T (dT T^T) on the CUDA cores (T lower triangular) ----
  {
    const int i0 = 4 * (tid & 15), j0 = 4 * (tid >> 4);
    float x[4][4] = {};
    for (int k = 0; k < j0 + 4; ++k) {
      float l[4], r[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        l[q] = sdT[(i0 + q) * LDF + k];
        r[q] = sT[(j0 + q) * LDF + k];
      }
#pragma unroll
      for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int q = 0; q < 4; ++q) x[p][q] += l[p] * r[q];
    }
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
      for (int q = 0; q < 4; ++q) sX[(i0 + p) * LDF + j0 + q] = x[p][q];
  }
  __syncthreads();
  {
    const int i0 = 4 * (tid >> 4), j0 = 4 * (tid & 15);
    float x[4][4] = {};
    for (int k = i0; k < CH; ++k) {
      float l[4], r[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        l[q] = sT[k * LDF + i0 + q];
        r[q] = sX[k * LDF + j0 + q];
      }
#pragma unroll
      for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int q = 0; q < 4; ++q) x[p][q] -= l[p] * r[q];
    }
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
      for (int q = 0; q < 4; ++q) sdT[(i0 + p) * LDF + j0 + q] = x[p][q];   // dT is dead: dA
  }
  // M = dKK + dKK^T is written over T (bf16): zero it first, then each thread of the A path
  // writes its strictly-lower entries and their mirror
  for (int e = tid; e < CH * CH / 8; e += TC_THREADS) reinterpret_cast<uint4*>(stb)[e] = make_uint4(0, 0, 0, 0);
  __syncthreads();

  // ---- P6: dA through A = beta_i (K K^T) E (strict lower), K K^T from TMEM lanes 64-127 ----
  if (ok && row >= CH) {
    const int i = row - CH;
    float kk[32];
    tc::tmem_ld32(lb + 32 * hf, kk);
    const float bi = sb[i], be = sbeta[i];
    float rowsum = 0.f, rb = 0.f, col[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) {
      const int j = 32 * hf + c;
      col[c] = 0.f;
      if (j < i) {
        const float ev = __expf(bi - sb[j]);
        const float da = sdT[i * LDF + j];
        const float kke = kk[c] * ev;
        const float ta = da * be * kke;
        rb += da * kke;
        rowsum += ta;
        col[c] = ta;
        const float m = da * ev * be;
        stsb(stb, swz(i, j, cb::ATOM64), m);
        stsb(stb, swz(j, i, cb::ATOM64), m);
      }
    }
    atomicAdd(sdb + i, rowsum);
    atomicAdd(sdbeta + i, rb);
#pragma unroll
    for (int c = 0; c < 32; ++c) {
      const float v = warp_sum(col[c]);
      if (lane == 0) atomicAdd(sdb + 32 * hf + c, -v);
    }
  }
  tc::fence_proxy_async();
  tc::fence_before();
  __syncthreads();

  // ---- P7: dK += M K; dK out; dG = reverse cumsum(db) with the b_C terms; dBeta ----
  if (ok && tid == 0) {
    tc::fence_after();
    constexpr uint32_t id = tc::idesc_bf16(128, 128, false, true);
#pragma unroll
    for (int k = 0; k < CH / 16; ++k) tc::mma_bf16(tmem + 192, kmaj(tb_a, cb::ATOM64, k), mnmaj(k_a, cb::ATOM_KQ, k), id, 1u);
  }
  commit_wait(68);
  if (ok && row < CH) {
    float x[32];
    float* dk = a.dK + toff + (size_t)row * DH;
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const int col = 64 * hf + 32 * h2;
      tc::tmem_ld32(lb + 192 + col, x);
#pragma unroll
      for (int q = 0; q < 32; q += 4) *reinterpret_cast<float4*>(dk + col + q) = make_float4(x[q], x[q + 1], x[q + 2], x[q + 3]);
    }
  }
  if (ok && warp == 0) {
    const float gamma = __expf(sb[CH - 1]);
    float d0 = sdb[2 * lane], d1 = sdb[2 * lane + 1];
    if (lane == 31) d1 += sscal[1] + sscal[0] * gamma;
    float s = d0 + d1;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const float v = __shfl_down_sync(0xffffffffu, s, off);
      if (lane + off < 32) s += v;
    }
    const float after = s - (d0 + d1);
    a.dG[(size_t)unit * CH + 2 * lane + 1] = after + d1;
    a.dG[(size_t)unit * CH + 2 * lane] = after + d1 + d0;
    a.dB[(size_t)unit * CH + 2 * lane] = sdbeta[2 * lane];
    a.dB[(size_t)unit * CH + 2 * lane + 1] = sdbeta[2 * lane + 1];
  }
  if (tid == 0) {   // nothing issued by this CTA is in flight when it retires (bounded)
    const unsigned long long t0 = tc::globaltimer();
    if (!loaded)
      while (!tc::mbar_try_wait(load_bar, 0) && tc::globaltimer() - t0 < tc::kWaitNs) {
      }
    if (!states_seen)
      while (!tc::mbar_try_wait(state_bar, 0) && tc::globaltimer() - t0 < tc::kWaitNs) {
      }
    if (pending)
      while (!tc::mbar_try_wait(mma_bar, (phase - 1) & 1) && tc::globaltimer() - t0 < tc::kWaitNs) {
      }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 512);
}

bool gdn_use_tc() {
  static const bool on = [] {
    const char* v = std::getenv("CQB_GDN_TC");
    return v == nullptr || std::string(v) != "0";
  }();
  return on;
}

void check_tile(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous() && t.scalar_type() == at::kBFloat16 && t.dim() == 4 &&
                  t.size(2) == CH && t.size(3) == DH,
              name, ": contiguous bf16 [Nc, H, 64, 128]");
}

}  // namespace

// Returns (W, U, P, Qd, Kt, gamma) of every (chunk, head).
std::vector<at::Tensor> gdn_prep(at::Tensor Q, at::Tensor K, at::Tensor V, at::Tensor G, at::Tensor B) {
  check_tile(Q, "Q");
  check_tile(K, "K");
  check_tile(V, "V");
  TORCH_CHECK(K.sizes() == Q.sizes() && V.sizes() == Q.sizes(), "Q, K, V shapes differ");
  const long Nc = Q.size(0), H = Q.size(1);
  for (const auto* t : {&G, &B})
    TORCH_CHECK(t->is_cuda() && t->is_contiguous() && t->scalar_type() == at::kFloat && t->numel() == Nc * H * CH,
                "G, B: contiguous fp32 [Nc, H, 64]");
  auto W = at::empty_like(Q), U = at::empty_like(Q), Qd = at::empty_like(Q), Kt = at::empty_like(Q);
  auto P = at::empty({Nc, H, CH, CH}, Q.options());
  auto gamma = at::empty({Nc, H}, G.options());
  if (Nc * H == 0) return {W, U, P, Qd, Kt, gamma};
  PrepArgs a{(const __nv_bfloat16*)Q.data_ptr(), (const __nv_bfloat16*)K.data_ptr(),
             (const __nv_bfloat16*)V.data_ptr(), G.data_ptr<float>(), B.data_ptr<float>(),
             (__nv_bfloat16*)W.data_ptr(), (__nv_bfloat16*)U.data_ptr(), (__nv_bfloat16*)P.data_ptr(),
             (__nv_bfloat16*)Qd.data_ptr(), (__nv_bfloat16*)Kt.data_ptr(), gamma.data_ptr<float>()};
  if (gdn_use_tc()) {
    static bool once_tc = [] {
      CQB_CHECK_CUDA(cudaFuncSetAttribute((const void*)gdn_prep_tc_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM));
      return true;
    }();
    (void)once_tc;
    const auto mq = tma_map_bf16(Q.view({Nc * H * CH, DH}), CH);
    const auto mk = tma_map_bf16(K.view({Nc * H * CH, DH}), CH);
    const auto mv = tma_map_bf16(V.view({Nc * H * CH, DH}), CH);
    gdn_prep_tc_kernel<<<(unsigned)(Nc * H), TC_THREADS, TC_SMEM, stream()>>>(mq, mk, mv, a, gdn_status_word());
  } else {
    static bool once = [] {
      CQB_CHECK_CUDA(cudaFuncSetAttribute((const void*)gdn_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)PREP_SMEM));
      return true;
    }();
    (void)once;
    gdn_prep_kernel<<<(unsigned)(Nc * H), THREADS_C, PREP_SMEM, stream()>>>(a);
  }
  CQB_LAUNCH_CHECK();
  count_launch();
  return {W, U, P, Qd, Kt, gamma};
}

// Status word of the tcgen05 GDN kernels (0 = no wait expired); optionally cleared.
int64_t gdn_status(bool reset) {
  int v = 0;
  CQB_CHECK_CUDA(cudaMemcpy(&v, gdn_status_word(), sizeof(int), cudaMemcpyDeviceToHost));
  if (reset && v) CQB_CHECK_CUDA(cudaMemset(gdn_status_word(), 0, sizeof(int)));
  return v;
}

// Returns (dQ, dK, dV fp32 [Nc, H, 64, 128], dG, dBeta fp32 [Nc, H, 64]).
// S, dS: fp32 (mma.sync kernel) or bf16 row-major [Nc, H, 128, 128] with dgamma = <S, dS> fp32 [Nc, H]
// (tcgen05 kernel: S and dS arrive by TMA).
std::vector<at::Tensor> gdn_chunk_bwd(at::Tensor Q, at::Tensor K, at::Tensor V, at::Tensor dO, at::Tensor G,
                                      at::Tensor B, at::Tensor S, at::Tensor dS, c10::optional<at::Tensor> dgamma) {
  check_tile(Q, "Q");
  check_tile(K, "K");
  check_tile(V, "V");
  check_tile(dO, "dO");
  TORCH_CHECK(K.sizes() == Q.sizes() && V.sizes() == Q.sizes() && dO.sizes() == Q.sizes(), "Q, K, V, dO shapes differ");
  const long Nc = Q.size(0), H = Q.size(1);
  for (const auto* t : {&G, &B})
    TORCH_CHECK(t->is_cuda() && t->is_contiguous() && t->scalar_type() == at::kFloat && t->numel() == Nc * H * CH,
                "G, B: contiguous fp32 [Nc, H, 64]");
  const bool tc_path = S.scalar_type() == at::kBFloat16;
  for (const auto* t : {&S, &dS})
    TORCH_CHECK(t->is_cuda() && t->is_contiguous() && t->scalar_type() == S.scalar_type() &&
                    (tc_path || t->scalar_type() == at::kFloat) && t->numel() == Nc * H * DH * DH,
                "S, dS: contiguous [Nc, H, 128, 128], both fp32 or both bf16");
  TORCH_CHECK(!tc_path || (dgamma.has_value() && dgamma->scalar_type() == at::kFloat && dgamma->is_contiguous() &&
                           dgamma->numel() == Nc * H),
              "bf16 states need dgamma: fp32 [Nc, H]");
  auto f32 = Q.options().dtype(at::kFloat);
  auto dQ = at::empty({Nc, H, CH, DH}, f32), dK = at::empty({Nc, H, CH, DH}, f32), dV = at::empty({Nc, H, CH, DH}, f32);
  auto dG = at::empty({Nc, H, CH}, f32), dB = at::empty({Nc, H, CH}, f32);
  if (Nc * H == 0) return {dQ, dK, dV, dG, dB};
  BwdArgs a{(const __nv_bfloat16*)Q.data_ptr(), (const __nv_bfloat16*)K.data_ptr(), (const __nv_bfloat16*)V.data_ptr(),
            (const __nv_bfloat16*)dO.data_ptr(), G.data_ptr<float>(), B.data_ptr<float>(),
            tc_path ? nullptr : S.data_ptr<float>(), tc_path ? nullptr : dS.data_ptr<float>(), dQ.data_ptr<float>(),
            dK.data_ptr<float>(), dV.data_ptr<float>(), dG.data_ptr<float>(), dB.data_ptr<float>(),
            tc_path ? dgamma->data_ptr<float>() : nullptr};
  if (tc_path) {
    static bool once_tc = [] {
      CQB_CHECK_CUDA(cudaFuncSetAttribute((const void*)gdn_chunk_bwd_tc_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cb::SMEM));
      return true;
    }();
    (void)once_tc;
    const auto mq = tma_map_bf16(Q.view({Nc * H * CH, DH}), CH);
    const auto mk = tma_map_bf16(K.view({Nc * H * CH, DH}), CH);
    const auto mv = tma_map_bf16(V.view({Nc * H * CH, DH}), CH);
    const auto mo = tma_map_bf16(dO.view({Nc * H * CH, DH}), CH);
    const auto ms = tma_map_bf16(S.view({Nc * H * DH, DH}), DH);
    const auto mds = tma_map_bf16(dS.view({Nc * H * DH, DH}), DH);
    gdn_chunk_bwd_tc_kernel<<<(unsigned)(Nc * H), TC_THREADS, cb::SMEM, stream()>>>(mq, mk, mv, mo, ms, mds, a,
                                                                                   gdn_status_word());
  } else {
    static bool once = [] {
      CQB_CHECK_CUDA(cudaFuncSetAttribute((const void*)gdn_chunk_bwd_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)BWD_SMEM));
      return true;
    }();
    (void)once;
    gdn_chunk_bwd_kernel<<<(unsigned)(Nc * H), THREADS_C, BWD_SMEM, stream()>>>(a);
  }
  CQB_LAUNCH_CHECK();
  count_launch();
  return {dQ, dK, dV, dG, dB};
}

}  // namespace cqb
