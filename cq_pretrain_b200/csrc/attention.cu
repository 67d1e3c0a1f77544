// Flash attention over per-row key ranges (forward, dQ, dK/dV) for sm_100a.
//
// Row r of a head reads keys [kstart[r], kend[r]) (the CQ visibility of a packed sequence, or
// the sample of a varlen DiT row); empty ranges output zero. The mask is computed on the fly
// from the two int32 vectors, and a 64-row block only visits key blocks inside the union of its
// rows' ranges, so skipped work is exact. GQA: head h reads kv head h / (Hq / Hkv).
// Online softmax in fp32 (exp2 domain); the forward stores the log-sum-exp per (head, row).
// Backward (FlashAttention-2 split): a dQ kernel over row blocks and a dK/dV kernel over key
// blocks (both recompute P from the saved LSE; no atomics). bf16 m16n8k16 tensor-core MMAs.
#include "common.cuh"
#include "mma_sync.cuh"

namespace cqb {

namespace {

using namespace ws;

constexpr int BM = 64, BN = 64, THREADS = 128;
constexpr float LOG2E = 1.4426950408889634f;

struct AttnArgs {
  const __nv_bfloat16* q;   // [rows, Hq, D]
  const __nv_bfloat16* k;   // [keys, Hkv, D]
  const __nv_bfloat16* v;   // [keys, Hkv, D]
  const __nv_bfloat16* o;   // [rows, Hq, D]   (backward)
  const __nv_bfloat16* dout;  // [rows, Hq, D] (backward)
  const int* kstart;        // [rows]
  const int* kend;          // [rows]
  const float* lse;         // [Hq, rows]      (backward)
  const float* dsum;        // [Hq, rows]      (backward)
  const int* qb_min;        // [q blocks]     (backward) key range union of each row block
  const int* qb_max;
  __nv_bfloat16* out;       // O / dQ / dK
  __nv_bfloat16* out2;      // dV
  float* lse_out;           // [Hq, rows]
  int rows, keys, Hq, Hkv;
  float scale;              // softmax scale
};

template <int D>
__device__ __forceinline__ void load_rows(__nv_bfloat16* dst, const __nv_bfloat16* src, int r0, int nrows, int stride,
                                          int tid) {
  constexpr int LD = D + 8;
  constexpr int VPR = D / 8;  // 16-byte vectors per row
  for (int i = tid; i < BM * VPR; i += THREADS) {
    const int r = i / VPR, c = (i % VPR) * 8;
    const bool ok = r0 + r < nrows;
    cp_async16(dst + r * LD + c, src + (size_t)(ok ? r0 + r : 0) * stride + c, ok);
  }
}

// ---- forward ------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(THREADS) attn_fwd_kernel(AttnArgs a) {
  constexpr int LD = D + 8;
  extern __shared__ __align__(16) __nv_bfloat16 sm[];
  __nv_bfloat16* qs = sm;
  __nv_bfloat16* ks = qs + BM * LD;   // [2][BN][LD]
  __nv_bfloat16* vs = ks + 2 * BN * LD;
  __shared__ int s_range[2];
  const int qb = blockIdx.x, h = blockIdx.y, hk = h / (a.Hq / a.Hkv);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int r0 = qb * BM;
  // union of the block's key ranges
  {
    int lo = INT_MAX, hi = 0;
    for (int r = tid; r < BM; r += THREADS) {
      const int row = r0 + r;
      if (row < a.rows) {
        const int s = a.kstart[row], e = a.kend[row];
        if (e > s) {
          lo = min(lo, s);
          hi = max(hi, e);
        }
      }
    }
    for (int o = 16; o; o >>= 1) {
      lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
      hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    if (tid == 0) s_range[0] = INT_MAX, s_range[1] = 0;
    __syncthreads();
    if (lane == 0) {
      atomicMin(&s_range[0], lo);
      atomicMax(&s_range[1], hi);
    }
    __syncthreads();
  }
  const int klo = s_range[0], khi = s_range[1];
  const int row_a = r0 + warp * 16 + g, row_b = row_a + 8;
  const int ks_a = row_a < a.rows ? a.kstart[row_a] : 0, ke_a = row_a < a.rows ? a.kend[row_a] : 0;
  const int ks_b = row_b < a.rows ? a.kstart[row_b] : 0, ke_b = row_b < a.rows ? a.kend[row_b] : 0;
  float acc[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  const float sl2 = a.scale * LOG2E;
  const int qstride = a.Hq * D, kstride = a.Hkv * D;
  if (klo < khi) {
    load_rows<D>(qs, a.q + (size_t)h * D, r0, a.rows, qstride, tid);
    const int nb0 = (klo / BN) * BN;
    load_rows<D>(ks, a.k + (size_t)hk * D, nb0, a.keys, kstride, tid);
    load_rows<D>(vs, a.v + (size_t)hk * D, nb0, a.keys, kstride, tid);
    cp_commit();
    int buf = 0;
    for (int n0 = nb0; n0 < khi; n0 += BN, buf ^= 1) {
      if (n0 + BN < khi) {
        load_rows<D>(ks + (buf ^ 1) * BN * LD, a.k + (size_t)hk * D, n0 + BN, a.keys, kstride, tid);
        load_rows<D>(vs + (buf ^ 1) * BN * LD, a.v + (size_t)hk * D, n0 + BN, a.keys, kstride, tid);
        cp_commit();
        cp_wait_1();
      } else {
        cp_wait_all();
      }
      __syncthreads();
      const __nv_bfloat16* kt = ks + buf * BN * LD;
      const __nv_bfloat16* vt = vs + buf * BN * LD;
      float s[BN / 8][4];
#pragma unroll
      for (int j = 0; j < BN / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < D; kk += 16) {
        uint32_t af[4];
        frag_a(af, qs, warp * 16, kk, LD, lane);
#pragma unroll
        for (int j = 0; j < BN / 8; j += 2) {
          uint32_t bf[4];
          frag_bt2(bf, kt, kk, j * 8, LD, lane);
          mma16816(s[j], af, bf[0], bf[1]);
          mma16816(s[j + 1], af, bf[2], bf[3]);
        }
      }
      // mask + online softmax (log2 domain)
      float mx_a = m_a, mx_b = m_b;
#pragma unroll
      for (int j = 0; j < BN / 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = n0 + j * 8 + 2 * t + e;
          s[j][e] = (key >= ks_a && key < ke_a) ? s[j][e] * sl2 : -INFINITY;
          s[j][2 + e] = (key >= ks_b && key < ke_b) ? s[j][2 + e] * sl2 : -INFINITY;
          mx_a = fmaxf(mx_a, s[j][e]);
          mx_b = fmaxf(mx_b, s[j][2 + e]);
        }
      }
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
      const float ref_a = mx_a == -INFINITY ? 0.f : mx_a, ref_b = mx_b == -INFINITY ? 0.f : mx_b;
      const float corr_a = exp2f((m_a == -INFINITY ? ref_a : m_a) - ref_a);
      const float corr_b = exp2f((m_b == -INFINITY ? ref_b : m_b) - ref_b);
      m_a = mx_a;
      m_b = mx_b;
      l_a *= corr_a;
      l_b *= corr_b;
#pragma unroll
      for (int j = 0; j < D / 8; ++j) {
        acc[j][0] *= corr_a;
        acc[j][1] *= corr_a;
        acc[j][2] *= corr_b;
        acc[j][3] *= corr_b;
      }
#pragma unroll
      for (int j = 0; j < BN / 8; ++j) {
        s[j][0] = exp2f(s[j][0] - ref_a);
        s[j][1] = exp2f(s[j][1] - ref_a);
        s[j][2] = exp2f(s[j][2] - ref_b);
        s[j][3] = exp2f(s[j][3] - ref_b);
        l_a += s[j][0] + s[j][1];
        l_b += s[j][2] + s[j][3];
      }
      // O += P V
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk) {
        uint32_t af[4];
        acc_to_a(af, s[2 * kk], s[2 * kk + 1]);
#pragma unroll
        for (int j = 0; j < D / 8; j += 2) {
          uint32_t bf[4];
          frag_b2(bf, vt, kk * 16, j * 8, LD, lane);
          mma16816(acc[j], af, bf[0], bf[1]);
          mma16816(acc[j + 1], af, bf[2], bf[3]);
        }
      }
      __syncthreads();  // this buffer may be refilled by the next prefetch
    }
  }
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
  const float inv_a = l_a > 0.f ? 1.f / l_a : 0.f, inv_b = l_b > 0.f ? 1.f / l_b : 0.f;
  if (row_a < a.rows) {
    __nv_bfloat16* dst = a.out + ((size_t)row_a * a.Hq + h) * D;
#pragma unroll
    for (int j = 0; j < D / 8; ++j)
      *reinterpret_cast<__nv_bfloat162*>(dst + j * 8 + 2 * t) = __floats2bfloat162_rn(acc[j][0] * inv_a, acc[j][1] * inv_a);
    if (t == 0) a.lse_out[(size_t)h * a.rows + row_a] = l_a > 0.f ? (m_a + log2f(l_a)) / LOG2E : INFINITY;
  }
  if (row_b < a.rows) {
    __nv_bfloat16* dst = a.out + ((size_t)row_b * a.Hq + h) * D;
#pragma unroll
    for (int j = 0; j < D / 8; ++j)
      *reinterpret_cast<__nv_bfloat162*>(dst + j * 8 + 2 * t) = __floats2bfloat162_rn(acc[j][2] * inv_b, acc[j][3] * inv_b);
    if (t == 0) a.lse_out[(size_t)h * a.rows + row_b] = l_b > 0.f ? (m_b + log2f(l_b)) / LOG2E : INFINITY;
  }
}

// ---- backward prep: Dsum = rowsum(dO * O), row-block key ranges -----------------------------
template <int D>
__global__ void attn_bwd_prep_kernel(AttnArgs a, float* dsum, int* qb_min, int* qb_max) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int total = a.rows * a.Hq;
  if (warp < total) {
    const int row = warp / a.Hq, h = warp % a.Hq;
    const __nv_bfloat16* o = a.o + ((size_t)row * a.Hq + h) * D;
    const __nv_bfloat16* d = a.dout + ((size_t)row * a.Hq + h) * D;
    float s = 0.f;
    for (int c = lane * 8; c < D; c += 256) {
      float ov[8], dv[8];
      load8(o + c, ov);
      load8(d + c, dv);
#pragma unroll
      for (int j = 0; j < 8; ++j) s += ov[j] * dv[j];
    }
    s = warp_sum(s);
    if (lane == 0) dsum[(size_t)h * a.rows + row] = s;
  }
  // block ranges: one thread per row block
  const int qb = blockIdx.x * blockDim.x + threadIdx.x;
  if (qb < (a.rows + BM - 1) / BM) {
    int lo = INT_MAX, hi = 0;
    for (int r = qb * BM; r < min(a.rows, qb * BM + BM); ++r) {
      const int s = a.kstart[r], e = a.kend[r];
      if (e > s) {
        lo = min(lo, s);
        hi = max(hi, e);
      }
    }
    qb_min[qb] = lo;
    qb_max[qb] = hi;
  }
}

// ---- backward dQ --------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(THREADS) attn_bwd_dq_kernel(AttnArgs a) {
  constexpr int LD = D + 8;
  extern __shared__ __align__(16) __nv_bfloat16 sm[];
  __nv_bfloat16* qs = sm;
  __nv_bfloat16* dos = qs + BM * LD;
  __nv_bfloat16* ks = dos + BM * LD;   // [2][BN][LD]
  __nv_bfloat16* vs = ks + 2 * BN * LD;
  const int qb = blockIdx.x, h = blockIdx.y, hk = h / (a.Hq / a.Hkv);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int r0 = qb * BM;
  const int klo = a.qb_min[qb], khi = a.qb_max[qb];
  const int row_a = r0 + warp * 16 + g, row_b = row_a + 8;
  const bool va = row_a < a.rows, vb = row_b < a.rows;
  const int ks_a = va ? a.kstart[row_a] : 0, ke_a = va ? a.kend[row_a] : 0;
  const int ks_b = vb ? a.kstart[row_b] : 0, ke_b = vb ? a.kend[row_b] : 0;
  const float lse_a = va ? a.lse[(size_t)h * a.rows + row_a] * LOG2E : INFINITY;
  const float lse_b = vb ? a.lse[(size_t)h * a.rows + row_b] * LOG2E : INFINITY;
  const float ds_a = va ? a.dsum[(size_t)h * a.rows + row_a] : 0.f;
  const float ds_b = vb ? a.dsum[(size_t)h * a.rows + row_b] : 0.f;
  float acc[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  const float sl2 = a.scale * LOG2E;
  const int qstride = a.Hq * D, kstride = a.Hkv * D;
  if (klo < khi) {
    load_rows<D>(qs, a.q + (size_t)h * D, r0, a.rows, qstride, tid);
    load_rows<D>(dos, a.dout + (size_t)h * D, r0, a.rows, qstride, tid);
    const int nb0 = (klo / BN) * BN;
    load_rows<D>(ks, a.k + (size_t)hk * D, nb0, a.keys, kstride, tid);
    load_rows<D>(vs, a.v + (size_t)hk * D, nb0, a.keys, kstride, tid);
    cp_commit();
    int buf = 0;
    for (int n0 = nb0; n0 < khi; n0 += BN, buf ^= 1) {
      if (n0 + BN < khi) {
        load_rows<D>(ks + (buf ^ 1) * BN * LD, a.k + (size_t)hk * D, n0 + BN, a.keys, kstride, tid);
        load_rows<D>(vs + (buf ^ 1) * BN * LD, a.v + (size_t)hk * D, n0 + BN, a.keys, kstride, tid);
        cp_commit();
        cp_wait_1();
      } else {
        cp_wait_all();
      }
      __syncthreads();
      const __nv_bfloat16* kt = ks + buf * BN * LD;
      const __nv_bfloat16* vt = vs + buf * BN * LD;
      float s[BN / 8][4], dp[BN / 8][4];
#pragma unroll
      for (int j = 0; j < BN / 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[j][e] = dp[j][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < D; kk += 16) {
        uint32_t aq[4], ad[4];
        frag_a(aq, qs, warp * 16, kk, LD, lane);
        frag_a(ad, dos, warp * 16, kk, LD, lane);
#pragma unroll
        for (int j = 0; j < BN / 8; j += 2) {
          uint32_t bk[4], bv[4];
          frag_bt2(bk, kt, kk, j * 8, LD, lane);
          frag_bt2(bv, vt, kk, j * 8, LD, lane);
          mma16816(s[j], aq, bk[0], bk[1]);
          mma16816(s[j + 1], aq, bk[2], bk[3]);
          mma16816(dp[j], ad, bv[0], bv[1]);
          mma16816(dp[j + 1], ad, bv[2], bv[3]);
        }
      }
#pragma unroll
      for (int j = 0; j < BN / 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = n0 + j * 8 + 2 * t + e;
          const float pa = (key >= ks_a && key < ke_a) ? exp2f(s[j][e] * sl2 - lse_a) : 0.f;
          const float pb = (key >= ks_b && key < ke_b) ? exp2f(s[j][2 + e] * sl2 - lse_b) : 0.f;
          s[j][e] = pa * (dp[j][e] - ds_a);
          s[j][2 + e] = pb * (dp[j][2 + e] - ds_b);
        }
      }
      // dQ += dS K
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk) {
        uint32_t af[4];
        acc_to_a(af, s[2 * kk], s[2 * kk + 1]);
#pragma unroll
        for (int j = 0; j < D / 8; j += 2) {
          uint32_t bf[4];
          frag_b2(bf, kt, kk * 16, j * 8, LD, lane);
          mma16816(acc[j], af, bf[0], bf[1]);
          mma16816(acc[j + 1], af, bf[2], bf[3]);
        }
      }
      __syncthreads();
    }
  }
  if (va) {
    __nv_bfloat16* dst = a.out + ((size_t)row_a * a.Hq + h) * D;
#pragma unroll
    for (int j = 0; j < D / 8; ++j)
      *reinterpret_cast<__nv_bfloat162*>(dst + j * 8 + 2 * t) =
          __floats2bfloat162_rn(acc[j][0] * a.scale, acc[j][1] * a.scale);
  }
  if (vb) {
    __nv_bfloat16* dst = a.out + ((size_t)row_b * a.Hq + h) * D;
#pragma unroll
    for (int j = 0; j < D / 8; ++j)
      *reinterpret_cast<__nv_bfloat162*>(dst + j * 8 + 2 * t) =
          __floats2bfloat162_rn(acc[j][2] * a.scale, acc[j][3] * a.scale);
  }
}

// ---- backward dK / dV (key blocks; value-dim slice DS per CTA) ------------------------------
template <int D, int DS>
__global__ void __launch_bounds__(THREADS) attn_bwd_dkv_kernel(AttnArgs a) {
  constexpr int LD = D + 8;
  extern __shared__ __align__(16) __nv_bfloat16 sm[];
  __nv_bfloat16* ks = sm;
  __nv_bfloat16* vs = ks + BN * LD;
  __nv_bfloat16* qs = vs + BN * LD;
  __nv_bfloat16* dos = qs + BM * LD;
  __shared__ float s_lse[BM], s_ds[BM];
  __shared__ int s_ks[BM], s_ke[BM];
  const int kb = blockIdx.x, hk = blockIdx.y, d0 = blockIdx.z * DS;
  const int group = a.Hq / a.Hkv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int n0 = kb * BN;
  const int key_a = n0 + warp * 16 + g, key_b = key_a + 8;
  const int qstride = a.Hq * D, kstride = a.Hkv * D;
  const float sl2 = a.scale * LOG2E;
  load_rows<D>(ks, a.k + (size_t)hk * D, n0, a.keys, kstride, tid);
  load_rows<D>(vs, a.v + (size_t)hk * D, n0, a.keys, kstride, tid);
  cp_commit();
  float dk[DS / 8][4], dv[DS / 8][4];
#pragma unroll
  for (int j = 0; j < DS / 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[j][e] = dv[j][e] = 0.f;
  const int nqb = (a.rows + BM - 1) / BM;
  for (int hh = 0; hh < group; ++hh) {
    const int h = hk * group + hh;
    for (int qb = 0; qb < nqb; ++qb) {
      const int lo = a.qb_min[qb], hi = a.qb_max[qb];
      if (!(lo < hi && lo < n0 + BN && hi > n0)) continue;  // uniform across the CTA
      const int r0 = qb * BM;
      __syncthreads();  // previous tiles consumed
      load_rows<D>(qs, a.q + (size_t)h * D, r0, a.rows, qstride, tid);
      load_rows<D>(dos, a.dout + (size_t)h * D, r0, a.rows, qstride, tid);
      cp_commit();
      for (int r = tid; r < BM; r += THREADS) {
        const int row = r0 + r;
        const bool ok = row < a.rows;
        s_lse[r] = ok ? a.lse[(size_t)h * a.rows + row] * LOG2E : INFINITY;
        s_ds[r] = ok ? a.dsum[(size_t)h * a.rows + row] : 0.f;
        s_ks[r] = ok ? a.kstart[row] : 0;
        s_ke[r] = ok ? a.kend[row] : 0;
      }
      cp_wait_all();
      __syncthreads();
      // S^T = K Q^T, dP^T = V dO^T  (16 keys x 64 rows per warp)
      float s[BM / 8][4], dp[BM / 8][4];
#pragma unroll
      for (int j = 0; j < BM / 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[j][e] = dp[j][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < D; kk += 16) {
        uint32_t ak[4], av[4];
        frag_a(ak, ks, warp * 16, kk, LD, lane);
        frag_a(av, vs, warp * 16, kk, LD, lane);
#pragma unroll
        for (int j = 0; j < BM / 8; j += 2) {
          uint32_t bq[4], bd[4];
          frag_bt2(bq, qs, kk, j * 8, LD, lane);
          frag_bt2(bd, dos, kk, j * 8, LD, lane);
          mma16816(s[j], ak, bq[0], bq[1]);
          mma16816(s[j + 1], ak, bq[2], bq[3]);
          mma16816(dp[j], av, bd[0], bd[1]);
          mma16816(dp[j + 1], av, bd[2], bd[3]);
        }
      }
      // P^T and dS^T (columns are rows of the q block)
#pragma unroll
      for (int j = 0; j < BM / 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int r = j * 8 + 2 * t + e;
          const int rs = s_ks[r], re = s_ke[r];
          const float lse = s_lse[r], dsr = s_ds[r];
          const float pa = (key_a >= rs && key_a < re) ? exp2f(s[j][e] * sl2 - lse) : 0.f;
          const float pb = (key_b >= rs && key_b < re) ? exp2f(s[j][2 + e] * sl2 - lse) : 0.f;
          s[j][e] = pa;
          s[j][2 + e] = pb;
          dp[j][e] = pa * (dp[j][e] - dsr);
          dp[j][2 + e] = pb * (dp[j][2 + e] - dsr);
        }
      }
      // dV += P^T dO[:, slice];  dK += dS^T Q[:, slice]
#pragma unroll
      for (int kk = 0; kk < BM / 16; ++kk) {
        uint32_t ap[4], ad[4];
        acc_to_a(ap, s[2 * kk], s[2 * kk + 1]);
        acc_to_a(ad, dp[2 * kk], dp[2 * kk + 1]);
#pragma unroll
        for (int j = 0; j < DS / 8; j += 2) {
          uint32_t bo[4], bq[4];
          frag_b2(bo, dos, kk * 16, d0 + j * 8, LD, lane);
          frag_b2(bq, qs, kk * 16, d0 + j * 8, LD, lane);
          mma16816(dv[j], ap, bo[0], bo[1]);
          mma16816(dv[j + 1], ap, bo[2], bo[3]);
          mma16816(dk[j], ad, bq[0], bq[1]);
          mma16816(dk[j + 1], ad, bq[2], bq[3]);
        }
      }
    }
  }
  cp_wait_all();
  if (key_a < a.keys) {
    __nv_bfloat16* dkd = a.out + ((size_t)key_a * a.Hkv + hk) * D + d0;
    __nv_bfloat16* dvd = a.out2 + ((size_t)key_a * a.Hkv + hk) * D + d0;
#pragma unroll
    for (int j = 0; j < DS / 8; ++j) {
      *reinterpret_cast<__nv_bfloat162*>(dkd + j * 8 + 2 * t) = __floats2bfloat162_rn(dk[j][0] * a.scale, dk[j][1] * a.scale);
      *reinterpret_cast<__nv_bfloat162*>(dvd + j * 8 + 2 * t) = __floats2bfloat162_rn(dv[j][0], dv[j][1]);
    }
  }
  if (key_b < a.keys) {
    __nv_bfloat16* dkd = a.out + ((size_t)key_b * a.Hkv + hk) * D + d0;
    __nv_bfloat16* dvd = a.out2 + ((size_t)key_b * a.Hkv + hk) * D + d0;
#pragma unroll
    for (int j = 0; j < DS / 8; ++j) {
      *reinterpret_cast<__nv_bfloat162*>(dkd + j * 8 + 2 * t) = __floats2bfloat162_rn(dk[j][2] * a.scale, dk[j][3] * a.scale);
      *reinterpret_cast<__nv_bfloat162*>(dvd + j * 8 + 2 * t) = __floats2bfloat162_rn(dv[j][2], dv[j][3]);
    }
  }
}

template <typename F>
void set_smem_once(F fn, size_t bytes) {
  CQB_CHECK_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
}

AttnArgs base_args(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& kstart,
                   const at::Tensor& kend, double scale) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && q.is_contiguous() && q.dim() == 3, "q: [rows,Hq,D] bf16");
  TORCH_CHECK(k.is_contiguous() && v.is_contiguous() && k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16,
              "k/v: contiguous bf16");
  TORCH_CHECK(kstart.scalar_type() == at::kInt && kend.scalar_type() == at::kInt && kstart.numel() == q.size(0) &&
                  kend.numel() == q.size(0),
              "kstart/kend: int32 [rows]");
  TORCH_CHECK(q.size(1) % k.size(1) == 0, "GQA ratio must be integral");
  AttnArgs a{};
  a.q = (const __nv_bfloat16*)q.data_ptr();
  a.k = (const __nv_bfloat16*)k.data_ptr();
  a.v = (const __nv_bfloat16*)v.data_ptr();
  a.kstart = kstart.data_ptr<int>();
  a.kend = kend.data_ptr<int>();
  a.rows = q.size(0);
  a.keys = k.size(0);
  a.Hq = q.size(1);
  a.Hkv = k.size(1);
  a.scale = (float)scale;
  return a;
}

template <int D>
size_t fwd_smem() { return (size_t)(BM + 4 * BN) * (D + 8) * 2; }
template <int D>
size_t dq_smem() { return (size_t)(2 * BM + 4 * BN) * (D + 8) * 2; }
template <int D>
size_t dkv_smem() { return (size_t)(2 * BN + 2 * BM) * (D + 8) * 2; }

#define ATTN_D_DISPATCH(D_, ...)                          \
  [&] {                                                   \
    if (D_ == 64) { constexpr int D = 64; __VA_ARGS__(); }  \
    else if (D_ == 128) { constexpr int D = 128; __VA_ARGS__(); } \
    else if (D_ == 256) { constexpr int D = 256; __VA_ARGS__(); } \
    else TORCH_CHECK(false, "attention head dim must be 64, 128 or 256"); \
  }()

}  // namespace

std::vector<at::Tensor> attn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor kstart, at::Tensor kend,
                                 double scale) {
  AttnArgs a = base_args(q, k, v, kstart, kend, scale);
  auto o = at::empty_like(q);
  auto lse = at::empty({q.size(1), q.size(0)}, q.options().dtype(at::kFloat));
  a.out = (__nv_bfloat16*)o.data_ptr();
  a.lse_out = lse.data_ptr<float>();
  if (a.rows == 0) return {o, lse};
  const int D_ = q.size(2);
  ATTN_D_DISPATCH(D_, [&] {
    static bool once = (set_smem_once(attn_fwd_kernel<D>, fwd_smem<D>()), true);
    (void)once;
    dim3 grid((a.rows + BM - 1) / BM, a.Hq);
    attn_fwd_kernel<D><<<grid, THREADS, fwd_smem<D>(), stream()>>>(a);
  });
  CQB_LAUNCH_CHECK();
  count_launch();
  return {o, lse};
}

std::vector<at::Tensor> attn_bwd(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o,
                                 at::Tensor lse, at::Tensor kstart, at::Tensor kend, double scale) {
  AttnArgs a = base_args(q, k, v, kstart, kend, scale);
  auto dq = at::empty_like(q);
  auto dk = at::empty_like(k);
  auto dv = at::empty_like(v);
  if (a.rows == 0) return {dq.zero_(), dk.zero_(), dv.zero_()};
  a.o = (const __nv_bfloat16*)o.data_ptr();
  a.dout = (const __nv_bfloat16*)dout.data_ptr();
  a.lse = lse.data_ptr<float>();
  const int nqb = (a.rows + BM - 1) / BM;
  auto dsum = at::empty({q.size(1), q.size(0)}, q.options().dtype(at::kFloat));
  auto qb_min = at::empty({nqb}, q.options().dtype(at::kInt));
  auto qb_max = at::empty({nqb}, q.options().dtype(at::kInt));
  a.dsum = dsum.data_ptr<float>();
  a.qb_min = qb_min.data_ptr<int>();
  a.qb_max = qb_max.data_ptr<int>();
  const int D_ = q.size(2);
  ATTN_D_DISPATCH(D_, [&] {
    const int warps = a.rows * a.Hq;
    const int blocks = std::max((warps * 32 + 255) / 256, (nqb + 255) / 256);
    attn_bwd_prep_kernel<D><<<blocks, 256, 0, stream()>>>(a, dsum.data_ptr<float>(), qb_min.data_ptr<int>(),
                                                          qb_max.data_ptr<int>());
    static bool once_q = (set_smem_once(attn_bwd_dq_kernel<D>, dq_smem<D>()), true);
    (void)once_q;
    a.out = (__nv_bfloat16*)dq.data_ptr();
    attn_bwd_dq_kernel<D><<<dim3(nqb, a.Hq), THREADS, dq_smem<D>(), stream()>>>(a);
    constexpr int DS = D > 128 ? 128 : D;
    static bool once_kv = (set_smem_once(attn_bwd_dkv_kernel<D, DS>, dkv_smem<D>()), true);
    (void)once_kv;
    a.out = (__nv_bfloat16*)dk.data_ptr();
    a.out2 = (__nv_bfloat16*)dv.data_ptr();
    attn_bwd_dkv_kernel<D, DS><<<dim3((a.keys + BN - 1) / BN, a.Hkv, D / DS), THREADS, dkv_smem<D>(), stream()>>>(a);
  });
  CQB_LAUNCH_CHECK();
  count_launch(3);
  return {dq, dk, dv};
}

}  // namespace cqb
