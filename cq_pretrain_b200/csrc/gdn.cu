// Gated-DeltaNet chunk recurrences (sequential over the chunks of one document).
//
// Per chunk c of a document (chunk length C = 64, key dim Dk = 128, value tile of BV columns),
// with chunk-local factors computed by the caller:
//   forward  D = U - W S;  O = Qd S + P D;  S <- gamma S + Kt^T D          (S entering chunk saved)
//   backward dD = P^T dO + Kt dS;  dS <- gamma dS + Qd^T dO - W^T dD        (dS entering saved)
// Columns of S (value dims) evolve independently, so each CTA owns one (document, head,
// value tile) and walks the document's chunks. 8 warps; bf16 tensor-core MMAs (m16n8k16) with
// fp32 accumulators; the fp32 state lives in registers, a bf16 copy in shared memory feeds
// the next products; chunk inputs are double-buffered with cp.async.
#include "common.cuh"
#include "tcgen05.cuh"

namespace cqb {

int* gdn_status_word();   // gdn_chunk.cu

namespace {

constexpr int C = 64, DK = 128, BV = 64, WARPS = 8, THREADS = WARPS * 32;
constexpr int LDK = DK + 8;   // padded row (elements) of 128-wide tiles
constexpr int LDV = BV + 8;   // padded row of 64-wide tiles
constexpr int TILE_K = C * LDK;          // W, Qd, Kt tiles
constexpr int TILE_V = C * LDV;          // U / dO tiles, P tile
constexpr int BUF = 3 * TILE_K + 2 * TILE_V;  // one chunk's inputs (elements)

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t* r, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t* r, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"((uint32_t)__cvta_generic_to_shared(p)));
}

__device__ __forceinline__ void mma16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A fragment (16x16) of a row-major [row][col] tile.
__device__ __forceinline__ void frag_a(uint32_t* r, const __nv_bfloat16* base, int row0, int col0, int ld, int lane) {
  ldsm_x4(r, base + (row0 + (lane & 15)) * ld + col0 + (lane >> 4) * 8);
}
// A fragment of A = X^T where X is row-major [k][m]: A[m][k] = X[k][m].
__device__ __forceinline__ void frag_at(uint32_t* r, const __nv_bfloat16* base, int m0, int k0, int ld, int lane) {
  // matrices: (m0..7,k0..7), (m8..15,k0..7), (m0..7,k8..15), (m8..15,k8..15) read transposed from X rows k
  const int k = k0 + (lane & 7) + ((lane >> 4) << 3);
  const int m = m0 + ((lane >> 3) & 1) * 8;
  ldsm_x4_t(r, base + k * ld + m);
}
// Two B fragments (k16 x n8 each, n-tiles n0 and n0+8) of B stored row-major [k][n].
__device__ __forceinline__ void frag_b2(uint32_t* r, const __nv_bfloat16* base, int k0, int n0, int ld, int lane) {
  // matrices: (k0..7, n0..7), (k8..15, n0..7), (k0..7, n8..15), (k8..15, n8..15)
  const int k = k0 + (lane & 7) + ((lane >> 3) & 1) * 8;
  const int n = n0 + (lane >> 4) * 8;
  ldsm_x4_t(r, base + k * ld + n);
}

// Store an m16n8 fp32 accumulator tile as bf16 into a row-major smem tile.
__device__ __forceinline__ void store_acc_bf16(__nv_bfloat16* base, int row0, int col0, int ld, const float* c,
                                               int lane) {
  const int g = lane >> 2, t = lane & 3;
  *reinterpret_cast<__nv_bfloat162*>(base + (row0 + g) * ld + col0 + 2 * t) = __floats2bfloat162_rn(c[0], c[1]);
  *reinterpret_cast<__nv_bfloat162*>(base + (row0 + g + 8) * ld + col0 + 2 * t) = __floats2bfloat162_rn(c[2], c[3]);
}

struct GdnArgs {
  const __nv_bfloat16* W;   // [Nc, H, C, DK]
  const __nv_bfloat16* Qd;  // [Nc, H, C, DK]
  const __nv_bfloat16* Kt;  // [Nc, H, C, DK]
  const __nv_bfloat16* P;   // [Nc, H, C, C]
  const __nv_bfloat16* UV;  // forward: U [Nc, H, C, DV]; backward: dO [Nc, H, C, DV]
  const float* gamma;       // [Nc, H]
  const int* chunk_start;   // [docs]
  const int* chunk_count;   // [docs]
  __nv_bfloat16* out;       // forward: O [Nc, H, C, DV] bf16
  float* states;            // [Nc, H, DK, DV] fp32: S entering (fwd) / dS entering from the right (bwd)
  float* final;             // forward, optional: [docs, H, DK, DV] fp32 state after each document
  int H, DV;
};

__device__ __forceinline__ void load_chunk(__nv_bfloat16* buf, const GdnArgs& a, int c, int h, int v0, bool backward,
                                           int tid) {
  const size_t kbase = ((size_t)c * a.H + h) * C * DK;
  const size_t vbase = ((size_t)c * a.H + h) * C * a.DV;
  const size_t pbase = ((size_t)c * a.H + h) * C * C;
  __nv_bfloat16* w = buf;
  __nv_bfloat16* q = buf + TILE_K;
  __nv_bfloat16* k = buf + 2 * TILE_K;
  __nv_bfloat16* u = buf + 3 * TILE_K;
  __nv_bfloat16* p = u + TILE_V;
  // 64 rows x 128 cols = 1024 16-byte vectors per K-wide tile
  for (int i = tid; i < C * DK / 8; i += THREADS) {
    const int r = i / (DK / 8), col = (i % (DK / 8)) * 8;
    cp_async16(w + r * LDK + col, a.W + kbase + r * DK + col);
    cp_async16(q + r * LDK + col, a.Qd + kbase + r * DK + col);
    cp_async16(k + r * LDK + col, a.Kt + kbase + r * DK + col);
  }
  for (int i = tid; i < C * BV / 8; i += THREADS) {
    const int r = i / (BV / 8), col = (i % (BV / 8)) * 8;
    cp_async16(u + r * LDV + col, a.UV + vbase + r * a.DV + v0 + col);
    cp_async16(p + r * LDV + col, a.P + pbase + r * C + col);
  }
  cp_commit();
  (void)backward;
}

// ---- forward ------------------------------------------------------------------------------
__global__ void __launch_bounds__(THREADS, 1) gdn_fwd_kernel(GdnArgs a) {
  extern __shared__ __align__(16) __nv_bfloat16 sm[];
  __nv_bfloat16* bufs[2] = {sm, sm + BUF};
  __nv_bfloat16* s_bf = sm + 2 * BUF;       // [DK][LDV]  state (bf16)
  __nv_bfloat16* d_bf = s_bf + DK * LDV;    // [C][LDV]   D (bf16)
  const int doc = blockIdx.z, h = blockIdx.y, v0 = blockIdx.x * BV;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int c0 = a.chunk_start[doc], nc = a.chunk_count[doc];
  if (nc == 0) {
    if (a.final)   // an empty document leaves the zero state
      for (int i = tid; i < DK * BV; i += THREADS)
        a.final[(((size_t)doc * a.H + h) * DK + i / BV) * a.DV + v0 + i % BV] = 0.f;
    return;
  }
  // state rows [16*warp, 16*warp+16) x BV columns, 8 n-tiles
  float st[BV / 8][4];
#pragma unroll
  for (int j = 0; j < BV / 8; ++j) st[j][0] = st[j][1] = st[j][2] = st[j][3] = 0.f;
  for (int i = tid; i < DK * LDV; i += THREADS) s_bf[i] = __float2bfloat16(0.f);
  load_chunk(bufs[0], a, c0, h, v0, false, tid);
  const int mt = warp & 3, nh = warp >> 2;  // steps 1-3: row tile mt (16 rows), column half nh (32 cols)
  for (int ci = 0; ci < nc; ++ci) {
    const int c = c0 + ci;
    __nv_bfloat16* buf = bufs[ci & 1];
    cp_wait_all();
    __syncthreads();  // chunk inputs + s_bf ready; previous reads of the other buffer done
    if (ci + 1 < nc) load_chunk(bufs[(ci + 1) & 1], a, c + 1, h, v0, false, tid);
    const __nv_bfloat16* W = buf;
    const __nv_bfloat16* Q = buf + TILE_K;
    const __nv_bfloat16* K = buf + 2 * TILE_K;
    const __nv_bfloat16* U = buf + 3 * TILE_K;
    const __nv_bfloat16* P = U + TILE_V;
    // save entering state (fp32) for the backward pass
    {
      float* dst = a.states + ((size_t)c * a.H + h) * DK * a.DV;
#pragma unroll
      for (int j = 0; j < BV / 8; ++j) {
        const int col = v0 + j * 8 + 2 * t;
        *reinterpret_cast<float2*>(dst + (size_t)(warp * 16 + g) * a.DV + col) = make_float2(st[j][0], st[j][1]);
        *reinterpret_cast<float2*>(dst + (size_t)(warp * 16 + g + 8) * a.DV + col) = make_float2(st[j][2], st[j][3]);
      }
    }
    // step 1-2: D = U - W S  (rows 16*mt, cols 32*nh)
    float x[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j][0] = x[j][1] = x[j][2] = x[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < DK; kk += 16) {
      uint32_t af[4];
      frag_a(af, W, mt * 16, kk, LDK, lane);
#pragma unroll
      for (int j = 0; j < 4; j += 2) {
        uint32_t bf[4];
        frag_b2(bf, s_bf, kk, nh * 32 + j * 8, LDV, lane);
        mma16816(x[j], af, bf[0], bf[1]);
        mma16816(x[j + 1], af, bf[2], bf[3]);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = nh * 32 + j * 8 + 2 * t;
      const float2 u0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(U + (mt * 16 + g) * LDV + col));
      const float2 u1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(U + (mt * 16 + g + 8) * LDV + col));
      x[j][0] = u0.x - x[j][0];
      x[j][1] = u0.y - x[j][1];
      x[j][2] = u1.x - x[j][2];
      x[j][3] = u1.y - x[j][3];
      store_acc_bf16(d_bf, mt * 16, nh * 32 + j * 8, LDV, x[j], lane);
    }
    __syncthreads();  // D visible
    // step 3: O = Qd S + P D
    float o[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < DK; kk += 16) {
      uint32_t af[4];
      frag_a(af, Q, mt * 16, kk, LDK, lane);
#pragma unroll
      for (int j = 0; j < 4; j += 2) {
        uint32_t bf[4];
        frag_b2(bf, s_bf, kk, nh * 32 + j * 8, LDV, lane);
        mma16816(o[j], af, bf[0], bf[1]);
        mma16816(o[j + 1], af, bf[2], bf[3]);
      }
    }
#pragma unroll
    for (int kk = 0; kk < C; kk += 16) {
      uint32_t af[4];
      frag_a(af, P, mt * 16, kk, LDV, lane);
#pragma unroll
      for (int j = 0; j < 4; j += 2) {
        uint32_t bf[4];
        frag_b2(bf, d_bf, kk, nh * 32 + j * 8, LDV, lane);
        mma16816(o[j], af, bf[0], bf[1]);
        mma16816(o[j + 1], af, bf[2], bf[3]);
      }
    }
    {
      __nv_bfloat16* dst = a.out + ((size_t)c * a.H + h) * C * a.DV;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col = v0 + nh * 32 + j * 8 + 2 * t;
        *reinterpret_cast<__nv_bfloat162*>(dst + (size_t)(mt * 16 + g) * a.DV + col) = __floats2bfloat162_rn(o[j][0], o[j][1]);
        *reinterpret_cast<__nv_bfloat162*>(dst + (size_t)(mt * 16 + g + 8) * a.DV + col) =
            __floats2bfloat162_rn(o[j][2], o[j][3]);
      }
    }
    // step 4: S = gamma S + Kt^T D   (state rows 16*warp)
    const float gm = a.gamma[(size_t)c * a.H + h];
#pragma unroll
    for (int j = 0; j < BV / 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) st[j][e] *= gm;
#pragma unroll
    for (int kk = 0; kk < C; kk += 16) {
      uint32_t af[4];
      frag_at(af, K, warp * 16, kk, LDK, lane);
#pragma unroll
      for (int j = 0; j < BV / 8; j += 2) {
        uint32_t bf[4];
        frag_b2(bf, d_bf, kk, j * 8, LDV, lane);
        mma16816(st[j], af, bf[0], bf[1]);
        mma16816(st[j + 1], af, bf[2], bf[3]);
      }
    }
    __syncthreads();  // every read of s_bf (steps 1, 3) is done
#pragma unroll
    for (int j = 0; j < BV / 8; ++j) store_acc_bf16(s_bf, warp * 16, j * 8, LDV, st[j], lane);
  }
  if (a.final) {   // prefill: the fp32 state leaving the document's last chunk
    float* dst = a.final + ((size_t)doc * a.H + h) * DK * a.DV;
#pragma unroll
    for (int j = 0; j < BV / 8; ++j) {
      const int col = v0 + j * 8 + 2 * t;
      *reinterpret_cast<float2*>(dst + (size_t)(warp * 16 + g) * a.DV + col) = make_float2(st[j][0], st[j][1]);
      *reinterpret_cast<float2*>(dst + (size_t)(warp * 16 + g + 8) * a.DV + col) = make_float2(st[j][2], st[j][3]);
    }
  }
}

// ---- backward -----------------------------------------------------------------------------
__global__ void __launch_bounds__(THREADS, 1) gdn_bwd_kernel(GdnArgs a) {
  extern __shared__ __align__(16) __nv_bfloat16 sm[];
  __nv_bfloat16* bufs[2] = {sm, sm + BUF};
  __nv_bfloat16* s_bf = sm + 2 * BUF;       // dS (bf16) [DK][LDV]
  __nv_bfloat16* d_bf = s_bf + DK * LDV;    // dD (bf16) [C][LDV]
  const int doc = blockIdx.z, h = blockIdx.y, v0 = blockIdx.x * BV;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int c0 = a.chunk_start[doc], nc = a.chunk_count[doc];
  if (nc == 0) return;
  float st[BV / 8][4];
#pragma unroll
  for (int j = 0; j < BV / 8; ++j) st[j][0] = st[j][1] = st[j][2] = st[j][3] = 0.f;
  for (int i = tid; i < DK * LDV; i += THREADS) s_bf[i] = __float2bfloat16(0.f);
  load_chunk(bufs[0], a, c0 + nc - 1, h, v0, true, tid);
  const int mt = warp & 3, nh = warp >> 2;
  for (int ci = nc - 1; ci >= 0; --ci) {
    const int c = c0 + ci;
    const int slot = (nc - 1 - ci) & 1;
    __nv_bfloat16* buf = bufs[slot];
    cp_wait_all();
    __syncthreads();
    if (ci > 0) load_chunk(bufs[slot ^ 1], a, c - 1, h, v0, true, tid);
    const __nv_bfloat16* W = buf;
    const __nv_bfloat16* Q = buf + TILE_K;
    const __nv_bfloat16* K = buf + 2 * TILE_K;
    const __nv_bfloat16* dO = buf + 3 * TILE_K;
    const __nv_bfloat16* P = dO + TILE_V;
    {
      float* dst = a.states + ((size_t)c * a.H + h) * DK * a.DV;
#pragma unroll
      for (int j = 0; j < BV / 8; ++j) {
        const int col = v0 + j * 8 + 2 * t;
        *reinterpret_cast<float2*>(dst + (size_t)(warp * 16 + g) * a.DV + col) = make_float2(st[j][0], st[j][1]);
        *reinterpret_cast<float2*>(dst + (size_t)(warp * 16 + g + 8) * a.DV + col) = make_float2(st[j][2], st[j][3]);
      }
    }
    // dD = P^T dO + Kt dS   (rows 16*mt, cols 32*nh)
    float x[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j][0] = x[j][1] = x[j][2] = x[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < C; kk += 16) {
      uint32_t af[4];
      frag_at(af, P, mt * 16, kk, LDV, lane);
#pragma unroll
      for (int j = 0; j < 4; j += 2) {
        uint32_t bf[4];
        frag_b2(bf, dO, kk, nh * 32 + j * 8, LDV, lane);
        mma16816(x[j], af, bf[0], bf[1]);
        mma16816(x[j + 1], af, bf[2], bf[3]);
      }
    }
#pragma unroll
    for (int kk = 0; kk < DK; kk += 16) {
      uint32_t af[4];
      frag_a(af, K, mt * 16, kk, LDK, lane);
#pragma unroll
      for (int j = 0; j < 4; j += 2) {
        uint32_t bf[4];
        frag_b2(bf, s_bf, kk, nh * 32 + j * 8, LDV, lane);
        mma16816(x[j], af, bf[0], bf[1]);
        mma16816(x[j + 1], af, bf[2], bf[3]);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) store_acc_bf16(d_bf, mt * 16, nh * 32 + j * 8, LDV, x[j], lane);
    __syncthreads();
    // dS = gamma dS + Qd^T dO - W^T dD   (dS rows 16*warp)
    const float gm = a.gamma[(size_t)c * a.H + h];
    float neg[BV / 8][4];
#pragma unroll
    for (int j = 0; j < BV / 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        st[j][e] *= gm;
        neg[j][e] = 0.f;
      }
#pragma unroll
    for (int kk = 0; kk < C; kk += 16) {
      uint32_t aq[4], aw[4];
      frag_at(aq, Q, warp * 16, kk, LDK, lane);
      frag_at(aw, W, warp * 16, kk, LDK, lane);
#pragma unroll
      for (int j = 0; j < BV / 8; j += 2) {
        uint32_t bo[4], bd[4];
        frag_b2(bo, dO, kk, j * 8, LDV, lane);
        frag_b2(bd, d_bf, kk, j * 8, LDV, lane);
        mma16816(st[j], aq, bo[0], bo[1]);
        mma16816(st[j + 1], aq, bo[2], bo[3]);
        mma16816(neg[j], aw, bd[0], bd[1]);
        mma16816(neg[j + 1], aw, bd[2], bd[3]);
      }
    }
#pragma unroll
    for (int j = 0; j < BV / 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) st[j][e] -= neg[j][e];
    __syncthreads();
#pragma unroll
    for (int j = 0; j < BV / 8; ++j) store_acc_bf16(s_bf, warp * 16, j * 8, LDV, st[j], lane);
  }
}

// ---- forward on tcgen05 ---------------------------------------------------------------------
//
// Same contract as gdn_fwd_kernel for a value dim of 128: one CTA per (document, head), 256 threads,
// one CTA per SM. The fp32 state S [dk x dv] stays in TMEM (lanes = dk, columns 0-127) for the whole
// document; per chunk, with S's bf16 copy in shared memory as the MN-major A operand S^T:
//   group 1: D^T = S^T W^T, O^T = S^T Qd^T                  (M = 128 value dims, N = 64 events)
//   epilogue: D^T <- U^T - D^T (bf16 K-major tile); S entering is written out (fp32) and scaled by
//             gamma in TMEM
//   group 2: O^T += D^T P^T; S += Kt^T D                     (Kt as the MN-major A operand)
//   epilogue: O leaves through a staging tile; the new S becomes the next chunk's bf16 operand.
// Thread 0 streams each chunk's W, Qd, Kt, U (two 64-column TMA boxes each) and P into a two-deep
// ring one chunk ahead and issues the MMAs; warp w reads TMEM lanes 32 (w % 4)..+31, warps w and
// w + 4 split the columns. Bounded waits (status codes 51-53); on expiry the CTA stops issuing,
// waits (bounded) for what it has in flight, frees its TMEM and returns.
constexpr int TF_THREADS = 256;
constexpr uint32_t TF_TILE = 64 * 128 * 2;                 // one [64][128] bf16 tile: 2 swizzle atoms of 8 KB
constexpr uint32_t TF_P = 64 * 64 * 2;
constexpr uint32_t TF_BUF = 4 * TF_TILE + TF_P;            // W, Qd, Kt, U, P
constexpr uint32_t TF_S = 2 * TF_BUF;                      // bf16 S [2 atoms][128 rows dk][128 B]
constexpr uint32_t TF_DT = TF_S + 2 * 128 * 128;           // bf16 D^T [128 rows dv][128 B (64 events)]
constexpr uint32_t TF_O = TF_DT + 128 * 128;               // bf16 O staging [64][128] row-major
constexpr uint32_t TF_BAR = TF_O + 64 * 128 * 2;
constexpr uint32_t TF_SMEM = TF_BAR + 64 + 1024;
constexpr int TF_TMEM_COLS = 256;                          // S 0-127, D^T 128-191, O^T 192-255
static_assert(TF_SMEM <= 232448, "forward recurrence tile set exceeds one CTA's shared memory");

__device__ __forceinline__ uint32_t sw128(uint32_t row, uint32_t col) {   // byte offset of (row, col) in a 64-col atom
  return row * 128 + ((((col >> 3) ^ row) & 7) << 4) + (col & 7) * 2;
}

__global__ void __launch_bounds__(TF_THREADS, 1)
    gdn_fwd_tc_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_q,
                      const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_u,
                      const __grid_constant__ CUtensorMap map_p, GdnArgs a, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sS = smem + TF_S;
  uint8_t* sDT = smem + TF_DT;
  __nv_bfloat16* sO = reinterpret_cast<__nv_bfloat16*>(smem + TF_O);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + TF_BAR);   // [2]
  uint64_t* bar1 = full + 2;
  uint64_t* bar2 = full + 3;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(full + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int doc = blockIdx.y, h = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, hf = warp >> 2, row = 32 * quad + lane;
  const int c0 = a.chunk_start[doc], nc = a.chunk_count[doc];
  if (nc == 0) {
    if (a.final)   // an empty document leaves the zero state
      for (int i = tid; i < DK * 128; i += TF_THREADS) a.final[((size_t)doc * a.H + h) * DK * 128 + i] = 0.f;
    return;
  }
  if (tid == 0) {
    tc::mbar_init(&full[0], 1);
    tc::mbar_init(&full[1], 1);
    tc::mbar_init(bar1, 1);
    tc::mbar_init(bar2, 1);
    *abort_flag = 0;
    tc::fence_mbar_init();
  }
  if (warp == 0) tc::tmem_alloc(tmem_slot, TF_TMEM_COLS);
  for (int i = tid; i < 2 * 128 * 128 / 16; i += TF_THREADS)   // S = 0: bf16 copy
    reinterpret_cast<uint4*>(sS)[i] = make_uint4(0, 0, 0, 0);
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = tmem + ((uint32_t)(32 * quad) << 16);
  {
    float z[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) z[j] = 0.f;
    tc::tmem_st32(lane_base + 64 * hf, z);         // S = 0 in TMEM (this warp's half of the columns)
    tc::tmem_st32(lane_base + 64 * hf + 32, z);
  }
  tc::fence_proxy_async();
  tc::fence_before();
  __syncthreads();

  auto issue_load = [&](int ci) {
    uint8_t* buf = smem + (ci & 1) * TF_BUF;
    uint64_t* bar = &full[ci & 1];
    const int r0 = ((c0 + ci) * a.H + h) * C;
    tc::mbar_expect_tx(bar, TF_BUF);
#pragma unroll
    for (int x = 0; x < 2; ++x) {
      tc::tma_load_2d(buf + x * (TF_TILE / 2), &map_w, bar, 64 * x, r0);
      tc::tma_load_2d(buf + TF_TILE + x * (TF_TILE / 2), &map_q, bar, 64 * x, r0);
      tc::tma_load_2d(buf + 2 * TF_TILE + x * (TF_TILE / 2), &map_k, bar, 64 * x, r0);
      tc::tma_load_2d(buf + 3 * TF_TILE + x * (TF_TILE / 2), &map_u, bar, 64 * x, r0);
    }
    tc::tma_load_2d(buf + 4 * TF_TILE, &map_p, bar, 0, r0);
  };
  int loads_issued = 0, loads_seen = 0;
  uint64_t* pending = nullptr;   // barrier of the MMA group thread 0 issued and has not seen complete
  uint32_t pending_parity = 0;
  if (tid == 0) {
    tc::prefetch_map(&map_w);
    tc::prefetch_map(&map_q);
    tc::prefetch_map(&map_k);
    tc::prefetch_map(&map_u);
    tc::prefetch_map(&map_p);
    issue_load(0);
    loads_issued = 1;
  }
  bool ok = true;
  constexpr uint32_t idesc_g1 = tc::idesc_bf16(128, 64, true, false);
  constexpr uint32_t idesc_o = tc::idesc_bf16(128, 64, false, false);
  constexpr uint32_t idesc_s = tc::idesc_bf16(128, 128, true, false);
  const uint32_t s_addr = tc::smem_u32(sS), dt_addr = tc::smem_u32(sDT);
  for (int ci = 0; ci < nc && ok; ++ci) {
    const int c = c0 + ci;
    uint8_t* buf = smem + (ci & 1) * TF_BUF;
    const uint32_t w_addr = tc::smem_u32(buf), q_addr = w_addr + TF_TILE, k_addr = w_addr + 2 * TF_TILE;
    const uint32_t p_addr = w_addr + 4 * TF_TILE;
    const uint8_t* sU = buf + 3 * TF_TILE;
    if (tid == 0) {
      if (ci + 1 < nc) {   // the other buffer's readers (chunk ci - 1) have all finished
        issue_load(ci + 1);
        ++loads_issued;
      }
      if (tc::mbar_wait(&full[ci & 1], (ci >> 1) & 1, status, abort_flag, 51)) {
        ++loads_seen;
        tc::fence_after();
#pragma unroll
        for (int k = 0; k < DK / 16; ++k) {
          const uint64_t st = tc::smem_desc(s_addr + k * 2048, 16384, 1024);
          const uint32_t boff = (k >> 2) * (TF_TILE / 2) + (k & 3) * 32;
          tc::mma_bf16(tmem + 128, st, tc::smem_desc(w_addr + boff, 16, 1024), idesc_g1, k > 0);
          tc::mma_bf16(tmem + 192, st, tc::smem_desc(q_addr + boff, 16, 1024), idesc_g1, k > 0);
        }
        tc::mma_commit(bar1);
        pending = bar1;
        pending_parity = (uint32_t)(ci & 1);
      }
    }
    const bool seen1 = tc::mbar_wait(bar1, ci & 1, status, abort_flag, 52);
    ok = __syncthreads_and(seen1);
    if (!ok) break;
    pending = nullptr;
    tc::fence_after();
    {
      // D^T rows (value dim v = row), events [32 hf, 32 hf + 32): D^T = U^T - S^T W^T
      float x[32];
      tc::tmem_ld32(lane_base + 128 + 32 * hf, x);
      const uint32_t uatom = (row >> 6) * (TF_TILE / 2), ucol = row & 63;
#pragma unroll
      for (int j8 = 0; j8 < 4; ++j8) {
        float d[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int i = 32 * hf + 8 * j8 + q;
          const float u = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(sU + uatom + sw128(i, ucol)));
          d[q] = u - x[8 * j8 + q];
        }
        store8(reinterpret_cast<__nv_bfloat16*>(sDT + sw128(row, 32 * hf + 8 * j8)), d);
      }
      // S rows (key dim d = row), value columns [64 hf, 64 hf + 64): save S entering, scale by gamma
      const float gm = a.gamma[(size_t)c * a.H + h];
      float* dst = a.states + (((size_t)c * a.H + h) * DK + row) * 128 + 64 * hf;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float sv[32];
        tc::tmem_ld32(lane_base + 64 * hf + 32 * half, sv);
#pragma unroll
        for (int q = 0; q < 32; q += 4)
          *reinterpret_cast<float4*>(dst + 32 * half + q) = make_float4(sv[q], sv[q + 1], sv[q + 2], sv[q + 3]);
#pragma unroll
        for (int q = 0; q < 32; ++q) sv[q] *= gm;
        tc::tmem_st32(lane_base + 64 * hf + 32 * half, sv);
      }
    }
    tc::fence_proxy_async();
    tc::fence_before();
    __syncthreads();
    if (tid == 0) {
      tc::fence_after();
#pragma unroll
      for (int k = 0; k < C / 16; ++k) {
        const uint64_t dt = tc::smem_desc(dt_addr + k * 32, 16, 1024);
        tc::mma_bf16(tmem + 192, dt, tc::smem_desc(p_addr + k * 32, 16, 1024), idesc_o, 1u);
        tc::mma_bf16(tmem, tc::smem_desc(k_addr + k * 2048, TF_TILE / 2, 1024), dt, idesc_s, 1u);
      }
      tc::mma_commit(bar2);
      pending = bar2;
      pending_parity = (uint32_t)(ci & 1);
    }
    const bool seen2 = tc::mbar_wait(bar2, ci & 1, status, abort_flag, 53);
    ok = __syncthreads_and(seen2);
    if (!ok) break;
    pending = nullptr;
    tc::fence_after();
    {
      float o[32];
      tc::tmem_ld32(lane_base + 192 + 32 * hf, o);   // O^T row v = row, events [32 hf, +32)
#pragma unroll
      for (int q = 0; q < 32; ++q) sO[(32 * hf + q) * 128 + row] = __float2bfloat16(o[q]);
      const bool last = ci + 1 == nc;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float sv[32];
        tc::tmem_ld32(lane_base + 64 * hf + 32 * half, sv);   // new S, row d = row
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8)
          store8(reinterpret_cast<__nv_bfloat16*>(sS + hf * 16384 + sw128(row, 32 * half + 8 * q8)), sv + 8 * q8);
        if (last && a.final) {
          float* fin = a.final + (((size_t)doc * a.H + h) * DK + row) * 128 + 64 * hf + 32 * half;
#pragma unroll
          for (int q = 0; q < 32; q += 4) *reinterpret_cast<float4*>(fin + q) = make_float4(sv[q], sv[q + 1], sv[q + 2], sv[q + 3]);
        }
      }
    }
    tc::fence_proxy_async();
    tc::fence_before();
    __syncthreads();
    {
      __nv_bfloat16* out = a.out + ((size_t)c * a.H + h) * C * 128;
      for (int e = tid; e < C * 128 / 8; e += TF_THREADS)
        reinterpret_cast<uint4*>(out)[e] = reinterpret_cast<const uint4*>(sO)[e];
    }
    __syncthreads();   // sO and this buffer's U are free again
  }
  if (tid == 0) {   // nothing issued by this CTA is in flight when it retires (bounded)
    const unsigned long long t0 = tc::globaltimer();
    for (int l = loads_seen; l < loads_issued; ++l)
      while (!tc::mbar_try_wait(&full[l & 1], (l >> 1) & 1) && tc::globaltimer() - t0 < tc::kWaitNs) {
      }
    if (pending != nullptr)
      while (!tc::mbar_try_wait(pending, pending_parity) && tc::globaltimer() - t0 < tc::kWaitNs) {
      }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, TF_TMEM_COLS);
}

// ---- backward recurrence on tcgen05 -------------------------------------------------------------
//
// Same contract as gdn_bwd_kernel for a value dim of 128: one CTA per (document, head) walks the
// chunks from last to first with dS [dk x dv] (fp32) in TMEM (lanes = dk, columns 0-127):
//   group 1: dD^T = dO^T P + dS^T Kt^T      (M = 128 value dims, N = 64 events; dO, P and dS as
//                                             MN-major operands)
//   epilogue: -dD^T -> bf16 K-major tile; dS entering from the right is written out (fp32) and
//             scaled by gamma in TMEM
//   group 2: dS += Qd^T dO + W^T (-dD)       (Qd, W as MN-major A operands)
//   epilogue: the new dS becomes the bf16 operand of the previous chunk.
// Loads, warp roles and bounded waits (status codes 54-56) as in gdn_fwd_tc_kernel.
__global__ void __launch_bounds__(TF_THREADS, 1)
    gdn_bwd_tc_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_q,
                      const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_do,
                      const __grid_constant__ CUtensorMap map_p, GdnArgs a, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sS = smem + TF_S;     // bf16 dS
  uint8_t* sDT = smem + TF_DT;   // bf16 -dD^T
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + TF_BAR);   // [2]
  uint64_t* bar1 = full + 2;
  uint64_t* bar2 = full + 3;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(full + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int doc = blockIdx.y, h = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, hf = warp >> 2, row = 32 * quad + lane;
  const int c0 = a.chunk_start[doc], nc = a.chunk_count[doc];
  if (nc == 0) return;
  if (tid == 0) {
    tc::mbar_init(&full[0], 1);
    tc::mbar_init(&full[1], 1);
    tc::mbar_init(bar1, 1);
    tc::mbar_init(bar2, 1);
    *abort_flag = 0;
    tc::fence_mbar_init();
  }
  if (warp == 0) tc::tmem_alloc(tmem_slot, TF_TMEM_COLS);
  for (int i = tid; i < 2 * 128 * 128 / 16; i += TF_THREADS) reinterpret_cast<uint4*>(sS)[i] = make_uint4(0, 0, 0, 0);
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = tmem + ((uint32_t)(32 * quad) << 16);
  {
    float z[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) z[j] = 0.f;
    tc::tmem_st32(lane_base + 64 * hf, z);
    tc::tmem_st32(lane_base + 64 * hf + 32, z);
  }
  tc::fence_proxy_async();
  tc::fence_before();
  __syncthreads();

  auto issue_load = [&](int it) {   // iteration it processes chunk c0 + nc - 1 - it
    uint8_t* buf = smem + (it & 1) * TF_BUF;
    uint64_t* bar = &full[it & 1];
    const int r0 = ((c0 + nc - 1 - it) * a.H + h) * C;
    tc::mbar_expect_tx(bar, TF_BUF);
#pragma unroll
    for (int x = 0; x < 2; ++x) {
      tc::tma_load_2d(buf + x * (TF_TILE / 2), &map_w, bar, 64 * x, r0);
      tc::tma_load_2d(buf + TF_TILE + x * (TF_TILE / 2), &map_q, bar, 64 * x, r0);
      tc::tma_load_2d(buf + 2 * TF_TILE + x * (TF_TILE / 2), &map_k, bar, 64 * x, r0);
      tc::tma_load_2d(buf + 3 * TF_TILE + x * (TF_TILE / 2), &map_do, bar, 64 * x, r0);
    }
    tc::tma_load_2d(buf + 4 * TF_TILE, &map_p, bar, 0, r0);
  };
  int loads_issued = 0, loads_seen = 0;
  uint64_t* pending = nullptr;
  uint32_t pending_parity = 0;
  if (tid == 0) {
    tc::prefetch_map(&map_w);
    tc::prefetch_map(&map_q);
    tc::prefetch_map(&map_k);
    tc::prefetch_map(&map_do);
    tc::prefetch_map(&map_p);
    issue_load(0);
    loads_issued = 1;
  }
  bool ok = true;
  constexpr uint32_t idesc_dop = tc::idesc_bf16(128, 64, true, true);     // dO^T P (both MN-major)
  constexpr uint32_t idesc_dsk = tc::idesc_bf16(128, 64, true, false);    // dS^T Kt^T
  constexpr uint32_t idesc_qdo = tc::idesc_bf16(128, 128, true, true);    // Qd^T dO
  constexpr uint32_t idesc_wdd = tc::idesc_bf16(128, 128, true, false);   // W^T (-dD)
  const uint32_t s_addr = tc::smem_u32(sS), dt_addr = tc::smem_u32(sDT);
  for (int it = 0; it < nc && ok; ++it) {
    const int c = c0 + nc - 1 - it;
    uint8_t* buf = smem + (it & 1) * TF_BUF;
    const uint32_t w_addr = tc::smem_u32(buf), q_addr = w_addr + TF_TILE, k_addr = w_addr + 2 * TF_TILE;
    const uint32_t do_addr = w_addr + 3 * TF_TILE, p_addr = w_addr + 4 * TF_TILE;
    if (tid == 0) {
      if (it + 1 < nc) {
        issue_load(it + 1);
        ++loads_issued;
      }
      if (tc::mbar_wait(&full[it & 1], (it >> 1) & 1, status, abort_flag, 54)) {
        ++loads_seen;
        tc::fence_after();
#pragma unroll
        for (int k = 0; k < C / 16; ++k)
          tc::mma_bf16(tmem + 128, tc::smem_desc(do_addr + k * 2048, TF_TILE / 2, 1024),
                       tc::smem_desc(p_addr + k * 2048, TF_TILE / 2, 1024), idesc_dop, k > 0);
#pragma unroll
        for (int k = 0; k < DK / 16; ++k)
          tc::mma_bf16(tmem + 128, tc::smem_desc(s_addr + k * 2048, 16384, 1024),
                       tc::smem_desc(k_addr + (k >> 2) * (TF_TILE / 2) + (k & 3) * 32, 16, 1024), idesc_dsk, 1u);
        tc::mma_commit(bar1);
        pending = bar1;
        pending_parity = (uint32_t)(it & 1);
      }
    }
    const bool seen1 = tc::mbar_wait(bar1, it & 1, status, abort_flag, 55);
    ok = __syncthreads_and(seen1);
    if (!ok) break;
    pending = nullptr;
    tc::fence_after();
    {
      float x[32];
      tc::tmem_ld32(lane_base + 128 + 32 * hf, x);   // dD^T row v = row, events [32 hf, +32)
#pragma unroll
      for (int q = 0; q < 32; ++q) x[q] = -x[q];
#pragma unroll
      for (int j8 = 0; j8 < 4; ++j8) store8(reinterpret_cast<__nv_bfloat16*>(sDT + sw128(row, 32 * hf + 8 * j8)), x + 8 * j8);
      const float gm = a.gamma[(size_t)c * a.H + h];
      float* dst = a.states + (((size_t)c * a.H + h) * DK + row) * 128 + 64 * hf;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float sv[32];
        tc::tmem_ld32(lane_base + 64 * hf + 32 * half, sv);
#pragma unroll
        for (int q = 0; q < 32; q += 4)
          *reinterpret_cast<float4*>(dst + 32 * half + q) = make_float4(sv[q], sv[q + 1], sv[q + 2], sv[q + 3]);
#pragma unroll
        for (int q = 0; q < 32; ++q) sv[q] *= gm;
        tc::tmem_st32(lane_base + 64 * hf + 32 * half, sv);
      }
    }
    tc::fence_proxy_async();
    tc::fence_before();
    __syncthreads();
    if (tid == 0) {
      tc::fence_after();
#pragma unroll
      for (int k = 0; k < C / 16; ++k) {
        tc::mma_bf16(tmem, tc::smem_desc(q_addr + k * 2048, TF_TILE / 2, 1024),
                     tc::smem_desc(do_addr + k * 2048, TF_TILE / 2, 1024), idesc_qdo, 1u);
        tc::mma_bf16(tmem, tc::smem_desc(w_addr + k * 2048, TF_TILE / 2, 1024), tc::smem_desc(dt_addr + k * 32, 16, 1024),
                     idesc_wdd, 1u);
      }
      tc::mma_commit(bar2);
      pending = bar2;
      pending_parity = (uint32_t)(it & 1);
    }
    const bool seen2 = tc::mbar_wait(bar2, it & 1, status, abort_flag, 56);
    ok = __syncthreads_and(seen2);
    if (!ok) break;
    pending = nullptr;
    tc::fence_after();
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float sv[32];
      tc::tmem_ld32(lane_base + 64 * hf + 32 * half, sv);
#pragma unroll
      for (int q8 = 0; q8 < 4; ++q8)
        store8(reinterpret_cast<__nv_bfloat16*>(sS + hf * 16384 + sw128(row, 32 * half + 8 * q8)), sv + 8 * q8);
    }
    tc::fence_proxy_async();
    tc::fence_before();
    __syncthreads();   // the new dS operand is visible; this buffer is free again
  }
  if (tid == 0) {
    const unsigned long long t0 = tc::globaltimer();
    for (int l = loads_seen; l < loads_issued; ++l)
      while (!tc::mbar_try_wait(&full[l & 1], (l >> 1) & 1) && tc::globaltimer() - t0 < tc::kWaitNs) {
      }
    if (pending != nullptr)
      while (!tc::mbar_try_wait(pending, pending_parity) && tc::globaltimer() - t0 < tc::kWaitNs) {
      }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, TF_TMEM_COLS);
}

bool gdn_fwd_use_tc(int dv) {
  static const bool on = [] {
    const char* v = std::getenv("CQB_GDN_TC");
    return v == nullptr || std::string(v) != "0";
  }();
  return on && dv == 128;
}

constexpr size_t SMEM = (size_t)(2 * BUF + DK * LDV + C * LDV) * sizeof(__nv_bfloat16);

void check(const at::Tensor& t, const char* name, at::ScalarType dtype) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous() && t.scalar_type() == dtype, name, " must be a contiguous CUDA tensor of ",
              dtype);
}

GdnArgs make_args(const at::Tensor& W, const at::Tensor& Qd, const at::Tensor& Kt, const at::Tensor& P,
                  const at::Tensor& UV, const at::Tensor& gamma, const at::Tensor& start, const at::Tensor& count) {
  check(W, "W", at::kBFloat16);
  check(Qd, "Qd", at::kBFloat16);
  check(Kt, "Kt", at::kBFloat16);
  check(P, "P", at::kBFloat16);
  check(UV, "U/dO", at::kBFloat16);
  check(gamma, "gamma", at::kFloat);
  check(start, "chunk_start", at::kInt);
  check(count, "chunk_count", at::kInt);
  TORCH_CHECK(W.dim() == 4 && W.size(2) == C && W.size(3) == DK, "W must be [Nc, H, 64, 128]");
  TORCH_CHECK(UV.size(3) % BV == 0, "value dim must be a multiple of 64");
  GdnArgs a{};
  a.W = (const __nv_bfloat16*)W.data_ptr();
  a.Qd = (const __nv_bfloat16*)Qd.data_ptr();
  a.Kt = (const __nv_bfloat16*)Kt.data_ptr();
  a.P = (const __nv_bfloat16*)P.data_ptr();
  a.UV = (const __nv_bfloat16*)UV.data_ptr();
  a.gamma = gamma.data_ptr<float>();
  a.chunk_start = start.data_ptr<int>();
  a.chunk_count = count.data_ptr<int>();
  a.H = W.size(1);
  a.DV = UV.size(3);
  return a;
}

void set_smem(const void* fn) {
  CQB_CHECK_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM));
}

}  // namespace

// Returns (O [Nc,H,C,DV] bf16, S_entering [Nc,H,DK,DV] fp32) and, with want_final, the fp32 state
// after each document [docs,H,DK,DV] (the prefill state of CQ decoding).
std::vector<at::Tensor> gdn_fwd(at::Tensor W, at::Tensor U, at::Tensor P, at::Tensor Qd, at::Tensor Kt,
                                at::Tensor gamma, at::Tensor start, at::Tensor count, bool want_final) {
  GdnArgs a = make_args(W, Qd, Kt, P, U, gamma, start, count);
  auto O = at::empty_like(U);
  const bool tc_path = gdn_fwd_use_tc(a.DV);
  auto S = at::empty({W.size(0), W.size(1), DK, U.size(3)}, W.options().dtype(at::kFloat));
  a.out = (__nv_bfloat16*)O.data_ptr();
  a.states = S.data_ptr<float>();
  at::Tensor F;
  if (want_final) {
    F = at::empty({start.size(0), W.size(1), DK, U.size(3)}, W.options().dtype(at::kFloat));
    a.final = F.data_ptr<float>();
  }
  if (tc_path) {
    static bool once_tc = [] {
      CQB_CHECK_CUDA(cudaFuncSetAttribute((const void*)gdn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)TF_SMEM));
      return true;
    }();
    (void)once_tc;
    const long rows = W.size(0) * W.size(1) * C;
    const auto mw = tma_map_bf16(W.view({rows, DK}), C);
    const auto mq = tma_map_bf16(Qd.view({rows, DK}), C);
    const auto mk = tma_map_bf16(Kt.view({rows, DK}), C);
    const auto mu = tma_map_bf16(U.view({rows, 128}), C);
    const auto mp = tma_map_bf16(P.view({rows, C}), C);
    gdn_fwd_tc_kernel<<<dim3(a.H, start.size(0)), TF_THREADS, TF_SMEM, stream()>>>(mw, mq, mk, mu, mp, a,
                                                                                  gdn_status_word());
  } else {
    static bool once = (set_smem((const void*)gdn_fwd_kernel), true);
    (void)once;
    dim3 grid(a.DV / BV, a.H, start.size(0));
    gdn_fwd_kernel<<<grid, THREADS, SMEM, stream()>>>(a);
  }
  CQB_LAUNCH_CHECK();
  count_launch();
  if (want_final) return {O, S, F};
  return {O, S};
}

// Returns dS_after [Nc,H,DK,DV] fp32: gradient w.r.t. the state leaving each chunk.
at::Tensor gdn_bwd(at::Tensor dO, at::Tensor W, at::Tensor P, at::Tensor Qd, at::Tensor Kt, at::Tensor gamma,
                   at::Tensor start, at::Tensor count) {
  GdnArgs a = make_args(W, Qd, Kt, P, dO, gamma, start, count);
  auto dS = at::empty({W.size(0), W.size(1), DK, dO.size(3)}, W.options().dtype(at::kFloat));
  a.states = dS.data_ptr<float>();
  if (gdn_fwd_use_tc(a.DV)) {
    static bool once_tc = [] {
      CQB_CHECK_CUDA(cudaFuncSetAttribute((const void*)gdn_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)TF_SMEM));
      return true;
    }();
    (void)once_tc;
    const long rows = W.size(0) * W.size(1) * C;
    const auto mw = tma_map_bf16(W.view({rows, DK}), C);
    const auto mq = tma_map_bf16(Qd.view({rows, DK}), C);
    const auto mk = tma_map_bf16(Kt.view({rows, DK}), C);
    const auto mo = tma_map_bf16(dO.view({rows, 128}), C);
    const auto mp = tma_map_bf16(P.view({rows, C}), C);
    gdn_bwd_tc_kernel<<<dim3(a.H, start.size(0)), TF_THREADS, TF_SMEM, stream()>>>(mw, mq, mk, mo, mp, a,
                                                                                  gdn_status_word());
  } else {
    static bool once = (set_smem((const void*)gdn_bwd_kernel), true);
    (void)once;
    dim3 grid(a.DV / BV, a.H, start.size(0));
    gdn_bwd_kernel<<<grid, THREADS, SMEM, stream()>>>(a);
  }
  CQB_LAUNCH_CHECK();
  count_launch();
  return dS;
}

}  // namespace cqb
