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

namespace cqb {

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
  auto S = at::empty({W.size(0), W.size(1), DK, U.size(3)}, W.options().dtype(at::kFloat));
  a.out = (__nv_bfloat16*)O.data_ptr();
  a.states = S.data_ptr<float>();
  at::Tensor F;
  if (want_final) {
    F = at::empty({start.size(0), W.size(1), DK, U.size(3)}, W.options().dtype(at::kFloat));
    a.final = F.data_ptr<float>();
  }
  static bool once = (set_smem((const void*)gdn_fwd_kernel), true);
  (void)once;
  dim3 grid(a.DV / BV, a.H, start.size(0));
  gdn_fwd_kernel<<<grid, THREADS, SMEM, stream()>>>(a);
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
  static bool once = (set_smem((const void*)gdn_bwd_kernel), true);
  (void)once;
  dim3 grid(a.DV / BV, a.H, start.size(0));
  gdn_bwd_kernel<<<grid, THREADS, SMEM, stream()>>>(a);
  CQB_LAUNCH_CHECK();
  count_launch();
  return dS;
}

}  // namespace cqb
