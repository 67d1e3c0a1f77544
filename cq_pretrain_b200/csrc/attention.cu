// Tensor-core (tcgen05) flash attention over per-row key ranges for sm_100a: forward, dQ, dK/dV.
//
// Row r of a head reads keys [kstart[r], kend[r]) (the CQ visibility of a packed sequence, or the
// sample of a varlen DiT row); GQA (head h reads kv head h / (Hq / Hkv)); empty ranges output zero
// with LSE = +inf; LSE in natural-log units. Key tiles outside the union of a block's ranges are
// skipped, so skipped work is exact. Forward: one CTA per (128-row block, head):
//  * warp 0 (one thread) streams the Q block once and K / V key tiles through a 2-deep ring
//    with TMA (128-byte swizzle; D / 64 boxes per tile);
//  * warp 1 allocates TMEM and issues the MMAs (one thread): S_j = Q K_j^T into one of two TMEM
//    score buffers (so S_{j+1} runs while the softmax reads S_j) and O += P_j V_j into a TMEM
//    accumulator that stays resident for the whole key loop (V is the MN-major B operand, so
//    no transpose);
//  * warps 2..5 own one query row per thread (TMEM lane = row): tcgen05.ld of the row's scores,
//    range mask, exp2-domain softmax without any cross-thread reduction, P_j written to shared
//    memory as bf16 in the 128B-swizzled K-major layout the MMA reads, and the epilogue
//    (tcgen05.ld of O, 1/l, bf16 stores, LSE).
// The running max is rescaled lazily: a row keeps its exponent reference until a tile's max
// exceeds it by more than 8 (P <= 2^8), and only then rescales its O row in TMEM (tcgen05.ld /
// st after the previous P V has retired). Numerator and denominator always share the
// reference, so the result is exact up to rounding.
// Tile sizes: BN = 64 keys at D = 256 (TMEM: 2 x 64 score + 256 O columns), 128 otherwise.
// Every wait is bounded; on expiry the kernel records a code in the status word, stops
// issuing, drains its TMA transactions and MMAs (bounded), frees TMEM and returns.
#include "common.cuh"
#include "tcgen05.cuh"

namespace cqb {

namespace {

constexpr float LOG2E_TC = 1.4426950408889634f;
constexpr float RESCALE_THRESHOLD = 8.f;  // log2 units

int* attn_status_word() {
  static int* word = [] {
    int* p = nullptr;
    CQB_CHECK_CUDA(cudaMalloc(&p, sizeof(int)));
    CQB_CHECK_CUDA(cudaMemset(p, 0, sizeof(int)));
    return p;
  }();
  return word;
}

// Longest-first launch order. Job 0 ranks the 128-row blocks by the number of `tile`-key tiles
// their rows' key-range union spans; job 1 ranks the 128-key blocks by the number of qblk-row
// blocks (qb_min / qb_max unions) that meet them. order[rank] = block, descending work, ties by
// index; CTAs take their block from the order, so the hardware's in-order dispatch starts the
// longest blocks first and the short ones fill the tail. Past kMaxScheduled blocks the order is
// the identity.
constexpr int kMaxScheduled = 4096;

__global__ void __launch_bounds__(1024) attn_schedule_kernel(const int* __restrict__ kstart, const int* __restrict__ kend,
                                                             int rows, int tile, int* __restrict__ order_rows,
                                                             const int* __restrict__ qb_min,
                                                             const int* __restrict__ qb_max, int nqb, int keys,
                                                             int* __restrict__ order_keys) {
  __shared__ int work[kMaxScheduled];
  const int job = blockIdx.x;
  const int n = job == 0 ? (rows + 127) / 128 : (keys + 127) / 128;
  int* order = job == 0 ? order_rows : order_keys;
  if (n > kMaxScheduled) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) order[i] = i;
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (job == 0) {
    for (int b = warp; b < n; b += 32) {
      int lo = INT_MAX, hi = 0;
      for (int r = b * 128 + lane; r < min(rows, b * 128 + 128); r += 32) {
        const int s = kstart[r], e = kend[r];
        if (e > s) lo = min(lo, s), hi = max(hi, e);
      }
      lo = __reduce_min_sync(0xffffffffu, lo);
      hi = __reduce_max_sync(0xffffffffu, hi);
      if (lane == 0) work[b] = lo < hi ? (hi - (lo / tile) * tile + tile - 1) / tile : 0;
    }
  } else {
    for (int b = warp; b < n; b += 32) {
      int c = 0;
      for (int q = lane; q < nqb; q += 32) {
        const int lo = qb_min[q], hi = qb_max[q];
        c += (lo < hi && lo < b * 128 + 128 && hi > b * 128) ? 1 : 0;
      }
      c = __reduce_add_sync(0xffffffffu, c);
      if (lane == 0) work[b] = c;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int w = work[i];
    int rank = 0;
    for (int j = 0; j < n; ++j) rank += (work[j] > w || (work[j] == w && j < i)) ? 1 : 0;
    order[rank] = i;
  }
}

template <int D>
struct FwdTc {
  static constexpr int BM = 128;
  static constexpr int BN = D == 256 ? 64 : 128;
  static constexpr int KB = D / 64;                      // 64-wide boxes per row
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;            // one K or V tile
  static constexpr int P_ATOM = BM * 128;                // 128 rows x 64 keys (bf16)
  static constexpr int P_BYTES = BM * BN * 2;
  static constexpr int SMEM = Q_BYTES + 4 * KV_BYTES + 2 * P_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t O_COL = 2 * BN;
};

struct FwdTcArgs {
  const int* kstart;
  const int* kend;
  const int* order;    // row blocks, longest first (null: index order, when all CTAs fit one wave)
  __nv_bfloat16* out;  // [rows, Hq, D]
  float* lse;          // [Hq, rows]
  int rows, keys, Hq, Hkv;
  float scale;
};

template <int D>
__global__ void __launch_bounds__(192, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                       const __grid_constant__ CUtensorMap map_v, FwdTcArgs a, int* status) {
  using C = FwdTc<D>;
  constexpr int BM = C::BM, BN = C::BN, KB = C::KB;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = smem;
  uint8_t* sk = sq + C::Q_BYTES;            // [2][KV_BYTES]
  uint8_t* sv = sk + 2 * C::KV_BYTES;       // [2][KV_BYTES]
  uint8_t* sp = sv + 2 * C::KV_BYTES;       // [2][P_BYTES]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sp + 2 * C::P_BYTES);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* p_full = bars + 11;  // [2]
  uint64_t* pv_done = bars + 13; // [2]
  uint64_t* drain = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* s_range = reinterpret_cast<int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = blockIdx.x / a.Hq, qb = a.order ? a.order[slot] : slot;
  const int h = blockIdx.x % a.Hq, hk = h / (a.Hq / a.Hkv);
  const int r0 = qb * BM;

  if (threadIdx.x == 0) {
    tc::mbar_init(q_full, 1);
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&k_full[b], 1);
      tc::mbar_init(&k_empty[b], 1);
      tc::mbar_init(&v_full[b], 1);
      tc::mbar_init(&v_empty[b], 1);
      tc::mbar_init(&s_full[b], 1);
      tc::mbar_init(&p_full[b], 128);
      tc::mbar_init(&pv_done[b], 1);
    }
    tc::mbar_init(drain, 1);
    *abort_flag = 0;
    s_range[0] = INT_MAX;
    s_range[1] = 0;
    tc::fence_mbar_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, C::TMEM_COLS);
  __syncthreads();
  // union of the block's key ranges -> key tiles [kt0, kt0 + nt * BN)
  if (threadIdx.x < BM) {
    const int row = r0 + threadIdx.x;
    int lo = INT_MAX, hi = 0;
    if (row < a.rows) {
      const int s = a.kstart[row], e = a.kend[row];
      if (e > s) lo = s, hi = e;
    }
    lo = __reduce_min_sync(0xffffffffu, lo);
    hi = __reduce_max_sync(0xffffffffu, hi);
    if (lane == 0) {
      atomicMin(&s_range[0], lo);
      atomicMax(&s_range[1], hi);
    }
  }
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;
  const int klo = s_range[0], khi = s_range[1];
  const int kt0 = klo < khi ? (klo / BN) * BN : 0;
  const int nt = klo < khi ? (khi - kt0 + BN - 1) / BN : 0;

  if (warp == 0) {
    if (lane == 0 && nt > 0) {
      tc::prefetch_map(&map_q);
      tc::prefetch_map(&map_k);
      tc::prefetch_map(&map_v);
      int armed_k[2] = {-1, -1}, armed_v[2] = {-1, -1};
      bool ok = true;
      tc::mbar_expect_tx(q_full, C::Q_BYTES);
#pragma unroll
      for (int i = 0; i < KB; ++i) tc::tma_load_2d(sq + i * BM * 128, &map_q, q_full, h * D + i * 64, r0);
      for (int j = 0; j < nt && ok; ++j) {
        const int b = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        const int n0 = kt0 + j * BN;
        if (!tc::mbar_wait(&k_empty[b], ph ^ 1, status, abort_flag, 31)) { ok = false; break; }
        tc::mbar_expect_tx(&k_full[b], C::KV_BYTES);
#pragma unroll
        for (int i = 0; i < KB; ++i)
          tc::tma_load_2d(sk + b * C::KV_BYTES + i * BN * 128, &map_k, &k_full[b], hk * D + i * 64, n0);
        armed_k[b] = (int)ph;
        if (!tc::mbar_wait(&v_empty[b], ph ^ 1, status, abort_flag, 32)) { ok = false; break; }
        tc::mbar_expect_tx(&v_full[b], C::KV_BYTES);
#pragma unroll
        for (int i = 0; i < KB; ++i)
          tc::tma_load_2d(sv + b * C::KV_BYTES + i * BN * 128, &map_v, &v_full[b], hk * D + i * 64, n0);
        armed_v[b] = (int)ph;
      }
      // drain: every issued transaction lands before the CTA's shared memory is released
      const unsigned long long t0 = tc::globaltimer();
      while (!tc::mbar_try_wait(q_full, 0) && tc::globaltimer() - t0 < tc::kWaitNs) {
      }
      for (int b = 0; b < 2; ++b) {
        if (armed_k[b] >= 0)
          while (!tc::mbar_try_wait(&k_full[b], (uint32_t)armed_k[b]) && tc::globaltimer() - t0 < tc::kWaitNs) {
          }
        if (armed_v[b] >= 0)
          while (!tc::mbar_try_wait(&v_full[b], (uint32_t)armed_v[b]) && tc::globaltimer() - t0 < tc::kWaitNs) {
          }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && nt > 0) {
      constexpr uint32_t idesc_s = tc::idesc_bf16(BM, BN, false, false);
      constexpr uint32_t idesc_o = tc::idesc_bf16(BM, D, false, true);
      const uint32_t q_addr = tc::smem_u32(sq), k_addr = tc::smem_u32(sk), v_addr = tc::smem_u32(sv),
                     p_addr = tc::smem_u32(sp);
      auto issue_s = [&](int j) -> bool {
        const int b = j & 1;
        if (!tc::mbar_wait(&k_full[b], (j >> 1) & 1, status, abort_flag, 33)) return false;
        tc::fence_after();
        const uint32_t kb_addr = k_addr + b * C::KV_BYTES;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint64_t ad = tc::smem_desc(q_addr + (k >> 2) * (BM * 128) + (k & 3) * 32, 16, 1024);
          const uint64_t bd = tc::smem_desc(kb_addr + (k >> 2) * (BN * 128) + (k & 3) * 32, 16, 1024);
          tc::mma_bf16(tmem + b * BN, ad, bd, idesc_s, k > 0 ? 1u : 0u);
        }
        tc::mma_commit(&k_empty[b]);
        tc::mma_commit(&s_full[b]);
        return true;
      };
      bool ok = tc::mbar_wait(q_full, 0, status, abort_flag, 34);
      if (ok) {
        tc::fence_after();
        ok = issue_s(0);
      }
      for (int j = 0; j < nt && ok; ++j) {
        if (j + 1 < nt && !issue_s(j + 1)) break;
        const int b = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!tc::mbar_wait(&p_full[b], ph, status, abort_flag, 35)) break;
        if (!tc::mbar_wait(&v_full[b], ph, status, abort_flag, 36)) break;
        tc::fence_after();
        const uint32_t vb_addr = v_addr + b * C::KV_BYTES, pb_addr = p_addr + b * C::P_BYTES;
#pragma unroll
        for (int k = 0; k < BN / 16; ++k) {
          const uint64_t ad = tc::smem_desc(pb_addr + (k >> 2) * C::P_ATOM + (k & 3) * 32, 16, 1024);
          const uint64_t bd = tc::smem_desc(vb_addr + k * 2048, BN * 128, 1024);
          tc::mma_bf16(tmem + C::O_COL, ad, bd, idesc_o, (j > 0 || k > 0) ? 1u : 0u);
        }
        tc::mma_commit(&v_empty[b]);
        tc::mma_commit(&pv_done[b]);
      }
      tc::mma_commit(drain);
      const unsigned long long t0 = tc::globaltimer();
      while (!tc::mbar_try_wait(drain, 0) && tc::globaltimer() - t0 < tc::kWaitNs) {
      }
    }
  } else {
    // softmax / epilogue: one query row per thread
    const int quarter = warp & 3;
    const int rl = quarter * 32 + lane, row = r0 + rl;
    const bool valid = row < a.rows;
    const int rks = valid ? a.kstart[row] : 0, rke = valid ? a.kend[row] : 0;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    const float sl2 = a.scale * LOG2E_TC;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    // warp-uniform bounded wait (the TMEM loads and stores that follow are warp-collective)
    auto wwait = [&](uint64_t* bar, uint32_t parity, int code) {
      return __all_sync(0xffffffffu, tc::mbar_wait(bar, parity, status, abort_flag, code));
    };
    for (int j = 0; j < nt; ++j) {
      const int b = j & 1;
      if (!wwait(&s_full[b], (j >> 1) & 1, 37)) { ok = false; break; }
      tc::fence_after();
      const int n0 = kt0 + j * BN;
      float s[BN];
#pragma unroll
      for (int c = 0; c < BN; c += 32) tc::tmem_ld32(lane_base + b * BN + c, s + c);
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < BN; ++c) {
        const int key = n0 + c;
        s[c] = (key >= rks && key < rke) ? s[c] * sl2 : -INFINITY;
        mt = fmaxf(mt, s[c]);
      }
      const bool need = mt > m_ref + RESCALE_THRESHOLD;
      const float corr = (need && m_ref != -INFINITY) ? exp2f(m_ref - mt) : 1.f;
      if (__any_sync(0xffffffffu, corr != 1.f)) {
        // O holds P_0..P_{j-1} V: wait for the last P V before rescaling this warp's rows
        if (!wwait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, 38)) { ok = false; break; }
        tc::fence_after();
#pragma unroll 1
        for (int c = 0; c < D; c += 32) {
          float o[32];
          tc::tmem_ld32(lane_base + C::O_COL + c, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= corr;
          tc::tmem_st32(lane_base + C::O_COL + c, o);
        }
      }
      if (need) m_ref = mt;
      l *= corr;
      const float mr = m_ref == -INFINITY ? 0.f : m_ref;
      // P buffer b was read by P_{j-2} V
      if (j >= 2 && !wwait(&pv_done[b], ((j >> 1) + 1) & 1, 39)) { ok = false; break; }
      uint8_t* prow = sp + b * C::P_BYTES + rl * 128;
#pragma unroll
      for (int c8 = 0; c8 < BN / 8; ++c8) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float p0 = exp2f(s[c8 * 8 + 2 * i] - mr), p1 = exp2f(s[c8 * 8 + 2 * i + 1] - mr);
          l += p0 + p1;
          __nv_bfloat162 v2 = __floats2bfloat162_rn(p0, p1);
          w[i] = *reinterpret_cast<uint32_t*>(&v2);
        }
        const int atom = c8 >> 3, chunk = (c8 & 7) ^ (rl & 7);
        *reinterpret_cast<uint4*>(prow + atom * C::P_ATOM + chunk * 16) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      tc::fence_proxy_async();
      tc::fence_before();
      tc::mbar_arrive(&p_full[b]);
    }
    if (ok && nt > 0 && !wwait(&pv_done[(nt - 1) & 1], ((nt - 1) >> 1) & 1, 40)) ok = false;
    if (ok) {
      tc::fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* dst = a.out + ((size_t)row * a.Hq + h) * D;
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        float o[32];
        if (nt > 0) {
          tc::tmem_ld32(lane_base + C::O_COL + c, o);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
        if (valid) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              __nv_bfloat162 v2 = __floats2bfloat162_rn(o[i + 2 * e] * inv, o[i + 2 * e + 1] * inv);
              w[e] = *reinterpret_cast<uint32_t*>(&v2);
            }
            *reinterpret_cast<uint4*>(dst + c + i) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
      if (valid) a.lse[(size_t)h * a.rows + row] = l > 0.f ? (m_ref + log2f(l)) / LOG2E_TC : INFINITY;
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after();
    tc::tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ---- backward -------------------------------------------------------------------------------
// Prep: per (head, row) the exponent reference lse * log2(e) (+inf for empty rows and padding)
// and Dsum = rowsum(dO * O), packed as float2 over rows padded to a multiple of 64; per row the
// (kstart, kend) pair (0, 0 in padding); per 64-row block the union of its rows' key ranges.
__global__ void attn_bwd_prep_tc_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                        const float* __restrict__ lse, const int* __restrict__ kstart,
                                        const int* __restrict__ kend, float2* __restrict__ lsd, int2* __restrict__ kse,
                                        int* __restrict__ qb_min, int* __restrict__ qb_max, int rows, int rows_pad,
                                        int Hq, int D) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp < rows_pad * Hq) {
    const int row = warp / Hq, h = warp % Hq;
    float s = 0.f, l2 = INFINITY;
    if (row < rows) {
      const __nv_bfloat16* op = o + ((size_t)row * Hq + h) * D;
      const __nv_bfloat16* dp = dout + ((size_t)row * Hq + h) * D;
      for (int c = lane * 8; c < D; c += 256) {
        float ov[8], dv[8];
        load8(op + c, ov);
        load8(dp + c, dv);
#pragma unroll
        for (int j = 0; j < 8; ++j) s += ov[j] * dv[j];
      }
      s = warp_sum(s);
      const float l = lse[(size_t)h * rows + row];
      l2 = l == INFINITY ? INFINITY : l * LOG2E_TC;
    }
    if (lane == 0) lsd[(size_t)h * rows_pad + row] = make_float2(l2, s);
    if (lane == 0 && h == 0) kse[row] = row < rows ? make_int2(kstart[row], kend[row]) : make_int2(0, 0);
  }
  const int qb = blockIdx.x * blockDim.x + threadIdx.x;
  if (qb < rows_pad / 64) {
    int lo = INT_MAX, hi = 0;
    for (int r = qb * 64; r < min(rows, qb * 64 + 64); ++r) {
      const int s = kstart[r], e = kend[r];
      if (e > s) {
        lo = min(lo, s);
        hi = max(hi, e);
      }
    }
    qb_min[qb] = lo;
    qb_max[qb] = hi;
  }
}

struct BwdTcArgs {
  const int* order_rows;  // 128-row blocks, longest first (dQ); null: index order
  const int* order_keys;  // 128-key blocks, longest first (dK/dV); null: index order
  const float2* lsd;   // [Hq, rows_pad]
  const int2* kse;     // [rows_pad]
  const int* qb_min;   // [rows_pad / 64]
  const int* qb_max;
  const __nv_bfloat16* vsrc;  // V [keys, Hkv, D] (dK/dV at D = 256 stores it into TMEM)
  const __nv_bfloat16* dosrc; // dO [rows, Hq, D] (dQ at D = 256 stores it into TMEM)
  __nv_bfloat16* dq;   // [rows, Hq, D]
  __nv_bfloat16* dk;   // [keys, Hkv, D]
  __nv_bfloat16* dv;
  int rows, rows_pad, keys, Hq, Hkv;
  float scale;
};

// dQ: one CTA per (128-row block, head); key tiles of 64. S = Q K^T and dP = dO V^T land in
// double-buffered TMEM; each softmax thread (one row) forms dS = P (dP - Dsum) and writes it to
// shared memory (bf16, 128B-swizzled K-major); dQ += dS K accumulates in TMEM (K is the MN-major B
// operand: the same shared tile that fed S).
template <int D>
struct DqTc {
  // D = 256: dO lives in TMEM as the A operand of dP = dO V^T and dS is written back over the S
  // columns as the A operand of dQ += dS K, so shared memory holds Q and two K / V stages.
  static constexpr bool DT = D > 128;
  static constexpr int BM = 128, BN = 64, KB = D / 64;
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int DS_BYTES = BM * BN * 2;
  static constexpr int STAGES = 2;
  static constexpr int NSB = DT ? 1 : 2;               // TMEM score buffers
  static constexpr int SMEM = (DT ? 1 : 2) * Q_BYTES + 2 * STAGES * KV_BYTES + (DT ? 0 : 2 * DS_BYTES) + 1024 + 256;
  static constexpr uint32_t DP_COL = NSB * BN, DQ_COL = 2 * NSB * BN;
  static constexpr uint32_t DO_COL = DQ_COL + D;       // DT only: D / 2 columns
  static_assert(!DT || DO_COL + D / 2 <= 512, "TMEM columns");
};

template <int D>
__global__ void __launch_bounds__(192, 1)
    attn_dq_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_do,
                      const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_v,
                      BwdTcArgs a, int* status) {
  using C = DqTc<D>;
  constexpr int BM = C::BM, BN = C::BN, KB = C::KB, ST = C::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = smem;
  uint8_t* sdo = sq + C::Q_BYTES;            // (not DT)
  uint8_t* sk = sdo + (C::DT ? 0 : C::Q_BYTES);  // [ST][KV_BYTES]
  uint8_t* sv = sk + ST * C::KV_BYTES;       // [ST][KV_BYTES]
  uint8_t* sds = sv + ST * C::KV_BYTES;      // [2][DS_BYTES] (not DT)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sds + (C::DT ? 0 : 2 * C::DS_BYTES));
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* k_empty = bars + 3;   // [2]
  uint64_t* v_full = bars + 5;    // [2]
  uint64_t* v_empty = bars + 7;   // [2]
  uint64_t* s_full = bars + 9;    // [2]
  uint64_t* ds_full = bars + 11;  // [2]
  uint64_t* dq_done = bars + 13;  // [2]
  uint64_t* drain = bars + 15;
  uint64_t* do_ready = bars + 16; // DT: dO stored into TMEM by the 128 softmax threads
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* s_range = reinterpret_cast<int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = blockIdx.x / a.Hq, qb = a.order_rows ? a.order_rows[slot] : slot;
  const int h = blockIdx.x % a.Hq, hk = h / (a.Hq / a.Hkv);
  const int r0 = qb * BM;
  if (threadIdx.x == 0) {
    tc::mbar_init(q_full, 1);
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&k_full[b], 1);
      tc::mbar_init(&k_empty[b], 1);
      tc::mbar_init(&v_full[b], 1);
      tc::mbar_init(&v_empty[b], 1);
      tc::mbar_init(&s_full[b], 1);
      tc::mbar_init(&ds_full[b], 128);
      tc::mbar_init(&dq_done[b], 1);
    }
    tc::mbar_init(drain, 1);
    tc::mbar_init(do_ready, 128);
    *abort_flag = 0;
    s_range[0] = INT_MAX;
    s_range[1] = 0;
    tc::fence_mbar_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, 512);
  __syncthreads();
  if (threadIdx.x < BM) {
    const int2 r = a.kse[min(r0 + (int)threadIdx.x, a.rows_pad - 1)];
    int lo = INT_MAX, hi = 0;
    if (r0 + (int)threadIdx.x < a.rows && r.y > r.x) lo = r.x, hi = r.y;
    lo = __reduce_min_sync(0xffffffffu, lo);
    hi = __reduce_max_sync(0xffffffffu, hi);
    if (lane == 0) {
      atomicMin(&s_range[0], lo);
      atomicMax(&s_range[1], hi);
    }
  }
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;
  const int klo = s_range[0], khi = s_range[1];
  const int kt0 = klo < khi ? (klo / BN) * BN : 0;
  const int nt = klo < khi ? (khi - kt0 + BN - 1) / BN : 0;

  if (warp == 0) {
    if (lane == 0 && nt > 0) {
      tc::prefetch_map(&map_q);
      tc::prefetch_map(&map_do);
      tc::prefetch_map(&map_k);
      tc::prefetch_map(&map_v);
      int armed_k[2] = {-1, -1}, armed_v[2] = {-1, -1};
      tc::mbar_expect_tx(q_full, (C::DT ? 1 : 2) * C::Q_BYTES);
#pragma unroll
      for (int i = 0; i < KB; ++i) {
        tc::tma_load_2d(sq + i * BM * 128, &map_q, q_full, h * D + i * 64, r0);
        if (!C::DT) tc::tma_load_2d(sdo + i * BM * 128, &map_do, q_full, h * D + i * 64, r0);
      }
      for (int j = 0; j < nt; ++j) {
        const int s = j % ST;
        const uint32_t ph = (j / ST) & 1;
        const int n0 = kt0 + j * BN;
        if (!tc::mbar_wait(&v_empty[s], ph ^ 1, status, abort_flag, 41)) break;
        tc::mbar_expect_tx(&v_full[s], C::KV_BYTES);
#pragma unroll
        for (int i = 0; i < KB; ++i)
          tc::tma_load_2d(sv + s * C::KV_BYTES + i * BN * 128, &map_v, &v_full[s], hk * D + i * 64, n0);
        armed_v[s] = (int)ph;
        if (!tc::mbar_wait(&k_empty[s], ph ^ 1, status, abort_flag, 42)) break;
        tc::mbar_expect_tx(&k_full[s], C::KV_BYTES);
#pragma unroll
        for (int i = 0; i < KB; ++i)
          tc::tma_load_2d(sk + s * C::KV_BYTES + i * BN * 128, &map_k, &k_full[s], hk * D + i * 64, n0);
        armed_k[s] = (int)ph;
      }
      const unsigned long long t0 = tc::globaltimer();
      while (!tc::mbar_try_wait(q_full, 0) && tc::globaltimer() - t0 < tc::kWaitNs) {
      }
      for (int s = 0; s < 2; ++s) {
        if (armed_k[s] >= 0)
          while (!tc::mbar_try_wait(&k_full[s], (uint32_t)armed_k[s]) && tc::globaltimer() - t0 < tc::kWaitNs) {
          }
        if (armed_v[s] >= 0)
          while (!tc::mbar_try_wait(&v_full[s], (uint32_t)armed_v[s]) && tc::globaltimer() - t0 < tc::kWaitNs) {
          }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && nt > 0) {
      constexpr uint32_t idesc_s = tc::idesc_bf16(BM, BN, false, false);
      constexpr uint32_t idesc_q = tc::idesc_bf16(BM, D, false, true);
      const uint32_t q_addr = tc::smem_u32(sq), do_addr = tc::smem_u32(sdo), k_addr = tc::smem_u32(sk),
                     v_addr = tc::smem_u32(sv), ds_addr = tc::smem_u32(sds);
      // X [BM x D] (K-major) times tile [BN x D]^T -> TMEM columns col
      auto rows_x_tile = [&](uint32_t x_addr, uint32_t t_addr, uint32_t col) {
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint64_t ad = tc::smem_desc(x_addr + (k >> 2) * (BM * 128) + (k & 3) * 32, 16, 1024);
          const uint64_t bd = tc::smem_desc(t_addr + (k >> 2) * (BN * 128) + (k & 3) * 32, 16, 1024);
          tc::mma_bf16(tmem + col, ad, bd, idesc_s, k > 0 ? 1u : 0u);
        }
      };
      auto issue_dp = [&](int j) -> bool {
        const int s = j % ST;
        if (!tc::mbar_wait(&v_full[s], (j / ST) & 1, status, abort_flag, 43)) return false;
        tc::fence_after();
        if (C::DT) {   // dO [BM x D] in TMEM (two bf16 per column) times V_j^T
          const uint32_t vt = v_addr + s * C::KV_BYTES;
#pragma unroll
          for (int k = 0; k < D / 16; ++k)
            tc::mma_bf16_ts(tmem + C::DP_COL, tmem + C::DO_COL + k * 8,
                            tc::smem_desc(vt + (k >> 2) * (BN * 128) + (k & 3) * 32, 16, 1024), idesc_s,
                            k > 0 ? 1u : 0u);
        } else {
          rows_x_tile(do_addr, v_addr + s * C::KV_BYTES, C::DP_COL + (j & 1) * BN);
        }
        tc::mma_commit(&v_empty[s]);
        return true;
      };
      auto issue_s = [&](int j) -> bool {
        const int s = j % ST, b = C::DT ? 0 : (j & 1);
        if (!tc::mbar_wait(&k_full[s], (j / ST) & 1, status, abort_flag, 44)) return false;
        tc::fence_after();
        rows_x_tile(q_addr, k_addr + s * C::KV_BYTES, b * BN);
        tc::mma_commit(&s_full[b]);
        return true;
      };
      auto issue_dq = [&](int j) -> bool {
        const int b = C::DT ? 0 : (j & 1), s = j % ST;
        if (!tc::mbar_wait(&ds_full[b], (C::DT ? j : j >> 1) & 1, status, abort_flag, 45)) return false;
        tc::fence_after();
        const uint32_t kt = k_addr + s * C::KV_BYTES, dst = ds_addr + b * C::DS_BYTES;
#pragma unroll
        for (int k = 0; k < BN / 16; ++k) {
          const uint64_t bd = tc::smem_desc(kt + k * 2048, BN * 128, 1024);
          const uint32_t acc = (j > 0 || k > 0) ? 1u : 0u;
          if (C::DT)   // dS over the S columns, two bf16 per column
            tc::mma_bf16_ts(tmem + C::DQ_COL, tmem + k * 8, bd, idesc_q, acc);
          else
            tc::mma_bf16(tmem + C::DQ_COL, tc::smem_desc(dst + k * 32, 16, 1024), bd, idesc_q, acc);
        }
        tc::mma_commit(&k_empty[s]);
        tc::mma_commit(&dq_done[b]);
        return true;
      };
      bool ok = tc::mbar_wait(q_full, 0, status, abort_flag, 46);
      if (ok && C::DT) ok = tc::mbar_wait(do_ready, 0, status, abort_flag, 60);
      if (ok) tc::fence_after();
      if (C::DT) {
        // single score buffer: dP_{j+1} (its columns are free once the softmax released dS_j) runs
        // while dQ_j does; S_{j+1} waits until dQ_j has read dS_j out of the S columns
        if (ok) ok = issue_dp(0);
        if (ok) ok = issue_s(0);
        for (int j = 0; j < nt && ok; ++j) {
          ok = issue_dq(j);
          if (ok && j + 1 < nt) ok = issue_dp(j + 1);
          if (ok && j + 1 < nt) ok = tc::mbar_wait(&dq_done[0], j & 1, status, abort_flag, 61);
          if (ok && j + 1 < nt) ok = issue_s(j + 1);
        }
      } else {
        for (int j = 0; j < nt && ok; ++j) {
          // S_j and dP_j run while the softmax threads turn S_{j-1} into dS_{j-1}
          ok = issue_dp(j);
          if (ok) ok = issue_s(j);
          if (ok && j > 0) ok = issue_dq(j - 1);
        }
        if (ok) issue_dq(nt - 1);
      }
      tc::mma_commit(drain);
      const unsigned long long t0 = tc::globaltimer();
      while (!tc::mbar_try_wait(drain, 0) && tc::globaltimer() - t0 < tc::kWaitNs) {
      }
    }
  } else {
    const int quarter = warp & 3;
    const int rl = quarter * 32 + lane, row = r0 + rl;
    const bool valid = row < a.rows;
    const float2 info = a.lsd[(size_t)h * a.rows_pad + min(row, a.rows_pad - 1)];
    const int2 rng = valid ? a.kse[row] : make_int2(0, 0);
    const float lse2 = valid ? info.x : INFINITY, dsum = info.y;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    const float sl2 = a.scale * LOG2E_TC;
    auto wwait = [&](uint64_t* bar, uint32_t parity, int code) {
      return __all_sync(0xffffffffu, tc::mbar_wait(bar, parity, status, abort_flag, code));
    };
    bool ok = true;
    if (C::DT && nt > 0) {
      // dO row of this thread -> TMEM columns DO_COL.. (two bf16 per column)
      const __nv_bfloat16* drow_src = a.dosrc + ((size_t)(valid ? row : 0) * a.Hq + h) * D;
#pragma unroll 1
      for (int c = 0; c < D / 2; c += 32) {
        float w[32];
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const uint4 u = valid ? *reinterpret_cast<const uint4*>(drow_src + 2 * (c + j)) : make_uint4(0, 0, 0, 0);
          w[j] = __uint_as_float(u.x);
          w[j + 1] = __uint_as_float(u.y);
          w[j + 2] = __uint_as_float(u.z);
          w[j + 3] = __uint_as_float(u.w);
        }
        tc::tmem_st32(lane_base + C::DO_COL + c, w);
      }
      tc::fence_before();
      tc::mbar_arrive(do_ready);
    }
    for (int j = 0; j < nt && ok; ++j) {
      const int b = C::DT ? 0 : (j & 1);
      if (!wwait(&s_full[b], (C::DT ? j : j >> 1) & 1, 47)) { ok = false; break; }
      tc::fence_after();
      const int n0 = kt0 + j * BN;
      if (C::DT) {
        // dS back into the first BN / 2 columns of the score buffer (halves read before writing)
        float dw[BN / 2];
#pragma unroll
        for (int c = 0; c < BN; c += 32) {
          float sv[32], pv[32];
          tc::tmem_ld32(lane_base + c, sv);
          tc::tmem_ld32(lane_base + C::DP_COL + c, pv);
#pragma unroll
          for (int i2 = 0; i2 < 16; ++i2) {
            float d2[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int i = 2 * i2 + u, key = n0 + c + i;
              const float p = (key >= rng.x && key < rng.y) ? exp2f(sv[i] * sl2 - lse2) : 0.f;
              d2[u] = p * (pv[i] - dsum);
            }
            __nv_bfloat162 v2 = __floats2bfloat162_rn(d2[0], d2[1]);
            dw[c / 2 + i2] = __uint_as_float(*reinterpret_cast<uint32_t*>(&v2));
          }
        }
        tc::tmem_st32(lane_base, dw);
        tc::fence_before();
        tc::mbar_arrive(&ds_full[0]);
        continue;
      }
      if (j >= 2 && !wwait(&dq_done[b], ((j >> 1) + 1) & 1, 48)) { ok = false; break; }
      uint8_t* drow = sds + b * C::DS_BYTES + rl * 128;
#pragma unroll
      for (int c = 0; c < BN; c += 32) {
        float sv[32], pv[32];
        tc::tmem_ld32(lane_base + b * BN + c, sv);
        tc::tmem_ld32(lane_base + C::DP_COL + b * BN + c, pv);
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float d2[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int i = c8 * 8 + 2 * e + u, key = n0 + c + i;
              const float p = (key >= rng.x && key < rng.y) ? exp2f(sv[i] * sl2 - lse2) : 0.f;
              d2[u] = p * (pv[i] - dsum);
            }
            __nv_bfloat162 v2 = __floats2bfloat162_rn(d2[0], d2[1]);
            w[e] = *reinterpret_cast<uint32_t*>(&v2);
          }
          const int chunk = ((c >> 3) + c8) ^ (rl & 7);
          *reinterpret_cast<uint4*>(drow + chunk * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      tc::fence_proxy_async();
      tc::fence_before();
      tc::mbar_arrive(&ds_full[b]);
    }
    if (ok && nt > 0 && !wwait(&dq_done[C::DT ? 0 : (nt - 1) & 1], (C::DT ? nt - 1 : (nt - 1) >> 1) & 1, 49))
      ok = false;
    if (ok) {
      tc::fence_after();
      __nv_bfloat16* dst = a.dq + ((size_t)row * a.Hq + h) * D;
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        float v[32];
        if (nt > 0) {
          tc::tmem_ld32(lane_base + C::DQ_COL + c, v);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0.f;
        }
        if (valid) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              __nv_bfloat162 v2 = __floats2bfloat162_rn(v[i + 2 * e] * a.scale, v[i + 2 * e + 1] * a.scale);
              w[e] = *reinterpret_cast<uint32_t*>(&v2);
            }
            *reinterpret_cast<uint4*>(dst + c + i) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

// dK / dV: one CTA per (128-key block, kv head, value-dim slice of DS). K and V stay in shared
// memory; for every (q head of the group, 64-row block) whose key ranges meet the block, Q and dO
// tiles (+ the rows' exponent references, Dsum and ranges) stream in by TMA. S^T = K Q^T and
// dP^T = V dO^T land in double-buffered TMEM; each softmax thread (one key) forms P^T and
// dS^T = P^T (dP^T - Dsum) into shared memory (bf16, 128B-swizzled K-major), and dV += P^T dO,
// dK += dS^T Q accumulate in TMEM over the value-dim slice (dO and Q tiles are the MN-major B
// operands). At D = 256 the slice is half the head (two CTAs per key block recompute S^T and
// dP^T), and V lives in TMEM as the A operand of dP^T = V dO^T (lane = key, two bf16 per column)
// while P^T and dS^T are written back over the S^T / dP^T columns with tcgen05.st and read by the
// dV / dK MMAs as TMEM A operands: shared memory then holds K and two Q / dO stages, so the next
// pair's tiles stream in while the current pair computes. The score columns are single-buffered
// there, so the MMA thread waits for the previous pair's dV / dK MMAs before overwriting them.
template <int D>
struct DkvTc {
  static constexpr bool VT = D > 128;                  // V, P^T, dS^T in TMEM (D = 256)
  static constexpr int BN = 128, BQ = 64, KB = D / 64;
  static constexpr int DS = D > 128 ? 128 : D;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int QT_BYTES = BQ * D * 2;
  static constexpr int INFO_BYTES = BQ * 16;           // float2 lsd + int2 kse per row
  static constexpr int STAGE_BYTES = 2 * QT_BYTES + INFO_BYTES;
  static constexpr int PT_BYTES = BN * BQ * 2;
  static constexpr int STAGES = 2;
  static constexpr int PBUF = VT ? 0 : 2;              // shared-memory P^T / dS^T buffers
  static constexpr int NSB = VT ? 1 : 2;               // TMEM score buffers
  static constexpr int SMEM = (VT ? 1 : 2) * KV_BYTES + STAGES * STAGE_BYTES + 2 * PBUF * PT_BYTES + 1024 + 256;
  static constexpr uint32_t DP_COL = NSB * BQ, DV_COL = 2 * NSB * BQ, DK_COL = 2 * NSB * BQ + DS;
  static constexpr uint32_t VT_COL = DK_COL + DS;      // V (VT only): D / 2 columns
  static_assert(!VT || VT_COL + D / 2 <= 512, "TMEM columns");
};

template <int D>
__global__ void __launch_bounds__(192, 1)
    attn_dkv_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_do,
                       const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_v,
                       BwdTcArgs a, int* status) {
  using C = DkvTc<D>;
  constexpr int BN = C::BN, BQ = C::BQ, KB = C::KB, DS = C::DS, ST = C::STAGES;
  constexpr int PB = C::PBUF ? C::PBUF : 1;   // shared-memory P^T buffers (unused when VT)
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sk = smem;
  uint8_t* sv = sk + C::KV_BYTES;                     // (not VT)
  uint8_t* stages = sv + (C::VT ? 0 : C::KV_BYTES);   // [ST][Q | dO | info]
  uint8_t* spt = stages + ST * C::STAGE_BYTES;        // [PB][P^T | dS^T] (not VT)
  uint64_t* bars = reinterpret_cast<uint64_t*>(spt + 2 * C::PBUF * C::PT_BYTES);
  uint64_t* kv_full = bars;
  uint64_t* qd_full = bars + 1;   // [2]
  uint64_t* qd_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* p_full = bars + 7;    // [2]
  uint64_t* pv_done = bars + 9;   // [2]
  uint64_t* drain = bars + 11;
  uint64_t* v_ready = bars + 12;  // VT: V stored into TMEM by the 128 softmax threads
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* s_count = reinterpret_cast<int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int NZ = D / DS;
  const int slot = blockIdx.x / (a.Hkv * NZ), kb = a.order_keys ? a.order_keys[slot] : slot;
  const int hk = (blockIdx.x / NZ) % a.Hkv, z = blockIdx.x % NZ;
  const int n0 = kb * BN, d0 = z * DS;
  const int group = a.Hq / a.Hkv, nqb = a.rows_pad / BQ;
  auto meets = [&](int qb) {
    const int lo = a.qb_min[qb], hi = a.qb_max[qb];
    return lo < hi && lo < n0 + BN && hi > n0;
  };
  if (threadIdx.x == 0) {
    tc::mbar_init(kv_full, 1);
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&qd_full[b], 1);
      tc::mbar_init(&qd_empty[b], 1);
      tc::mbar_init(&s_full[b], 1);
      tc::mbar_init(&p_full[b], 128);
      tc::mbar_init(&pv_done[b], 1);
    }
    tc::mbar_init(drain, 1);
    tc::mbar_init(v_ready, 128);
    *abort_flag = 0;
    *s_count = 0;
    tc::fence_mbar_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, 512);
  __syncthreads();
  {
    int c = 0;
    for (int qb = threadIdx.x; qb < nqb; qb += blockDim.x) c += meets(qb) ? 1 : 0;
    c = __reduce_add_sync(0xffffffffu, c);
    if (lane == 0 && c) atomicAdd(s_count, c);
  }
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;
  const int np = *s_count * group;   // (head, row block) pairs, heads outermost

  if (warp == 0) {
    if (lane == 0 && np > 0) {
      tc::prefetch_map(&map_q);
      tc::prefetch_map(&map_do);
      tc::prefetch_map(&map_k);
      tc::prefetch_map(&map_v);
      int armed[2] = {-1, -1};
      tc::mbar_expect_tx(kv_full, (C::VT ? 1 : 2) * C::KV_BYTES);
#pragma unroll
      for (int i = 0; i < KB; ++i) {
        tc::tma_load_2d(sk + i * BN * 128, &map_k, kv_full, hk * D + i * 64, n0);
        if (!C::VT) tc::tma_load_2d(sv + i * BN * 128, &map_v, kv_full, hk * D + i * 64, n0);
      }
      int i = 0;
      for (int hh = 0; hh < group && i < np; ++hh) {
        const int h = hk * group + hh;
        bool ok = true;
        for (int qb = 0; qb < nqb && ok; ++qb) {
          if (!meets(qb)) continue;
          const int s = i % ST;
          const uint32_t ph = (i / ST) & 1;
          if (!tc::mbar_wait(&qd_empty[s], ph ^ 1, status, abort_flag, 51)) { ok = false; break; }
          uint8_t* st = stages + s * C::STAGE_BYTES;
          tc::mbar_expect_tx(&qd_full[s], C::STAGE_BYTES);
#pragma unroll
          for (int c = 0; c < KB; ++c) {
            tc::tma_load_2d(st + c * BQ * 128, &map_q, &qd_full[s], h * D + c * 64, qb * BQ);
            tc::tma_load_2d(st + C::QT_BYTES + c * BQ * 128, &map_do, &qd_full[s], h * D + c * 64, qb * BQ);
          }
          tc::bulk_load(st + 2 * C::QT_BYTES, a.lsd + (size_t)h * a.rows_pad + qb * BQ, BQ * 8, &qd_full[s]);
          tc::bulk_load(st + 2 * C::QT_BYTES + BQ * 8, a.kse + qb * BQ, BQ * 8, &qd_full[s]);
          armed[s] = (int)ph;
          ++i;
        }
        if (!ok) break;
      }
      const unsigned long long t0 = tc::globaltimer();
      while (!tc::mbar_try_wait(kv_full, 0) && tc::globaltimer() - t0 < tc::kWaitNs) {
      }
      for (int s = 0; s < 2; ++s)
        if (armed[s] >= 0)
          while (!tc::mbar_try_wait(&qd_full[s], (uint32_t)armed[s]) && tc::globaltimer() - t0 < tc::kWaitNs) {
          }
    }
  } else if (warp == 1) {
    if (lane == 0 && np > 0) {
      constexpr uint32_t idesc_s = tc::idesc_bf16(BN, BQ, false, false);
      constexpr uint32_t idesc_g = tc::idesc_bf16(BN, DS, false, true);
      const uint32_t k_addr = tc::smem_u32(sk), v_addr = tc::smem_u32(sv), st_addr = tc::smem_u32(stages),
                     pt_addr = tc::smem_u32(spt);
      auto issue_scores = [&](int i) -> bool {
        const int s = i % ST, b = C::VT ? 0 : (i & 1);
        if (C::VT && i > 0) {
          // single score buffer: the previous pair's dV / dK MMAs read P^T / dS^T from it
          if (!tc::mbar_wait(&pv_done[0], (i - 1) & 1, status, abort_flag, 58)) return false;
        }
        if (!tc::mbar_wait(&qd_full[s], (i / ST) & 1, status, abort_flag, 52)) return false;
        tc::fence_after();
        const uint32_t qt = st_addr + s * C::STAGE_BYTES, dt = qt + C::QT_BYTES;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (k >> 2) * (BN * 128) + (k & 3) * 32, toff = (k >> 2) * (BQ * 128) + (k & 3) * 32;
          tc::mma_bf16(tmem + b * BQ, tc::smem_desc(k_addr + off, 16, 1024), tc::smem_desc(qt + toff, 16, 1024),
                       idesc_s, k > 0 ? 1u : 0u);
          if (C::VT)
            tc::mma_bf16_ts(tmem + C::DP_COL, tmem + C::VT_COL + k * 8, tc::smem_desc(dt + toff, 16, 1024), idesc_s,
                            k > 0 ? 1u : 0u);
          else
            tc::mma_bf16(tmem + C::DP_COL + b * BQ, tc::smem_desc(v_addr + off, 16, 1024),
                         tc::smem_desc(dt + toff, 16, 1024), idesc_s, k > 0 ? 1u : 0u);
        }
        tc::mma_commit(&s_full[b]);
        return true;
      };
      auto issue_grads = [&](int i) -> bool {
        const int s = i % ST, pb = C::VT ? 0 : i % PB;
        if (!tc::mbar_wait(&p_full[pb], (C::VT ? i : i / PB) & 1, status, abort_flag, 53)) return false;
        tc::fence_after();
        const uint32_t qt = st_addr + s * C::STAGE_BYTES + (d0 / 64) * (BQ * 128), dt = qt + C::QT_BYTES;
        const uint32_t pt = pt_addr + pb * 2 * C::PT_BYTES, dst = pt + C::PT_BYTES;
#pragma unroll
        for (int k = 0; k < BQ / 16; ++k) {
          const uint64_t bo = tc::smem_desc(dt + k * 2048, BQ * 128, 1024), bq = tc::smem_desc(qt + k * 2048, BQ * 128, 1024);
          const uint32_t acc = (i > 0 || k > 0) ? 1u : 0u;
          if (C::VT) {   // P^T / dS^T over the score columns, two bf16 per column
            tc::mma_bf16_ts(tmem + C::DV_COL, tmem + k * 8, bo, idesc_g, acc);
            tc::mma_bf16_ts(tmem + C::DK_COL, tmem + C::DP_COL + k * 8, bq, idesc_g, acc);
          } else {
            tc::mma_bf16(tmem + C::DV_COL, tc::smem_desc(pt + k * 32, 16, 1024), bo, idesc_g, acc);
            tc::mma_bf16(tmem + C::DK_COL, tc::smem_desc(dst + k * 32, 16, 1024), bq, idesc_g, acc);
          }
        }
        tc::mma_commit(&qd_empty[s]);
        tc::mma_commit(&pv_done[pb]);
        return true;
      };
      bool ok = tc::mbar_wait(kv_full, 0, status, abort_flag, 54);
      if (ok && C::VT) ok = tc::mbar_wait(v_ready, 0, status, abort_flag, 59);
      if (ok) tc::fence_after();
      for (int i = 0; i < np && ok; ++i) {
        ok = issue_scores(i);
        if (ok && C::VT) ok = issue_grads(i);            // the next scores need these columns back
        else if (ok && i > 0) ok = issue_grads(i - 1);   // S^T_i / dP^T_i overlap softmax_{i-1}
      }
      if (ok && !C::VT) issue_grads(np - 1);
      tc::mma_commit(drain);
      const unsigned long long t0 = tc::globaltimer();
      while (!tc::mbar_try_wait(drain, 0) && tc::globaltimer() - t0 < tc::kWaitNs) {
      }
    }
  } else {
    // one key per thread
    const int quarter = warp & 3;
    const int kl = quarter * 32 + lane, key = n0 + kl;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    const float sl2 = a.scale * LOG2E_TC;
    auto wwait = [&](uint64_t* bar, uint32_t parity, int code) {
      return __all_sync(0xffffffffu, tc::mbar_wait(bar, parity, status, abort_flag, code));
    };
    bool ok = true;
    if (C::VT && np > 0) {
      // V row of this thread's key -> TMEM columns VT_COL.. (two bf16 per column)
      const bool kv = key < a.keys;
      const __nv_bfloat16* vrow = a.vsrc + ((size_t)(kv ? key : 0) * a.Hkv + hk) * D;
#pragma unroll 1
      for (int c = 0; c < D / 2; c += 32) {
        float w[32];
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const uint4 u = kv ? *reinterpret_cast<const uint4*>(vrow + 2 * (c + j)) : make_uint4(0, 0, 0, 0);
          w[j] = __uint_as_float(u.x);
          w[j + 1] = __uint_as_float(u.y);
          w[j + 2] = __uint_as_float(u.z);
          w[j + 3] = __uint_as_float(u.w);
        }
        tc::tmem_st32(lane_base + C::VT_COL + c, w);
      }
      tc::fence_before();
      tc::mbar_arrive(v_ready);
    }
    for (int i = 0; i < np && ok; ++i) {
      const int b = C::VT ? 0 : (i & 1), s = i % ST, pb = C::VT ? 0 : i % PB;
      if (!wwait(&s_full[b], (C::VT ? i : i >> 1) & 1, 55)) { ok = false; break; }
      tc::fence_after();
      if (!C::VT && i >= PB && !wwait(&pv_done[pb], ((i - PB) / PB) & 1, 56)) { ok = false; break; }
      const uint8_t* info = stages + s * C::STAGE_BYTES + 2 * C::QT_BYTES;
      const float2* lsd = reinterpret_cast<const float2*>(info);
      const int2* kse = reinterpret_cast<const int2*>(info + BQ * 8);
      if (C::VT) {
        // P^T and dS^T back into the first BQ / 2 columns of the score buffers; the 32-column
        // halves of S^T / dP^T are read before anything is stored over them
        float pw[BQ / 2], dw[BQ / 2];
#pragma unroll
        for (int c = 0; c < BQ; c += 32) {
          float sv[32], dv[32];
          tc::tmem_ld32(lane_base + c, sv);
          tc::tmem_ld32(lane_base + C::DP_COL + c, dv);
#pragma unroll
          for (int r2 = 0; r2 < 16; ++r2) {
            float p2[2], d2[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int j = 2 * r2 + u, r = c + j;
              const float2 ld = lsd[r];
              const int2 rg = kse[r];
              const float p = (key >= rg.x && key < rg.y) ? exp2f(sv[j] * sl2 - ld.x) : 0.f;
              p2[u] = p;
              d2[u] = p * (dv[j] - ld.y);
            }
            __nv_bfloat162 a2 = __floats2bfloat162_rn(p2[0], p2[1]);
            __nv_bfloat162 b2 = __floats2bfloat162_rn(d2[0], d2[1]);
            pw[c / 2 + r2] = __uint_as_float(*reinterpret_cast<uint32_t*>(&a2));
            dw[c / 2 + r2] = __uint_as_float(*reinterpret_cast<uint32_t*>(&b2));
          }
        }
        tc::tmem_st32(lane_base, pw);
        tc::tmem_st32(lane_base + C::DP_COL, dw);
        tc::fence_before();
        tc::mbar_arrive(&p_full[0]);
        continue;
      }
      uint8_t* prow = spt + pb * 2 * C::PT_BYTES + kl * 128;
      uint8_t* drow = prow + C::PT_BYTES;
#pragma unroll
      for (int c = 0; c < BQ; c += 32) {
        float sv[32], dv[32];
        tc::tmem_ld32(lane_base + b * BQ + c, sv);
        tc::tmem_ld32(lane_base + C::DP_COL + b * BQ + c, dv);
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          uint32_t wp[4], wd[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float p2[2], d2[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int r = c + c8 * 8 + 2 * e + u, i2 = c8 * 8 + 2 * e + u;
              const float2 ld = lsd[r];
              const int2 rg = kse[r];
              const float p = (key >= rg.x && key < rg.y) ? exp2f(sv[i2] * sl2 - ld.x) : 0.f;
              p2[u] = p;
              d2[u] = p * (dv[i2] - ld.y);
            }
            __nv_bfloat162 a2 = __floats2bfloat162_rn(p2[0], p2[1]);
            __nv_bfloat162 b2 = __floats2bfloat162_rn(d2[0], d2[1]);
            wp[e] = *reinterpret_cast<uint32_t*>(&a2);
            wd[e] = *reinterpret_cast<uint32_t*>(&b2);
          }
          const int chunk = ((c >> 3) + c8) ^ (kl & 7);
          *reinterpret_cast<uint4*>(prow + chunk * 16) = make_uint4(wp[0], wp[1], wp[2], wp[3]);
          *reinterpret_cast<uint4*>(drow + chunk * 16) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
        }
      }
      tc::fence_proxy_async();
      tc::fence_before();
      tc::mbar_arrive(&p_full[pb]);
    }
    if (ok && np > 0 && !wwait(&pv_done[C::VT ? 0 : (np - 1) % PB], (C::VT ? np - 1 : (np - 1) / PB) & 1, 57))
      ok = false;
    if (ok) {
      tc::fence_after();
      const bool valid = key < a.keys;
      __nv_bfloat16* dkd = a.dk + ((size_t)key * a.Hkv + hk) * D + d0;
      __nv_bfloat16* dvd = a.dv + ((size_t)key * a.Hkv + hk) * D + d0;
#pragma unroll 1
      for (int c = 0; c < DS; c += 32) {
        float gk[32], gv[32];
        if (np > 0) {
          tc::tmem_ld32(lane_base + C::DK_COL + c, gk);
          tc::tmem_ld32(lane_base + C::DV_COL + c, gv);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) gk[i] = gv[i] = 0.f;
        }
        if (valid) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint32_t wk[4], wv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              __nv_bfloat162 k2 = __floats2bfloat162_rn(gk[i + 2 * e] * a.scale, gk[i + 2 * e + 1] * a.scale);
              __nv_bfloat162 v2 = __floats2bfloat162_rn(gv[i + 2 * e], gv[i + 2 * e + 1]);
              wk[e] = *reinterpret_cast<uint32_t*>(&k2);
              wv[e] = *reinterpret_cast<uint32_t*>(&v2);
            }
            *reinterpret_cast<uint4*>(dkd + c + i) = make_uint4(wk[0], wk[1], wk[2], wk[3]);
            *reinterpret_cast<uint4*>(dvd + c + i) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
          }
        }
      }
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

}  // namespace

// q [rows, Hq, D], k/v [keys, Hkv, D] bf16 contiguous, kstart/kend int32 [rows]; D in {64, 128,
// 256}. Returns {O [rows, Hq, D] bf16, LSE [Hq, rows] fp32}.
std::vector<at::Tensor> attn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor kstart, at::Tensor kend,
                                    double scale) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && q.is_contiguous() && q.dim() == 3, "q: [rows,Hq,D] bf16");
  TORCH_CHECK(k.is_contiguous() && v.is_contiguous() && k.scalar_type() == at::kBFloat16 &&
                  v.scalar_type() == at::kBFloat16 && k.dim() == 3 && v.sizes() == k.sizes(),
              "k/v: contiguous bf16 [keys, Hkv, D]");
  TORCH_CHECK(kstart.scalar_type() == at::kInt && kend.scalar_type() == at::kInt && kstart.numel() == q.size(0) &&
                  kend.numel() == q.size(0) && kstart.is_contiguous() && kend.is_contiguous(),
              "kstart/kend: int32 [rows]");
  const int rows = q.size(0), Hq = q.size(1), D = q.size(2), keys = k.size(0), Hkv = k.size(1);
  TORCH_CHECK(k.size(2) == D && Hq % Hkv == 0, "head dims / GQA ratio");
  auto o = at::empty_like(q);
  auto lse = at::empty({Hq, rows}, q.options().dtype(at::kFloat));
  if (rows == 0) return {o, lse};
  const int nqb = (rows + 127) / 128;
  const bool schedule = (long)nqb * Hq > sm_count();
  auto order = at::empty({schedule ? nqb : 0}, q.options().dtype(at::kInt));
  FwdTcArgs a{kstart.data_ptr<int>(), kend.data_ptr<int>(), schedule ? order.data_ptr<int>() : nullptr,
              (__nv_bfloat16*)o.data_ptr(), lse.data_ptr<float>(), rows, keys, Hq, Hkv, (float)scale};
  auto launch = [&](auto dtag) {
    constexpr int DD = decltype(dtag)::value;
    using C = FwdTc<DD>;
    auto mq = tma_map_bf16(q.view({rows, Hq * DD}), C::BM);
    auto mk = tma_map_bf16(k.view({keys, Hkv * DD}), C::BN);
    auto mv = tma_map_bf16(v.view({keys, Hkv * DD}), C::BN);
    static bool once = [] {
      CQB_CHECK_CUDA(cudaFuncSetAttribute(attn_fwd_tc_kernel<DD>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
      return true;
    }();
    (void)once;
    if (schedule) {
      attn_schedule_kernel<<<1, 1024, 0, stream()>>>(kstart.data_ptr<int>(), kend.data_ptr<int>(), rows, C::BN,
                                                     order.data_ptr<int>(), nullptr, nullptr, 0, 0, nullptr);
      CQB_LAUNCH_CHECK();
      count_launch();
    }
    attn_fwd_tc_kernel<DD><<<nqb * Hq, 192, C::SMEM, stream()>>>(mq, mk, mv, a, attn_status_word());
  };
  if (D == 64) launch(std::integral_constant<int, 64>{});
  else if (D == 128) launch(std::integral_constant<int, 128>{});
  else if (D == 256) launch(std::integral_constant<int, 256>{});
  else TORCH_CHECK(false, "attn_fwd: head dim must be 64, 128 or 256");
  CQB_LAUNCH_CHECK();
  count_launch();
  return {o, lse};
}

// Gradients of attn_fwd from dO, the inputs and the forward's O and LSE: returns {dq, dk, dv}. Deterministic (no atomics): a dQ kernel over row blocks and a dK/dV kernel over
// key blocks, both on tcgen05.
std::vector<at::Tensor> attn_bwd(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o,
                                    at::Tensor lse, at::Tensor kstart, at::Tensor kend, double scale) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && q.is_contiguous() && q.dim() == 3, "q: [rows,Hq,D] bf16");
  TORCH_CHECK(k.is_contiguous() && v.is_contiguous() && k.scalar_type() == at::kBFloat16 &&
                  v.scalar_type() == at::kBFloat16 && k.dim() == 3 && v.sizes() == k.sizes(),
              "k/v: contiguous bf16 [keys, Hkv, D]");
  TORCH_CHECK(o.sizes() == q.sizes() && dout.sizes() == q.sizes() && o.is_contiguous() && dout.is_contiguous() &&
                  o.scalar_type() == at::kBFloat16 && dout.scalar_type() == at::kBFloat16,
              "o / dout: contiguous bf16 like q");
  TORCH_CHECK(kstart.scalar_type() == at::kInt && kend.scalar_type() == at::kInt && kstart.numel() == q.size(0) &&
                  kend.numel() == q.size(0) && kstart.is_contiguous() && kend.is_contiguous(),
              "kstart/kend: int32 [rows]");
  const int rows = q.size(0), Hq = q.size(1), D = q.size(2), keys = k.size(0), Hkv = k.size(1);
  TORCH_CHECK(k.size(2) == D && Hq % Hkv == 0, "head dims / GQA ratio");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.is_contiguous() && lse.numel() == (int64_t)Hq * rows,
              "lse: fp32 [Hq, rows]");
  auto dq = at::empty_like(q);
  auto dk = at::empty_like(k);
  auto dv = at::empty_like(v);
  if (rows == 0 || keys == 0) return {dq.zero_(), dk.zero_(), dv.zero_()};
  const int rows_pad = (rows + 63) / 64 * 64;
  auto lsd = at::empty({Hq, rows_pad, 2}, q.options().dtype(at::kFloat));
  auto kse = at::empty({rows_pad, 2}, q.options().dtype(at::kInt));
  auto qb_min = at::empty({rows_pad / 64}, q.options().dtype(at::kInt));
  auto qb_max = at::empty({rows_pad / 64}, q.options().dtype(at::kInt));
  {
    const long warps = (long)rows_pad * Hq;
    const int blocks = (int)std::max<long>((warps * 32 + 255) / 256, (rows_pad / 64 + 255) / 256);
    attn_bwd_prep_tc_kernel<<<blocks, 256, 0, stream()>>>(
        (const __nv_bfloat16*)o.data_ptr(), (const __nv_bfloat16*)dout.data_ptr(), lse.data_ptr<float>(),
        kstart.data_ptr<int>(), kend.data_ptr<int>(), reinterpret_cast<float2*>(lsd.data_ptr<float>()),
        reinterpret_cast<int2*>(kse.data_ptr<int>()), qb_min.data_ptr<int>(), qb_max.data_ptr<int>(), rows, rows_pad,
        Hq, D);
    CQB_LAUNCH_CHECK();
  }
  const int nqb128 = (rows + 127) / 128, nkb = (keys + 127) / 128;
  // longest-first orders pay off once the two kernels' CTAs exceed one wave
  const bool schedule = (long)nqb128 * Hq + (long)nkb * Hkv * (D > 128 ? 2 : 1) > sm_count();
  auto orders = at::empty({schedule ? nqb128 + nkb : 0}, q.options().dtype(at::kInt));
  BwdTcArgs a{schedule ? orders.data_ptr<int>() : nullptr, schedule ? orders.data_ptr<int>() + nqb128 : nullptr,
              reinterpret_cast<const float2*>(lsd.data_ptr<float>()), reinterpret_cast<const int2*>(kse.data_ptr<int>()),
              qb_min.data_ptr<int>(), qb_max.data_ptr<int>(), (const __nv_bfloat16*)v.data_ptr(),
              (const __nv_bfloat16*)dout.data_ptr(), (__nv_bfloat16*)dq.data_ptr(),
              (__nv_bfloat16*)dk.data_ptr(), (__nv_bfloat16*)dv.data_ptr(), rows, rows_pad, keys, Hq, Hkv,
              (float)scale};
  auto launch = [&](auto dtag) {
    constexpr int DD = decltype(dtag)::value;
    using Q = DqTc<DD>;
    using K = DkvTc<DD>;
    auto q2 = q.view({rows, Hq * DD}), do2 = dout.view({rows, Hq * DD});
    auto k2 = k.view({keys, Hkv * DD}), v2 = v.view({keys, Hkv * DD});
    static bool once = [] {
      CQB_CHECK_CUDA(cudaFuncSetAttribute(attn_dq_tc_kernel<DD>, cudaFuncAttributeMaxDynamicSharedMemorySize, Q::SMEM));
      CQB_CHECK_CUDA(cudaFuncSetAttribute(attn_dkv_tc_kernel<DD>, cudaFuncAttributeMaxDynamicSharedMemorySize, K::SMEM));
      return true;
    }();
    (void)once;
    if (schedule) {
      attn_schedule_kernel<<<2, 1024, 0, stream()>>>(kstart.data_ptr<int>(), kend.data_ptr<int>(), rows, Q::BN,
                                                     orders.data_ptr<int>(), qb_min.data_ptr<int>(),
                                                     qb_max.data_ptr<int>(), rows_pad / 64, keys,
                                                     orders.data_ptr<int>() + nqb128);
      CQB_LAUNCH_CHECK();
      count_launch();
    }
    // dK/dV (fewer, longer CTAs) first on this stream; dQ on a side stream fills the SMs its tail
    // leaves idle (one CTA per SM each: their shared memory does not fit twice).
    cudaStream_t main = stream();
    at::cuda::CUDAStream side = at::cuda::getStreamFromPool(false, q.get_device());
    cudaEvent_t ready, done;
    CQB_CHECK_CUDA(cudaEventCreateWithFlags(&ready, cudaEventDisableTiming));
    CQB_CHECK_CUDA(cudaEventCreateWithFlags(&done, cudaEventDisableTiming));
    CQB_CHECK_CUDA(cudaEventRecord(ready, main));
    attn_dkv_tc_kernel<DD><<<nkb * Hkv * (DD / K::DS), 192, K::SMEM, main>>>(
        tma_map_bf16(q2, K::BQ), tma_map_bf16(do2, K::BQ), tma_map_bf16(k2, K::BN), tma_map_bf16(v2, K::BN), a,
        attn_status_word());
    CQB_LAUNCH_CHECK();
    CQB_CHECK_CUDA(cudaStreamWaitEvent(side.stream(), ready, 0));
    attn_dq_tc_kernel<DD><<<nqb128 * Hq, 192, Q::SMEM, side.stream()>>>(
        tma_map_bf16(q2, Q::BM), tma_map_bf16(do2, Q::BM), tma_map_bf16(k2, Q::BN), tma_map_bf16(v2, Q::BN), a,
        attn_status_word());
    CQB_LAUNCH_CHECK();
    CQB_CHECK_CUDA(cudaEventRecord(done, side.stream()));
    CQB_CHECK_CUDA(cudaStreamWaitEvent(main, done, 0));
    CQB_CHECK_CUDA(cudaEventDestroy(ready));
    CQB_CHECK_CUDA(cudaEventDestroy(done));
  };
  if (D == 64) launch(std::integral_constant<int, 64>{});
  else if (D == 128) launch(std::integral_constant<int, 128>{});
  else if (D == 256) launch(std::integral_constant<int, 256>{});
  else TORCH_CHECK(false, "attn_bwd: head dim must be 64, 128 or 256");
  count_launch(3);
  return {dq, dk, dv};
}

int attn_status(bool reset) {
  int v = 0;
  CQB_CHECK_CUDA(cudaMemcpy(&v, attn_status_word(), sizeof(int), cudaMemcpyDeviceToHost));
  if (reset && v) CQB_CHECK_CUDA(cudaMemset(attn_status_word(), 0, sizeof(int)));
  return v;
}

}  // namespace cqb
