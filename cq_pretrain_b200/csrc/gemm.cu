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
//  * epilogues: 0 = bf16 TMA store (+ bias); 1 = fp32 TMA reduce-add into an existing fp32
//    matrix (the main_grad accumulation of weight gradients); 2 = bf16 stores of each tile
//    straight into the receive buffer of the TP rank that owns its rows, over NVLink peer
//    memory (the communication half of GEMM -> reduce-scatter, overlapped tile by tile);
//    3 = cross-entropy statistics: nothing is stored; each thread (one output row) folds the
//    tile's 256 logits into an online (max, sum exp) pair and picks out its target logit, and
//    writes one partial per (row, column tile) (the LM-head forward never writes logits);
//    4 = cross-entropy gradient: (exp(logit - lse) - [col == target]) * dloss as bf16 TMA stores;
//    5 = GEMM -> reduce-scatter in one kernel: tiles of rows owned by another TP rank are
//    stored (bf16) into that rank's receive slab and published with a per-(tile, source, warp)
//    epoch stamp; tiles of this rank's own rows come last in the tile order, and their epilogue
//    waits for the peers' stamps, then adds the peers' partials to its own fp32 accumulator
//    (still in TMEM) and the bias, and TMA-stores the reduced rows;
//  * a second operand pair (A2, B2, contraction K2) may follow the first in the k loop, so
//    D = A B^T + A2 B2^T runs as one accumulation (e.g. dX = dY1 W1 + dY2 W2 of two projections
//    of one gathered input); rows of A2 past its own extent read as zero;
//  * GATHER: two extra warps pull the A row blocks of every TP rank (peer memory, plain loads)
//    into this GPU's gather buffer and publish a flag per 16-row sub-chunk; the TMA producer waits
//    for a block's flags before loading it, and tiles of this rank's own rows go first, read by
//    TMA straight from the caller's shard while the copy warps publish it to the peers and pull
//    theirs (all-gather -> GEMM in one kernel; each remote byte crosses NVLink once).
//
// Waits are bounded (tcgen05.cuh); on expiry the kernel records an error code, stops issuing,
// waits for its outstanding TMA transactions (bounded), frees TMEM and exits.
#include "common.cuh"
#include "tcgen05.cuh"

#include <cstdlib>
#include <mutex>

namespace cqb {

namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int GATHER_SUB = 16;   // rows per all-gather copy unit (and per publication flag)
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_BOX = 32;                                   // 32 x 32 output box per warp store
constexpr int STAGING_BYTES = 4 /*warps*/ * 2 /*buffers*/ * EPI_BOX * EPI_BOX * 4;  // sized for fp32
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + STAGING_BYTES + 1024 /*align*/ + 256 /*barriers*/;
constexpr int RS_MAX_TP = 8;    // flag slots per tile: [tile][source < RS_MAX_TP][epilogue warp < 4]

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
  void* out;                  // EPI 0/1: bf16 / fp32 [M, ldo]
  int ldo;
  const __nv_bfloat16* bias;  // [N] or null
  // EPI 2 (scatter to owners): tile rows belong to rank m / rows_per_rank and land at
  //   peer_out[owner] + ((src_rank * rows_per_rank) + m - owner * rows_per_rank) * N + n
  void* const* peer_out;
  int rows_per_rank, src_rank, tp;
  // GATHER: A rows of rank s live at peer_in[s] + local_row * K; gathered into a_local.
  const __nv_bfloat16* const* peer_in;
  __nv_bfloat16* a_local;
  const long long* ready;     // this rank's flag area: ready[s] >= epoch when rank s published
  // GATHER with in-kernel staging: the tensor cores read this rank's rows straight from x_local
  // (map_a2); the copy warps first write them into send_mine (the symmetric send buffer the peers
  // read) and, once every own sub-chunk is there (own_done counts them), publish the epoch into
  // slot src_rank of every peer's flag area (peer_ready[p]); then they pull the peers' rows into
  // the gather buffer (published per sub-chunk) and last copy the own rows into it (output only).
  const __nv_bfloat16* x_local;
  __nv_bfloat16* send_mine;
  long long* const* peer_ready;
  unsigned* own_done;
  long long* chunk_flags;     // [M / 16] per-sub-chunk publication flags (local)
  long long epoch;
  int group_m;                // tile raster: groups of group_m row blocks sweep all column blocks
  int split_k;                // EPI 1 only: equal k-ranges per tile (1 = whole tiles), chosen by launch()
  // EPI 3/4 (cross-entropy over a vocabulary shard [lo, lo + N)):
  const long long* targets;   // [M] global token ids
  long long lo;
  float2* ce_part;            // EPI 3: [M, tiles_n] (max, sum exp(x - max)) per column tile
  float* ce_target;           // EPI 3: [M] target logit (rows whose target is in this shard)
  const float* ce_lse;        // EPI 4: [M] log-sum-exp over the full vocabulary
  const float* ce_scale;      // EPI 4: device scalar dloss / rows
  // Second operand pair (K2 > 0): k blocks [kb(K), kb(K) + kb(K2)) read map_a2 / map_b2.
  int K2;
  // EPI 5: receive slabs [tp][rows_per_rank][N] bf16 of this call's parity (peer bases and ours)
  // and the per-tile stamp areas [tiles][RS_MAX_TP][4] int64 (peer bases and ours).
  const __nv_bfloat16* my_recv;
  long long* const* rs_flags_peer;
  const long long* rs_flags_mine;
  // Graph-safe epochs (epoch_ctr non-null): the call's epoch is *epoch_ctr + 1, read by every CTA at
  // the start; the last CTA to finish stores it back (epoch_done counts finished CTAs), so the next
  // call of the kind, ordered after this one on the stream, sees it, also inside a CUDA-graph
  // replay. The epoch's parity then picks the double-buffered symmetric buffers on the device:
  // the *_odd pointers are used for odd epochs (host-chosen epochs pass the call's buffers only).
  long long* epoch_ctr;
  unsigned* epoch_done;
  const __nv_bfloat16* const* peer_in_odd;
  __nv_bfloat16* send_mine_odd;
  void* const* peer_out_odd;
  const __nv_bfloat16* my_recv_odd;
};

__device__ __forceinline__ long long ld_acquire_sys(const long long* p) {
  long long v;
  asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ long long ld_acquire_gpu(const long long* p) {
  long long v;
  asm volatile("ld.acquire.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(long long* p, long long v) {
  asm volatile("st.release.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_release_sys(long long* p, long long v) {
  asm volatile("st.release.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint4 ld_cg_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Bounded spin until *flag >= target; false (status recorded) on timeout or abort.
template <bool SYS>
__device__ __forceinline__ bool wait_flag(const long long* flag, long long target, int* status, volatile int* abort,
                                          int code) {
  const unsigned long long start = tc::globaltimer();
  while ((SYS ? ld_acquire_sys(flag) : ld_acquire_gpu(flag)) < target) {
    if (*abort) return false;
    if (tc::globaltimer() - start > tc::kWaitNs) {
      atomicCAS(status, 0, code);
      *abort = 1;
      return false;
    }
  }
  return true;
}

// Tile order: groups of `group_m` row blocks; inside a group m is fastest and the group sweeps
// every column block before the next group starts, so the CTAs in flight share a few A row
// blocks and B column blocks that stay in L2 (an m-fastest order over all rows re-reads A from
// DRAM once per column block when A exceeds L2). With GATHER the m index is rotated so this
// rank's own rows come first.
__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int group_m, int rotate, int& m0,
                                            int& n0) {
  const int per_group = group_m * tiles_n;
  const int first = (t / per_group) * group_m;
  const int rows = min(group_m, tiles_m - first);
  const int r = t % per_group;
  const int mi = (first + r % rows + rotate) % tiles_m;
  m0 = mi * BM;
  n0 = (r / rows) * BN;
}

// Work of one CTA: units handed out round-robin over the grid. A unit is a whole tile, or (split_k
// = S > 1, epilogue 1 only) one of S equal k-ranges of a tile, numbered split-major (unit u is
// range u / tiles of tile u % tiles), so the CTAs of one wave sweep the same contraction range and
// share its A/B slices in L2. Partial sums of a tile from several units meet in the reduce-add
// epilogue, so no fix-up pass is needed; S is picked on the host to even out the last wave.
struct WorkIter {
  int u, units, kblocks, tiles, splits;
  __device__ WorkIter(int splits_, int tiles_, int kblocks_)
      : u(blockIdx.x), units(tiles_ * max(1, splits_)), kblocks(kblocks_), tiles(tiles_), splits(max(1, splits_)) {}
  __device__ bool next(int& tile, int& kb0, int& kb1) {
    if (u >= units) return false;
    const int s = u / tiles;
    tile = u % tiles;
    kb0 = (int)((long long)s * kblocks / splits);
    kb1 = (int)((long long)(s + 1) * kblocks / splits);
    u += gridDim.x;
    return true;
  }
};

template <bool A_MN, bool B_MN, int EPI, bool GATHER>
__global__ void __launch_bounds__(GATHER ? 256 : 192, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const __grid_constant__ CUtensorMap map_out, const __grid_constant__ CUtensorMap map_a2,
                const __grid_constant__ CUtensorMap map_b2, GemmArgs args, int* status) {
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
  __shared__ long long s_epoch;
  if (threadIdx.x == 0)
    s_epoch = epoch_begin(args.epoch_ctr, args.epoch);
  const int tiles_m = (args.M + BM - 1) / BM, tiles_n = (args.N + BN - 1) / BN;
  const int tiles = tiles_m * tiles_n;
  const int kb_first = (args.K + BK - 1) / BK;   // k blocks of the first operand pair
  const int kblocks = kb_first + (args.K2 > 0 ? (args.K2 + BK - 1) / BK : 0);
  // GATHER: this rank's rows first; EPI 5: the next rank's rows first and this rank's rows last.
  const int rotate = GATHER ? (args.src_rank * args.rows_per_rank) / BM
                            : (EPI == 5 ? (((args.src_rank + 1) % args.tp) * args.rows_per_rank) / BM : 0);

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
  const long long epoch = s_epoch;
  const bool odd = (epoch & 1) != 0;
  const __nv_bfloat16* const* peer_in = (odd && args.peer_in_odd) ? args.peer_in_odd : args.peer_in;
  __nv_bfloat16* send_mine = (odd && args.send_mine_odd) ? args.send_mine_odd : args.send_mine;
  void* const* peer_out = (odd && args.peer_out_odd) ? args.peer_out_odd : args.peer_out;
  const __nv_bfloat16* my_recv = (odd && args.my_recv_odd) ? args.my_recv_odd : args.my_recv;

  if (warp == 0) {
    if (lane == 0) {
      tc::prefetch_map(&map_a);
      tc::prefetch_map(&map_b);
      if (args.K2 > 0) {
        tc::prefetch_map(&map_a2);
        tc::prefetch_map(&map_b2);
      } else if (GATHER && args.x_local) {
        tc::prefetch_map(&map_a2);
      }
      int stage = 0;
      uint32_t phase = 0;
      int armed[STAGES];  // parity of the last armed phase of each stage, -1 = never armed
#pragma unroll
      for (int s = 0; s < STAGES; ++s) armed[s] = -1;
      bool ok = true;
      WorkIter work(EPI == 1 ? args.split_k : 1, tiles, kblocks);
      int t, kb0, kb1;
      int ready_m0 = -1;   // GATHER: the last row block seen published (consecutive tiles often share it)
      while (ok && work.next(t, kb0, kb1)) {
        int m0, n0;
        tile_coords(t, tiles_m, tiles_n, args.group_m, rotate, m0, n0);
        // GATHER with staging: this rank's row blocks come from x_local (map_a2), never waited for
        const int own_row = m0 - args.src_rank * args.rows_per_rank;
        const bool own_tile = GATHER && args.x_local != nullptr && own_row >= 0 && own_row < args.rows_per_rank;
        if (GATHER && !own_tile && m0 != ready_m0) {
          // the row block is ready once all of its 16-row sub-chunks are published
          for (int j = 0; j < BM / GATHER_SUB && ok; ++j)
            ok = wait_flag<false>(args.chunk_flags + m0 / GATHER_SUB + j, epoch, status, abort_flag, 5);
          if (!ok) break;
          fence_proxy_async_global();
          ready_m0 = m0;
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!tc::mbar_wait(&empty[stage], phase ^ 1, status, abort_flag, 1)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          tc::mbar_expect_tx(&full[stage], STAGE_BYTES);
          const bool second = kb >= kb_first;
          const CUtensorMap* ma = (second || own_tile) ? &map_a2 : &map_a;
          const CUtensorMap* mb = second ? &map_b2 : &map_b;
          const int k0 = (second ? kb - kb_first : kb) * BK;
          const int am0 = own_tile ? own_row : m0;
          if (A_MN) {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tc::tma_load_2d(sa + j * (BK * 128), ma, &full[stage], am0 + j * 64, k0);
          } else {
            tc::tma_load_2d(sa, ma, &full[stage], k0, am0);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tc::tma_load_2d(sb + j * (BK * 128), mb, &full[stage], n0 + j * 64, k0);
          } else {
            tc::tma_load_2d(sb, mb, &full[stage], k0, n0);
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
      WorkIter work(EPI == 1 ? args.split_k : 1, tiles, kblocks);
      int t, kb0, kb1;
      for (; ok && work.next(t, kb0, kb1); ++local) {
        const int buf = local & 1;
        const uint32_t use = (local >> 1) & 1;
        if (!tc::mbar_wait(&tempty[buf], use ^ 1, status, abort_flag, 2)) break;
        tc::fence_after();
        const uint32_t d = tmem + buf * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
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
            tc::mma_bf16(d, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
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
  } else if (warp < 6) {
    // Epilogue warps 2..5 -> TMEM lane quarter (warp % 4). Each warp owns 32 rows of the tile:
    // TMEM -> registers (tcgen05.ld) -> dense 32x32 smem box -> TMA store (bf16), TMA reduce-add
    // (fp32 accumulate) or coalesced stores into the owning rank's receive buffer (peer memory).
    const int quarter = warp & 3;
    uint8_t* my_stage = staging + quarter * 2 * EPI_BOX * EPI_BOX * 4;
    int local = 0, chunk = 0;
    if (lane == 0 && EPI != 2 && EPI != 3) tc::prefetch_map(&map_out);
    WorkIter work(EPI == 1 ? args.split_k : 1, tiles, kblocks);
    int t, kb0, kb1;
    for (; work.next(t, kb0, kb1); ++local) {
      const int buf = local & 1;
      const uint32_t use = (local >> 1) & 1;
      if (!tc::mbar_wait(&tfull[buf], use, status, abort_flag, 4)) break;
      tc::fence_after();
      int m0, n0;
      tile_coords(t, tiles_m, tiles_n, args.group_m, rotate, m0, n0);
      const uint32_t base = tmem + buf * BN + ((uint32_t)(quarter * 32) << 16);
      if (EPI == 3) {
        // online softmax statistics of this thread's row over the tile's columns
        const int row = m0 + quarter * 32 + lane;
        const long long tgt = row < args.M ? args.targets[row] - args.lo : -1;
        float mx = -INFINITY, se = 0.f, tv = 0.f;
        bool found = false;
#pragma unroll 1
        for (int c = 0; c < BN; c += EPI_BOX) {
          float v[32];
          tc::tmem_ld32(base + c, v);
          const int col0 = n0 + c;
          if (col0 >= args.N) continue;
          const int valid = min(32, args.N - col0);
          float bm = -INFINITY;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (j < valid) bm = fmaxf(bm, v[j]);
            if (col0 + j == tgt) {
              tv = v[j];
              found = true;
            }
          }
          const float nm = fmaxf(mx, bm);
          float add = 0.f;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < valid) add += __expf(v[j] - nm);
          se = se * __expf(mx - nm) + add;
          mx = nm;
        }
        if (row < args.M) {
          args.ce_part[(size_t)row * tiles_n + n0 / BN] = make_float2(mx, se);
          if (found) args.ce_target[row] = tv;
        }
        tc::fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&tempty[buf]);
        continue;
      }
      // EPI 5: tiles of this rank's rows reduce the peers' partials; other tiles go to their owner.
      const int owner = (EPI == 5 || EPI == 2) ? m0 / args.rows_per_rank : 0;
      const bool own = EPI == 5 && owner == args.src_rank;
      const int owner_tile = EPI == 5 ? ((m0 - owner * args.rows_per_rank) / BM) * tiles_n + n0 / BN : 0;
      if (own) {
        bool ok = true;
        if (lane == 0)
          for (int s = 0; s < args.tp && ok; ++s)
            if (s != args.src_rank)
              ok = wait_flag<true>(args.rs_flags_mine + ((size_t)owner_tile * RS_MAX_TP + s) * 4 + quarter,
                                   epoch, status, abort_flag, 7);
        ok = __shfl_sync(0xffffffffu, ok, 0) != 0;  // the warp barrier orders lane 0's acquire before all lanes' reads
        if (!ok) break;
      }
      const __nv_bfloat16* bias = (EPI == 5 && !own) ? nullptr : args.bias;
      float ce_l = 0.f, ce_f = 0.f;
      long long ce_t = -1;
      if (EPI == 4) {
        const int row = m0 + quarter * 32 + lane;
        if (row < args.M) {
          ce_l = args.ce_lse[row];
          ce_t = args.targets[row] - args.lo;
        }
        ce_f = *args.ce_scale;
      }
#pragma unroll 1
      for (int c = 0; c < BN; c += EPI_BOX, ++chunk) {
        float v[32];
        tc::tmem_ld32(base + c, v);
        const int col0 = n0 + c;
        if (col0 >= args.N) continue;  // whole box outside the matrix (uniform across the warp)
        uint8_t* box = my_stage + (chunk & 1) * EPI_BOX * EPI_BOX * 4;
        if (own) {
          // peers' bf16 partials of this thread's row (local memory, written by the peers' kernels)
          const int lrow = m0 - args.src_rank * args.rows_per_rank + quarter * 32 + lane;
          const int valid = min(32, args.N - col0);
          for (int s = 0; s < args.tp; ++s) {
            if (s == args.src_rank) continue;
            const __nv_bfloat16* src = my_recv + ((size_t)s * args.rows_per_rank + lrow) * args.N + col0;
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              if (j < valid) {
                const uint4 u = ld_cg_u4(src + j);
                const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  const float2 f = __bfloat1622float2(h[q]);
                  v[j + 2 * q] += f.x;
                  v[j + 2 * q + 1] += f.y;
                }
              }
            }
          }
        }
        if (EPI != 2) {
          if (lane == 0) tc::bulk_wait_read1();  // the store that last used this buffer finished reading
          __syncwarp();
        }
        if (EPI == 4) {
          __nv_bfloat16* row = reinterpret_cast<__nv_bfloat16*>(box) + lane * EPI_BOX;
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            float o[8];
#pragma unroll
            for (int q = 0; q < 8; ++q)
              o[q] = (__expf(v[j + q] - ce_l) - (col0 + j + q == ce_t ? 1.f : 0.f)) * ce_f;
            store8(row + j, o);
          }
        } else if (EPI == 0 || EPI == 2 || EPI == 5) {
          __nv_bfloat16* row = reinterpret_cast<__nv_bfloat16*>(box) + lane * EPI_BOX;
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            float o[8];
#pragma unroll
            for (int q = 0; q < 8; ++q)
              o[q] = v[j + q] + ((bias && col0 + j + q < args.N) ? __bfloat162float(bias[col0 + j + q]) : 0.f);
            store8(row + j, o);
          }
        } else {
          float* row = reinterpret_cast<float*>(box) + lane * EPI_BOX;
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(row + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        }
        if (EPI == 2 || (EPI == 5 && !own)) {
          __syncwarp();
          const int lrow0 = args.src_rank * args.rows_per_rank + (m0 - owner * args.rows_per_rank) + quarter * 32;
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(peer_out[owner]) + (size_t)lrow0 * args.N + col0;
          const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(box);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int cidx = lane + 32 * i;        // 128 16-byte pieces: 32 rows x 4
            const int r = cidx >> 2, part = cidx & 3;
            if (m0 + quarter * 32 + r < args.M && col0 + part * 8 < args.N)
              *reinterpret_cast<uint4*>(dst + (size_t)r * args.N + part * 8) =
                  *reinterpret_cast<const uint4*>(src + r * EPI_BOX + part * 8);
          }
          __syncwarp();
        } else {
          tc::fence_proxy_async();
          __syncwarp();
          if (lane == 0) {
            if (EPI == 5)
              tc::tma_store_2d(&map_out, box, col0, m0 - args.src_rank * args.rows_per_rank + quarter * 32);
            else if (EPI == 0 || EPI == 4)
              tc::tma_store_2d(&map_out, box, col0, m0 + quarter * 32);
            else
              tc::tma_reduce_add_2d(&map_out, box, col0, m0 + quarter * 32);
            tc::bulk_commit();
          }
        }
      }
      // every TMEM read of this buffer is done: hand it back to the MMA warp before the publication
      // below, so the next tile's accumulation is not held up by the system-scope fence
      tc::fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&tempty[buf]);
      if (EPI == 5 && !own) {
        // publish this warp's 32 rows of the tile to the owner: system-scope fence by every lane,
        // then one release store of the epoch into the (tile, source, warp) slot
        __threadfence_system();
        __syncwarp();
        if (lane == 0)
          st_release_sys(args.rs_flags_peer[owner] + ((size_t)owner_tile * RS_MAX_TP + args.src_rank) * 4 + quarter,
                         epoch);
      }
    }
    if (EPI != 2 && EPI != 3 && lane == 0) tc::bulk_wait_all();
    __syncwarp();
  } else if (GATHER) {
    // Copy warps 6..7 of every CTA move 16-row sub-chunks, handed out round-robin over the CTAs.
    // Without x_local: every rank's rows (peer_in[s]; this rank's own send buffer included) into
    // the gather buffer, in tile order (this rank's rows first), each sub-chunk published with the
    // call's epoch for the TMA producer. With x_local, three phases: (1) this rank's rows into
    // send_mine, the last of them publishing the shard to the peers; (2) the peers' rows into the
    // gather buffer, published per sub-chunk (the tensor cores read this rank's rows from x_local
    // meanwhile); (3) this rank's rows into the gather buffer, which only the caller reads.
    const int ct = threadIdx.x - 192;  // 0..63
    const int subs = args.M / GATHER_SUB;
    const int rot = rotate * (BM / GATHER_SUB);
    const bool staged = args.x_local != nullptr;
    const int own_subs = args.rows_per_rank / GATHER_SUB;
    const int items = staged ? subs + own_subs : subs;
    for (int i = blockIdx.x; i < items; i += gridDim.x) {
      // phase of item i and its sub-chunk (phase 0: the unstaged single pass)
      const int phase = !staged ? 0 : (i < own_subs ? 1 : (i < subs ? 2 : 3));
      const int sub = phase == 1 ? rot + i : (phase == 3 ? rot + (i - subs) : (i + rot) % subs);
      const int row0 = sub * GATHER_SUB;
      const int s = row0 / args.rows_per_rank;
      const int lrow = row0 - s * args.rows_per_rank;
      bool ok = true;
      if (ct == 0 && s != args.src_rank) ok = wait_flag<true>(args.ready + s, epoch, status, abort_flag, 6);
      asm volatile("bar.sync 1, 64;" ::: "memory");
      if (*abort_flag || !ok) break;
      const bool from_local = phase == 1 || phase == 3;
      const uint4* src = reinterpret_cast<const uint4*>((from_local ? args.x_local : peer_in[s]) + (size_t)lrow * args.K);
      uint4* dst = phase == 1 ? reinterpret_cast<uint4*>(send_mine + (size_t)lrow * args.K)
                              : reinterpret_cast<uint4*>(args.a_local + (size_t)row0 * args.K);
      const int vecs = GATHER_SUB * args.K / 8;
      // 16 independent 16-byte loads in flight per thread: NVLink latency is hidden by
      // memory-level parallelism rather than by occupancy.
      constexpr int UNROLL = 16;
      int v = ct;
      for (; v + 64 * (UNROLL - 1) < vecs; v += 64 * UNROLL) {
        uint4 r[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) r[u] = __ldcg(src + v + 64 * u);
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) dst[v + 64 * u] = r[u];
      }
      for (; v < vecs; v += 64) dst[v] = __ldcg(src + v);
      if (phase == 3) continue;   // output rows only: the kernel's completion publishes them
      if (phase == 1) {
        __threadfence_system();
      } else {
        fence_proxy_async_global();
        __threadfence();
      }
      asm volatile("bar.sync 1, 64;" ::: "memory");
      if (ct == 0) {
        if (phase != 1) st_release_gpu(args.chunk_flags + sub, epoch);
        if (phase == 1) {
          // the last own sub-chunk staged (over all CTAs) publishes this rank's shard to the peers
          if (atomicAdd(args.own_done, 1u) + 1u == (unsigned)own_subs) {
            atomicExch(args.own_done, 0u);
            __threadfence_system();
            for (int p = 0; p < args.tp; ++p)
              if (p != args.src_rank) st_release_sys(args.peer_ready[p] + args.src_rank, epoch);
          }
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc::fence_after();
    tc::tmem_dealloc(tmem, 2 * BN);
  }
  if (threadIdx.x == 0) epoch_end(args.epoch_ctr, args.epoch_done, epoch);   // last CTA publishes the epoch
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

}  // namespace

CUtensorMap tma_map_bf16(const at::Tensor& t, int box_rows) { return make_map(t, box_rows); }

namespace {

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

template <bool A_MN, bool B_MN, int EPI, bool GATHER>
void launch(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo, GemmArgs args,
            const CUtensorMap* ma2 = nullptr, const CUtensorMap* mb2 = nullptr) {
  auto kernel = gemm_kernel<A_MN, B_MN, EPI, GATHER>;
  static std::once_flag once;
  std::call_once(once, [&] {
    CQB_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
  });
  const int tiles_m = (args.M + BM - 1) / BM;
  const int tiles = tiles_m * ((args.N + BN - 1) / BN);
  // Row-block group: the group's A blocks (BM x K bf16 each) should fill about 48 MB of L2.
  const long long a_block = (long long)BM * args.K * 2;
  args.group_m = (int)std::max(1LL, std::min<long long>(tiles_m, (48LL << 20) / std::max(1LL, a_block)));
  // All-gather: tiles follow the ranks' row ranges (own rows first), so the first tiles need no
  // peer data and the copy of the other ranks' rows overlaps them. One row block per group (all
  // column tiles of a row block before the next block): a wave of tiles then needs only the next
  // ~148 / tiles_n row blocks, in the order the copy warps publish them, instead of every block of
  // a 32-block group; the row block's 12-24 column tiles share it in L2 and B stays resident.
  if (GATHER) args.group_m = 1;
  // GEMM -> reduce-scatter: groups must not straddle two owners, so that this rank's own row
  // blocks (rotated to the end of the order) form the last groups.
  if (EPI == 5) {
    const int blocks = args.rows_per_rank / BM;
    int g = std::min(args.group_m, blocks);
    while (blocks % g) --g;
    args.group_m = g;
  }
  if (args.K2 > 0) TORCH_CHECK(ma2 != nullptr && mb2 != nullptr, "second operand pair without tensor maps");
  // GATHER needs every CTA resident (copy blocks are handed out by CTA index): one per SM.
  // Split-K (reduce-add epilogue): every SM takes an equal share of the tiles x k-blocks units.
  // Split-K (reduce-add epilogue only): S equal k-ranges per tile, S in 1..4 with at least 16 k
  // blocks per range, chosen for the best fill of the last wave (ties go to the smaller S).
  const int kblocks = (int)((args.K + BK - 1) / BK);
  if (EPI == 1 && args.split_k) {
    int best = 1;
    double best_fill = 0.0;
    for (int s = 1; s <= 4; ++s) {
      if (s > 1 && kblocks / s < 16) break;
      const long long units = (long long)tiles * s;
      const long long waves = (units + sm_count() - 1) / sm_count();
      const double fill = (double)units / (double)(waves * sm_count());
      if (fill > best_fill + 0.02) {
        best_fill = fill;
        best = s;
      }
    }
    args.split_k = best;
  } else {
    args.split_k = 1;
  }
  const int grid = std::max(1, std::min(tiles * args.split_k, sm_count()));
  kernel<<<grid, GATHER ? 256 : 192, SMEM_BYTES, stream()>>>(ma, mb, mo, ma2 ? *ma2 : ma, mb2 ? *mb2 : mb, args,
                                                              status_word());
  CQB_LAUNCH_CHECK();
  count_launch();
}

// Inner (contiguous) TMA extents must be multiples of 8 elements (16 bytes); outer extents are free.
void check_dims(int64_t m, int64_t n, int64_t k, bool k_inner = true) {
  TORCH_CHECK(m > 0 && n > 0 && k > 0, "empty GEMM");
  TORCH_CHECK(n % 16 == 0, "GEMM N must be a multiple of 16");
  TORCH_CHECK(!k_inner || k % 16 == 0, "GEMM K must be a multiple of 16");
}

GemmArgs plain_args(int64_t M, int64_t N, int64_t K, void* out, int64_t ldo, const __nv_bfloat16* bias) {
  GemmArgs a{};
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.out = out;
  a.ldo = (int)ldo;
  a.bias = bias;
  return a;
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
  auto args = plain_args(M, N, K, y.data_ptr(), N, b.defined() ? (const __nv_bfloat16*)b.data_ptr() : nullptr);
  launch<false, false, 0, false>(ma, mb, make_out_map(y), args);
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
  launch<false, true, 0, false>(ma, mb, make_out_map(y), plain_args(M, N, K, y.data_ptr(), N, nullptr));
  return y;
}

// y[M,N] = x w (+) x2 w2 with two operand pairs in one k loop: w [N,K] (or [K,N] with w_mn_major), x2
// may have fewer rows than x (missing rows count as zero). The single-GPU form of the pair that the
// GEMM -> reduce-scatter kernel runs (the input gradient of two projections of one input).
at::Tensor gemm_dual(at::Tensor x, at::Tensor w, at::Tensor x2, at::Tensor w2, bool w_mn_major) {
  const int64_t M = x.size(0), K = x.size(1), N = w_mn_major ? w.size(1) : w.size(0);
  const int64_t K2 = x2.size(1);
  TORCH_CHECK(w_mn_major ? w.size(0) == K : w.size(1) == K, "gemm_dual: inner dims differ");
  TORCH_CHECK(w_mn_major ? (w2.size(0) == K2 && w2.size(1) == N) : (w2.size(1) == K2 && w2.size(0) == N),
              "gemm_dual: second pair shapes");
  TORCH_CHECK(x2.size(0) <= M && x2.size(0) > 0 && K2 % 16 == 0, "gemm_dual: x2 rows in [1, M], K2 % 16 == 0");
  check_dims(M, N, K);
  auto y = at::empty({M, N}, x.options());
  auto ma = make_map(x, BM);
  auto mb = w_mn_major ? make_map(w, BK) : make_map(w, BN);
  auto ma2 = make_map(x2, BM);
  auto mb2 = w_mn_major ? make_map(w2, BK) : make_map(w2, BN);
  auto args = plain_args(M, N, K, y.data_ptr(), N, nullptr);
  args.K2 = (int)K2;
  if (w_mn_major)
    launch<false, true, 0, false>(ma, mb, make_out_map(y), args, &ma2, &mb2);
  else
    launch<false, false, 0, false>(ma, mb, make_out_map(y), args, &ma2, &mb2);
  return y;
}

// Split-K for the reduce-add weight-gradient GEMM unless CQB_DETERMINISTIC=1: the fp32 partial sums
// of a tile then reach main_grad in an order that varies from run to run (values differ in the
// last bits); deterministic mode keeps one CTA per tile.
bool split_k_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("CQB_DETERMINISTIC");
    return !(v && v[0] == '1');
  }();
  return on;
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
  auto args = plain_args(N, K, M, out.data_ptr(), K, nullptr);
  args.split_k = split_k_enabled() ? 1 : 0;
  launch<true, true, 1, false>(ma, mb, make_out_map(out.view({N, K})), args);
}

// GEMM -> reduce-scatter, communication half: every tile of x[M,K] w^T (w [N,K]) or x w
// (w [K,N], w_mn_major) is stored into the receive buffer of the rank that owns its rows.
void gemm_scatter(at::Tensor x, at::Tensor w, bool w_mn_major, at::Tensor peer_out_ptrs, int64_t rows_per_rank,
                  int64_t src_rank, int64_t tp) {
  const int64_t M = x.size(0), K = x.size(1), N = w_mn_major ? w.size(1) : w.size(0);
  check_dims(M, N, K);
  TORCH_CHECK(rows_per_rank % BM == 0 && M == rows_per_rank * tp, "rows per rank must be a multiple of 128");
  TORCH_CHECK(peer_out_ptrs.is_cuda() && peer_out_ptrs.numel() == tp, "peer pointers: cuda int64 [tp]");
  auto ma = make_map(x, BM);
  auto mb = w_mn_major ? make_map(w, BK) : make_map(w, BN);
  auto args = plain_args(M, N, K, nullptr, N, nullptr);
  args.peer_out = reinterpret_cast<void* const*>(peer_out_ptrs.data_ptr());
  args.rows_per_rank = (int)rows_per_rank;
  args.src_rank = (int)src_rank;
  args.tp = (int)tp;
  if (w_mn_major)
    launch<false, true, 2, false>(ma, mb, ma, args);
  else
    launch<false, false, 2, false>(ma, mb, ma, args);
}

// GEMM -> reduce-scatter in one kernel (epilogue 5). Returns this rank's reduced rows
// out[rows_per_rank, N] = sum over ranks of (x w^T + x2 w2^T)[own rows] + bias, where the rank
// order of x's rows is [rank 0 rows, rank 1 rows, ...]. w is [N, K] (or [K, N] with w_mn_major);
// x2 / w2 (optional) form a second operand pair with the same layouts, contraction K2, and x2 may
// have fewer rows than x (missing rows count as zero). peer_recv: int64 [tp] receive-slab bases
// ([tp][rows_per_rank][N] bf16, this call's parity) of every rank; my_recv: ours. peer_flags:
// int64 [tp] stamp-area bases; my_flags: ours (tiles * 8 * 4 int64 slots).
at::Tensor gemm_scatter_reduce(at::Tensor x, at::Tensor w, bool w_mn_major, c10::optional<at::Tensor> x2,
                               c10::optional<at::Tensor> w2, c10::optional<at::Tensor> bias, at::Tensor peer_recv,
                               int64_t my_recv, at::Tensor peer_flags, int64_t my_flags, int64_t flag_slots,
                               int64_t epoch, int64_t rows_per_rank, int64_t src_rank, int64_t tp,
                               int64_t epoch_ctr, int64_t epoch_done, c10::optional<at::Tensor> peer_recv_odd,
                               int64_t my_recv_odd) {
  const int64_t M = x.size(0), K = x.size(1), N = w_mn_major ? w.size(1) : w.size(0);
  TORCH_CHECK(w_mn_major ? w.size(0) == K : w.size(1) == K, "gemm_scatter_reduce: inner dims differ");
  check_dims(M, N, K);
  TORCH_CHECK(tp >= 2 && tp <= RS_MAX_TP, "gemm_scatter_reduce: TP must be 2..", RS_MAX_TP);
  TORCH_CHECK(rows_per_rank % BM == 0 && M == rows_per_rank * tp, "rows per rank must be a multiple of 128");
  TORCH_CHECK(peer_recv.is_cuda() && peer_recv.numel() == tp && peer_flags.is_cuda() && peer_flags.numel() == tp,
              "peer pointers: cuda int64 [tp]");
  const int64_t own_tiles = (rows_per_rank / BM) * ((N + BN - 1) / BN);
  TORCH_CHECK(own_tiles * RS_MAX_TP * 4 <= flag_slots, "gemm_scatter_reduce: too many tiles for the stamp area");
  auto out = at::empty({rows_per_rank, N}, x.options());
  auto ma = make_map(x, BM);
  auto mb = w_mn_major ? make_map(w, BK) : make_map(w, BN);
  at::Tensor b;
  if (bias && bias->defined()) b = bias->to(at::kBFloat16).contiguous();
  auto args = plain_args(M, N, K, out.data_ptr(), N, b.defined() ? (const __nv_bfloat16*)b.data_ptr() : nullptr);
  args.peer_out = reinterpret_cast<void* const*>(peer_recv.data_ptr());
  args.my_recv = reinterpret_cast<const __nv_bfloat16*>(my_recv);
  args.rs_flags_peer = reinterpret_cast<long long* const*>(peer_flags.data_ptr());
  args.rs_flags_mine = reinterpret_cast<const long long*>(my_flags);
  args.epoch = epoch;
  args.rows_per_rank = (int)rows_per_rank;
  args.src_rank = (int)src_rank;
  args.tp = (int)tp;
  if (epoch_ctr) {   // graph-safe epochs: the kernel reads and advances the device counter
    TORCH_CHECK(epoch_done != 0 && peer_recv_odd && peer_recv_odd->is_cuda() && peer_recv_odd->numel() == tp &&
                    my_recv_odd != 0,
                "gemm_scatter_reduce: device epochs need the done counter and the odd-parity buffers");
    args.epoch_ctr = reinterpret_cast<long long*>(epoch_ctr);
    args.epoch_done = reinterpret_cast<unsigned*>(epoch_done);
    args.peer_out_odd = reinterpret_cast<void* const*>(peer_recv_odd->data_ptr());
    args.my_recv_odd = reinterpret_cast<const __nv_bfloat16*>(my_recv_odd);
  }
  CUtensorMap ma2, mb2;
  const bool dual = x2 && x2->defined();
  if (dual) {
    TORCH_CHECK(w2 && w2->defined(), "second operand pair needs both x2 and w2");
    const int64_t K2 = x2->size(1);
    TORCH_CHECK(x2->size(0) <= M && x2->size(0) > 0, "x2 rows must be in [1, rows of x]");
    TORCH_CHECK(w_mn_major ? (w2->size(0) == K2 && w2->size(1) == N) : (w2->size(1) == K2 && w2->size(0) == N),
                "gemm_scatter_reduce: second pair shapes");
    TORCH_CHECK(K2 % 16 == 0, "K2 must be a multiple of 16");
    ma2 = make_map(*x2, BM);
    mb2 = w_mn_major ? make_map(*w2, BK) : make_map(*w2, BN);
    args.K2 = (int)K2;
  }
  auto mo = make_out_map(out);
  if (w_mn_major)
    launch<false, true, 5, false>(ma, mb, mo, args, dual ? &ma2 : nullptr, dual ? &mb2 : nullptr);
  else
    launch<false, false, 5, false>(ma, mb, mo, args, dual ? &ma2 : nullptr, dual ? &mb2 : nullptr);
  return out;
}

// All-gather -> GEMM: y[M,N] = gather(x)[M,K] w[N,K]^T (+ bias); the gathered rows land in a_local.
// mn_major: w is [K, N] (the row-parallel backward dX = all_gather(dY) @ W), else [N, K].
// With x_local (this rank's shard [rows_per_rank, K]) the kernel stages it itself: copy warps write
// it into the gather buffer and into send_mine (this rank's symmetric send buffer, which the peers
// read), then publish the epoch into slot src_rank of every peer's flag area (peer_ready bases,
// own_done: a zeroed device counter). Without x_local the caller staged and published the shard.
at::Tensor gather_gemm(at::Tensor a_local, at::Tensor w, c10::optional<at::Tensor> bias, at::Tensor peer_in_ptrs,
                       int64_t ready_ptr, at::Tensor chunk_flags, int64_t epoch, int64_t rows_per_rank, int64_t src_rank,
                       int64_t tp, bool mn_major, c10::optional<at::Tensor> x_local, int64_t send_mine,
                       c10::optional<at::Tensor> peer_ready, int64_t own_done, int64_t epoch_ctr, int64_t epoch_done,
                       c10::optional<at::Tensor> peer_in_odd, int64_t send_mine_odd) {
  const int64_t M = a_local.size(0), K = a_local.size(1), N = mn_major ? w.size(1) : w.size(0);
  TORCH_CHECK(!mn_major || w.size(0) == K, "gather_gemm: inner dims differ");
  check_dims(M, N, K);
  TORCH_CHECK(rows_per_rank % BM == 0 && M == rows_per_rank * tp, "rows per rank must be a multiple of 128");
  TORCH_CHECK(chunk_flags.scalar_type() == at::kLong && chunk_flags.numel() >= M / GATHER_SUB,
              "chunk flags too small: one per 16 rows");
  auto y = at::empty({M, N}, a_local.options());
  auto ma = make_map(a_local, BM);
  auto mb = make_map(w, mn_major ? BK : BN);
  at::Tensor b;
  if (bias && bias->defined()) b = bias->to(at::kBFloat16).contiguous();
  auto args = plain_args(M, N, K, y.data_ptr(), N, b.defined() ? (const __nv_bfloat16*)b.data_ptr() : nullptr);
  args.peer_in = reinterpret_cast<const __nv_bfloat16* const*>(peer_in_ptrs.data_ptr());
  args.a_local = (__nv_bfloat16*)a_local.data_ptr();
  args.ready = reinterpret_cast<const long long*>(ready_ptr);
  args.chunk_flags = reinterpret_cast<long long*>(chunk_flags.data_ptr());
  args.epoch = epoch;
  args.rows_per_rank = (int)rows_per_rank;
  args.src_rank = (int)src_rank;
  args.tp = (int)tp;
  if (x_local && x_local->defined()) {
    TORCH_CHECK(x_local->is_contiguous() && x_local->size(0) == rows_per_rank && x_local->size(1) == K &&
                    x_local->scalar_type() == at::kBFloat16 && reinterpret_cast<uintptr_t>(x_local->data_ptr()) % 16 == 0,
                "gather_gemm: x_local must be a contiguous aligned bf16 [rows_per_rank, K]");
    TORCH_CHECK(peer_ready && peer_ready->is_cuda() && peer_ready->numel() == tp && send_mine != 0 && own_done != 0,
                "gather_gemm: in-kernel staging needs send_mine, peer_ready and own_done");
    TORCH_CHECK(rows_per_rank % GATHER_SUB == 0 && K % 8 == 0, "gather_gemm: rows per rank / K alignment");
    args.x_local = reinterpret_cast<const __nv_bfloat16*>(x_local->data_ptr());
    args.send_mine = reinterpret_cast<__nv_bfloat16*>(send_mine);
    args.peer_ready = reinterpret_cast<long long* const*>(peer_ready->data_ptr());
    args.own_done = reinterpret_cast<unsigned*>(own_done);
  }
  if (epoch_ctr) {   // graph-safe epochs: the kernel reads and advances the device counter
    TORCH_CHECK(epoch_done != 0 && peer_in_odd && peer_in_odd->is_cuda() && peer_in_odd->numel() == tp &&
                    (!args.x_local || send_mine_odd != 0),
                "gather_gemm: device epochs need the done counter and the odd-parity buffers");
    args.epoch_ctr = reinterpret_cast<long long*>(epoch_ctr);
    args.epoch_done = reinterpret_cast<unsigned*>(epoch_done);
    args.peer_in_odd = reinterpret_cast<const __nv_bfloat16* const*>(peer_in_odd->data_ptr());
    args.send_mine_odd = reinterpret_cast<__nv_bfloat16*>(send_mine_odd);
  }
  CUtensorMap mx;
  if (args.x_local) mx = make_map(*x_local, BM);   // this rank's rows, read by the tensor cores directly
  if (mn_major)
    launch<false, true, 0, true>(ma, mb, make_out_map(y), args, args.x_local ? &mx : nullptr);
  else
    launch<false, false, 0, true>(ma, mb, make_out_map(y), args, args.x_local ? &mx : nullptr);
  return y;
}

namespace {

// (max, sum exp) merge of the per-tile partials of each row: one warp per row.
__global__ void ce_merge_kernel(const float2* __restrict__ part, int rows, int tiles, float* __restrict__ mx_out,
                                float* __restrict__ se_out) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  // (m, s) pairs merge as s = s e^{m - M} + s' e^{m' - M}; a lane without tiles holds (-inf, 0)
  // and two such lanes must stay (-inf, 0) instead of forming e^{-inf - (-inf)}.
  auto merge = [](float& m, float& s, float om, float os) {
    const float nm = fmaxf(m, om);
    if (nm == -INFINITY) return;
    s = s * __expf(m - nm) + os * __expf(om - nm);
    m = nm;
  };
  float m = -INFINITY, s = 0.f;
  for (int t = lane; t < tiles; t += 32) {
    const float2 p = part[(size_t)warp * tiles + t];
    merge(m, s, p.x, p.y);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o), os = __shfl_xor_sync(0xffffffffu, s, o);
    merge(m, s, om, os);
  }
  if (lane == 0) {
    mx_out[warp] = m;
    se_out[warp] = s;
  }
}

void check_ce(const at::Tensor& h, const at::Tensor& w, const at::Tensor& targets) {
  TORCH_CHECK(h.is_cuda() && h.scalar_type() == at::kBFloat16 && h.is_contiguous() && h.dim() == 2, "h: bf16 [rows, K]");
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.is_contiguous() && w.size(1) == h.size(1), "w: bf16 [V, K]");
  TORCH_CHECK(targets.scalar_type() == at::kLong && targets.is_contiguous() && targets.numel() == h.size(0),
              "targets: int64 [rows]");
  check_dims(h.size(0), w.size(0), h.size(1));
}

}  // namespace

// LM-head GEMM with the statistics epilogue only: returns the per-(row, column tile) (max, sum exp)
// partials [rows, tiles, 2] and the target logit [rows] (0 where the target is outside [lo, lo + V)).
std::vector<at::Tensor> ce_partials(at::Tensor h, at::Tensor w, at::Tensor targets, int64_t lo) {
  check_ce(h, w, targets);
  const int64_t M = h.size(0), K = h.size(1), N = w.size(0);
  const int tiles_n = (int)((N + BN - 1) / BN);
  auto f32 = h.options().dtype(at::kFloat);
  auto part = at::empty({M, tiles_n, 2}, f32);
  auto tgt = at::zeros({M}, f32);
  auto ma = make_map(h, BM);
  auto mb = make_map(w, BN);
  auto args = plain_args(M, N, K, nullptr, N, nullptr);
  args.targets = reinterpret_cast<const long long*>(targets.data_ptr<int64_t>());
  args.lo = lo;
  args.ce_part = reinterpret_cast<float2*>(part.data_ptr<float>());
  args.ce_target = tgt.data_ptr<float>();
  launch<false, false, 3, false>(ma, mb, ma, args);
  return {part, tgt};
}

// Vocabulary-shard statistics of logits = h w^T without materialising them:
// returns (row max, target logit (0 where the target is outside [lo, lo + V)), sum exp(logit - max)).
std::vector<at::Tensor> ce_stats(at::Tensor h, at::Tensor w, at::Tensor targets, int64_t lo) {
  auto pt = ce_partials(h, w, targets, lo);
  auto part = pt[0], tgt = pt[1];
  const int64_t M = h.size(0);
  const int tiles_n = (int)part.size(1);
  auto mx = at::empty({M}, tgt.options()), se = at::empty({M}, tgt.options());
  ce_merge_kernel<<<(unsigned)((M * 32 + 255) / 256), 256, 0, stream()>>>(
      reinterpret_cast<const float2*>(part.data_ptr<float>()), (int)M, tiles_n, mx.data_ptr<float>(),
      se.data_ptr<float>());
  CQB_LAUNCH_CHECK();
  count_launch();
  return {mx, tgt, se};
}

// dlogits = (softmax(h w^T) - onehot(target - lo)) * scale as bf16 [rows, V] (scale: device scalar).
at::Tensor ce_grad_logits(at::Tensor h, at::Tensor w, at::Tensor targets, at::Tensor lse, int64_t lo,
                          at::Tensor scale) {
  check_ce(h, w, targets);
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.is_contiguous() && lse.numel() == h.size(0), "lse: fp32 [rows]");
  auto sc = scale.to(at::kFloat).reshape({1}).contiguous();
  TORCH_CHECK(sc.is_cuda(), "scale must live on the GPU");
  const int64_t M = h.size(0), K = h.size(1), N = w.size(0);
  auto y = at::empty({M, N}, h.options());
  auto ma = make_map(h, BM);
  auto mb = make_map(w, BN);
  auto args = plain_args(M, N, K, y.data_ptr(), N, nullptr);
  args.targets = reinterpret_cast<const long long*>(targets.data_ptr<int64_t>());
  args.lo = lo;
  args.ce_lse = lse.data_ptr<float>();
  args.ce_scale = sc.data_ptr<float>();
  launch<false, false, 4, false>(ma, mb, make_out_map(y), args);
  return y;
}

int gemm_status(bool reset) {
  int v = 0;
  CQB_CHECK_CUDA(cudaMemcpy(&v, status_word(), sizeof(int), cudaMemcpyDeviceToHost));
  if (reset && v) CQB_CHECK_CUDA(cudaMemset(status_word(), 0, sizeof(int)));
  return v;
}

}  // namespace cqb
