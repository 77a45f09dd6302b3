// Dense matmul on CTA pairs (tcgen05 cta_group::2) for 16-bit inputs: the
// same contraction, rounding and epilogues as gemm_kernel, with a 256x256
// output tile per pair of SMs.
//
// A cluster of two CTAs computes one tile with M=256, N=256 MMAs issued by
// rank 0: each CTA holds its own 128 rows of A and half (128 columns) of B per
// K block, and each CTA's TMEM receives its 128 rows x 256 columns.  Per SM
// that halves the B bytes loaded from L2 and read by the tensor core per FLOP
// (A 16 KB + B 16 KB per 64-deep K block instead of 16 + 32 KB), so six stages
// fit where the single-CTA kernel holds four.
//
// Synchronisation (every wait bounded, as in gemm_kernel):
//   full[s]       rank 0's barrier counts both CTAs' TMA bytes of stage s; its
//                 producer posts the expected bytes, both producers' loads
//                 complete on it (the peer's through its cluster address);
//   empty[s]      in both CTAs, one commit from rank 0's MMA thread with a
//                 two-CTA mask frees stage s in both;
//   acc_full[b]   in both CTAs, committed the same way after a tile's MMAs;
//   acc_empty[b]  rank 0's, eight arrivals: the four epilogue warps of each
//                 CTA, the peer's through its cluster address;
//   dealloc       each CTA's, one arrival from the other CTA: neither frees
//                 TMEM before both are done with it.
// A CTA never exits while something can still land in its shared memory:
// its producer waits for the final commit of every stage, its epilogue for
// every tile's accumulator, and the dealloc handshake orders the peer's last
// remote arrivals before rank 0 leaves.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "fa_internal.h"
#include "ptx.cuh"

// 1: whole-tile launches of the pair kernel start one cluster per tile and
// hand out tiles dynamically (cluster launch control); 0: one cluster per
// resident pair, tiles round robin.  Measured on B200 at 16384^3: the round
// robin lets pairs drift apart, so pairs sharing an A or B panel stop
// meeting in L2 (28 GB of DRAM traffic for 1.5 GB of operands and result);
// the dynamic order keeps the tiles in flight a window of consecutive raster
// positions.  1430 -> 1555 TF/s in short bursts and 1041 -> 1317 TF/s
// sustained under the power cap (SM clock 915 -> 1155 MHz); the TTFT shapes
// within +-2 %.
#ifndef FAB_GEMM_DYNAMIC
#define FAB_GEMM_DYNAMIC 1
#endif

namespace fab {

// kBN: 256, or 224 where that width leaves fewer idle pairs in the last wave
// (e.g. N = 3584 = 16 x 224).  B's half per CTA is kBN / 2 columns in two
// 64-column swizzle atoms (the second one partly used at 224).
template <int kBN_ = 256>
struct GemmPairCfg {
  static constexpr int kBM = 256;                     // rows per pair tile (128 per CTA)
  static constexpr int kBMc = 128;                    // rows per CTA
  static constexpr int kBN = kBN_;                    // columns per tile
  static constexpr int kBNc = kBN / 2;                // B columns each CTA holds
  static constexpr int kAccStride = 256;              // TMEM columns between the two accumulators
  static constexpr int kBK = 64;                      // one 128-byte swizzle atom of 16-bit K
  static constexpr int kStages = 6;
  static constexpr int kKInstr = 16;
  static constexpr int kABytes = kBMc * 128;          // 128 rows x one atom
  static constexpr int kBAtomN = 64;
  static constexpr int kBAtomBytes = kBK * 128;
  static constexpr int kBAtoms = (kBNc + kBAtomN - 1) / kBAtomN;
  static constexpr int kBBytes = kBAtoms * kBAtomBytes;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kThreads = 256;
  static constexpr int kTmemCols = 512;               // 2 accumulators, kAccStride apart
  // full/empty per stage, acc full/empty x 2, dealloc, then the dynamic
  // schedule's ring (full/empty x 2) and its cluster-launch-control barrier.
  static constexpr int kNumBars = 2 * kStages + 4 + 1 + 5;
  // After the barriers: TMEM address, abort flag, (unused), the ring's two
  // tile words at +8, the 16-byte scheduler response at +12.
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kNumBars * 8 + 64;
  static_assert(kNumBars % 2 == 0 && kStageBytes % 16 == 0, "scheduler response 16-byte aligned");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static_assert(kBN % 32 == 0 && kBN <= kAccStride && kBNc % 16 == 0, "tile width");
};

// ---------------------------------------------------------------- stream-K
// With T tiles on P pairs, T % P tiles would leave most pairs idle in the
// last wave.  Stream-K runs the first P * (T / P) tiles whole, round robin,
// and cuts the K blocks of the remaining tiles into P equal ranges, one per
// pair.  A tile cut this way is finished by its owner, the pair whose range
// holds its last K block: the other pairs' pieces of it (partial fp32 sums)
// wait in their workspace slots, and the owner adds them in pair order
// (deterministic) before its epilogue.  A range is at most one tile long, so
// a pair has at most one piece for another pair's tile; it computes that
// piece first, so every owner finds its pieces computed at the start of the
// stream-K phase.  No piece waits for anything, and all pairs are resident,
// so an owner's wait always ends.
enum PairItemKind : int { kItemFull = 0, kItemPart = 1, kItemOwner = 2 };

struct PairItem {
  int tile, kb0, kb1, kind;  // K blocks [kb0, kb1) of the tile
};

struct PairSched {
  int num_pairs, nkb, dp_tiles;
  long long sk_blocks;  // K blocks of the tiles after dp_tiles (0: stream-K off)
  __host__ __device__ long long begin(int pair) const { return sk_blocks * pair / num_pairs; }
};

// Item i of a pair's work (false past the last): its whole tiles, then its
// piece for another pair's tile, then its own (owned or whole) tile.
__host__ __device__ inline bool pair_item(const PairSched& S, int pair, int i, PairItem* out) {
  const int ndp = pair < S.dp_tiles ? (S.dp_tiles - 1 - pair) / S.num_pairs + 1 : 0;
  if (i < ndp) {
    *out = PairItem{pair + i * S.num_pairs, 0, S.nkb, kItemFull};
    return true;
  }
  i -= ndp;
  const long long s = S.begin(pair), e = S.begin(pair + 1);
  if (s >= e || i > 1) return false;
  const long long nkb = S.nkb;
  const int ts = static_cast<int>(s / nkb), te = static_cast<int>((e - 1) / nkb);
  PairItem a;
  a.tile = S.dp_tiles + ts;
  a.kb0 = static_cast<int>(s - ts * nkb);
  a.kb1 = static_cast<int>((e < (ts + 1) * nkb ? e : (ts + 1) * nkb) - ts * nkb);
  a.kind = a.kb1 < S.nkb ? kItemPart : (a.kb0 == 0 ? kItemFull : kItemOwner);
  if (te == ts) {
    if (i != 0) return false;
    *out = a;
    return true;
  }
  PairItem b;
  b.tile = S.dp_tiles + te;
  b.kb0 = 0;
  b.kb1 = static_cast<int>(e - te * nkb);
  b.kind = b.kb1 < S.nkb ? kItemPart : kItemFull;
  *out = i == 0 ? b : a;
  return true;
}

// The pairs whose pieces the owner of `tile` adds: [first, owner).
__host__ __device__ inline int pair_first_piece(const PairSched& S, int owner, int tile) {
  const long long start = static_cast<long long>(tile - S.dp_tiles) * S.nkb;
  int q = owner;
  while (q > 0 && S.begin(q) > start) --q;
  return q;
}

// Float4 index of (16-byte column group g, row r) in one CTA's partial tile:
// group-major, so a warp's 32 rows are 512 contiguous bytes.
__device__ __forceinline__ int part_index(int g, int r) { return g * 128 + r; }

// A piece's epilogue: the raw fp32 accumulator row into this pair's slot.
template <int kWidth>
__device__ __forceinline__ void store_partial_row(uint32_t acc, float4* slab, int r) {
#pragma unroll 1
  for (int cc = 0; cc < kWidth / 32; ++cc) {
    uint32_t v[32];
    tmem_ld32(acc + cc * 32, v);
    tmem_wait_ld();
#pragma unroll
    for (int q = 0; q < 8; ++q)
      __stcg(slab + part_index(cc * 8 + q, r), make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                                                           __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3])));
  }
}

// An owner's epilogue (plain store): accumulator + the pieces of pairs
// [first, owner) in pair order, times the row scale, stored as C's type.
template <typename Tout, int kWidth>
__device__ __forceinline__ void store_owned_row(const GemmKernelParams& p, uint32_t acc, int row, int n0,
                                                const float4* part0, int64_t part_stride, int npart, int r) {
  const float rs = (p.row_scale != nullptr && row < p.M) ? p.row_scale[row] : 1.0f;
  Tout* crow = reinterpret_cast<Tout*>(p.c) + static_cast<int64_t>(row) * p.ldc + n0;
#pragma unroll 1
  for (int cc = 0; cc < kWidth / 32; ++cc) {
    uint32_t rr[32];
    tmem_ld32(acc + cc * 32, rr);
    tmem_wait_ld();
    float v[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(rr[e]);
    for (int j = 0; j < npart; ++j) {
      const float4* src = part0 + j * part_stride;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 x = __ldcg(src + part_index(cc * 8 + q, r));
        v[4 * q] += x.x;
        v[4 * q + 1] += x.y;
        v[4 * q + 2] += x.z;
        v[4 * q + 3] += x.w;
      }
    }
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] *= rs;
    const int ncols = min(32, p.N - n0 - cc * 32);
    if (row < p.M && ncols > 0) gemm_store_chunk<Tout>(crow + cc * 32, v, ncols, p.round_f16 != 0);
  }
}

template <typename Tin, typename Tout, int kBN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(256, 1)
    gemm_pair_kernel(const __grid_constant__ GemmKernelParams p, const __grid_constant__ CUtensorMap tm_a,
                     const __grid_constant__ CUtensorMap tm_b) {
  using C = GemmPairCfg<kBN>;
  static_assert(sizeof(Tin) == 2, "CTA-pair GEMM: 16-bit inputs");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* bar_full = bars;
  uint64_t* bar_empty = bars + C::kStages;
  uint64_t* bar_acc_full = bar_empty + C::kStages;
  uint64_t* bar_acc_empty = bar_acc_full + 2;
  uint64_t* bar_dealloc = bar_acc_empty + 2;
  uint64_t* bar_sched_full = bar_dealloc + 1;    // [2]
  uint64_t* bar_sched_empty = bar_sched_full + 2;  // [2], rank 0's is the one used
  uint64_t* bar_clc = bar_sched_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_clc + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* sched_tile = reinterpret_cast<volatile int*>(tmem_slot + 8);  // [2]
  const uint32_t clc_resp = smem_u32(tmem_slot + 12);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t peer = rank ^ 1u;
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int num_pairs = static_cast<int>(gridDim.x >> 1);
  const int num_pid_m = (p.M + C::kBM - 1) / C::kBM;
  const int num_pid_n = (p.N + C::kBN - 1) / C::kBN;
  const int num_tiles = num_pid_m * num_pid_n;
  const int nkb = (p.K + C::kBK - 1) / C::kBK;
  PairSched sched;
  sched.num_pairs = num_pairs;
  sched.nkb = nkb;
  sched.dp_tiles = p.sk_part != nullptr ? p.sk_dp_tiles : num_tiles;
  sched.sk_blocks = static_cast<long long>(num_tiles - sched.dp_tiles) * nkb;
  if (sched.sk_blocks < num_pairs) {
    // An empty range would leave a gap in an owner's run of pieces: whole tiles.
    sched.dp_tiles = num_tiles;
    sched.sk_blocks = 0;
  }
  // Item i of this pair.  Static schedule: pair_item.  Dynamic (whole tiles,
  // one cluster launched per tile): item 0 is the cluster's own tile, item
  // i >= 1 the tile rank 0's scheduler thread took from a cluster that had
  // not started, published in both CTAs' two-slot ring (slot (i-1) % 2); -1
  // ends the run.  Epilogue warps read last, so they free the slot (`epi`,
  // called by whole warps).
  const bool dyn = p.dyn_sched != 0;
  auto next_item = [&](int i, PairItem* out, bool epi) -> bool {
    if (!dyn) return pair_item(sched, pair, i, out);
    int tile = pair;
    if (i > 0) {
      const int q = i - 1, s = q & 1;
      bool got = mbar_wait_cluster(bar_sched_full + s, (q >> 1) & 1, abort_flag, kDevTimeoutSched);
      if (epi) got = __all_sync(0xffffffffu, got) != 0;
      if (!got) return false;
      tile = sched_tile[s];
      if (epi) {
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive_cluster(mapa_shared(smem_u32(bar_sched_empty + s), 0));
      }
    }
    if (tile < 0 || tile >= num_tiles) return false;
    *out = PairItem{tile, 0, nkb, kItemFull};
    return true;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(bar_full + s, 1);
      mbar_init(bar_empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_acc_full + b, 1);
      mbar_init(bar_acc_empty + b, 8);  // 4 epilogue warps x 2 CTAs (rank 0's is the one used)
    }
    mbar_init(bar_dealloc, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_sched_full + b, 1);
      mbar_init(bar_sched_empty + b, 8);  // 4 epilogue warps x 2 CTAs
    }
    mbar_init(bar_clc, 1);
    *abort_flag = *reinterpret_cast<volatile int*>(&g_fab_device_error) != 0 ? 1 : 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, C::kTmemCols);
    tmem_relinquish_pair();
  }
  // Both CTAs' barriers exist and both TMEM allocations are made before
  // either CTA touches the other's shared memory.
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const bool skip = *abort_flag != 0;

  if (!skip && warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    int it = 0;
    bool ok = true;
    PairItem w;
    for (int i = 0; ok && next_item(i, &w, false); ++i) {
      int pm, pn;
      gemm_tile_coords(w.tile, num_pid_m, num_pid_n, p.group_m, &pm, &pn);
      const int m0 = pm * C::kBM + static_cast<int>(rank) * C::kBMc;
      const int n0 = pn * C::kBN + static_cast<int>(rank) * C::kBNc;
      for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
        const int s = it % C::kStages;
        const uint32_t ph = (it / C::kStages) & 1;
        if (!(ok = mbar_wait(bar_empty + s, ph ^ 1, abort_flag, kDevTimeoutEmpty))) break;
        uint8_t* st = smem + s * C::kStageBytes;
        if (rank == 0) mbar_arrive_expect_tx(bar_full + s, 2 * C::kStageBytes);
        const uint32_t full_s = mapa_shared(smem_u32(bar_full + s), 0);  // rank 0's full[s]
        tma_load_2d_pair(st, &tm_a, full_s, kb * C::kBK, m0);
#pragma unroll
        for (int a = 0; a < C::kBAtoms; ++a)
          tma_load_2d_pair(st + C::kABytes + a * C::kBAtomBytes, &tm_b, full_s, n0 + a * C::kBAtomN, kb * C::kBK);
      }
    }
    // Every stage's last use is over (its data landed and the MMAs that read
    // it completed) once its final release has arrived here.
    volatile int no_abort = 0;
    for (int x = max(0, it - C::kStages); x < it; ++x)
      mbar_wait(bar_empty + (x % C::kStages), (x / C::kStages) & 1, &no_abort, kDevTimeoutTeardown);
  } else if (!skip && warp == 1 && lane == 0 && rank == 0) {
    // ------------------------------------------------------------ MMA issuer (rank 0, for the pair)
    constexpr uint32_t idesc = umma_idesc(GemmFmt<Tin>::kFmt, C::kBM, C::kBN, 0, 1);
    constexpr uint32_t kHiA = umma_desc_hi(1024, kLayoutSw128);
    constexpr uint32_t kHiB = umma_desc_hi(1024, kLayoutSw128);
    const uint32_t a_lo0 = umma_desc_lo(smem_u32(smem), 16);
    const uint32_t b_lo0 = umma_desc_lo(smem_u32(smem) + C::kABytes, C::kBAtomBytes);
    constexpr uint16_t kBoth = 0x3;
    int it = 0, tcount = 0;
    bool ok = true;
    PairItem w;
    for (int i = 0; ok && next_item(i, &w, false); ++i, ++tcount) {
      const int buf = tcount & 1;
      const uint32_t use = tcount >> 1;
      if (!(ok = mbar_wait(bar_acc_empty + buf, (use & 1) ^ 1, abort_flag, kDevTimeoutAcc))) break;
      tc_fence_after();
      const uint32_t d = tmem + buf * C::kAccStride;
      for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
        const int s = it % C::kStages;
        const uint32_t ph = (it / C::kStages) & 1;
        if (!(ok = mbar_wait(bar_full + s, ph, abort_flag, kDevTimeoutKV))) break;
        tc_fence_after();
        uint32_t a_lo = a_lo0 + s * (C::kStageBytes >> 4);
        uint32_t b_lo = b_lo0 + s * (C::kStageBytes >> 4);
        asm volatile("" : "+r"(a_lo), "+r"(b_lo));
#pragma unroll
        for (int kk = 0; kk < C::kBK / C::kKInstr; ++kk) {
          const uint64_t ad = umma_desc_join(a_lo + ((kk * 32) >> 4), kHiA);
          const uint64_t bd = umma_desc_join(b_lo + ((kk * C::kKInstr * 128) >> 4), kHiB);
          mma_ss_f16_pair(d, ad, bd, idesc, (kb > w.kb0 || kk > 0) ? 1u : 0u);
        }
        mma_commit_pair(bar_empty + s, kBoth);
      }
      if (!ok) break;
      mma_commit_pair(bar_acc_full + buf, kBoth);
    }
  } else if (!skip && dyn && warp == 2 && lane == 0 && rank == 0) {
    // ------------------------------------------------------------ tile scheduler (rank 0, dynamic)
    // Takes the pair's next tile from a cluster of this grid that has not
    // started (cluster launch control: the hardware hands out clusters in
    // launch order, so the tiles in flight stay a window of consecutive
    // raster positions) while the current one runs, and publishes it in
    // both CTAs' ring.  A slot is reused once all eight epilogue warps read
    // it.  Every request's response lands before this thread moves on.
    volatile int no_abort = 0;
    for (int q = 0;; ++q) {
      const int s = q & 1;
      if (q >= 2 && !mbar_wait_cluster(bar_sched_empty + s, ((q - 2) >> 1) & 1, abort_flag, kDevTimeoutSched)) break;
      mbar_arrive_expect_tx(bar_clc, 16);
      clc_try_cancel(clc_resp, bar_clc);
      if (!mbar_wait(bar_clc, q & 1, &no_abort, kDevTimeoutSched)) break;
      const int x = clc_first_cta_x(clc_resp);
      const int tile = x < 0 ? -1 : (x >> 1);
      sched_tile[s] = tile;
      st_cluster_u32(mapa_shared(smem_u32(const_cast<int*>(sched_tile + s)), 1), static_cast<uint32_t>(tile));
      mbar_arrive(bar_sched_full + s);
      mbar_arrive_cluster(mapa_shared(smem_u32(bar_sched_full + s), 1));
      if (tile < 0) break;
    }
  } else if (!skip && warp >= 4) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(wq * 32) << 16;
    // One partial tile per pair and CTA: kBN / 4 16-byte groups x 128 rows.
    constexpr int64_t kSlab = static_cast<int64_t>(C::kBN / 4) * 128;
    int tcount = 0;
    PairItem w;
    for (int i = 0; next_item(i, &w, true); ++i, ++tcount) {
      const int buf = tcount & 1;
      const uint32_t use = tcount >> 1;
      if (!mbar_wait_warp(bar_acc_full + buf, use & 1, abort_flag, kDevTimeoutAcc)) break;
      tc_fence_after();
      int pm, pn;
      gemm_tile_coords(w.tile, num_pid_m, num_pid_n, p.group_m, &pm, &pn);
      const uint32_t acc = tmem + lane_base + buf * C::kAccStride;
      const int row = pm * C::kBM + static_cast<int>(rank) * C::kBMc + r;
      if (w.kind == kItemFull) {
        gemm_store_tile_row<Tout, kBN>(p, acc, row, pn * C::kBN);
      } else if (w.kind == kItemPart) {
        // This pair's slot: every lane's row, then one flag per warp, set
        // after all 32 rows are visible at GPU scope.
        float4* slab = reinterpret_cast<float4*>(p.sk_part) + (static_cast<int64_t>(pair) * 2 + rank) * kSlab;
        store_partial_row<kBN>(acc, slab, r);
        __threadfence();
        __syncwarp();
        if (lane == 0) st_release_gpu(p.sk_flags + (pair * 2 + static_cast<int>(rank)) * 4 + wq, 1);
      } else {
        // Owner: wait (bounded) for every piece of this tile, add them in
        // pair order, store, and clear the pieces' flags for the next call.
        const int first = pair_first_piece(sched, pair, w.tile);
        bool got = true;
        if (lane == 0)
          for (int q = first; got && q < pair; ++q)
            got = wait_flag_set(p.sk_flags + (q * 2 + static_cast<int>(rank)) * 4 + wq, abort_flag,
                                kDevTimeoutPartial);
        got = __shfl_sync(0xffffffffu, got ? 1 : 0, 0) != 0;
        if (got) {
          const float4* part0 =
              reinterpret_cast<const float4*>(p.sk_part) + (static_cast<int64_t>(first) * 2 + rank) * kSlab;
          store_owned_row<Tout, kBN>(p, acc, row, pn * C::kBN, part0, 2 * kSlab, pair - first, r);
          __syncwarp();
          if (lane == 0)
            for (int q = first; q < pair; ++q) p.sk_flags[(q * 2 + static_cast<int>(rank)) * 4 + wq] = 0;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(bar_acc_empty + buf), 0));  // rank 0's
    }
  }

  // ------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    if (lane == 0) {
      // Tell the other CTA this one is done with the pair's TMEM and smem,
      // then wait (bounded) for the same word from it.
      mbar_arrive_cluster(mapa_shared(smem_u32(bar_dealloc), peer));
      volatile int no_abort = 0;
      mbar_wait(bar_dealloc, 0, &no_abort, kDevTimeoutTeardown);
      if (*abort_flag) {
        // After a failed wait MMAs may still be running: let them finish
        // (bounded) before the accumulators are released.
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 20000u) __nanosleep(1000);
      }
    }
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem, C::kTmemCols);
  }
}

// Resident clusters (pairs) of one launch of the kBN-wide kernel: an owner
// waits for other pairs' pieces, so a stream-K grid never exceeds this.
template <typename Tin, typename Tout, int kBN>
static int gemm_pair_capacity() {
  using C = GemmPairCfg<kBN>;
  static int cached = -1;
  if (cached >= 0) return cached;
  auto kern = gemm_pair_kernel<Tin, Tout, kBN>;
  if (ensure_smem_attr(reinterpret_cast<const void*>(kern), C::kSmemBytes)) return 0;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * 64);
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, reinterpret_cast<const void*>(kern), &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  cached = n;
  return n;
}

// How a CTA-pair GEMM is laid out: tile width, pairs in the grid and the
// tiles run whole (all of them without stream-K).
struct PairChoice {
  int bn;
  int pairs;
  int dp_tiles;
  int tiles;
  bool stream_k;
};

// Whole tiles with more tiles than resident pairs take the dynamic schedule.
static bool pair_dynamic(const PairChoice& c) { return FAB_GEMM_DYNAMIC != 0 && !c.stream_k && c.tiles > c.pairs; }

static long long pair_tiles(const GemmLaunch& L, int bn) {
  return static_cast<long long>((L.M + 255) / 256) * ((L.N + bn - 1) / bn);
}

// Stream-K workspace of a layout: one flag word per pair, CTA and epilogue
// warp (a 256-byte aligned block), then one fp32 partial tile per pair and CTA.
static size_t pair_sk_flag_bytes(int pairs) { return (static_cast<size_t>(pairs) * 8 * sizeof(int) + 255) / 256 * 256; }
static size_t pair_sk_bytes(const PairChoice& c) {
  return c.stream_k ? pair_sk_flag_bytes(c.pairs) + static_cast<size_t>(c.pairs) * 2 * 128 * c.bn * sizeof(float) : 0;
}

// Whole-tile layout with the fewest idle pair-slots: tiles 256 wide, or 224
// where that leaves fewer pairs idle in the last wave and K is short (a
// 224-wide tile's B halves start off the 128-byte line, which costs L2
// traffic in long main loops; measured on B200: N = 3584 gains 7 % at
// K = 3584, loses 2-7 % at K = 18944).  The SwiGLU and bias + RoPE
// epilogues need 256-wide tiles.
static PairChoice gemm_pair_whole(const GemmLaunch& L, int half_sms) {
  PairChoice best{256, 0, 0, 0, false};
  double best_cost = 1e300;
  for (int bn : {256, 224}) {
    if (bn == 224 && (gemm_fixed_width(L) || L.K > 8192)) continue;
    const long long tiles = pair_tiles(L, bn);
    if (tiles <= 0 || half_sms <= 0) continue;
    const int pairs = static_cast<int>(tiles < half_sms ? tiles : half_sms);
    const double cost = static_cast<double>((tiles + pairs - 1) / pairs) * bn;
    if (cost < best_cost) {
      best_cost = cost;
      best = PairChoice{bn, pairs, static_cast<int>(tiles), static_cast<int>(tiles), false};
    }
  }
  return best;
}

// The chosen layout.  Stream-K (256-wide tiles, plain store epilogue, deep
// K) is taken when the tiles leave part of the last wave idle and the estimate --
// tiles / pairs waves plus ~4 % for writing and adding the pieces -- beats
// the best whole-tile layout; it also needs at least two K blocks per pair
// and ranges of at least a quarter tile (so an owner adds a handful of
// pieces at most), and a workspace from the caller (with_workspace).
template <typename Tin, typename Tout>
static PairChoice gemm_pair_choice(const GemmLaunch& L, bool with_workspace) {
  const int half_sms = num_sms() / 2;
  PairChoice best = gemm_pair_whole(L, half_sms);
#ifndef FAB_GEMM_NO_STREAMK
  if (!with_workspace || gemm_fixed_width(L) || best.pairs <= 0) return best;
  const double whole_cost = static_cast<double>((best.tiles + best.pairs - 1) / best.pairs) * best.bn;
  const long long tiles = pair_tiles(L, 256);
  const int cap = gemm_pair_capacity<Tin, Tout, 256>();
  const int P = cap < half_sms ? cap : half_sms;
  const long long nkb = (L.K + 63) / 64;
  // K >= 8192 only: measured on B200, stream-K beat whole tiles at the TTFT
  // down_proj (K = 18944: 1386 -> 1512 TF/s) but lost 3-5 % at K = 3584 and
  // 4096, where its fixed costs (writing and adding the pieces, the owners'
  // tails) weigh more, and where whole tiles' part-idle last wave runs the
  // busy SMs at a higher clock under the power cap.
  if (P >= 1 && tiles > P && tiles % P != 0 && L.K >= 8192) {
    const long long dp = tiles / P * P;
    const long long sk_blocks = (tiles - dp) * nkb;
    const double sk_cost = static_cast<double>(tiles) / P * 256 * 1.04;
    if (sk_blocks >= 2LL * P && 4 * sk_blocks >= P * nkb && sk_cost < whole_cost)
      best = PairChoice{256, P, static_cast<int>(dp), static_cast<int>(tiles), true};
  }
#endif
  return best;
}

template <typename Tin, typename Tout>
static PairChoice gemm_pair_layout(const GemmLaunch& L) {
  PairChoice c = gemm_pair_choice<Tin, Tout>(L, true);
  if (c.stream_k && (L.workspace == nullptr || (reinterpret_cast<uintptr_t>(L.workspace) & 255u) != 0 ||
                     L.workspace_bytes < pair_sk_bytes(c)))
    c = gemm_pair_whole(L, num_sms() / 2);
  return c;
}

template <typename Tin, typename Tout, int kBN>
static int launch_gemm_pair_w(const GemmLaunch& L, const PairChoice& c, cudaStream_t stream) {
  using C = GemmPairCfg<kBN>;
  auto kern = gemm_pair_kernel<Tin, Tout, kBN>;
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), C::kSmemBytes);
  if (rc) return rc;
  const CUtensorMapDataType dt =
      L.in_dtype == kDtypeBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ta, tb;
  rc = make_2d_map(&ta, L.a, dt, 2, L.K, L.M, L.lda, C::kBK, C::kBMc, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_2d_map(&tb, L.b, dt, 2, L.N, L.K, L.ldb, C::kBAtomN, C::kBK, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  GemmKernelParams kp;
  kp.c = L.c;
  kp.ldc = L.ldc;
  kp.M = L.M;
  kp.N = L.N;
  kp.K = L.K;
  kp.group_m = L.group_m > 0 ? L.group_m : 8;
  kp.round_f16 = L.round_f16;
  kp.swiglu = L.swiglu;
  kp.bias_rope = L.bias_rope;
  kp.rope_cols = L.rope_cols;
  kp.head_dim = L.head_dim;
  kp.bias = L.bias;
  kp.rope_cos = L.rope_cos;
  kp.rope_sin = L.rope_sin;
  kp.row_scale = L.row_scale;
  kp.sk_dp_tiles = c.tiles;
  kp.sk_part = nullptr;
  kp.sk_flags = nullptr;
  kp.dyn_sched = 0;
  if (c.tiles <= 0) return 0;
  if (c.pairs < 1) return kErrLaunch;
  int clusters = c.pairs;
  if (c.stream_k) {
    uint8_t* ws = static_cast<uint8_t*>(L.workspace);
    kp.sk_dp_tiles = c.dp_tiles;
    kp.sk_flags = reinterpret_cast<int*>(ws);
    kp.sk_part = reinterpret_cast<float*>(ws + pair_sk_flag_bytes(c.pairs));
  } else if (pair_dynamic(c)) {
    kp.dyn_sched = 1;
    clusters = c.tiles;
  }
  kern<<<2 * clusters, C::kThreads, C::kSmemBytes, stream>>>(kp, ta, tb);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrLaunch;
}

template <typename Tin, typename Tout>
static int launch_gemm_pair(const GemmLaunch& L, cudaStream_t stream) {
  const PairChoice c = gemm_pair_layout<Tin, Tout>(L);
  if (c.bn == 224) return launch_gemm_pair_w<Tin, Tout, 224>(L, c, stream);
  return launch_gemm_pair_w<Tin, Tout, 256>(L, c, stream);
}

// The layout the launch for L takes (the capacity query is per tile width,
// the same for every output type).
static PairChoice gemm_pair_layout_any(const GemmLaunch& L) {
  return L.in_dtype == kDtypeBF16 ? gemm_pair_layout<__nv_bfloat16, __nv_bfloat16>(L)
                                  : gemm_pair_layout<__half, __half>(L);
}

// Stream-K workspace bytes the launch for L would use with a workspace.
static size_t gemm_pair_workspace(const GemmLaunch& L) {
  if (L.in_dtype != kDtypeBF16 && L.in_dtype != kDtypeF16) return 0;
  const PairChoice c = L.in_dtype == kDtypeBF16 ? gemm_pair_choice<__nv_bfloat16, __nv_bfloat16>(L, true)
                                                : gemm_pair_choice<__half, __half>(L, true);
  return pair_sk_bytes(c);
}

// The pair kernel serves 16-bit inputs when the problem fills at least one
// wave of pairs; smaller problems keep the single-CTA kernel's finer tiles.
static bool gemm_use_pair(const GemmLaunch& L) {
#ifdef FAB_GEMM_NO_PAIR
  return false;
#else
  if (L.in_dtype != kDtypeBF16 && L.in_dtype != kDtypeF16) return false;
  const int sms = num_sms();
  const long long tiles = static_cast<long long>((L.M + 255) / 256) * ((L.N + 255) / 256);
  return sms >= 2 && tiles >= sms / 2;
#endif
}

}  // namespace fab
