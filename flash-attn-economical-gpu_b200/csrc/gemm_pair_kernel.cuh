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
  static constexpr int kNumBars = 2 * kStages + 4 + 1;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kNumBars * 8 + 64;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static_assert(kBN % 32 == 0 && kBN <= kAccStride && kBNc % 16 == 0, "tile width");
};

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
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_dealloc + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

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
    for (int t = pair; ok && t < num_tiles; t += num_pairs) {
      int pm, pn;
      gemm_tile_coords(t, num_pid_m, num_pid_n, p.group_m, &pm, &pn);
      const int m0 = pm * C::kBM + static_cast<int>(rank) * C::kBMc;
      const int n0 = pn * C::kBN + static_cast<int>(rank) * C::kBNc;
      for (int kb = 0; kb < nkb; ++kb, ++it) {
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
    for (int t = pair; ok && t < num_tiles; t += num_pairs, ++tcount) {
      const int buf = tcount & 1;
      const uint32_t use = tcount >> 1;
      if (!(ok = mbar_wait(bar_acc_empty + buf, (use & 1) ^ 1, abort_flag, kDevTimeoutAcc))) break;
      tc_fence_after();
      const uint32_t d = tmem + buf * C::kAccStride;
      for (int kb = 0; kb < nkb; ++kb, ++it) {
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
          mma_ss_f16_pair(d, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit_pair(bar_empty + s, kBoth);
      }
      if (!ok) break;
      mma_commit_pair(bar_acc_full + buf, kBoth);
    }
  } else if (!skip && warp >= 4) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(wq * 32) << 16;
    int tcount = 0;
    for (int t = pair; t < num_tiles; t += num_pairs, ++tcount) {
      const int buf = tcount & 1;
      const uint32_t use = tcount >> 1;
      if (!mbar_wait_warp(bar_acc_full + buf, use & 1, abort_flag, kDevTimeoutAcc)) break;
      tc_fence_after();
      int pm, pn;
      gemm_tile_coords(t, num_pid_m, num_pid_n, p.group_m, &pm, &pn);
      gemm_store_tile_row<Tout, kBN>(p, tmem + lane_base + buf * C::kAccStride,
                                     pm * C::kBM + static_cast<int>(rank) * C::kBMc + r, pn * C::kBN);
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

// Pair tiles (256 x kBN) in a grid of up to one pair per two SMs.
template <typename Tin, typename Tout, int kBN>
static int launch_gemm_pair_w(const GemmLaunch& L, cudaStream_t stream) {
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
  const int tiles = ((L.M + C::kBM - 1) / C::kBM) * ((L.N + C::kBN - 1) / C::kBN);
  if (tiles <= 0) return 0;
  const int sms = num_sms();
  if (sms < 2) return kErrLaunch;
  const int pairs = tiles < sms / 2 ? tiles : sms / 2;
  kern<<<2 * pairs, C::kThreads, C::kSmemBytes, stream>>>(kp, ta, tb);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrLaunch;
}

// Relative time of a pair-tile width: full waves of pairs times the work of
// one tile (proportional to its width).
static long long gemm_pair_cost(const GemmLaunch& L, int bn, int pairs) {
  const long long tiles = static_cast<long long>((L.M + 255) / 256) * ((L.N + bn - 1) / bn);
  return (tiles + pairs - 1) / pairs * bn;
}

template <typename Tin, typename Tout>
static int launch_gemm_pair(const GemmLaunch& L, cudaStream_t stream) {
  const int pairs = num_sms() / 2;
  // 224-wide tiles only where they leave less of the last wave idle and K is
  // short: a 224-wide tile's B halves start off the 128-byte line, which
  // costs L2 traffic in long main loops (measured on B200: N = 3584 gains 7 %
  // at K = 3584, loses 2-7 % at K = 18944).  The SwiGLU epilogue pairs
  // 64-column gate/up blocks within 256-wide tiles.
  if (!gemm_fixed_width(L) && pairs > 0 && L.K <= 8192 && gemm_pair_cost(L, 224, pairs) < gemm_pair_cost(L, 256, pairs))
    return launch_gemm_pair_w<Tin, Tout, 224>(L, stream);
  return launch_gemm_pair_w<Tin, Tout, 256>(L, stream);
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
