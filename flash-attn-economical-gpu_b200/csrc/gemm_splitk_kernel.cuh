// Split-K matmul for problems with few output tiles and a deep K (e.g. a few
// rows times a large weight): 16-bit inputs, the same 128x256 tiles,
// rounding and stores as gemm_kernel.
//
// A cluster of kSplit CTAs computes one output tile.  CTA r of the cluster
// runs the K blocks [r*nkb/kSplit, (r+1)*nkb/kSplit) through the usual TMA
// ring into its own TMEM accumulator.  The partial sums then meet in
// distributed shared memory: column slice q (256/kSplit columns) of every
// CTA's partial goes to CTA q, which adds the kSplit slices in rank order
// (deterministic) and stores them.  No global workspace and no counters, so
// calls on different streams or inside CUDA graphs need nothing extra.
//
// Order of events, every wait bounded except the two cluster barriers, which
// every thread of the cluster reaches on every path:
//   1. producer / MMA / epilogue as in gemm_kernel, one tile, one accumulator;
//   2. the epilogue warps wait for the accumulator (all MMAs done, so the
//      stage memory is idle), then cluster barrier 1;
//   3. each epilogue warp sends its 32 rows' slices to their owners' receive
//      buffers (which reuse the stage memory), 32x32 blocks at a time,
//      transposed through its own stage memory so the remote stores write
//      whole 128-byte row pieces; then cluster barrier 2;
//   4. each epilogue thread adds the slices of its row it owns and stores.
// After barrier 2 no CTA touches another's shared memory, so any can exit.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "fa_internal.h"
#include "ptx.cuh"

namespace fab {

template <typename Tin, typename Tout, int kSplit>
__global__ void __cluster_dims__(kSplit, 1, 1) __launch_bounds__(256, 1)
    gemm_splitk_kernel(const __grid_constant__ GemmKernelParams p, const __grid_constant__ CUtensorMap tm_a,
                       const __grid_constant__ CUtensorMap tm_b) {
  using C = GemmCfg<sizeof(Tin)>;
  static_assert(sizeof(Tin) == 2, "16-bit inputs");
  constexpr int kW = C::kBN / kSplit;  // columns each CTA adds up and stores
  constexpr int kRowF = kW + 4;        // receive row stride in floats: the 16-byte pad spreads rows over banks
  static_assert(kW % 32 == 0, "slices of whole 32-column chunks");
  constexpr int kRecvBytes = kSplit * C::kBM * kRowF * 4;
  constexpr int kStageRowF = 36;  // warp transpose block: 32 rows of 32 floats + 16-byte pad
  static_assert(kRecvBytes + 4 * 32 * kStageRowF * 4 <= C::kStages * C::kStageBytes,
                "receive buffers and transpose blocks fit the stages");
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint64_t* bar_full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* bar_empty = bar_full + C::kStages;
  uint64_t* bar_acc = bar_empty + C::kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_acc + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // [kSplit source ranks][128 rows][kRowF] fp32, over the idle stages.
  float* recv = reinterpret_cast<float*>(smem);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = static_cast<int>(cluster_ctarank());
  const int num_pid_m = (p.M + C::kBM - 1) / C::kBM;
  const int num_pid_n = (p.N + C::kBN - 1) / C::kBN;
  int pm, pn;
  gemm_tile_coords(static_cast<int>(blockIdx.x) / kSplit, num_pid_m, num_pid_n, p.group_m, &pm, &pn);
  const int nkb = (p.K + C::kBK - 1) / C::kBK;
  const int kb0 = nkb * rank / kSplit;
  const int kb1 = nkb * (rank + 1) / kSplit;  // non-empty: the launcher keeps nkb >= kSplit

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(bar_full + s, 1);
      mbar_init(bar_empty + s, 1);
    }
    mbar_init(bar_acc, 1);
    *abort_flag = *reinterpret_cast<volatile int*>(&g_fab_device_error) != 0 ? 1 : 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const bool skip = *abort_flag != 0;
  bool acc_ok = false;

  if (!skip && warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    const int m0 = pm * C::kBM, n0 = pn * C::kBN;
    int it = 0;
    for (int kb = kb0; kb < kb1; ++kb, ++it) {
      const int s = it % C::kStages;
      const uint32_t ph = (it / C::kStages) & 1;
      if (!mbar_wait(bar_empty + s, ph ^ 1, abort_flag, kDevTimeoutEmpty)) break;
      uint8_t* st = smem + s * C::kStageBytes;
      mbar_arrive_expect_tx(bar_full + s, C::kStageBytes);
      tma_load_2d(st, &tm_a, bar_full + s, kb * C::kBK, m0);
#pragma unroll
      for (int a = 0; a < C::kBN / C::kBAtomN; ++a)
        tma_load_2d(st + C::kABytes + a * C::kBAtomBytes, &tm_b, bar_full + s, n0 + a * C::kBAtomN, kb * C::kBK);
    }
    // Wait (bounded) for the last copy issued into every stage.
    volatile int no_abort = 0;
    for (int x = max(0, it - C::kStages); x < it; ++x)
      mbar_wait(bar_full + (x % C::kStages), (x / C::kStages) & 1, &no_abort, kDevTimeoutTeardown);
  } else if (!skip && warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = umma_idesc(GemmFmt<Tin>::kFmt, C::kBM, C::kBN, 0, 1);
    constexpr uint32_t kHiA = umma_desc_hi(1024, kLayoutSw128);
    constexpr uint32_t kHiB = umma_desc_hi(1024, kLayoutSw128);
    const uint32_t a_lo0 = umma_desc_lo(smem_u32(smem), 16);
    const uint32_t b_lo0 = umma_desc_lo(smem_u32(smem) + C::kABytes, C::kBAtomBytes);
    int it = 0;
    bool ok = true;
    for (int kb = kb0; kb < kb1; ++kb, ++it) {
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
        mma_ss_f16(tmem, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
      }
      mma_commit(bar_empty + s);
    }
    // Also after a failed wait: the commit tracks the MMAs already issued, so
    // the epilogue's wait ends once nothing reads the stages any more.
    mma_commit(bar_acc);
  } else if (!skip && warp >= 4) {
    acc_ok = mbar_wait_warp(bar_acc, 0, abort_flag, kDevTimeoutAcc);
    tc_fence_after();
  }
  __syncwarp();
  // Barrier 1: every CTA's accumulator is final and its stage memory idle.
  cluster_sync_all();
  const int wq = warp & 3;
  const int r = wq * 32 + lane;  // tile row of this epilogue thread
  if (warp >= 4 && acc_ok) {
    // Each 32-column chunk of the warp's 32 rows goes through a warp-private
    // block of this CTA's (idle) stage memory, so that every remote store
    // instruction writes four whole 128-byte row pieces rather than 32
    // scattered 16-byte ones.
    const uint32_t lane_base = static_cast<uint32_t>(wq * 32) << 16;
    float* blk = reinterpret_cast<float*>(smem + kRecvBytes) + wq * 32 * kStageRowF;
#pragma unroll 1
    for (int cc = 0; cc < C::kBN / 32; ++cc) {
      uint32_t rr[32];
      tmem_ld32(tmem + lane_base + cc * 32, rr);
      tmem_wait_ld();
      float4* mine = reinterpret_cast<float4*>(blk + lane * kStageRowF);
#pragma unroll
      for (int e = 0; e < 8; ++e)
        mine[e] = make_float4(__uint_as_float(rr[4 * e]), __uint_as_float(rr[4 * e + 1]),
                              __uint_as_float(rr[4 * e + 2]), __uint_as_float(rr[4 * e + 3]));
      __syncwarp();
      const int owner = (cc * 32) / kW;
      const uint32_t dst = mapa_shared(smem_u32(recv + (rank * C::kBM + wq * 32) * kRowF + (cc * 32) % kW),
                                       static_cast<uint32_t>(owner));
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int br = 4 * i + (lane >> 3);  // block row; lane & 7 picks its 16-byte piece
        const float4 x = reinterpret_cast<const float4*>(blk + br * kStageRowF)[lane & 7];
        st_cluster_v4(dst + (br * kRowF + (lane & 7) * 4) * 4, x.x, x.y, x.z, x.w);
      }
      __syncwarp();
    }
  }
  __syncwarp();
  // Barrier 2: every slice has landed with its owner.
  cluster_sync_all();
  if (warp >= 4 && acc_ok) {
    const int row = pm * C::kBM + r;
#pragma unroll 1
    for (int ch = 0; ch < kW / 32; ++ch) {
      float v[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) v[e] = 0.f;
#pragma unroll 1
      for (int src = 0; src < kSplit; ++src) {
        const float4* in = reinterpret_cast<const float4*>(recv + (src * C::kBM + r) * kRowF + ch * 32);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float4 x = in[e];
          v[4 * e] += x.x;
          v[4 * e + 1] += x.y;
          v[4 * e + 2] += x.z;
          v[4 * e + 3] += x.w;
        }
      }
      const int col = pn * C::kBN + rank * kW + ch * 32;
      const int ncols = min(32, p.N - col);
      if (row < p.M && ncols > 0)
        gemm_store_chunk<Tout>(reinterpret_cast<Tout*>(p.c) + static_cast<int64_t>(row) * p.ldc + col, v, ncols,
                               p.round_f16 != 0);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kBN);
  }
}

// Resident clusters of one kSplit launch (0 if the query fails).
template <typename Tin, typename Tout, int kSplit>
static int gemm_splitk_capacity() {
  using C = GemmCfg<sizeof(Tin)>;
  static int cached = -1;
  if (cached >= 0) return cached;
  auto kern = gemm_splitk_kernel<Tin, Tout, kSplit>;
  if (ensure_smem_attr(reinterpret_cast<const void*>(kern), C::kSmemBytes)) return 0;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(kSplit * 64);
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

template <typename Tin, typename Tout, int kSplit>
static int launch_gemm_splitk_k(const GemmLaunch& L, cudaStream_t stream) {
  using C = GemmCfg<sizeof(Tin)>;
  auto kern = gemm_splitk_kernel<Tin, Tout, kSplit>;
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), C::kSmemBytes);
  if (rc) return rc;
  const CUtensorMapDataType dt = L.in_dtype == kDtypeBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                          : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ta, tb;
  rc = make_2d_map(&ta, L.a, dt, 2, L.K, L.M, L.lda, C::kBK, C::kBM, CU_TENSOR_MAP_SWIZZLE_128B);
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
  kp.swiglu = 0;
  kp.bias_rope = 0;
  kp.rope_cols = 0;
  kp.head_dim = 0;
  kp.bias = kp.rope_cos = kp.rope_sin = nullptr;
  kp.row_scale = nullptr;
  kp.sk_dp_tiles = 0;
  kp.sk_part = nullptr;
  kp.sk_flags = nullptr;
  kp.dyn_sched = 0;
  const long long tiles = static_cast<long long>((L.M + C::kBM - 1) / C::kBM) * ((L.N + C::kBN - 1) / C::kBN);
  kern<<<static_cast<unsigned>(tiles * kSplit), C::kThreads, C::kSmemBytes, stream>>>(kp, ta, tb);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrLaunch;
}

// How many CTAs share each tile's K: the largest of 8, 4, 2 whose clusters all
// fit on the GPU at once.  Splitting saves each CTA (1 - 1/kSplit) of its
// 48 KB per K block of loads (a single CTA ingests ~100 GB/s) and costs it
// (1 - 1/kSplit) x 128 KB of partial sums over distributed shared memory,
// which moves only ~16-20 GB/s per SM on B200: it pays from about 48 K blocks
// (K >= 3072 for 16-bit inputs), and only with few tiles (at most a quarter
// of the SMs; more tiles already spread the loads).  1 (no split) otherwise,
// and for tf32, SwiGLU or K = 0.
constexpr int kSplitMinKBlocks = 48;

template <typename Tin, typename Tout>
static int gemm_splitk_factor(const GemmLaunch& L) {
  using C = GemmCfg<2>;
  // The split kernel has no row-scaled epilogue: such GEMMs are not split.
  if (L.in_dtype == kDtypeF32 || gemm_fixed_width(L) || L.row_scale != nullptr || L.K <= 0) return 1;
  const long long tiles = static_cast<long long>((L.M + C::kBM - 1) / C::kBM) * ((L.N + C::kBN - 1) / C::kBN);
  const int nkb = (L.K + C::kBK - 1) / C::kBK;
  const int sms = num_sms();
  if (sms <= 0 || 4 * tiles > sms || nkb < kSplitMinKBlocks) return 1;
  if (tiles <= gemm_splitk_capacity<Tin, Tout, 8>()) return 8;
  if (tiles <= gemm_splitk_capacity<Tin, Tout, 4>()) return 4;
  if (tiles <= gemm_splitk_capacity<Tin, Tout, 2>()) return 2;
  return 1;
}

// Split-K launch if it pays for this shape (*taken says whether it did).
template <typename Tin, typename Tout>
static int launch_gemm_splitk(const GemmLaunch& L, cudaStream_t stream, bool* taken) {
  *taken = true;
#ifndef FAB_GEMM_NO_SPLITK
  switch (gemm_splitk_factor<Tin, Tout>(L)) {
    case 8:
      return launch_gemm_splitk_k<Tin, Tout, 8>(L, stream);
    case 4:
      return launch_gemm_splitk_k<Tin, Tout, 4>(L, stream);
    case 2:
      return launch_gemm_splitk_k<Tin, Tout, 2>(L, stream);
    default:
      break;
  }
#endif
  *taken = false;
  return 0;
}

}  // namespace fab
