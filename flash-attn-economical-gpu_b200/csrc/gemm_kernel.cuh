// Dense matmul for sm_100a: C[M,N] = A[M,K] * B[K,N], row-major A and B,
// fp32 accumulation in TMEM.  Same contraction and output rounding as the
// reference's Triton `_matmul_contiguous_kernel` (mma.py:8-52): the fp32
// accumulator is rounded to fp16 before the store when `round_f16` is set
// (the reference always does `accumulator.to(tl.float16)`, mma.py:52), then
// stored in C's dtype.
//
// B200 structure: persistent grid (one CTA per SM), 128x256 output tiles in
// grouped order (GROUP_M rows of tiles share B in L2, as mma.py:22-30 does),
// a 4-stage TMA ring of A (K-major) and B (N-major) tiles, one thread issuing
// tcgen05.mma (M=128, N=256) into a double-buffered TMEM accumulator, and a
// 128-thread epilogue that drains one accumulator while the next tile's main
// loop runs.
//
// With kAR the same kernel also all-reduces C over the ranks of a
// tensor-parallel group through NVLink peer memory (GemmArParams):
//   1. each finished partial tile is stored straight into the inbox of the
//      rank that owns it (tile t -> rank t % world) and counted there with a
//      system-scope release, while the next tile's MMAs run;
//   2. meanwhile the two otherwise idle warps of every CTA take the tiles its
//      rank owns, wait (bounded) until all ranks' partials are in, sum them
//      in fp32 and write the result into every rank's output buffer, then
//      count it in each rank's done counter; once the CTA's own GEMM tiles
//      are out, its four epilogue warps take owned tiles too (both groups
//      claim them from one shared counter, so each is reduced once).  For
//      GEMMs of fewer than three waves of tiles the two warps stay out: the
//      overlap is too short to pay for their slower 64-thread reduction;
//   3. CTA 0 waits (bounded) until every tile of C has landed locally.
// Each counter is reset to zero by the one thread that waits on it, once it
// has seen the count it waits for; no rank can add to it again before that
// (its next call's partials go out only after its previous call saw every
// tile land, which the owners signal after their resets).  Nothing waits on
// a step that waits on it, and the CTAs of one rank are all resident
// (cooperative launch), so the only failure mode is a missing rank, which
// ends every wait at its time limit with a device error code; the counters
// are then left mid-count and the buffers must be replaced.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "fa_internal.h"
#include "ptx.cuh"

namespace fab {

// kBN_: output tile width, 256 by default; 128 or 64 (with more stages) for
// problems whose 256-wide tiles would leave many SMs idle.
template <int kElt, int kBN_ = 256, int kStages_ = 4>
struct GemmCfg {
  static constexpr int kBM = 128;
  static constexpr int kBN = kBN_;
  static constexpr int kBK = 128 / kElt;             // one 128-byte swizzle atom of K
  static constexpr int kStages = kStages_;
  static constexpr int kKInstr = 32 / kElt;
  static constexpr int kABytes = kBM * 128;          // 128 rows x one atom
  static constexpr int kBAtomN = 128 / kElt;         // N elements per B atom
  static constexpr int kBAtomBytes = kBK * 128;      // kBK rows x 128 B
  static constexpr int kBBytes = (kBN / kBAtomN) * kBAtomBytes;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kThreads = 256;
  static constexpr int kTmemCols = 2 * kBN;          // two fp32 accumulators
  static_assert(kBN == 64 || kBN == 128 || kBN == 256, "tile width");
  static constexpr int kNumBars = 2 * kStages + 4 + 1;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kNumBars * 8 + 64;  // + 16 status words
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

template <typename Tin>
struct GemmFmt;
template <>
struct GemmFmt<__nv_bfloat16> {
  static constexpr uint32_t kFmt = kFmtBF16;
};
template <>
struct GemmFmt<__half> {
  static constexpr uint32_t kFmt = kFmtF16;
};
template <>
struct GemmFmt<float> {
  static constexpr uint32_t kFmt = kFmtTF32;
};

__device__ __forceinline__ void gemm_tile_coords(int t, int num_pid_m, int num_pid_n, int group_m, int* pm, int* pn) {
  const int per_group = group_m * num_pid_n;
  const int g = t / per_group;
  const int first_m = g * group_m;
  const int gsize = min(num_pid_m - first_m, group_m);
  const int local = t - g * per_group;
  *pm = first_m + local % gsize;
  *pn = local / gsize;
}

template <typename Tout>
__device__ __forceinline__ void gemm_store_chunk(Tout* dst, const float (&v)[32], int ncols, bool round_f16) {
  float w[32];
#pragma unroll
  for (int e = 0; e < 32; ++e) w[e] = round_f16 ? __half2float(__float2half_rn(v[e])) : v[e];
  if constexpr (sizeof(Tout) == 2) {
    uint32_t pk[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      if constexpr (std::is_same<Tout, __nv_bfloat16>::value) {
        __nv_bfloat162 h = __floats2bfloat162_rn(w[2 * e], w[2 * e + 1]);
        pk[e] = *reinterpret_cast<uint32_t*>(&h);
      } else {
        __half2 h = __floats2half2_rn(w[2 * e], w[2 * e + 1]);
        pk[e] = *reinterpret_cast<uint32_t*>(&h);
      }
    }
    if (ncols >= 32) {
      uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int e = 0; e < 4; ++e) d4[e] = make_uint4(pk[4 * e], pk[4 * e + 1], pk[4 * e + 2], pk[4 * e + 3]);
    } else {
      // Ragged edge: static indices only, so pk stays in registers.
      uint32_t* d2 = reinterpret_cast<uint32_t*>(dst);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        if (2 * e + 1 < ncols)
          d2[e] = pk[e];
        else if (2 * e < ncols)
          reinterpret_cast<uint16_t*>(dst)[2 * e] = static_cast<uint16_t>(pk[e] & 0xFFFFu);
      }
    }
  } else {
    if (ncols >= 32) {
      float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
      for (int e = 0; e < 8; ++e) d4[e] = make_float4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e)
        if (e < ncols) dst[e] = w[e];
    }
  }
}

// x rounded to T's precision and back.
template <typename T>
__device__ __forceinline__ float round_to(float x) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    return __bfloat162float(__float2bfloat16_rn(x));
  else
    return __half2float(__float2half_rn(x));
}

// One thread's row of a finished accumulator tile, from TMEM to C: `acc` is
// the row's TMEM address of column 0, `row` its row of C, `n0` the tile's
// first column of B, `width` the tile's columns (multiple of 32).  Plain
// store (optionally through fp16), or with p.swiglu the SwiGLU of each
// 64-column gate block and the up block after it: a 256-wide tile holds
// gate 0-63, up 0-63, gate 64-127, up 64-127 of output columns n0/2 ... n0/2+127.
template <typename Tout>
__device__ __forceinline__ void load8(const void* src, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(src);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    if constexpr (std::is_same<Tout, __nv_bfloat16>::value) {
      f[2 * e] = __uint_as_float(w[e] << 16);
      f[2 * e + 1] = __uint_as_float(w[e] & 0xFFFF0000u);
    } else {
      const __half2 h = *reinterpret_cast<const __half2*>(&w[e]);
      const float2 x = __half22float2(h);
      f[2 * e] = x.x;
      f[2 * e + 1] = x.y;
    }
  }
}

// The bias + RoPE epilogue for one row of a 256-column tile: whole heads of
// p.head_dim columns (n0 is a multiple of it).  Rounds where the two-pass
// path rounds (GEMM output, + bias, each product and the sum), so it equals
// fab_gemm followed by fab_bias_rope bit for bit.
template <typename Tout>
__device__ __forceinline__ void gemm_store_bias_rope_row(const GemmKernelParams& p, uint32_t acc, int row, int n0) {
  // Every lane runs the TMEM loads (warp-collective) and the arithmetic; rows
  // past M read table row 0 and store nothing.
  const bool row_ok = row < p.M;
  const int trow = row_ok ? row : 0;
  const float rs = p.row_scale != nullptr ? p.row_scale[trow] : 1.0f;  // x * 1.0f == x: no-op without a scale
  const int hd = p.head_dim, half = hd / 2;
  Tout* crow = reinterpret_cast<Tout*>(p.c) + static_cast<int64_t>(trow) * p.ldc;
  const Tout* bias = static_cast<const Tout*>(p.bias);
  const Tout* cs = static_cast<const Tout*>(p.rope_cos) + static_cast<int64_t>(trow) * hd;
  const Tout* sn = static_cast<const Tout*>(p.rope_sin) + static_cast<int64_t>(trow) * hd;
#pragma unroll 1
  for (int h0 = 0; h0 < 256; h0 += hd) {
    const int col = n0 + h0;  // first column of this head
    if (col >= p.N) break;
    const bool rot = col < p.rope_cols;
#pragma unroll 1
    for (int c = 0; c < half; c += 32) {
      uint32_t rl[32], rh[32];
      tmem_ld32(acc + h0 + c, rl);
      tmem_ld32(acc + h0 + half + c, rh);
      tmem_wait_ld();
      float lo[32], hi[32];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        float bl[8], bh[8], cl[8], ch[8], sl[8], sh[8];
        if (bias != nullptr) {
          load8<Tout>(bias + col + c + 8 * g, bl);
          load8<Tout>(bias + col + half + c + 8 * g, bh);
        }
        if (rot) {
          load8<Tout>(cs + c + 8 * g, cl);
          load8<Tout>(cs + half + c + 8 * g, ch);
          load8<Tout>(sn + c + 8 * g, sl);
          load8<Tout>(sn + half + c + 8 * g, sh);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float l = round_to<Tout>(__uint_as_float(rl[8 * g + e]) * rs);
          float h = round_to<Tout>(__uint_as_float(rh[8 * g + e]) * rs);
          if (bias != nullptr) {
            l = round_to<Tout>(l + bl[e]);
            h = round_to<Tout>(h + bh[e]);
          }
          if (rot) {
            const float nl = round_to<Tout>(round_to<Tout>(l * cl[e]) + round_to<Tout>(-h * sl[e]));
            const float nh = round_to<Tout>(round_to<Tout>(h * ch[e]) + round_to<Tout>(l * sh[e]));
            l = nl;
            h = nh;
          }
          lo[8 * g + e] = l;
          hi[8 * g + e] = h;
        }
      }
      if (row_ok) {
        gemm_store_chunk<Tout>(crow + col + c, lo, 32, false);
        gemm_store_chunk<Tout>(crow + col + half + c, hi, 32, false);
      }
    }
  }
}

template <typename Tout, int kWidth>
__device__ __forceinline__ void gemm_store_tile_row(const GemmKernelParams& p, uint32_t acc, int row, int n0) {
  const float rs = (p.row_scale != nullptr && row < p.M) ? p.row_scale[row] : 1.0f;
  if constexpr (sizeof(Tout) == 2 && kWidth == 256) {
    if (p.bias_rope) {
      gemm_store_bias_rope_row<Tout>(p, acc, row, n0);
      return;
    }
    if (p.swiglu) {
      const int o0 = n0 / 2;
      Tout* orow = reinterpret_cast<Tout*>(p.c) + static_cast<int64_t>(row) * p.ldc + o0;
#pragma unroll 1
      for (int q = 0; q < 4; ++q) {  // 32 output columns each
        const int cg = (q >> 1) * 4 + (q & 1);
        uint32_t rg[32], ru[32];
        tmem_ld32(acc + cg * 32, rg);
        tmem_ld32(acc + (cg + 2) * 32, ru);
        tmem_wait_ld();
        float v[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float g = round_to<Tout>(__uint_as_float(rg[e]) * rs);
          const float u = round_to<Tout>(__uint_as_float(ru[e]) * rs);
          v[e] = round_to<Tout>(g / (1.0f + expf(-g))) * u;
        }
        const int ncols = min(32, p.N / 2 - o0 - q * 32);
        if (row < p.M && ncols > 0) gemm_store_chunk<Tout>(orow + q * 32, v, ncols, false);
      }
      return;
    }
  }
  Tout* crow = reinterpret_cast<Tout*>(p.c) + static_cast<int64_t>(row) * p.ldc + n0;
#pragma unroll 1
  for (int cc = 0; cc < kWidth / 32; ++cc) {
    uint32_t rr[32];
    tmem_ld32(acc + cc * 32, rr);
    tmem_wait_ld();
    float v[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(rr[e]) * rs;
    const int ncols = min(32, p.N - n0 - cc * 32);
    if (row < p.M && ncols > 0) gemm_store_chunk<Tout>(crow + cc * 32, v, ncols, p.round_f16 != 0);
  }
}

// 32 fp32 values as four 16-byte groups of 16-bit values.
template <typename Tout>
__device__ __forceinline__ void pack_chunk(const float (&v)[32], uint4 (&out)[4]) {
  uint32_t pk[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    if constexpr (std::is_same<Tout, __nv_bfloat16>::value) {
      __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
      pk[e] = *reinterpret_cast<uint32_t*>(&h);
    } else {
      __half2 h = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
      pk[e] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) out[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
}

// Partial tiles in the inboxes are stored column-group major: the 16-byte
// group g (8 columns) of row r sits at 16-byte index g * 128 + r, so the 32
// lanes of a warp (32 consecutive rows) write and read 512 contiguous bytes.
__device__ __forceinline__ int inbox_index(int group, int row) { return group * 128 + row; }

// Sums 32 columns (16-byte groups 4*cc .. 4*cc+3) of row r over the ranks' inbox slots.
template <typename Tout>
__device__ __forceinline__ void sum_partials(const uint4* slot0, int64_t src_stride16, int world, int cc, int r,
                                             float (&acc)[32]) {
#pragma unroll
  for (int e = 0; e < 32; ++e) acc[e] = 0.f;
  for (int src = 0; src < world; ++src) {
    const uint4* s4 = slot0 + src * src_stride16;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 x = __ldcg(s4 + inbox_index(4 * cc + q, r));  // L2: written by another GPU
      const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f;
        if constexpr (std::is_same<Tout, __nv_bfloat16>::value)
          f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[e]));
        else
          f = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
        acc[8 * q + 2 * e] += f.x;
        acc[8 * q + 2 * e + 1] += f.y;
      }
    }
  }
}

// Claims the next owned tile of this CTA (j = blockIdx.x + k * gridDim.x)
// once all ranks' partials of it are in: the reducer warps and, after their
// GEMM tiles, the epilogue warps call this, and whichever sees the tile ready
// first takes it, so a tile is never held by a group that is slower to reduce
// it while its partials are still missing.  Returns the tile, -1 when none is
// left, or -2 when the wait ran out (device error recorded).
__device__ __forceinline__ int claim_ready_tile(int* next, const GemmArParams& ar, int num_tiles,
                                                volatile int* abort) {
  uint64_t t0 = globaltimer_ns();
  int seen = -1;
  uint32_t spins = 0;
  while (true) {
    const int k = *reinterpret_cast<volatile int*>(next);
    const int j = static_cast<int>(blockIdx.x) + k * static_cast<int>(gridDim.x);
    if (j >= ar.tiles_per_owner || j * ar.world + ar.rank >= num_tiles) return -1;
    if (k != seen) {  // a new tile to wait for: restart its clock
      seen = k;
      t0 = globaltimer_ns();
    }
    if (ld_acquire_sys(ar.arrive[ar.rank] + j) >= static_cast<unsigned long long>(ar.world)) {
      if (atomicCAS(next, k, k + 1) == k) return j;
      continue;  // the other group took it
    }
    __nanosleep(64);
    if ((++spins & 63u) == 0u) {
      if (*abort) return -2;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        record_device_error(kDevTimeoutPeerTile);
        *abort = 1;
        return -2;
      }
    }
  }
}

template <typename Tin, typename Tout, bool kAR, int kBN = 256, int kStages = 4>
__global__ void __launch_bounds__(256, 1)
    gemm_kernel(const __grid_constant__ GemmKernelParams p, const __grid_constant__ CUtensorMap tm_a,
                const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ GemmArParams ar) {
  using C = GemmCfg<sizeof(Tin), kBN, kStages>;
  static_assert(!kAR || kBN == 256, "the fused all-reduce epilogue moves 256-column rows");
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* bar_full = bars;
  uint64_t* bar_empty = bars + C::kStages;
  uint64_t* bar_acc_full = bar_empty + C::kStages;
  uint64_t* bar_acc_empty = bar_acc_full + 2;
  uint64_t* bar_teardown = bar_acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_teardown + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // Epilogue-warpgroup agreement words (fused all-reduce only).
  volatile int* ep_ok = reinterpret_cast<volatile int*>(tmem_slot + 2);  // [4], one per epilogue warp
  volatile int* red_have = reinterpret_cast<volatile int*>(tmem_slot + 7);
  int* red_next = reinterpret_cast<int*>(tmem_slot + 6);  // next unclaimed owned tile of this CTA
  // Reducer staging: 32 rows x 32 16-byte groups, after the barrier words.
  uint4* red_stage =
      reinterpret_cast<uint4*>(smem + (C::kStages * C::kStageBytes + C::kNumBars * 8 + 64 + 127) / 128 * 128);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
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
      mbar_init(bar_acc_empty + b, 128);
    }
    mbar_init(bar_teardown, 1);
    *red_next = 0;
    *abort_flag = *reinterpret_cast<volatile int*>(&g_fab_device_error) != 0 ? 1 : 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const bool skip = *abort_flag != 0;

  if (!skip && warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
      int pm, pn;
      gemm_tile_coords(t, num_pid_m, num_pid_n, p.group_m, &pm, &pn);
      const int m0 = pm * C::kBM, n0 = pn * C::kBN;
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % C::kStages;
        const uint32_t ph = (it / C::kStages) & 1;
        if (!(ok = mbar_wait(bar_empty + s, ph ^ 1, abort_flag, kDevTimeoutEmpty))) break;
        uint8_t* st = smem + s * C::kStageBytes;
        mbar_arrive_expect_tx(bar_full + s, C::kStageBytes);
        tma_load_2d(st, &tm_a, bar_full + s, kb * C::kBK, m0);
#pragma unroll
        for (int a = 0; a < C::kBN / C::kBAtomN; ++a)
          tma_load_2d(st + C::kABytes + a * C::kBAtomBytes, &tm_b, bar_full + s, n0 + a * C::kBAtomN, kb * C::kBK);
      }
    }
    // Wait (bounded) for the last copy issued into every stage.
    volatile int no_abort = 0;
    for (int x = max(0, it - C::kStages); x < it; ++x)
      mbar_wait(bar_full + (x % C::kStages), (x / C::kStages) & 1, &no_abort, kDevTimeoutTeardown);
  } else if (!skip && warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = umma_idesc(GemmFmt<Tin>::kFmt, C::kBM, C::kBN, 0, 1);
    // Descriptors from precomputed words (see umma_desc_lo): per MMA only the
    // low word's address field moves.
    constexpr uint32_t kHiA = umma_desc_hi(1024, kLayoutSw128);
    constexpr uint32_t kHiB = sizeof(Tin) == 4 ? umma_desc_hi(512, kLayoutSw128Base32B) : umma_desc_hi(1024, kLayoutSw128);
    const uint32_t a_lo0 = umma_desc_lo(smem_u32(smem), 16);
    const uint32_t b_lo0 = umma_desc_lo(smem_u32(smem) + C::kABytes, C::kBAtomBytes);
    int it = 0, tcount = 0;
    bool ok = true, any = false;
    for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x, ++tcount) {
      const int buf = tcount & 1;
      const uint32_t use = tcount >> 1;
      if (!(ok = mbar_wait(bar_acc_empty + buf, (use & 1) ^ 1, abort_flag, kDevTimeoutAcc))) break;
      tc_fence_after();
      const uint32_t d = tmem + buf * C::kBN;
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % C::kStages;
        const uint32_t ph = (it / C::kStages) & 1;
        if (!(ok = mbar_wait(bar_full + s, ph, abort_flag, kDevTimeoutKV))) break;
        tc_fence_after();
        uint32_t a_lo = a_lo0 + s * (C::kStageBytes >> 4);
        uint32_t b_lo = b_lo0 + s * (C::kStageBytes >> 4);
        asm volatile("" : "+r"(a_lo), "+r"(b_lo));  // formed per stage, not hoisted into registers
#pragma unroll
        for (int kk = 0; kk < C::kBK / C::kKInstr; ++kk) {
          const uint64_t ad = umma_desc_join(a_lo + ((kk * 32) >> 4), kHiA);
          const uint64_t bd = umma_desc_join(b_lo + ((kk * C::kKInstr * 128) >> 4), kHiB);
          const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
          if constexpr (sizeof(Tin) == 4)
            mma_ss_tf32(d, ad, bd, idesc, acc);
          else
            mma_ss_f16(d, ad, bd, idesc, acc);
        }
        mma_commit(bar_empty + s);
        any = true;
      }
      if (!ok) break;
      mma_commit(bar_acc_full + buf);
    }
    if (any) {
      volatile int no_abort = 0;
      mma_commit(bar_teardown);
      mbar_wait(bar_teardown, 0, &no_abort, kDevTimeoutTeardown);
    }
  } else if (!skip && warp >= 4) {
    // ------------------------------------------------------------ epilogue
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(wq * 32) << 16;
    if constexpr (!kAR) {
      int tcount = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tcount) {
        const int buf = tcount & 1;
        const uint32_t use = tcount >> 1;
        if (!mbar_wait_warp(bar_acc_full + buf, use & 1, abort_flag, kDevTimeoutAcc)) break;
        tc_fence_after();
        int pm, pn;
        gemm_tile_coords(t, num_pid_m, num_pid_n, p.group_m, &pm, &pn);
        gemm_store_tile_row<Tout, C::kBN>(p, tmem + lane_base + buf * C::kBN, pm * C::kBM + r, pn * C::kBN);
        tc_fence_before();
        mbar_arrive(bar_acc_empty + buf);
      }
    } else {
      // The epilogue warpgroup synchronises with a named barrier, which has
      // no time limit, so no warp leaves these loops early: a failed wait
      // only clears `ok`, and decisions every warp must share are taken by
      // thread 0 and read back after a barrier.
      const int64_t slot_elems = static_cast<int64_t>(C::kBM) * C::kBN;
      const int64_t src_stride = static_cast<int64_t>(ar.tiles_per_owner) * slot_elems;
      bool ok = true;
      int tcount = 0;
      // 1. partial tiles into their owners' inboxes
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tcount) {
        const int buf = tcount & 1;
        const uint32_t use = tcount >> 1;
        if (ok) ok = mbar_wait_warp(bar_acc_full + buf, use & 1, abort_flag, kDevTimeoutAcc);
        const int owner = t % ar.world;
        const int j = t / ar.world;
        if (ok) {
          tc_fence_after();
          uint4* slot = reinterpret_cast<uint4*>(ar.inbox[owner]) + (ar.rank * src_stride + j * slot_elems) / 8;
#pragma unroll 1
          for (int cc = 0; cc < C::kBN / 32; ++cc) {
            uint32_t rr[32];
            tmem_ld32(tmem + lane_base + buf * C::kBN + cc * 32, rr);
            tmem_wait_ld();
            float v[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(rr[e]);
            uint4 g[4];
            pack_chunk<Tout>(v, g);
#pragma unroll
            for (int q = 0; q < 4; ++q) slot[inbox_index(4 * cc + q, r)] = g[q];
          }
          tc_fence_before();
          mbar_arrive(bar_acc_empty + buf);
        }
        if (lane == 0) ep_ok[wq] = ok ? 1 : 0;
        named_barrier_sync(1, 128);
        if (r == 0 && ep_ok[0] && ep_ok[1] && ep_ok[2] && ep_ok[3]) {
          fence_acq_rel_sys();
          red_release_sys_add(ar.arrive[owner] + j, 1ull);
        }
        named_barrier_sync(1, 128);  // ep_ok is rewritten next iteration
      }
      // 2b. help with the owned tiles the reducer warps have not claimed.  The
      // K/V stages are idle now (this CTA's last MMAs completed before its last
      // accumulator was drained): stage a whole reduced tile there so each
      // warp writes 512-byte rows.
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      uint4* stage = reinterpret_cast<uint4*>(smem);  // [128 rows][32 groups]
      const uint4* inbox = reinterpret_cast<const uint4*>(ar.inbox[ar.rank]);
      const int64_t src_stride16 = src_stride / 8;
      volatile int* ep_claim = ep_ok;  // reused: ep_ok is no longer needed
      while (true) {
        if (r == 0) ep_claim[0] = claim_ready_tile(red_next, ar, num_tiles, abort_flag);
        named_barrier_sync(1, 128);
        const int j = ep_claim[0];
        if (j < 0) break;  // read by all 128 threads after the barrier: the same for all
        const bool have = true;
        int pm = 0, pn = 0;
        if (have) {
          gemm_tile_coords(j * ar.world + ar.rank, num_pid_m, num_pid_n, p.group_m, &pm, &pn);
          const uint4* slot0 = inbox + j * slot_elems / 8;
#pragma unroll 1
          for (int cc = 0; cc < C::kBN / 32; ++cc) {
            float acc[32];
            sum_partials<Tout>(slot0, src_stride16, ar.world, cc, r, acc);
            uint4 g[4];
            pack_chunk<Tout>(acc, g);
#pragma unroll
            for (int q = 0; q < 4; ++q) stage[r * 32 + ((4 * cc + q) ^ (r & 31))] = g[q];
          }
        }
        named_barrier_sync(1, 128);
        if (have) {
          const int col = pn * C::kBN + lane * 8;
#pragma unroll 1
          for (int i = wq * 32; i < wq * 32 + 32; ++i) {
            const int row = pm * C::kBM + i;
            if (row < p.M && col < p.N) {
              const uint4 val = stage[i * 32 + (lane ^ (i & 31))];
              for (int dst = 0; dst < ar.world; ++dst)
                *reinterpret_cast<uint4*>(reinterpret_cast<Tout*>(ar.out[dst]) + static_cast<int64_t>(row) * ar.ldo +
                                          col) = val;
            }
          }
        }
        named_barrier_sync(1, 128);
        if (r == 0 && have) {
          atomicExch(ar.arrive[ar.rank] + j, 0ull);  // every partial of tile j has been read
          fence_acq_rel_sys();
          for (int dst = 0; dst < ar.world; ++dst) red_release_sys_add(ar.done[dst], 1ull);
        }
      }
      // 3. every tile of C has landed in this rank's output
      if (blockIdx.x == 0 && r == 0 &&
          wait_counter_at_least(ar.done[ar.rank], static_cast<unsigned long long>(num_tiles), abort_flag,
                                kDevTimeoutPeerDone))
        atomicExch(ar.done[ar.rank], 0ull);
    }
  } else if constexpr (kAR) {
    if (!skip && ar.overlap && (warp == 2 || warp == 3)) {
      // ------------------------------------------------------------ reducer
      // 2. reduce the tiles this rank owns as their partials arrive, while
      // the GEMM runs.  32 rows at a time: each thread sums 128 columns of one
      // row into the staging buffer (16-byte groups XOR-swizzled by row),
      // then each warp writes 16 whole 512-byte rows to every rank.  Named
      // barrier 2 spans these 64 threads; no thread leaves a loop early.
      const int rr = threadIdx.x - 64;
      const int half = rr >> 5;  // which 128 columns
      const int64_t slot_elems = static_cast<int64_t>(C::kBM) * C::kBN;
      const int64_t src_stride16 = static_cast<int64_t>(ar.tiles_per_owner) * slot_elems / 8;
      const uint4* inbox = reinterpret_cast<const uint4*>(ar.inbox[ar.rank]);
      volatile int* red_claim = red_have;  // the claimed tile, or < 0
      while (true) {
        if (rr == 0) *red_claim = claim_ready_tile(red_next, ar, num_tiles, abort_flag);
        named_barrier_sync(2, 64);
        const int j = *red_claim;
        if (j < 0) break;  // read by all 64 threads after the barrier: the same for all
        const int t = j * ar.world + ar.rank;
        const bool have = true;
        if (have) {
          int pm, pn;
          gemm_tile_coords(t, num_pid_m, num_pid_n, p.group_m, &pm, &pn);
          const int n0 = pn * C::kBN;
          const uint4* slot0 = inbox + j * slot_elems / 8;
#pragma unroll 1
          for (int rb = 0; rb < C::kBM / 32; ++rb) {
            const int r = rb * 32 + (rr & 31);
#pragma unroll 1
            for (int c4 = 0; c4 < 4; ++c4) {  // 32 columns = 4 groups at a time
              const int cc = half * 4 + c4;
              float acc[32];
              sum_partials<Tout>(slot0, src_stride16, ar.world, cc, r, acc);
              uint4 g[4];
              pack_chunk<Tout>(acc, g);
#pragma unroll
              for (int q = 0; q < 4; ++q) red_stage[(r & 31) * 32 + ((4 * cc + q) ^ (r & 31))] = g[q];
            }
            named_barrier_sync(2, 64);
            const int col = n0 + (rr & 31) * 8;
#pragma unroll 1
            for (int i = half * 16; i < half * 16 + 16; ++i) {
              const int row = pm * C::kBM + rb * 32 + i;
              if (row < p.M && col < p.N) {
                const uint4 val = red_stage[i * 32 + ((rr & 31) ^ i)];
                for (int dst = 0; dst < ar.world; ++dst)
                  *reinterpret_cast<uint4*>(reinterpret_cast<Tout*>(ar.out[dst]) + static_cast<int64_t>(row) * ar.ldo +
                                            col) = val;
              }
            }
            named_barrier_sync(2, 64);
          }
          if (rr == 0) {
            atomicExch(ar.arrive[ar.rank] + j, 0ull);  // every partial of tile j has been read
            fence_acq_rel_sys();
            for (int dst = 0; dst < ar.world; ++dst) red_release_sys_add(ar.done[dst], 1ull);
          }
        }
        named_barrier_sync(2, 64);  // red_claim is rewritten next iteration
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

template <typename Tin, typename Tout, bool kAR = false, int kBN = 256, int kStages = 4>
static int launch_gemm(const GemmLaunch& L, cudaStream_t stream, const GemmArParams* ar = nullptr) {
  using C = GemmCfg<sizeof(Tin), kBN, kStages>;
  auto kern = gemm_kernel<Tin, Tout, kAR, kBN, kStages>;
  constexpr int kSmem = C::kSmemBytes + (kAR ? 128 + 32 * 32 * 16 : 0);  // reducer staging
  static_assert(kSmem <= 232448, "shared memory budget");
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), kSmem);
  if (rc) return rc;
  const int elt = sizeof(Tin);
  const CUtensorMapDataType dt = elt == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : L.in_dtype == kDtypeBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                            : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ta, tb;
  rc = make_2d_map(&ta, L.a, dt, elt, L.K, L.M, L.lda, C::kBK, C::kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  // B is the MN-major operand: tf32 needs the 32-byte-chunk swizzle there.
  rc = make_2d_map(&tb, L.b, dt, elt, L.N, L.K, L.ldb, C::kBAtomN, C::kBK,
                   elt == 4 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B);
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
  kp.sk_dp_tiles = 0;  // stream-K is the CTA-pair kernel's
  kp.sk_part = nullptr;
  kp.sk_flags = nullptr;
  kp.dyn_sched = 0;
  const int tiles = ((L.M + C::kBM - 1) / C::kBM) * ((L.N + C::kBN - 1) / C::kBN);
  if (tiles <= 0) return 0;
  int sms = num_sms();
  if (sms <= 0) return kErrLaunch;
  const int grid = tiles < sms ? tiles : sms;
  GemmArParams arp{};
  if constexpr (kAR) {
    // CTAs wait on one another's tiles: launch them all resident together.
    arp = *ar;
    arp.overlap = tiles >= 3 * grid ? 1 : 0;
    void* args[] = {&kp, &ta, &tb, &arp};
    const cudaError_t e = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(kern), dim3(grid),
                                                      dim3(C::kThreads), args, kSmem, stream);
    return e == cudaSuccess ? 0 : kErrLaunch;
  } else {
    kern<<<grid, C::kThreads, kSmem, stream>>>(kp, ta, tb, arp);
    return cudaGetLastError() == cudaSuccess ? 0 : kErrLaunch;
  }
}

int gemm_ar_tiles(int M, int N) {
  return ((M + GemmCfg<2>::kBM - 1) / GemmCfg<2>::kBM) * ((N + GemmCfg<2>::kBN - 1) / GemmCfg<2>::kBN);
}

int gemm_allreduce(const GemmLaunch& L, const GemmArParams& ar, cudaStream_t stream) {
  if (L.M <= 0 || L.N <= 0 || L.K <= 0) return kErrInvalidArg;
  if (L.in_dtype != L.out_dtype) return kErrUnsupported;
  if (L.in_dtype == kDtypeBF16) return launch_gemm<__nv_bfloat16, __nv_bfloat16, true>(L, stream, &ar);
  if (L.in_dtype == kDtypeF16) return launch_gemm<__half, __half, true>(L, stream, &ar);
  return kErrUnsupported;
}

}  // namespace fab

#include "gemm_pair_kernel.cuh"
#include "gemm_splitk_kernel.cuh"

namespace fab {

template <typename Tin>
static int gemm_splitk_factor_out(const GemmLaunch& L) {
  if (L.out_dtype == kDtypeF16) return gemm_splitk_factor<Tin, __half>(L);
  if (L.out_dtype == kDtypeBF16) return gemm_splitk_factor<Tin, __nv_bfloat16>(L);
  if (L.out_dtype == kDtypeF32) return gemm_splitk_factor<Tin, float>(L);
  return 1;
}

// Output tile width of the single-CTA kernel: 256, unless that leaves more
// than a quarter of the SMs without a tile; then the widest of 128 and 64
// that gives at least 3/4 of the SMs a tile (64 if neither does).  Narrow
// tiles spread a small problem's loads over more SMs and keep more stages in
// flight per CTA (6 and 8), which is what a short kernel with a cold L2
// waits on.  16-bit inputs without the SwiGLU epilogue only.
static int gemm_single_width(const GemmLaunch& L) {
  if (gemm_fixed_width(L) || (L.in_dtype != kDtypeF16 && L.in_dtype != kDtypeBF16)) return 256;
  const int sms = num_sms();
  if (sms <= 0) return 256;
  const long long rows = (L.M + 127) / 128;
  auto tiles = [&](int w) { return rows * ((L.N + w - 1) / w); };
  if (4 * tiles(256) >= 3LL * sms) return 256;
  if (4 * tiles(128) >= 3LL * sms) return 128;
  return 64;
}

// Which kernel gemm_forward runs for L: 0 single CTA per tile (*tile_n wide),
// 1 CTA pairs (*tile_n wide tiles), 2 split K over a cluster of *split CTAs
// per tile, 3 CTA pairs with the stream-K schedule (L carries a workspace).
int gemm_plan(const GemmLaunch& L, int* kernel, int* split, int* tile_n) {
  *kernel = 0;
  *split = 1;
  *tile_n = 256;
  if (L.M <= 0 || L.N <= 0 || L.K <= 0) return 0;
#ifndef FAB_GEMM_NO_SPLITK
  if (L.in_dtype == kDtypeF16 || L.in_dtype == kDtypeBF16) {
    const int s = L.in_dtype == kDtypeF16 ? gemm_splitk_factor_out<__half>(L) : gemm_splitk_factor_out<__nv_bfloat16>(L);
    if (s > 1) {
      *kernel = 2;
      *split = s;
      return 0;
    }
  }
#endif
  if (gemm_use_pair(L)) {
    const PairChoice c = gemm_pair_layout_any(L);
    *kernel = c.stream_k ? 3 : 1;
    *tile_n = c.bn;
  } else {
    *tile_n = gemm_single_width(L);
  }
  return 0;
}

size_t gemm_workspace_bytes(const GemmLaunch& L) {
  int kernel = 0, split = 1, tile_n = 256;
  if (L.M <= 0 || L.N <= 0 || L.K <= 0) return 0;
  gemm_plan(L, &kernel, &split, &tile_n);
  if (kernel == 2 || !gemm_use_pair(L)) return 0;
  return gemm_pair_workspace(L);
}

long long gemm_grid_ctas(const GemmLaunch& L) {
  int kernel = 0, split = 1, tile_n = 256;
  if (L.M <= 0 || L.N <= 0 || L.K <= 0) return 0;
  gemm_plan(L, &kernel, &split, &tile_n);
  const int sms = num_sms();
  if (kernel == 2) return static_cast<long long>((L.M + 127) / 128) * ((L.N + 255) / 256) * split;
  if (kernel == 1 || kernel == 3) {
    const PairChoice c = gemm_pair_layout_any(L);
    return 2LL * (pair_dynamic(c) ? c.tiles : c.pairs);
  }
  const long long tiles = static_cast<long long>((L.M + 127) / 128) * ((L.N + tile_n - 1) / tile_n);
  return tiles < sms ? tiles : sms;
}

template <typename Tin, typename Tout>
static int launch_gemm_single(const GemmLaunch& L, cudaStream_t stream) {
  if constexpr (sizeof(Tin) == 2) {
    const int w = gemm_single_width(L);
    if (w == 64) return launch_gemm<Tin, Tout, false, 64, 8>(L, stream);
    if (w == 128) return launch_gemm<Tin, Tout, false, 128, 6>(L, stream);
  }
  return launch_gemm<Tin, Tout>(L, stream);
}

template <typename Tin>
static int gemm_forward_splitk(const GemmLaunch& L, cudaStream_t stream, bool* taken) {
  if (L.out_dtype == kDtypeF16) return launch_gemm_splitk<Tin, __half>(L, stream, taken);
  if (L.out_dtype == kDtypeBF16) return launch_gemm_splitk<Tin, __nv_bfloat16>(L, stream, taken);
  if (L.out_dtype == kDtypeF32) return launch_gemm_splitk<Tin, float>(L, stream, taken);
  *taken = false;
  return 0;
}

int gemm_forward(const GemmLaunch& L, cudaStream_t stream) {
  if (L.M < 0 || L.N < 0 || L.K < 0) return kErrInvalidArg;
  if (L.M == 0 || L.N == 0) return 0;
  const int in = L.in_dtype, out = L.out_dtype;
  if (L.K > 0 && (in == kDtypeF16 || in == kDtypeBF16)) {
    // Too few output tiles for the SMs: the CTAs of a cluster share each tile's K.
    bool taken = false;
    const int rc = in == kDtypeF16 ? gemm_forward_splitk<__half>(L, stream, &taken)
                                   : gemm_forward_splitk<__nv_bfloat16>(L, stream, &taken);
    if (taken) return rc;
  }
  if (L.K > 0 && gemm_use_pair(L)) {
    if (in == kDtypeF16) {
      if (out == kDtypeF16) return launch_gemm_pair<__half, __half>(L, stream);
      if (out == kDtypeBF16) return launch_gemm_pair<__half, __nv_bfloat16>(L, stream);
      if (out == kDtypeF32) return launch_gemm_pair<__half, float>(L, stream);
    } else {
      if (out == kDtypeF16) return launch_gemm_pair<__nv_bfloat16, __half>(L, stream);
      if (out == kDtypeBF16) return launch_gemm_pair<__nv_bfloat16, __nv_bfloat16>(L, stream);
      if (out == kDtypeF32) return launch_gemm_pair<__nv_bfloat16, float>(L, stream);
    }
    return kErrInvalidArg;
  }
  if (in == kDtypeF16) {
    if (out == kDtypeF16) return launch_gemm_single<__half, __half>(L, stream);
    if (out == kDtypeBF16) return launch_gemm_single<__half, __nv_bfloat16>(L, stream);
    if (out == kDtypeF32) return launch_gemm_single<__half, float>(L, stream);
  } else if (in == kDtypeBF16) {
    if (out == kDtypeF16) return launch_gemm_single<__nv_bfloat16, __half>(L, stream);
    if (out == kDtypeBF16) return launch_gemm_single<__nv_bfloat16, __nv_bfloat16>(L, stream);
    if (out == kDtypeF32) return launch_gemm_single<__nv_bfloat16, float>(L, stream);
  } else if (in == kDtypeF32) {
    if (out == kDtypeF16) return launch_gemm<float, __half>(L, stream);
    if (out == kDtypeBF16) return launch_gemm<float, __nv_bfloat16>(L, stream);
    if (out == kDtypeF32) return launch_gemm<float, float>(L, stream);
  }
  return kErrInvalidArg;
}

int gemm_kernel_attrs(int in_dtype, int* regs, int* smem, int* threads) {
  cudaFuncAttributes a{};
  const void* k = in_dtype == kDtypeF32    ? reinterpret_cast<const void*>(gemm_kernel<float, __half, false>)
                  : in_dtype == kDtypeBF16 ? reinterpret_cast<const void*>(gemm_kernel<__nv_bfloat16, __half, false>)
                                           : reinterpret_cast<const void*>(gemm_kernel<__half, __half, false>);
  if (cudaFuncGetAttributes(&a, k) != cudaSuccess) return kErrLaunch;
  *regs = a.numRegs;
  *smem = in_dtype == kDtypeF32 ? GemmCfg<4>::kSmemBytes : GemmCfg<2>::kSmemBytes;
  *threads = 256;
  return 0;
}

}  // namespace fab
