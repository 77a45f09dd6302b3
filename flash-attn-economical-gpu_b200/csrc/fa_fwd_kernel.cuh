// FlashAttention forward for sm_100a: O = softmax(scale * Q K^T [+ causal mask]) V,
// optional LSE = rowmax + log(rowsum) in natural-log units.
//
// Same mathematics as the reference's three Triton kernels
// (flash_atten.py:14-133 basic, :136-258 optimize_shared_mem, :261-361
// block_d_nomask_contiguous): online softmax over KV tiles in fp32, P rounded
// to the input dtype before the P*V product, final O = acc / l.
//
// B200 structure (one CTA per SM, 128 + NQ*128 threads; the one-tile,
// one-S-buffer family runs two CTAs per SM):
//   warp 0      TMA producer: Q tile 0, K_0, the other Q tiles (each Q tile
//               on its own barrier), then K and V tiles through one ring of
//               kRing tile slots, in the order the MMA thread uses them (K_j,
//               V_j alternating with one S buffer; K_0, K_1, then V_j,
//               K_{j+2} with two), so every slot the Q tiles leave free in
//               shared memory adds load lead time.
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer.
//   warps 4..   one 128-thread softmax group per 128-row Q tile; thread r of
//               the group owns row r (TMEM lane r) for the whole kernel.
// Per KV tile j and Q tile i:
//   S_i   = Q_i K_j^T            tcgen05.mma SS, fp32 in TMEM
//   P_i   = exp2(S_i*c - m_i)    softmax group: tcgen05.ld S, tcgen05.st P
//                                (P overwrites the first columns of its S buffer)
//   O_i  += P_i V_j              tcgen05.mma TS (A = P from TMEM)
// Two ways to keep the tensor core busy while a softmax runs:
//   * two Q tiles per CTA (head dims up to 128): the tensor core computes one
//     tile's products while the other tile's softmax runs;
//   * two S buffers for one Q tile (head dim 256, fp32 128): S(j+1) is
//     computed while softmax(j) runs.
// The S product that reuses an S buffer is issued right after the P*V product
// that reads the P held there; tcgen05.mma instructions from one thread
// execute in issue order, so the write cannot overtake the read.  The running
// max is only moved when it grows by more than 2^8, so O is rescaled rarely;
// the final O / l is unaffected.
// Epilogue: dense 16-bit O is staged in its Q tile's shared memory (idle by
// then) and written by TMA tensor stores; other layouts are stored directly.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>

#include "fa_internal.h"
#include "ptx.cuh"

// 1: the MMA issuer is a converged warp whose elected lane issues (descriptor
// arithmetic stays warp-uniform); 0: a single thread.  Measured on B200
// together with 4 of 16 polynomial pairs below: +2.7 % at B4 H32 S8192 D128,
// +4 % causal, +6.5 % S4096 causal; within +-2 % on the short shapes.
#ifndef FAB_FA_WARP_MMA
#define FAB_FA_WARP_MMA 1
#endif
constexpr bool kWarpMma = FAB_FA_WARP_MMA != 0;

// Of every 16 pairs of scores, this many are exponentiated by exp2_poly2 on
// the FMA pipe and the rest by ex2.approx on the MUFU unit.
#ifndef FAB_FA_POLY_PAIRS_PER_16
#define FAB_FA_POLY_PAIRS_PER_16 4
#endif

// 1: with one S buffer per Q tile, the softmax releases P in two halves of
// the key tile, so the MMA issuer starts P*V on the first half while the
// second half is still being exponentiated; 0: one release per tile.
// Measured on B200 (three interleaved rounds against 0): +1.5 % at
// B4 H32 S8192 D128 (non-causal and causal), +6 % at S2048 causal and on
// Qwen2.5-7B's 28/4-head GQA prefill, +4 % at D64.
#ifndef FAB_FA_P_HALVES
#define FAB_FA_P_HALVES 1
#endif
constexpr bool kPHalves = FAB_FA_P_HALVES != 0;

// 1 (with P halves): a third release after three quarters of the keys, so the
// P*V left after the last release covers a quarter of the tile.  Measured on
// B200 in two sets of three interleaved rounds against halves only: +0.7 and
// +3.9 % at B4 H32 S8192 D128, +1.0 / +2.1 % at S4096, +3.4 / +2.0 % at
// S2048, +3.6 / +3.1 % at D64; short causal shapes and Qwen2.5-7B's GQA
// prefill within +-2.5 % either way.
#ifndef FAB_FA_P_3Q
#define FAB_FA_P_3Q 1
#endif
constexpr bool kP3Q = kPHalves && FAB_FA_P_3Q != 0;

namespace fab {

// Test hook (fab_debug_starve_kv_load): the producer of every CTA skips the
// K/V ring load with this index, so the wait for it runs out and the kernel
// takes its give-up path.  -1, the default, skips nothing.
static __device__ int g_fab_starve_kv_load = -1;

template <int kElt, int kDP, int kNQ, int kBN, int kRing, int kSB>
struct FaCfg {
  static constexpr int kBM = 128;                    // rows per Q tile (TMEM lanes)
  static constexpr int kAtom = 128 / kElt;           // elements per 128-byte swizzle atom
  static constexpr int kNumAtoms = kDP / kAtom;      // atoms across the head dim
  static constexpr int kQAtomBytes = kBM * 128;
  static constexpr int kQTileBytes = kQAtomBytes * kNumAtoms;
  static constexpr int kKVAtomBytes = kBN * 128;
  static constexpr int kKVTileBytes = kKVAtomBytes * kNumAtoms;
  static constexpr int kKInstr = 32 / kElt;          // K extent of one MMA instruction
  static constexpr int kThreads = 128 + kNQ * 128;
  // One Q tile with one S buffer: small enough (<= ~112 KB of shared memory,
  // 256 TMEM columns, 128 registers a thread) that two CTAs share an SM, and
  // the tensor core alternates between their tiles.
  static constexpr bool kDual = kNQ == 1 && kSB == 1;
  static constexpr int kCtasPerSm = kDual ? 2 : 1;
  // Register split: the launch gives every thread kLaunchRegs; the TMA/MMA
  // warpgroup gives registers back so the softmax warpgroups can hold a
  // whole 128-column S row.  384 threads: 65536 / 384 rounded down to 8;
  // two 256-thread CTAs: 32768 / 256.
  static constexpr bool kSplitRegs = kNQ == 2 || kDual;
  static constexpr int kLaunchRegs = kDual ? 128 : 168;
  static constexpr int kProducerRegs = kDual ? 56 : 72;
  static constexpr int kSoftmaxRegs = kDual ? 200 : 216;
  static_assert(!kSplitRegs || 128 * kProducerRegs + kNQ * 128 * kSoftmaxRegs <= kThreads * kLaunchRegs,
                "register split exceeds the block's launch allocation");
  static constexpr int kSlots = kNQ * kSB;           // S/P buffers in TMEM
  static constexpr int kTmemUsed = kSlots * kBN + kNQ * kDP;
  static constexpr int kTmemAlloc = kTmemUsed <= 32 ? 32 : kTmemUsed <= 64 ? 64 : kTmemUsed <= 128 ? 128
                                    : kTmemUsed <= 256 ? 256 : 512;
  static constexpr int kNumBars = kNQ + 2 * kRing + 4 * kSlots + kNQ + 2;
  static constexpr int kDataBytes = kNQ * kQTileBytes + kRing * kKVTileBytes;
  // With two S buffers the MMA thread holds V_j while it waits for K_{j+2}:
  // ring tiles 2j+1 .. 2j+4 are resident together.
  // The ring holds tiles in the order the MMA thread uses them, so at most
  // V_j and K_{j+2} (two S buffers) or V_j and K_{j+1} (one) are held at once.
  static_assert(kRing >= 2, "K/V ring too short");
  // After the barriers: the TMEM address, the abort flag, the split-merge flag.
  static constexpr int kSmemBytes = 1024 + kDataBytes + kNumBars * 8 + 16;
  static_assert(kDP % kAtom == 0, "head dim must fill whole swizzle atoms");
  static_assert(kTmemUsed <= 512, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static_assert(!kDual || (2 * (kSmemBytes + 1024) <= 233472 && kTmemAlloc <= 256), "two CTAs per SM");
  __host__ __device__ static constexpr int tmem_s(int slot) { return slot * kBN; }
  __host__ __device__ static constexpr int tmem_o(int i) { return kSlots * kBN + i * kDP; }
};

// Ring positions with two S buffers: the MMA thread uses K_0, K_1, then V_j
// followed by K_{j+2} while that exists (P*V_j, then the S product that
// reuses the buffer), and the producer loads them in that order.
__host__ __device__ constexpr int ring_pos_k2(int j) { return j <= 1 ? j : 2 * j - 1; }
__host__ __device__ constexpr int ring_pos_v2(int j, int nt) {
  return nt == 1 ? 1 : (j <= nt - 3 ? 2 + 2 * j : nt + j);
}
// Ring positions of K_j and V_j for either S buffering (one: 2j and 2j+1).
template <int kSB>
__host__ __device__ constexpr int ring_pos_k(int j) {
  if constexpr (kSB == 2) return ring_pos_k2(j);
  else return 2 * j;
}
template <int kSB>
__host__ __device__ constexpr int ring_pos_v(int j, int nt) {
  if constexpr (kSB == 2) return ring_pos_v2(j, nt);
  else return 2 * j + 1;
}
static_assert(ring_pos_v2(0, 1) == 1 && ring_pos_k2(1) == 1 && ring_pos_v2(0, 2) == 2 && ring_pos_v2(1, 2) == 3 &&
                  ring_pos_k2(2) == 3 && ring_pos_v2(1, 3) == 4 && ring_pos_v2(2, 3) == 5 && ring_pos_k2(3) == 5 &&
                  ring_pos_v2(2, 4) == 6 && ring_pos_v2(3, 4) == 7,
              "ring order K0 K1 V0 K2 V1 K3 ... V(nt-2) V(nt-1)");

template <typename T>
struct ElemOps;

template <>
struct ElemOps<__nv_bfloat16> {
  static constexpr uint32_t kFmt = kFmtBF16;
  __device__ static uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

template <>
struct ElemOps<__half> {
  static constexpr uint32_t kFmt = kFmtF16;
  __device__ static uint32_t pack2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

template <>
struct ElemOps<float> {
  static constexpr uint32_t kFmt = kFmtTF32;
  __device__ static uint32_t pack2(float a, float) { return __float_as_uint(a); }
};

// Store 32 fp32 values (already normalised) as one 32-column chunk of an O row.
// Every array index is static so the values stay in registers.
template <typename T>
__device__ __forceinline__ void store_o_chunk(T* dst, const float (&v)[32], int ncols) {
  if constexpr (sizeof(T) == 2) {
    uint32_t w[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) w[e] = ElemOps<T>::pack2(v[2 * e], v[2 * e + 1]);
    if (ncols >= 32) {
      uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int e = 0; e < 4; ++e) d4[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
    } else {
      uint32_t* d2 = reinterpret_cast<uint32_t*>(dst);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        if (2 * e + 1 < ncols)
          d2[e] = w[e];
        else if (2 * e < ncols)
          reinterpret_cast<uint16_t*>(dst)[2 * e] = static_cast<uint16_t>(w[e] & 0xFFFFu);
      }
    }
  } else {
    if (ncols >= 32) {
      float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
      for (int e = 0; e < 8; ++e) d4[e] = make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e)
        if (e < ncols) dst[e] = v[e];
    }
  }
}

// The key splits of one row group (the CTAs blockIdx.x of every blockIdx.y)
// each leave their rows' normalised O and LSE in o_part / lse_part.  Every
// CTA counts itself in split_cnt[blockIdx.x] once its 128 softmax threads
// have stored; the last to arrive merges the group's rows:
// O = sum_s w_s O_s / sum_s w_s and LSE = max + log(sum_s w_s), with
// w_s = exp(LSE_s - max) (zero for an empty split), and sets the counter back
// to zero for the next call.  The group's rows are consecutive in o_part, so
// the merge runs over all 128 threads in row chunks: the chunk's LSEs into
// `scratch` (the idle K/V ring), per-row max and weights there, then each
// thread sums 4-column pieces of O (single columns for head dims that are
// not a multiple of 4) over the splits in split order, eight splits' loads in
// flight at a time.  Called by the four softmax warps of a
// one-query-tile CTA on every path (the named barriers have no time limit).
template <typename T>
__device__ __forceinline__ void split_merge(const FaKernelParams& p, int m0, int b, int h, int wq, int lane,
                                            uint32_t* merge_flag, float* scratch, int scratch_floats,
                                            uint64_t* bar, volatile int* abort_flag) {
  __threadfence();  // this thread's partial row, visible GPU-wide before the count
  named_barrier_sync(1, 128);
  if (wq == 0 && lane == 0) {
    const unsigned int prev = atomicAdd(p.split_cnt + blockIdx.x, 1u);
    *reinterpret_cast<volatile uint32_t*>(merge_flag) = prev + 1 == gridDim.y ? 1u : 0u;
  }
  named_barrier_sync(1, 128);
  if (*reinterpret_cast<volatile uint32_t*>(merge_flag) == 0) return;
  __threadfence();
  const int tid = wq * 32 + lane;
  const int splits = static_cast<int>(gridDim.y);
  const int64_t split_rows = static_cast<int64_t>(p.B) * p.Hq * p.Mq;
  // o_part / lse_part row of group row 0: rows m0.. of one (batch, head) or,
  // packed, of the query heads sharing key/value head h -- consecutive.
  const int64_t row_base = static_cast<int64_t>(b) * p.Hq * p.Mq +
                           (p.pack_gqa ? static_cast<int64_t>(h) * p.group * p.Mq : static_cast<int64_t>(h) * p.Mq) + m0;
  const int nrows = min(128, p.M - m0);
  const bool vec4 = (p.D & 3) == 0;  // o_part rows are then 16-byte aligned
  // Staged: per chunk of rows, every split's partial rows are bulk-copied
  // into the scratch at once (one round trip instead of one per eight
  // splits), then summed from shared memory.  Per chunk row: splits x D
  // partial values, splits weights, its max and 1/sum.
  const int staged_rows = vec4 ? min(nrows, scratch_floats / (splits * (p.D + 1) + 2)) : 0;
  if (staged_rows > 0) {
    uint32_t phase = 0;
    for (int r0 = 0; r0 < nrows; r0 += staged_rows, phase ^= 1u) {
      const int nr = min(staged_rows, nrows - r0);
      float* part = scratch;                    // [splits][nr][D]
      float* wsc = part + splits * nr * p.D;    // [splits][nr]
      float* rmax = wsc + splits * nr;
      float* rinv = rmax + nr;
      if (tid == 0) {
        fence_proxy_async_global();  // the other CTAs' rows, seen through the counter, before the copies
        fence_proxy_async_smem();    // this CTA's earlier reads of the scratch, before the copies overwrite it
        const uint32_t bytes = static_cast<uint32_t>(nr * p.D * 4);
        mbar_arrive_expect_tx(bar, bytes * static_cast<uint32_t>(splits));
        for (int sp = 0; sp < splits; ++sp)
          bulk_load_g2s(part + sp * nr * p.D, p.o_part + (sp * split_rows + row_base + r0) * p.D, bytes, bar);
      }
      for (int idx = tid; idx < splits * nr; idx += 128) {
        const int sp = idx / nr, rr = idx - sp * nr;
        wsc[idx] = __ldcg(p.lse_part + sp * split_rows + row_base + r0 + rr);
      }
      named_barrier_sync(1, 128);
      for (int rr = tid; rr < nr; rr += 128) {
        float mx = -INFINITY;
        for (int sp = 0; sp < splits; ++sp) mx = fmaxf(mx, wsc[sp * nr + rr]);
        float wsum = 0.f;
        if (mx != -INFINITY) {
          for (int sp = 0; sp < splits; ++sp) {
            const float ls = wsc[sp * nr + rr];
            const float w = ls == -INFINITY ? 0.f : expf(ls - mx);  // an empty split carries zeros
            wsc[sp * nr + rr] = w;
            wsum += w;
          }
        }
        rmax[rr] = mx;
        rinv[rr] = 1.f / wsum;
        const int row = m0 + r0 + rr;
        const int oh = p.pack_gqa ? h * p.group + row / p.Mq : h;
        const int qpos = p.pack_gqa ? row % p.Mq : row;
        if (p.lse != nullptr)
          p.lse[b * p.l_sb + oh * p.l_sh + static_cast<int64_t>(qpos) * p.l_sm] =
              mx == -INFINITY ? -INFINITY : mx + logf(wsum);
      }
      named_barrier_sync(1, 128);
      const bool got = mbar_wait(bar, phase, abort_flag, kDevTimeoutMerge);
      const int upr = p.D / 4;
      for (int u = tid; got && u < nr * upr; u += 128) {
        const int rr = u / upr, c0 = (u - rr * upr) * 4;
        const int row = m0 + r0 + rr;
        const int oh = p.pack_gqa ? h * p.group + row / p.Mq : h;
        const int qpos = p.pack_gqa ? row % p.Mq : row;
        T* orow = reinterpret_cast<T*>(p.o) + b * p.o_sb + oh * p.o_sh + static_cast<int64_t>(qpos) * p.o_sm + c0;
        if (rmax[rr] == -INFINITY) {
          for (int e = 0; e < 4; ++e) orow[e] = static_cast<T>(NAN);  // no split saw a key: 0/0
          continue;
        }
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int sp = 0; sp < splits; ++sp) {
          const float w = wsc[sp * nr + rr];
          const float4 x = *reinterpret_cast<const float4*>(part + (sp * nr + rr) * p.D + c0);
          acc[0] = fmaf(w, x.x, acc[0]);
          acc[1] = fmaf(w, x.y, acc[1]);
          acc[2] = fmaf(w, x.z, acc[2]);
          acc[3] = fmaf(w, x.w, acc[3]);
        }
        const float inv = rinv[rr];
        for (int e = 0; e < 4; ++e) orow[e] = static_cast<T>(acc[e] * inv);
      }
      named_barrier_sync(1, 128);  // the next chunk's copies overwrite the scratch
    }
    if (wq == 0 && lane == 0) p.split_cnt[blockIdx.x] = 0u;
    return;
  }
  // Otherwise (head dims not a multiple of 4, or too many splits for one row
  // in the scratch): plain loads, eight splits in flight at a time.
  // Per chunk row: splits weights, then max and 1/sum.
  const int chunk = min(nrows, scratch_floats / (splits + 2));
  float* wsc = scratch;
  for (int r0 = 0; r0 < nrows; r0 += chunk) {
    const int nr = min(chunk, nrows - r0);
    float* rmax = wsc + splits * nr;
    float* rinv = rmax + nr;
    for (int idx = tid; idx < splits * nr; idx += 128) {
      const int sp = idx / nr, rr = idx - sp * nr;
      wsc[idx] = __ldcg(p.lse_part + sp * split_rows + row_base + r0 + rr);
    }
    named_barrier_sync(1, 128);
    for (int rr = tid; rr < nr; rr += 128) {
      float mx = -INFINITY;
      for (int sp = 0; sp < splits; ++sp) mx = fmaxf(mx, wsc[sp * nr + rr]);
      float wsum = 0.f;
      if (mx != -INFINITY) {
        for (int sp = 0; sp < splits; ++sp) {
          const float ls = wsc[sp * nr + rr];
          const float w = ls == -INFINITY ? 0.f : expf(ls - mx);  // an empty split carries zeros
          wsc[sp * nr + rr] = w;
          wsum += w;
        }
      }
      rmax[rr] = mx;
      rinv[rr] = 1.f / wsum;
      const int row = m0 + r0 + rr;
      const int oh = p.pack_gqa ? h * p.group + row / p.Mq : h;
      const int qpos = p.pack_gqa ? row % p.Mq : row;
      if (p.lse != nullptr)
        p.lse[b * p.l_sb + oh * p.l_sh + static_cast<int64_t>(qpos) * p.l_sm] =
            mx == -INFINITY ? -INFINITY : mx + logf(wsum);
    }
    named_barrier_sync(1, 128);
    // Units of 4 columns (float4) when the head dim allows, else single columns.
    const int uw = vec4 ? 4 : 1;
    const int upr = p.D / uw;  // units per row
    for (int u = tid; u < nr * upr; u += 128) {
      const int rr = u / upr, c0 = (u - rr * upr) * uw;
      const int row = m0 + r0 + rr;
      const int oh = p.pack_gqa ? h * p.group + row / p.Mq : h;
      const int qpos = p.pack_gqa ? row % p.Mq : row;
      T* orow = reinterpret_cast<T*>(p.o) + b * p.o_sb + oh * p.o_sh + static_cast<int64_t>(qpos) * p.o_sm + c0;
      if (rmax[rr] == -INFINITY) {
        // No split saw a key: 0/0 like the single-pass kernel.
        for (int e = 0; e < uw; ++e) orow[e] = static_cast<T>(NAN);
        continue;
      }
      const float* src = p.o_part + (row_base + r0 + rr) * p.D + c0;
      const int64_t sstride = split_rows * p.D;  // floats between splits
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int sp0 = 0; sp0 < splits; sp0 += 8) {
        float4 x[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          if (sp0 + k < splits) {
            const float* q = src + (sp0 + k) * sstride;
            x[k] = vec4 ? __ldcg(reinterpret_cast<const float4*>(q)) : make_float4(__ldcg(q), 0.f, 0.f, 0.f);
          }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          if (sp0 + k < splits) {
            const float w = wsc[(sp0 + k) * nr + rr];
            acc[0] = fmaf(w, x[k].x, acc[0]);
            acc[1] = fmaf(w, x[k].y, acc[1]);
            acc[2] = fmaf(w, x[k].z, acc[2]);
            acc[3] = fmaf(w, x[k].w, acc[3]);
          }
        }
      }
      const float inv = rinv[rr];
      for (int e = 0; e < uw; ++e) orow[e] = static_cast<T>(acc[e] * inv);
    }
    named_barrier_sync(1, 128);  // the next chunk reuses the scratch
  }
  if (wq == 0 && lane == 0) p.split_cnt[blockIdx.x] = 0u;
}

template <typename T, int kDP, int kNQ, int kBN, int kRing, int kSB>
__global__ void __launch_bounds__(128 + kNQ * 128, (kNQ == 1 && kSB == 1) ? 2 : 1)
    fa_fwd_kernel(const __grid_constant__ FaKernelParams p, const __grid_constant__ CUtensorMap tm_q,
                  const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                  const __grid_constant__ CUtensorMap tm_o) {
  using C = FaCfg<sizeof(T), kDP, kNQ, kBN, kRing, kSB>;
  constexpr float kNegInf = -INFINITY;
  static_assert(!(kSB == 1 && kPHalves) || kBN % 64 == 0, "P halves are whole 32-key chunks");

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + kNQ * C::kQTileBytes;  // [kRing] K or V tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + kRing * C::kKVTileBytes);
  uint64_t* bar_q_full = bars;                    // [kNQ], one per Q tile
  uint64_t* bar_kv_full = bars + kNQ;             // [kRing]
  uint64_t* bar_kv_empty = bar_kv_full + kRing;   // [kRing]
  uint64_t* bar_s_full = bar_kv_empty + kRing;    // [kSlots]
  uint64_t* bar_p_full = bar_s_full + C::kSlots; // [kSlots]
  uint64_t* bar_o_done = bar_p_full + C::kSlots; // [kNQ]
  uint64_t* bar_teardown = bar_o_done + kNQ;
  uint64_t* bar_p_half = bar_teardown + 1;        // [kSlots], P of the first half of the keys
  uint64_t* bar_p_3q = bar_p_half + C::kSlots;    // [kSlots], P of three quarters of the keys
  uint64_t* bar_merge = bar_p_3q + C::kSlots;     // split-KV merge: partial rows copied in
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_merge + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Work item: (batch, head) items are dealt in groups of head_group, the
  // slow index, so CTAs resident together share the group's K/V in L2;
  // within a group the row blocks go longest (causal) first across all its
  // items, so the grid's last CTAs are short ones and the SMs finish
  // together.  Rows are the query positions of one (batch, query head), or
  // with pack_gqa the (query head, position) pairs of the query heads sharing
  // one key/value head.  blockIdx.y selects a split of split_len keys.
  const int heads = p.pack_gqa ? p.Hq / p.group : p.Hq;
  int bh, mblk;
  {
    const int items = static_cast<int>(gridDim.x) / p.num_m_blocks;
    const int per_group = p.head_group * p.num_m_blocks;
    const int grp = static_cast<int>(blockIdx.x) / per_group;
    const int in_grp = min(p.head_group, items - grp * p.head_group);
    const int r = static_cast<int>(blockIdx.x) - grp * per_group;
    bh = grp * p.head_group + r % in_grp;
    mblk = p.num_m_blocks - 1 - r / in_grp;
  }
  const int b = bh / heads;
  const int h = bh % heads;  // query head; key/value head when packed
  const int hk = p.pack_gqa ? h : h / p.group;
  const int m0 = mblk * kNQ * C::kBM;
  // Lengths and first rows of this batch entry; packed variable-length
  // batches read them from the cumulative offsets and index one flat tensor.
  int seq_m = p.M, seq_n = p.N, q_row0 = 0, k_row0 = 0, map_b = b;
  int64_t o_boff = b * p.o_sb, l_boff = b * p.l_sb;
  if (p.cu_q != nullptr) {
    q_row0 = p.cu_q[b];
    seq_m = p.cu_q[b + 1] - q_row0;
    k_row0 = p.cu_k[b];
    seq_n = p.cu_k[b + 1] - k_row0;
    map_b = 0;
    o_boff = static_cast<int64_t>(q_row0) * p.o_sm;
    l_boff = static_cast<int64_t>(q_row0) * p.l_sm;
    // The grid covers the longest sequence; row blocks past this one's end
    // leave before touching shared memory, TMEM or a barrier.
    if (m0 >= seq_m) return;
  }
  const int n_begin = static_cast<int>(blockIdx.y) * p.split_len;
  const int n_key_end = min(seq_n, n_begin + p.split_len);  // keys of this split
  int n_end = n_key_end;                                      // keys any row of this CTA may see
  if (p.causal) n_end = min(n_end, p.pack_gqa ? p.Mq : min(seq_m, m0 + kNQ * C::kBM));
  const int nt = n_end > n_begin ? (n_end - n_begin + kBN - 1) / kBN : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNQ; ++i) mbar_init(bar_q_full + i, 1);
    for (int s = 0; s < kRing; ++s) {
      mbar_init(bar_kv_full + s, 1);
      mbar_init(bar_kv_empty + s, 1);
    }
    for (int x = 0; x < C::kSlots; ++x) {
      mbar_init(bar_s_full + x, 1);
      mbar_init(bar_p_full + x, 4);  // one arrival per softmax warp
      mbar_init(bar_p_half + x, 4);
      mbar_init(bar_p_3q + x, 4);
    }
    for (int i = 0; i < kNQ; ++i) mbar_init(bar_o_done + i, 1);
    mbar_init(bar_teardown, 1);
    mbar_init(bar_merge, 1);
    *abort_flag = *reinterpret_cast<volatile int*>(&g_fab_device_error) != 0 ? 1 : 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemAlloc);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const bool skip = *abort_flag != 0;
  // Role dispatch.  Warpgroup 0 (TMA producer, MMA issuer, two spare warps)
  // and the softmax warpgroups each re-split registers first, unconditionally
  // and warpgroup-uniformly, so the release always happens and the softmax
  // increase can always be satisfied; each role's code stays inside its
  // warpgroup's branch.
  if (warp < 4) {
    if constexpr (C::kSplitRegs) setmaxnreg_dec<C::kProducerRegs>();
  if (!skip && warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    auto load_q = [&](int i) {
      mbar_arrive_expect_tx(bar_q_full + i, C::kQTileBytes);
      for (int a = 0; a < C::kNumAtoms; ++a)
        tma_load_4d(sQ + i * C::kQTileBytes + a * C::kQAtomBytes, &tm_q, bar_q_full + i, a * C::kAtom,
                    q_row0 + m0 + i * C::kBM, h, map_b);
    };
    // Q tile 0, then K_0 (all the first S product needs), then the other Q
    // tiles; with no keys only Q tile 0 is loaded (the MMA thread waits for
    // nothing else).
    load_q(0);
    int q_loaded = 1;
    const int starve = g_fab_starve_kv_load;
    // Ring tile t: K_{t/2} for even t, V_{t/2} for odd t, in slot t % kRing.
    // With one S buffer the MMA thread frees V_j and K_{j+1} with one commit
    // (release group j+1; group 0 is K_0), on barrier group % kRing; with two,
    // every slot has its own release.
    int issued = 0;
    for (int t = 0; t < 2 * nt; ++t) {
      const int s = t % kRing;
      const uint32_t ph = (t / kRing) & 1;
      if constexpr (kSB == 1) {
        if (t >= kRing) {
          const int g = (t - kRing + 1) >> 1;  // release group of the slot's previous tile
          if (!mbar_wait(bar_kv_empty + g % kRing, (g / kRing) & 1, abort_flag, kDevTimeoutEmpty)) break;
        }
      } else {
        if (!mbar_wait(bar_kv_empty + s, ph ^ 1, abort_flag, kDevTimeoutEmpty)) break;
      }
      if (t == starve) {
        issued = t + 1;
        if (t == 0)
          for (; q_loaded < kNQ; ++q_loaded) load_q(q_loaded);
        continue;
      }
      mbar_arrive_expect_tx(bar_kv_full + s, C::kKVTileBytes);
      // Which tile is ring position t: alternating K/V with one S buffer;
      // K_0, K_1, then V_j, K_{j+2} with two.
      const CUtensorMap* map;
      int row;
      if constexpr (kSB == 2) {
        bool is_v;
        int tj;
        if (t == 0 || (t == 1 && nt > 1)) {
          is_v = false;
          tj = t;
        } else if (nt == 1) {
          is_v = true;
          tj = 0;
        } else {
          const int q = t - 2, pairs = nt - 2;  // (V_j, K_{j+2}) pairs, then the last two V
          if (q < 2 * pairs) {
            is_v = (q & 1) == 0;
            tj = (q >> 1) + (is_v ? 0 : 2);
          } else {
            is_v = true;
            tj = pairs + (q - 2 * pairs);
          }
        }
        map = is_v ? &tm_v : &tm_k;
        row = k_row0 + n_begin + tj * kBN;
      } else {
        map = (t & 1) ? &tm_v : &tm_k;
        row = k_row0 + n_begin + (t >> 1) * kBN;
      }
      for (int a = 0; a < C::kNumAtoms; ++a)
        tma_load_4d(sKV + s * C::kKVTileBytes + a * C::kKVAtomBytes, map, bar_kv_full + s, a * C::kAtom, row, hk,
                    map_b);
      issued = t + 1;
      if (t == 0)
        for (; q_loaded < kNQ; ++q_loaded) load_q(q_loaded);
    }
    // Never leave this CTA with bulk copies still landing in its smem: wait
    // (bounded) for the last load issued into every slot.
    volatile int no_abort = 0;
    for (int i = 0; i < q_loaded; ++i) mbar_wait(bar_q_full + i, 0, &no_abort, kDevTimeoutTeardown);
    for (int x = max(0, issued - kRing); x < issued; ++x)
      mbar_wait(bar_kv_full + (x % kRing), (x / kRing) & 1, &no_abort, kDevTimeoutTeardown);
  } else if (!skip && warp == 1 && (kWarpMma || lane == 0)) {
    // ------------------------------------------------------------ MMA issuer
    // One thread issues every tcgen05.mma and commit (the commits track that
    // thread's products).  With kWarpMma the whole warp runs this code and
    // waits together, and its elected lane issues.
    const bool leader = kWarpMma ? elect_one() : true;
    auto wait = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
      if constexpr (kWarpMma) {
        return mbar_wait_warp(bar, parity, abort_flag, code);
      } else {
        return mbar_wait(bar, parity, abort_flag, code);
      }
    };
    constexpr uint32_t kFmt = ElemOps<T>::kFmt;
    constexpr uint32_t idesc_qk = umma_idesc(kFmt, C::kBM, kBN, 0, 0);
    constexpr uint32_t idesc_pv = umma_idesc(kFmt, C::kBM, kDP, 0, 1);
    // Descriptors are built from precomputed words: per MMA only the low
    // word's address field moves (see umma_desc_lo), which keeps this
    // thread's instruction stream short -- it shares its SM sub-partition
    // with two softmax warps.
    constexpr uint32_t kHiK = umma_desc_hi(1024, kLayoutSw128);
    constexpr uint32_t kHiV = sizeof(T) == 4 ? umma_desc_hi(512, kLayoutSw128Base32B) : umma_desc_hi(1024, kLayoutSw128);
    const uint32_t q_lo = umma_desc_lo(smem_u32(sQ), 16);
    const uint32_t k_lo = umma_desc_lo(smem_u32(sKV), 16);
    const uint32_t v_lo = umma_desc_lo(smem_u32(sKV), C::kKVAtomBytes);
    // Ring slot and phase of K_j and V_j: tiles 2j and 2j+1 with one S buffer,
    // the ring_pos_*2 order with two.
    auto kslot = [](int j) { return ring_pos_k<kSB>(j) % kRing; };
    auto kpar = [](int j) { return static_cast<uint32_t>((ring_pos_k<kSB>(j) / kRing) & 1); };
    auto vslot = [=](int j) { return ring_pos_v<kSB>(j, nt) % kRing; };
    auto vpar = [=](int j) { return static_cast<uint32_t>((ring_pos_v<kSB>(j, nt) / kRing) & 1); };
    auto issue_qk = [&](int i, int slot, int s) {
      const uint32_t d = tmem + C::tmem_s(slot);
      uint32_t qa = q_lo + i * (C::kQTileBytes >> 4);
      uint32_t kb = k_lo + s * (C::kKVTileBytes >> 4);
      // Opaque to the optimiser, so the per-step words are formed here rather
      // than hoisted out of the tile loop into registers this warp lacks.
      asm volatile("" : "+r"(qa), "+r"(kb));
#pragma unroll
      for (int kk = 0; kk < kDP / C::kKInstr; ++kk) {
        const int a = kk >> 2;
        const uint32_t off = (kk & 3) * 32;
        const uint64_t ad = umma_desc_join(qa + ((a * C::kQAtomBytes + off) >> 4), kHiK);
        const uint64_t bd = umma_desc_join(kb + ((a * C::kKVAtomBytes + off) >> 4), kHiK);
        if (leader) {
          if constexpr (sizeof(T) == 4) {
            mma_ss_tf32(d, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
          } else {
            mma_ss_f16(d, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
          }
        }
      }
    };
    // P*V over the key steps [kk0, kk1) of the tile (kBN / kKInstr in all).
    auto issue_pv = [&](int i, int slot, int s, bool acc, int kk0 = 0, int kk1 = kBN / C::kKInstr) {
      const uint32_t d = tmem + C::tmem_o(i);
      const uint32_t pa = tmem + C::tmem_s(slot);
      uint32_t vb = v_lo + s * (C::kKVTileBytes >> 4);
      asm volatile("" : "+r"(vb));
#pragma unroll
      for (int kk = kk0; kk < kk1; ++kk) {
        const uint64_t bd = umma_desc_join(vb + ((kk * C::kKInstr * 128) >> 4), kHiV);
        const uint32_t a_t = pa + kk * (C::kKInstr * static_cast<int>(sizeof(T)) / 4);
        const uint32_t accum = (acc || kk > 0) ? 1u : 0u;
        if (leader) {
          if constexpr (sizeof(T) == 4) {
            mma_ts_tf32(d, a_t, bd, idesc_pv, accum);
          } else {
            mma_ts_f16(d, a_t, bd, idesc_pv, accum);
          }
        }
      }
    };

    bool ok = wait(bar_q_full, 0, kDevTimeoutQ);  // Q tile 0
    bool any_issued = false;
    // Prologue: S for the first kSB KV tiles of every Q tile.  Q tiles after
    // the first land behind K_0, so tile 0's product starts without them.
    for (int j = 0; ok && j < min(kSB, nt); ++j) {
      if (!(ok = wait(bar_kv_full + kslot(j), kpar(j), kDevTimeoutKV))) break;
      tc_fence_after();
      for (int i = 0; i < kNQ; ++i) {
        if (j == 0 && i > 0) {
          if (!(ok = wait(bar_q_full + i, 0, kDevTimeoutQ))) break;
          tc_fence_after();
        }
        issue_qk(i, i * kSB + j, kslot(j));
        any_issued = true;
        { if (leader) mma_commit(bar_s_full + i * kSB + j); }
      }
      if (!ok) break;
      { if (leader) mma_commit(bar_kv_empty + kslot(j)); }
    }
    for (int j = 0; ok && j < nt; ++j) {
      const int s = vslot(j);
      const int jn = j + kSB;  // the KV tile whose S product reuses this S buffer
      const int sn = kslot(jn);
      if (!(ok = wait(bar_kv_full + s, vpar(j), kDevTimeoutKV))) break;
      if constexpr (kSB == 1) {
        // Two Q tiles.  Each MMA burst is followed by a stall of a few hundred
        // cycles before the issuing thread's next instruction, so P_i*V(j)
        // and S_i(j+1) go out back to back: K(j+1) (loaded an iteration ago)
        // is waited for up front and the K/V release commits come last.
        if (jn < nt && !(ok = wait(bar_kv_full + sn, kpar(jn), kDevTimeoutKV))) break;
        for (int i = 0; i < kNQ; ++i) {
          const int slot = i;
          if constexpr (kPHalves) {
            constexpr int kHalf = kBN / C::kKInstr / 2;
            if (!(ok = wait(bar_p_half + slot, j & 1, kDevTimeoutP))) break;
            tc_fence_after();
            issue_pv(i, slot, s, j > 0, 0, kHalf);
            if constexpr (kP3Q) {
              constexpr int k3q = 3 * kBN / C::kKInstr / 4;
              if (!(ok = wait(bar_p_3q + slot, j & 1, kDevTimeoutP))) break;
              tc_fence_after();
              issue_pv(i, slot, s, true, kHalf, k3q);
              if (!(ok = wait(bar_p_full + slot, j & 1, kDevTimeoutP))) break;
              tc_fence_after();
              issue_pv(i, slot, s, true, k3q, 2 * kHalf);
            } else {
              if (!(ok = wait(bar_p_full + slot, j & 1, kDevTimeoutP))) break;
              tc_fence_after();
              issue_pv(i, slot, s, true, kHalf, 2 * kHalf);
            }
          } else {
            if (!(ok = wait(bar_p_full + slot, j & 1, kDevTimeoutP))) break;
            tc_fence_after();
            issue_pv(i, slot, s, j > 0);
          }
          if (jn < nt) issue_qk(i, slot, sn);
          if (j == nt - 1) { if (leader) mma_commit(bar_o_done + i); }  // nobody reads O before the end
          if (jn < nt) { if (leader) mma_commit(bar_s_full + slot); }
        }
        if (!ok) break;
        { if (leader) mma_commit(bar_kv_empty + (j + 1) % kRing); }  // release group j+1: V_j and K_{j+1}
      } else {
        // Two S buffers per Q tile: S_i(j+1) is already in TMEM while the
        // softmax works on tile j.  The softmax of tile j+1 waits for
        // P_i*V(j) before it may rescale O, and the producer's next V and K
        // loads wait for V(j)'s slot: release both right after the P*V
        // products; K(j+2) is issued only after V(j+1), so wait for it
        // afterwards.
        for (int i = 0; i < kNQ; ++i) {
          const int slot = i * kSB + j % kSB;
          if (!(ok = wait(bar_p_full + slot, (j / kSB) & 1, kDevTimeoutP))) break;
          tc_fence_after();
          issue_pv(i, slot, s, j > 0);
          { if (leader) mma_commit(bar_o_done + i); }
        }
        if (!ok) break;
        { if (leader) mma_commit(bar_kv_empty + s); }
        if (jn < nt) {
          if (!(ok = wait(bar_kv_full + sn, kpar(jn), kDevTimeoutKV))) break;
          tc_fence_after();
          for (int i = 0; i < kNQ; ++i) {
            const int slot = i * kSB + j % kSB;
            issue_qk(i, slot, sn);
            { if (leader) mma_commit(bar_s_full + slot); }
          }
          { if (leader) mma_commit(bar_kv_empty + sn); }
        }
      }
    }
    if (any_issued) {
      // Drain the tensor pipe before TMEM is released.
      volatile int no_abort = 0;
      { if (leader) mma_commit(bar_teardown); }
      mbar_wait(bar_teardown, 0, &no_abort, kDevTimeoutTeardown);
    }
  }
  } else {
    if constexpr (C::kSplitRegs) setmaxnreg_inc<C::kSoftmaxRegs>();
  if (!skip) {
    // ------------------------------------------------------------ softmax
    const int i = (warp - 4) >> 2;
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const int row = m0 + i * C::kBM + r;
    const int oh = p.pack_gqa ? h * p.group + row / p.Mq : h;  // query head of this row
    const int qpos = p.pack_gqa ? row % p.Mq : row;            // its query position
    const uint32_t lane_base = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t t_o = tmem + lane_base + C::tmem_o(i);
    const float c = p.scale_log2;
    float m_run = kNegInf;
    float l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      const int slot = i * kSB + (j % kSB);
      const uint32_t t_s = tmem + lane_base + C::tmem_s(slot);
      if (!(ok = mbar_wait_warp(bar_s_full + slot, (j / kSB) & 1, abort_flag, kDevTimeoutS))) break;
      tc_fence_after();
      float s[kBN];
#pragma unroll
      for (int cc = 0; cc < kBN / 32; ++cc) {
        uint32_t rr[32];
        tmem_ld32(t_s + cc * 32, rr);
#pragma unroll
        for (int e = 0; e < 32; ++e) s[cc * 32 + e] = __uint_as_float(rr[e]);
      }
      tmem_wait_ld();
      const int col0 = n_begin + j * kBN;
      const bool need_mask = (col0 + kBN > n_key_end) || (p.causal && col0 + kBN - 1 > qpos);
      if (need_mask) {
        const int lim = p.causal ? min(n_key_end, qpos + 1) : n_key_end;
#pragma unroll
        for (int e = 0; e < kBN; ++e)
          if (col0 + e >= lim) s[e] = kNegInf;
      }
      // Row max: eight independent chains seeded with columns 0-7, then
      // three-input max over 16 columns per step, then a last 8 if left.
      float mxv[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) mxv[a] = s[a];
      constexpr int kSteps16 = (kBN - 8) / 16;
#pragma unroll
      for (int t = 0; t < kSteps16; ++t)
#pragma unroll
        for (int a = 0; a < 8; ++a) mxv[a] = fmax3(mxv[a], s[8 + 16 * t + a], s[16 + 16 * t + a]);
      static_assert(kBN % 8 == 0, "BLOCK_N is a multiple of 8");
      if constexpr (8 + 16 * kSteps16 < kBN)
#pragma unroll
        for (int a = 0; a < 8; ++a) mxv[a] = fmaxf(mxv[a], s[8 + 16 * kSteps16 + a]);
      const float mx = fmax3(fmax3(mxv[0], mxv[1], mxv[2]), fmax3(mxv[3], mxv[4], mxv[5]), fmaxf(mxv[6], mxv[7]));
      const float m_cand = fmaxf(m_run, mx * c);
      const bool rescale = m_cand > m_run + 8.0f;
      const float m_new = rescale ? m_cand : m_run;
      const float alpha = rescale ? ex2_approx(m_run - m_new) : 1.0f;
      const float m_base = (m_new == kNegInf) ? 0.f : m_new;
      // With P released in halves, P*V(j) may start before this tile's
      // softmax ends, so O is rescaled first.  One S buffer: S_i(j) was issued
      // after P*V of tile j-1 and its commit covers that product, so O_i is
      // final here.
      constexpr bool kEarlyRescale = kSB == 1 && kPHalves;
      if constexpr (kEarlyRescale) {
        if (j > 0 && __any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
          for (int cc = 0; cc < kDP / 32; ++cc) {
            uint32_t rr[32];
            tmem_ld32(t_o + cc * 32, rr);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) rr[e] = __float_as_uint(__uint_as_float(rr[e]) * alpha);
            tmem_st32(t_o + cc * 32, rr);
          }
        }
      }
      // p = 2^(s*c - m_base), two scores at a time.
      const float2 c2 = make_float2(c, c);
      const float2 nmb2 = make_float2(-m_base, -m_base);
      float2 lsum2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int cc = 0; cc < kBN / 32; ++cc) {
        constexpr int kPk = sizeof(T) == 2 ? 16 : 32;
        uint32_t pk[kPk];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float2 x = __ffma2_rn(make_float2(s[cc * 32 + 2 * e], s[cc * 32 + 2 * e + 1]), c2, nmb2);
          float2 pp;
          // Spread FAB_FA_POLY_PAIRS_PER_16 polynomial pairs evenly among the 16.
          if ((e * FAB_FA_POLY_PAIRS_PER_16) % 16 < FAB_FA_POLY_PAIRS_PER_16) {
            pp = exp2_poly2(x);
          } else {
            pp = make_float2(ex2_approx(x.x), ex2_approx(x.y));
          }
          lsum2[e & 1] = __fadd2_rn(lsum2[e & 1], pp);
          if constexpr (sizeof(T) == 2) {
            pk[e] = ElemOps<T>::pack2(pp.x, pp.y);
          } else {
            pk[2 * e] = __float_as_uint(pp.x);
            pk[2 * e + 1] = __float_as_uint(pp.y);
          }
        }
        if constexpr (kEarlyRescale) {
          // P of the first kBN/2 keys (chunks 0 .. kBN/64 - 1) is in TMEM:
          // release it, then store this chunk.
          if (cc == kBN / 64) {
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_p_half + slot);
          }
          if constexpr (kP3Q) {
            if (cc == 3 * kBN / 128) {
              tmem_wait_st();
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(bar_p_3q + slot);
            }
          }
        }
        if constexpr (sizeof(T) == 2) {
          tmem_st16(t_s + cc * 16, pk);
        } else {
          tmem_st32(t_s + cc * 32, pk);
        }
      }
      const float2 lsum_pair = __fadd2_rn(lsum2[0], lsum2[1]);
      const float lsum = lsum_pair.x + lsum_pair.y;
      tmem_wait_st();
      if (!kEarlyRescale && j > 0) {
        // With one S buffer, S_i(j) was issued after P*V of tile j-1 and its
        // commit covers that product, so O_i is already final here.  With two
        // S buffers that product may still be running: wait for it.
        if constexpr (kSB == 2) {
          if (!(ok = mbar_wait_warp(bar_o_done + i, (j - 1) & 1, abort_flag, kDevTimeoutO))) break;
          tc_fence_after();
        }
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
          for (int cc = 0; cc < kDP / 32; ++cc) {
            uint32_t rr[32];
            tmem_ld32(t_o + cc * 32, rr);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) rr[e] = __float_as_uint(__uint_as_float(rr[e]) * alpha);
            tmem_st32(t_o + cc * 32, rr);
          }
          tmem_wait_st();
        }
      }
      l_run = l_run * alpha + lsum;
      m_run = m_new;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_p_full + slot);
    }

    // ------------------------------------------------------------ epilogue
    // Single pass: O in the input dtype and LSE at the caller's strides.  Key
    // splits: this split's normalised O in fp32 and its LSE, in the partial
    // buffers the combine kernel reads.
    const bool row_ok = row < (p.cu_q != nullptr ? seq_m : p.M);
    const int64_t part_row = (static_cast<int64_t>(blockIdx.y) * p.B + b) * p.Hq * static_cast<int64_t>(p.Mq) +
                             static_cast<int64_t>(oh) * p.Mq + qpos;
    T* orow = reinterpret_cast<T*>(p.o) + o_boff + oh * p.o_sh + static_cast<int64_t>(qpos) * p.o_sm;
    float* prow = p.o_part != nullptr ? p.o_part + part_row * p.D : nullptr;
    float* lse_out = p.o_part != nullptr ? p.lse_part + part_row
                     : p.lse != nullptr  ? p.lse + l_boff + oh * p.l_sh + static_cast<int64_t>(qpos) * p.l_sm
                                         : nullptr;
    bool via_tma = false;
    if constexpr (sizeof(T) == 2) {
      if (nt > 0 && p.o_tma) {
        via_tma = true;
        // Dense 16-bit O: the tile is staged in this Q tile's shared memory,
        // idle once O is final (every S product has completed by then), in
        // the 128-byte swizzled layout of a tm_o box, and written by one TMA
        // tensor store per 64-column atom: whole lines, clipped at the
        // tensor's bounds, instead of 16-byte pieces of 128 rows.  All four
        // warps reach the named barrier on every path.
        const uint32_t last_phase = kSB == 2 ? ((nt - 1) & 1) : 0u;
        const bool got = ok && mbar_wait_warp(bar_o_done + i, last_phase, abort_flag, kDevTimeoutO);
        tc_fence_after();
        uint8_t* stage = sQ + i * C::kQTileBytes;
        if (got) {
          const float inv_l = 1.0f / l_run;
#pragma unroll 1
          for (int cc = 0; cc < kDP / 32; ++cc) {
            uint32_t rr[32];
            tmem_ld32(t_o + cc * 32, rr);
            tmem_wait_ld();
            uint32_t pk[16];
#pragma unroll
            for (int e = 0; e < 16; ++e)
              pk[e] = ElemOps<T>::pack2(__uint_as_float(rr[2 * e]) * inv_l, __uint_as_float(rr[2 * e + 1]) * inv_l);
            uint8_t* rowp = stage + ((cc * 32) / C::kAtom) * C::kQAtomBytes + r * 128;
            const int chunk0 = ((cc * 32) % C::kAtom) * static_cast<int>(sizeof(T)) / 16;
#pragma unroll
            for (int q = 0; q < 4; ++q)
              *reinterpret_cast<uint4*>(rowp + (((chunk0 + q) ^ (r & 7)) * 16)) =
                  make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
          }
        }
        fence_proxy_async_smem();
        // Compile-time ids, so the kernel reserves only the barriers it names.
        if (i == 0)
          named_barrier_sync(1, 128);
        else
          named_barrier_sync(2, 128);
        if (r == 0 && got) {
#pragma unroll
          for (int a = 0; a < C::kNumAtoms; ++a)
            tma_store_4d(&tm_o, stage + a * C::kQAtomBytes, a * C::kAtom, m0 + i * C::kBM, h, b);
          bulk_commit_group();
          bulk_wait_read_all();
        }
        if (got && lse_out != nullptr && row_ok) {
          const float m_base = (m_run == kNegInf) ? 0.f : m_run;
          *lse_out = (m_base + log2f(l_run)) * 0.6931471805599453f;
        }
      }
    }
    if (via_tma) {
      // written above
    } else if (ok && nt > 0) {
      // One S buffer: O's only commit comes after the last product (phase 0);
      // two: one commit per KV tile.
      const uint32_t last_phase = kSB == 2 ? ((nt - 1) & 1) : 0u;
      ok = mbar_wait_warp(bar_o_done + i, last_phase, abort_flag, kDevTimeoutO);
      if (ok) {
        tc_fence_after();
        const float inv_l = 1.0f / l_run;
#pragma unroll 1
        for (int cc = 0; cc < kDP / 32; ++cc) {
          uint32_t rr[32];
          tmem_ld32(t_o + cc * 32, rr);
          tmem_wait_ld();
          float v[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(rr[e]) * inv_l;
          const int ncols = min(32, p.D - cc * 32);
          if (row_ok && ncols > 0) {
            if (p.o_part != nullptr)
              store_o_chunk<float>(prow + cc * 32, v, ncols);
            else
              store_o_chunk<T>(orow + cc * 32, v, ncols);
          }
        }
        if (lse_out != nullptr && row_ok) {
          const float m_base = (m_run == kNegInf) ? 0.f : m_run;
          *lse_out = (m_base + log2f(l_run)) * 0.6931471805599453f;
        }
      }
    } else if (ok && nt == 0 && row_ok) {
      if (p.o_part != nullptr) {
        // An empty split: weight zero in the combine.
        for (int d = 0; d < p.D; ++d) prow[d] = 0.f;
      } else {
        // No keys at all: 0/0 like the reference's acc / l_i.
        for (int d = 0; d < p.D; ++d) orow[d] = static_cast<T>(NAN);
      }
      if (lse_out != nullptr) *lse_out = kNegInf;
    }
    if constexpr (kNQ == 1) {
      // The K/V ring is idle here: every tile it held was consumed by
      // products that completed before O was final.
      if (p.split_cnt != nullptr)
        split_merge<T>(p, m0, b, h, wq, lane, tmem_slot + 2, reinterpret_cast<float*>(sKV),
                       kRing * C::kKVTileBytes / 4, bar_merge, abort_flag);
    }
  }
  }

  // ------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemAlloc);
  }
}

// ---------------------------------------------------------------- host side

// Causal launches deal (batch, head) items in groups whose K and V together
// take at most this much of the 126 MB L2 (see fa_fwd_kernel's work item).
#ifndef FAB_CAUSAL_GROUP_L2_MB
#define FAB_CAUSAL_GROUP_L2_MB 48
#endif
constexpr long long kCausalGroupL2Bytes = static_cast<long long>(FAB_CAUSAL_GROUP_L2_MB) << 20;

template <typename T, int kDP, int kNQ, int kBN, int kRing, int kSB>
static int launch_fa(const FaLaunch& L, cudaStream_t stream) {
  using C = FaCfg<sizeof(T), kDP, kNQ, kBN, kRing, kSB>;
  auto kern = fa_fwd_kernel<T, kDP, kNQ, kBN, kRing, kSB>;
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), C::kSmemBytes);
  if (rc) return rc;
  if constexpr (C::kSplitRegs) {
    // The register split assumes the launch allocation it was sized for;
    // refuse to launch a build that was compiled to anything else.
    cudaFuncAttributes a{};
    if (cudaFuncGetAttributes(&a, reinterpret_cast<const void*>(kern)) != cudaSuccess) return kErrLaunch;
    if (a.numRegs != C::kLaunchRegs) return kErrUnsupported;
  }
  CUtensorMap tq, tk, tv;
  const int elt = sizeof(T);
  const CUtensorMapDataType dt = elt == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : L.dtype == kDtypeBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  // V is the MN-major operand of P*V: tf32 needs the 32-byte-chunk swizzle there.
  const CUtensorMapSwizzle v_swz = elt == 4 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B;
  const int group = L.Hq / L.Hkv;
  // Rows of the kernel's query tiles: positions of one head, or with pack_gqa
  // the (head, position) pairs of one key/value head's query heads, which the
  // caller has checked are evenly spaced in memory.
  const int rows = L.pack_gqa ? group * L.M : L.M;
  const bool varlen = L.cu_q != nullptr;
  if (varlen) {
    // One flat [total, heads, D] tensor per operand; batch extent 1.
    rc = make_bhsd_map(&tq, L.q, dt, elt, L.D, L.total_q, L.Hq, 1, L.q_ss, L.q_sh, 0, C::kAtom, C::kBM,
                       CU_TENSOR_MAP_SWIZZLE_128B);
  } else if (L.pack_gqa) {
    const int64_t row_stride = L.M == 1 ? L.q_sh : L.q_ss;
    rc = make_bhsd_map(&tq, L.q, dt, elt, L.D, rows, L.Hkv, L.B, row_stride, group * L.q_sh, L.q_sb, C::kAtom,
                       C::kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    rc = make_bhsd_map(&tq, L.q, dt, elt, L.D, L.M, L.Hq, L.B, L.q_ss, L.q_sh, L.q_sb, C::kAtom, C::kBM,
                       CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (rc) return rc;
  // With no keys the kernel never reads K/V, but a tensor map needs extents >= 1.
  const int n_rows = varlen ? L.total_k : L.N;
  const int n_map = n_rows > 0 ? n_rows : 1;
  const int kv_b = varlen ? 1 : L.B;
  rc = make_bhsd_map(&tk, L.k, dt, elt, L.D, n_map, L.Hkv, kv_b, L.k_ss, L.k_sh, L.k_sb, C::kAtom, kBN,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_bhsd_map(&tv, L.v, dt, elt, L.D, n_map, L.Hkv, kv_b, L.v_ss, L.v_sh, L.v_sb, C::kAtom, kBN, v_swz);
  if (rc) return rc;
  FaKernelParams kp;
  kp.o = L.o;
  kp.lse = L.lse;
  kp.o_sb = L.o_sb;
  kp.o_sh = L.o_sh;
  kp.o_sm = L.o_ss;
  kp.l_sb = L.l_sb;
  kp.l_sh = L.l_sh;
  kp.l_sm = L.l_ss;
  kp.B = L.B;
  kp.Hq = L.Hq;
  kp.M = rows;
  kp.N = L.N;
  kp.D = L.D;
  kp.group = group;
  kp.scale_log2 = L.sm_scale * 1.4426950408889634f;
  kp.causal = L.causal;
  kp.num_m_blocks = (rows + kNQ * C::kBM - 1) / (kNQ * C::kBM);
  const int splits = L.num_splits > 0 ? L.num_splits : 1;
  kp.split_len = L.num_splits > 0 ? L.split_len : (L.N > 0 ? L.N : 1);
  kp.pack_gqa = L.pack_gqa;
  kp.Mq = L.M;
  kp.o_part = L.o_part;
  kp.lse_part = L.lse_part;
  kp.split_cnt = L.o_part != nullptr ? L.split_cnt : nullptr;
  kp.cu_q = L.cu_q;
  kp.cu_k = L.cu_k;
  // O through TMA tensor stores where the map allows it (dense, one query
  // head per row block, 16-bit, 16-byte-aligned base and strides).
  CUtensorMap to = tq;  // not read when o_tma is 0
  kp.o_tma = 0;
  if (elt == 2 && !varlen && !L.pack_gqa && L.o_part == nullptr && L.M > 0) {
    if (make_bhsd_map(&to, L.o, dt, elt, L.D, L.M, L.Hq, L.B, L.o_ss, L.o_sh, L.o_sb, C::kAtom, C::kBM,
                      CU_TENSOR_MAP_SWIZZLE_128B) == 0)
      kp.o_tma = 1;
    else
      to = tq;
  }
  const int items = L.B * (L.pack_gqa ? L.Hkv : L.Hq);
  const long long grid = static_cast<long long>(kp.num_m_blocks) * items;
  if (grid <= 0) return 0;
  // Causal row blocks differ in length: deal the (batch, head) items in
  // groups whose K and V fit in a slice of L2 and run each group's row blocks
  // longest first.  Without a mask every block is as long, and one item per
  // group keeps a head's blocks together.
  kp.head_group = 1;
  if (L.causal) {
    // K and V bytes per item: the query heads of one key/value head share it.
    const long long kv_bytes = 2LL * (L.N > 0 ? L.N : 1) * L.D * elt / (L.pack_gqa ? 1 : group);
    const long long fit = kCausalGroupL2Bytes / (kv_bytes > 0 ? kv_bytes : 1);
    kp.head_group = static_cast<int>(fit < 1 ? 1 : (fit > items ? items : fit));
  }
  if (grid > 0x7fffffffLL || splits > 65535) return kErrInvalidArg;
  kern<<<dim3(static_cast<unsigned>(grid), static_cast<unsigned>(splits)), C::kThreads, C::kSmemBytes, stream>>>(
      kp, tq, tk, tv, to);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrLaunch;
}

// Merges the key splits of every output row: with split s holding the
// normalised O_s and LSE_s of its keys, O = sum_s w_s O_s / sum_s w_s and
// LSE = max + log(sum_s w_s), w_s = exp(LSE_s - max).  One CTA per row: the
// weights are computed once, one split per thread, into shared memory; then
// each of the eight warps adds every eighth split's O_s (several loads in
// flight per warp) and the warps' sums meet in shared memory.
constexpr int kCombineWarps = 8;
constexpr int kCombineSmemSplits = 1024;  // more splits recompute their weight from the LSE

template <typename T>
__global__ void __launch_bounds__(kCombineWarps * 32) fa_split_combine_kernel(
    const float* __restrict__ o_part, const float* __restrict__ lse_part, T* o, float* lse, int64_t o_sb,
    int64_t o_sh, int64_t o_sm, int64_t l_sb, int64_t l_sh, int64_t l_sm, int Hq, int M, int D, int splits,
    int64_t rows) {
  constexpr int kMaxPerLane = 8;  // head dims up to 256
  __shared__ float s_red[kCombineWarps];
  __shared__ float s_w[kCombineSmemSplits];
  __shared__ float s_acc[kCombineWarps][kMaxPerLane * 32];
  const int64_t row = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m = static_cast<int>(row % M);
  const int h = static_cast<int>((row / M) % Hq);
  const int64_t b = row / (static_cast<int64_t>(M) * Hq);
  T* orow = o + b * o_sb + h * o_sh + m * o_sm;

  float mx = -INFINITY;
  for (int sp = threadIdx.x; sp < splits; sp += blockDim.x) mx = fmaxf(mx, lse_part[sp * rows + row]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if (lane == 0) s_red[warp] = mx;
  __syncthreads();
  mx = s_red[0];
#pragma unroll
  for (int w = 1; w < kCombineWarps; ++w) mx = fmaxf(mx, s_red[w]);
  if (mx == -INFINITY) {
    // No split saw a key: 0/0 like the single-pass kernel.
    for (int d = threadIdx.x; d < D; d += blockDim.x) orow[d] = static_cast<T>(NAN);
    if (lse != nullptr && threadIdx.x == 0) lse[b * l_sb + h * l_sh + m * l_sm] = -INFINITY;
    return;
  }
  auto weight = [&](int sp) {
    const float ls = lse_part[sp * rows + row];
    return ls == -INFINITY ? 0.f : expf(ls - mx);  // an empty split carries zeros
  };
  for (int sp = threadIdx.x; sp < min(splits, kCombineSmemSplits); sp += blockDim.x) s_w[sp] = weight(sp);
  __syncthreads();
  float acc[kMaxPerLane];
#pragma unroll
  for (int e = 0; e < kMaxPerLane; ++e) acc[e] = 0.f;
  float wsum = 0.f;
#pragma unroll 4
  for (int sp = warp; sp < splits; sp += kCombineWarps) {
    const float w = sp < kCombineSmemSplits ? s_w[sp] : weight(sp);
    wsum += w;
    const float* src = o_part + (sp * rows + row) * D;
#pragma unroll
    for (int e = 0; e < kMaxPerLane; ++e) {
      const int d = lane + 32 * e;
      if (d < D) acc[e] = fmaf(w, src[d], acc[e]);
    }
  }
  __syncthreads();  // every warp is done with s_red before it is reused for the weight sums
#pragma unroll
  for (int e = 0; e < kMaxPerLane; ++e) s_acc[warp][lane + 32 * e] = acc[e];
  if (lane == 0) s_red[warp] = wsum;
  __syncthreads();
  float total_w = 0.f;
#pragma unroll
  for (int w = 0; w < kCombineWarps; ++w) total_w += s_red[w];
  const float inv = 1.f / total_w;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < kCombineWarps; ++w) sum += s_acc[w][d];
    orow[d] = static_cast<T>(sum * inv);
  }
  if (lse != nullptr && threadIdx.x == 0) lse[b * l_sb + h * l_sh + m * l_sm] = mx + logf(total_w);
}

// The sm_100a tile table: one instantiation per (element size, padded head
// dim).  Columns: element size, padded head dim, Q tiles per CTA, BLOCK_N,
// K/V ring slots (as many tiles as fit beside the Q tiles), S buffers.
#define FAB_FA_TABLE(X)                                    \
  X(2, 64, 2, 128, 10, 1)   /* 16-bit, head dim <= 64 */    \
  X(2, 128, 2, 128, 5, 1)   /* 16-bit, head dim <= 128 */   \
  X(2, 256, 1, 128, 2, 2)   /* 16-bit, head dim <= 256 */   \
  X(4, 64, 2, 128, 5, 1)    /* fp32/tf32, head dim <= 64 */ \
  X(4, 128, 1, 128, 2, 2)   /* fp32/tf32, head dim <= 128 */

static bool fa_table_lookup(int elt, int D, int* d_pad) {
  int best = 0;
#define FAB_FA_PICK(E, DP, NQ, BN, ST, SB) \
  if (elt == E && D <= DP && (best == 0 || DP < best)) best = DP;
  FAB_FA_TABLE(FAB_FA_PICK)
#undef FAB_FA_PICK
  *d_pad = best;
  return best != 0;
}

int fa_select_config(int dtype, int D, FaConfigInfo* out) {
  if (D <= 0) return kErrInvalidArg;
  if (dtype != kDtypeF16 && dtype != kDtypeBF16 && dtype != kDtypeF32) return kErrInvalidArg;
  const int elt = dtype == kDtypeF32 ? 4 : 2;
  int dp = 0;
  if (!fa_table_lookup(elt, D, &dp)) return kErrUnsupported;
#define FAB_FA_FILL(E, DP, NQ, BN, ST, SB)                                                         \
  if (elt == E && dp == DP) {                                                                     \
    using Cf = FaCfg<E, DP, NQ, BN, ST, SB>;                                                      \
    *out = FaConfigInfo{DP, NQ, BN, ST, Cf::kThreads, Cf::kSmemBytes, Cf::kTmemAlloc, SB};        \
    return 0;                                                                                     \
  }
  FAB_FA_TABLE(FAB_FA_FILL)
#undef FAB_FA_FILL
  return kErrUnsupported;
}

// Dispatch helpers: templates, so the branch for the other element size is
// discarded instead of instantiated.
template <int E, int DP, int NQ, int BN, int ST, int SB>
static int launch_entry(const FaLaunch& L, cudaStream_t stream) {
  if constexpr (E == 4) {
    return launch_fa<float, DP, NQ, BN, ST, SB>(L, stream);
  } else {
    if (L.dtype == kDtypeBF16) return launch_fa<__nv_bfloat16, DP, NQ, BN, ST, SB>(L, stream);
    return launch_fa<__half, DP, NQ, BN, ST, SB>(L, stream);
  }
}

template <int E, int DP, int NQ, int BN, int ST, int SB>
static const void* kernel_entry(int dtype) {
  if constexpr (E == 4) {
    return reinterpret_cast<const void*>(fa_fwd_kernel<float, DP, NQ, BN, ST, SB>);
  } else {
    if (dtype == kDtypeBF16) return reinterpret_cast<const void*>(fa_fwd_kernel<__nv_bfloat16, DP, NQ, BN, ST, SB>);
    return reinterpret_cast<const void*>(fa_fwd_kernel<__half, DP, NQ, BN, ST, SB>);
  }
}

int fa_forward(const FaLaunch& L, cudaStream_t stream) {
  FaConfigInfo c;
  int rc = fa_select_config(L.dtype, L.D, &c);
  if (rc) return rc;
  const int elt = L.dtype == kDtypeF32 ? 4 : 2;
#define FAB_FA_LAUNCH(E, DP, NQ, BN, ST, SB) \
  if (elt == E && c.d_pad == DP) return launch_entry<E, DP, NQ, BN, ST, SB>(L, stream);
  FAB_FA_TABLE(FAB_FA_LAUNCH)
#undef FAB_FA_LAUNCH
  return kErrUnsupported;
}

// Tiles for split-KV launches (short query blocks against long key ranges):
// one 128-row query tile per CTA with two S buffers, so S(j+1) is computed
// while the softmax of tile j runs and the CTA streams K/V at the rate the
// memory system gives it.
#define FAB_FA_SPLIT_TABLE(X)                              \
  X(2, 64, 1, 128, 8, 2)    /* 16-bit, head dim <= 64 */    \
  X(2, 128, 1, 128, 6, 2)   /* 16-bit, head dim <= 128 */   \
  X(2, 256, 1, 128, 2, 2)   /* 16-bit, head dim <= 256 */   \
  X(4, 64, 1, 128, 6, 2)    /* fp32/tf32, head dim <= 64 */ \
  X(4, 128, 1, 128, 2, 2)   /* fp32/tf32, head dim <= 128 */

// The one-query-tile family run as a single pass (FAB_FA_VARIANT_ONE_TILE,
// picked for shapes with few query tiles): two CTAs per SM with one S buffer
// each where that fits and the launch has at least 1.5 CTAs per SM, so that
// most SMs hold two tiles that take turns on the tensor core; otherwise (or
// with too few CTAs, when a lone one-buffer CTA would leave its tensor core
// idle during every softmax) the split-KV tiles, whose two S buffers overlap
// S(j+1) with softmax(j) inside one CTA.
#define FAB_FA_ONE_TILE_TABLE(X)                                         \
  X(2, 64, 1, 128, 4, 1)    /* 16-bit, head dim <= 64: 2 CTAs/SM */      \
  X(2, 128, 1, 128, 2, 1)   /* 16-bit, head dim <= 128: 2 CTAs/SM */     \
  X(2, 256, 1, 128, 2, 2)   /* 16-bit, head dim <= 256 */                \
  X(4, 64, 1, 128, 2, 1)    /* fp32/tf32, head dim <= 64: 2 CTAs/SM */   \
  X(4, 128, 1, 128, 2, 2)   /* fp32/tf32, head dim <= 128 */

int fa_select_one_tile_config(int dtype, int D, FaConfigInfo* out) {
  if (D <= 0) return kErrInvalidArg;
  if (dtype != kDtypeF16 && dtype != kDtypeBF16 && dtype != kDtypeF32) return kErrInvalidArg;
  const int elt = dtype == kDtypeF32 ? 4 : 2;
  int best = 0;
#define FAB_FA_OPICK(E, DP, NQ, BN, ST, SB) \
  if (elt == E && D <= DP && (best == 0 || DP < best)) best = DP;
  FAB_FA_ONE_TILE_TABLE(FAB_FA_OPICK)
#undef FAB_FA_OPICK
  if (best == 0) return kErrUnsupported;
#define FAB_FA_OFILL(E, DP, NQ, BN, ST, SB)                                                      \
  if (elt == E && best == DP) {                                                                 \
    using Cf = FaCfg<E, DP, NQ, BN, ST, SB>;                                                    \
    *out = FaConfigInfo{DP, NQ, BN, ST, Cf::kThreads, Cf::kSmemBytes, Cf::kTmemAlloc, SB};      \
    return 0;                                                                                   \
  }
  FAB_FA_ONE_TILE_TABLE(FAB_FA_OFILL)
#undef FAB_FA_OFILL
  return kErrUnsupported;
}

int fa_forward_split(const FaLaunch& L, cudaStream_t stream);

// CTAs in the grid of a non-varlen launch whose tile holds nq query tiles.
static long long fa_grid_ctas(const FaLaunch& L, int nq) {
  const long long rows = L.pack_gqa ? static_cast<long long>(L.Hq / L.Hkv) * L.M : L.M;
  const long long per_cta = 128LL * nq;
  return (rows + per_cta - 1) / per_cta * L.B * (L.pack_gqa ? L.Hkv : L.Hq) * std::max(L.num_splits, 1);
}

int fa_plan(const FaLaunch& L, int variant, FaPlanInfo* out) {
  int rc;
  out->split_table = false;
  if (variant == 0) {
    rc = fa_select_config(L.dtype, L.D, &out->cfg);
  } else {
    rc = fa_select_one_tile_config(L.dtype, L.D, &out->cfg);
    if (rc == 0 && out->cfg.s_bufs == 1) {
      // Two CTAs per SM only pay when most SMs get two: below 1.5 CTAs per
      // SM the split tiles (two S buffers in one CTA) run the pass instead.
      const int sms = num_sms();
      if (sms <= 0) return kErrCuda;
      if (2 * fa_grid_ctas(L, out->cfg.nq) < 3LL * sms) {
        rc = fa_select_split_config(L.dtype, L.D, &out->cfg);
        out->split_table = true;
      }
    }
  }
  if (rc) return rc;
  out->ctas = fa_grid_ctas(L, out->cfg.nq);
  out->ctas_per_sm = (out->cfg.nq == 1 && out->cfg.s_bufs == 1) ? 2 : 1;
  return kOk;
}

int fa_forward_one_tile(const FaLaunch& L, cudaStream_t stream) {
  FaPlanInfo plan;
  int rc = fa_plan(L, 1, &plan);
  if (rc) return rc;
  if (plan.split_table) return fa_forward_split(L, stream);
  const FaConfigInfo& c = plan.cfg;
  const int elt = L.dtype == kDtypeF32 ? 4 : 2;
  rc = kErrUnsupported;
#define FAB_FA_OLAUNCH(E, DP, NQ, BN, ST, SB) \
  if (elt == E && c.d_pad == DP) rc = launch_entry<E, DP, NQ, BN, ST, SB>(L, stream);
  FAB_FA_ONE_TILE_TABLE(FAB_FA_OLAUNCH)
#undef FAB_FA_OLAUNCH
  return rc;
}

int fa_select_split_config(int dtype, int D, FaConfigInfo* out) {
  if (D <= 0) return kErrInvalidArg;
  if (dtype != kDtypeF16 && dtype != kDtypeBF16 && dtype != kDtypeF32) return kErrInvalidArg;
  const int elt = dtype == kDtypeF32 ? 4 : 2;
  int best = 0;
#define FAB_FA_SPICK(E, DP, NQ, BN, ST, SB) \
  if (elt == E && D <= DP && (best == 0 || DP < best)) best = DP;
  FAB_FA_SPLIT_TABLE(FAB_FA_SPICK)
#undef FAB_FA_SPICK
  if (best == 0) return kErrUnsupported;
#define FAB_FA_SFILL(E, DP, NQ, BN, ST, SB)                                                      \
  if (elt == E && best == DP) {                                                                 \
    using Cf = FaCfg<E, DP, NQ, BN, ST, SB>;                                                    \
    *out = FaConfigInfo{DP, NQ, BN, ST, Cf::kThreads, Cf::kSmemBytes, Cf::kTmemAlloc, SB};      \
    return 0;                                                                                   \
  }
  FAB_FA_SPLIT_TABLE(FAB_FA_SFILL)
#undef FAB_FA_SFILL
  return kErrUnsupported;
}

static size_t align256(size_t x) { return (x + 255) / 256 * 256; }

// Key splits on the two-CTAs-per-SM one-tile kernel (one S buffer per CTA,
// two CTAs sharing each SM) instead of the two-S-buffer tile, with twice the
// CTAs.
#ifndef FAB_SPLIT_DUAL
#define FAB_SPLIT_DUAL 0
#endif

int fa_split_plan(const FaLaunch& L, int num_splits, FaSplitPlan* plan) {
  FaConfigInfo cfg;
  int rc = fa_select_split_config(L.dtype, L.D, &cfg);
  if (rc) return rc;
  int per_sm = 1;
  plan->dual = 0;
  if (FAB_SPLIT_DUAL) {
    FaConfigInfo one;
    if (fa_select_one_tile_config(L.dtype, L.D, &one) == 0 && one.s_bufs == 1) {
      cfg = one;
      per_sm = 2;
      plan->dual = 1;
    }
  }
  const int group = L.Hq / L.Hkv;
  // Pack a key/value head's query heads into one tile when their rows are
  // evenly spaced: every query position of a head, then the next head.
  const bool even = L.M == 1 || L.q_sh == static_cast<int64_t>(L.M) * L.q_ss;
  plan->pack_gqa = (group > 1 && even) ? 1 : 0;
  const int64_t rows = plan->pack_gqa ? static_cast<int64_t>(group) * L.M : L.M;
  const int64_t rows_per_cta = static_cast<int64_t>(cfg.nq) * 128;
  const int64_t base_ctas = (rows + rows_per_cta - 1) / rows_per_cta * L.B * (plan->pack_gqa ? L.Hkv : L.Hq);
  const int tiles = L.N > 0 ? (L.N + cfg.bn - 1) / cfg.bn : 0;
  int splits = num_splits;
  if (splits <= 0) {
    // As many splits as keep every CTA in one wave (at most one per SM): a
    // few CTAs past the wave would run their whole range after it.
    const int sms = num_sms();
    if (sms <= 0) return kErrCuda;
    splits = static_cast<int>(static_cast<long long>(per_sm) * sms / (base_ctas > 0 ? base_ctas : 1));
  }
  splits = std::max(1, std::min({splits, std::max(tiles, 1), 65535}));
  const int tiles_per_split = tiles > 0 ? (tiles + splits - 1) / splits : 1;
  plan->split_len = tiles_per_split * cfg.bn;
  plan->num_splits = L.N > 0 ? (L.N + plan->split_len - 1) / plan->split_len : 1;
  if (plan->num_splits <= 1) plan->dual = 0;  // a single pass keeps the two-S-buffer tile
  plan->rows = static_cast<int64_t>(L.B) * L.Hq * L.M;
  plan->workspace_bytes = 0;
  plan->lse_offset = 0;
  plan->counter_offset = 0;
  plan->groups = base_ctas;
  if (plan->num_splits > 1) {
    plan->lse_offset = align256(sizeof(float) * plan->num_splits * plan->rows * L.D);
    plan->counter_offset = plan->lse_offset + align256(sizeof(float) * plan->num_splits * plan->rows);
    plan->workspace_bytes = plan->counter_offset + align256(sizeof(unsigned int) * base_ctas);
  }
  return 0;
}

int fa_forward_split(const FaLaunch& L, cudaStream_t stream) {
  FaConfigInfo c;
  int rc = L.split_dual ? fa_select_one_tile_config(L.dtype, L.D, &c) : fa_select_split_config(L.dtype, L.D, &c);
  if (rc) return rc;
  const int elt = L.dtype == kDtypeF32 ? 4 : 2;
  rc = kErrUnsupported;
#define FAB_FA_SLAUNCH(E, DP, NQ, BN, ST, SB) \
  if (elt == E && c.d_pad == DP) rc = launch_entry<E, DP, NQ, BN, ST, SB>(L, stream);
  if (L.split_dual) {
    FAB_FA_ONE_TILE_TABLE(FAB_FA_SLAUNCH)
  } else {
    FAB_FA_SPLIT_TABLE(FAB_FA_SLAUNCH)
  }
#undef FAB_FA_SLAUNCH
  // Merged inside the split kernel when the launch carries the counters.
  if (rc || L.num_splits <= 1 || L.o_part == nullptr || L.split_cnt != nullptr) return rc;
  const int64_t rows = static_cast<int64_t>(L.B) * L.Hq * L.M;
  const long long blocks = rows;  // one CTA per output row
  if (blocks > 0x7fffffffLL) return kErrInvalidArg;
  const unsigned g = static_cast<unsigned>(blocks);
  if (L.dtype == kDtypeBF16) {
    fa_split_combine_kernel<__nv_bfloat16><<<g, kCombineWarps * 32, 0, stream>>>(
        L.o_part, L.lse_part, static_cast<__nv_bfloat16*>(L.o), L.lse, L.o_sb, L.o_sh, L.o_ss, L.l_sb, L.l_sh, L.l_ss,
        L.Hq, L.M, L.D, L.num_splits, rows);
  } else if (L.dtype == kDtypeF16) {
    fa_split_combine_kernel<__half><<<g, kCombineWarps * 32, 0, stream>>>(L.o_part, L.lse_part, static_cast<__half*>(L.o), L.lse,
                                                           L.o_sb, L.o_sh, L.o_ss, L.l_sb, L.l_sh, L.l_ss, L.Hq, L.M,
                                                           L.D, L.num_splits, rows);
  } else {
    fa_split_combine_kernel<float><<<g, kCombineWarps * 32, 0, stream>>>(L.o_part, L.lse_part, static_cast<float*>(L.o), L.lse,
                                                          L.o_sb, L.o_sh, L.o_ss, L.l_sb, L.l_sh, L.l_ss, L.Hq, L.M,
                                                          L.D, L.num_splits, rows);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : kErrLaunch;
}

int fa_kernel_attrs(int dtype, int D, int* regs, int* smem, int* threads, bool one_tile) {
  FaConfigInfo c;
  int rc = one_tile ? fa_select_one_tile_config(dtype, D, &c) : fa_select_config(dtype, D, &c);
  if (rc) return rc;
  const int elt = dtype == kDtypeF32 ? 4 : 2;
  const void* k = nullptr;
#define FAB_FA_ATTR(E, DP, NQ, BN, ST, SB) \
  if (elt == E && c.d_pad == DP) k = kernel_entry<E, DP, NQ, BN, ST, SB>(dtype);
  if (one_tile) {
    FAB_FA_ONE_TILE_TABLE(FAB_FA_ATTR)
  } else {
    FAB_FA_TABLE(FAB_FA_ATTR)
  }
#undef FAB_FA_ATTR
  if (k == nullptr) return kErrUnsupported;
  cudaFuncAttributes a{};
  if (cudaFuncGetAttributes(&a, k) != cudaSuccess) return kErrLaunch;
  *regs = a.numRegs;
  *smem = c.smem_bytes;
  *threads = c.threads;
  return 0;
}

}  // namespace fab
