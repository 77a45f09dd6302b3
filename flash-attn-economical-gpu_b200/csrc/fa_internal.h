// Internal (C++) declarations shared by the kernels and the C-ABI layer.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace fab {

// Return codes (mirrored by the public FAB_* constants in include/fa_b200.h).
enum : int {
  kOk = 0,
  kErrInvalidArg = 1,
  kErrUnsupported = 2,
  kErrLaunch = 3,
  kErrDeviceTimeout = 4,
  kErrCuda = 5,
  kErrWorkspace = 6,
};

enum : int { kDtypeF16 = 0, kDtypeBF16 = 1, kDtypeF32 = 2 };

// What the FlashAttention kernel reads from its parameter block.
struct FaKernelParams {
  void* o;
  float* lse;
  int64_t o_sb, o_sh, o_sm;
  int64_t l_sb, l_sh, l_sm;
  int B, Hq, M, N, D;
  int group;
  float scale_log2;
  int causal;
  int num_m_blocks;
  // blockIdx.x walks groups of head_group (batch, head) items; inside a group
  // the row block is the slow index (longest first) and the item the fast one.
  int head_group;
  // Key splits: CTA (x, y) attends to keys [y * split_len, (y + 1) * split_len).
  // Without splitting split_len >= N and gridDim.y == 1.
  int split_len;
  // pack_gqa: the M rows are (query head, position) pairs of the `group`
  // query heads that share one key/value head, position = row % Mq.
  int pack_gqa;
  int Mq;
  // With key splits each CTA writes its split's normalised O (fp32,
  // [split][B][Hq][Mq][D]) and LSE ([split][B][Hq][Mq]) here instead of o/lse.
  float* o_part;
  float* lse_part;
  // With key splits: one counter per row group (blockIdx.x), zero between
  // calls.  The last split CTA of a group to finish merges the group's
  // partials into o / lse and sets the counter back to zero.
  unsigned int* split_cnt;
  // Packed variable-length batches: sequence b's query rows are
  // [cu_q[b], cu_q[b+1]) of a [total, heads, D] tensor (keys likewise with
  // cu_k); M and N are then the longest lengths.  NULL for dense batches.
  const int* cu_q;
  const int* cu_k;
  // 1: O (dense, 16-bit, 16-byte-aligned strides) is written by TMA tensor
  // stores from shared memory through the tm_o map; 0: direct stores.
  int o_tma;
};

// A fully validated attention launch (element strides, unit stride on D).
struct FaLaunch {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  float* lse;
  int64_t q_sb, q_sh, q_ss;
  int64_t k_sb, k_sh, k_ss;
  int64_t v_sb, v_sh, v_ss;
  int64_t o_sb, o_sh, o_ss;
  int64_t l_sb, l_sh, l_ss;
  int B, Hq, Hkv, M, N, D;
  int dtype;
  float sm_scale;
  int causal;
  // Split-KV launches only (zero for the single-pass path).
  int num_splits;
  int split_len;
  int pack_gqa;
  float* o_part;
  float* lse_part;
  unsigned int* split_cnt;  // see FaKernelParams
  int split_dual;           // key splits on the two-CTAs-per-SM one-tile kernel (see FaSplitPlan)
  // Packed variable-length batches (see FaKernelParams); the tensor maps
  // then span total_q / total_k rows with batch extent 1.
  const int* cu_q;
  const int* cu_k;
  int total_q;
  int total_k;
};

// Plan of a split-KV launch: the tile config it runs and the workspace it needs.
struct FaSplitPlan {
  int num_splits;
  int split_len;
  int pack_gqa;
  int64_t rows;            // B * Hq * M output rows
  size_t workspace_bytes;  // o_part, lse_part, then the row groups' counters, each 256-byte aligned
  size_t lse_offset;       // byte offset of lse_part in the workspace
  size_t counter_offset;   // byte offset of the counters (which start at zero)
  int64_t groups;          // row groups (CTAs per key split): one counter each
  int dual;                // 1: the splits run on the two-CTAs-per-SM one-tile kernel, two CTAs per SM
};

struct FaConfigInfo {
  int d_pad;
  int nq;
  int bn;
  int stages;
  int threads;
  int smem_bytes;
  int tmem_cols;
  int s_bufs;
};

struct GemmKernelParams {
  void* c;
  int64_t ldc;
  int M, N, K;
  int group_m;
  int round_f16;
  // SwiGLU epilogue: B's columns alternate 64 gate / 64 up columns, and C
  // receives round(round(silu(round(g))) * round(u)), N / 2 columns.
  int swiglu;
  // Bias + rotate-half RoPE epilogue (bias_rope 1): every column gets
  // round(round(acc) + bias), and the heads of head_dim columns among the
  // first rope_cols are rotated with row r's cos/sin ([M][head_dim] tables).
  int bias_rope;
  int rope_cols;
  int head_dim;
  const void* bias;  // [N] or null
  const void* rope_cos;
  const void* rope_sin;
  // [M] fp32 or null: row r's accumulator is multiplied by row_scale[r]
  // before any epilogue rounding (an RMSNorm's 1/rms folded into the GEMM
  // that consumes the normalised rows; its weight is folded into B).
  const float* row_scale;
  // Stream-K schedule of the CTA-pair kernel (plain store epilogue only):
  // tiles [0, sk_dp_tiles) run whole, round robin over the pairs; the K
  // blocks of the remaining tiles are split evenly over all pairs, and each
  // such tile is finished by the pair holding its last K block (its owner),
  // which adds the partial sums the other pairs left in sk_part.
  // sk_part == nullptr turns stream-K off.
  int sk_dp_tiles;
  float* sk_part;  // [pairs][2 CTAs][kBN / 4][128 rows] float4: one partial tile per pair and CTA
  int* sk_flags;   // [pairs][2 CTAs][4 epilogue warps]; zero between calls
  // CTA-pair kernel, whole tiles: 1 launches one cluster per tile, and a
  // running cluster takes the tile of the next cluster that has not started
  // (cluster launch control) instead of a fixed round robin; 0 launches one
  // cluster per resident pair.
  int dyn_sched;
};

// Fused GEMM + all-reduce over NVLink peer memory (tensor-parallel output
// projections).  Pointers index by rank; this rank's own entries are local.
constexpr int kMaxTpRanks = 8;
struct GemmArParams {
  void* inbox[kMaxTpRanks];                 // [world][tiles_per_owner][128][256] partial tiles, per rank
  void* out[kMaxTpRanks];                   // [M][ldo] reduced output, per rank
  unsigned long long* arrive[kMaxTpRanks];  // [tiles_per_owner] partial-tile arrivals, per rank
  unsigned long long* done[kMaxTpRanks];    // reduced tiles landed, one counter per rank
  int64_t ldo;
  int world;
  int rank;
  int tiles_per_owner;
  int overlap;  // the two idle warps of each CTA reduce owned tiles during the GEMM
};

struct GemmLaunch {
  const void* a;
  const void* b;
  void* c;
  int64_t lda, ldb, ldc;
  int M, N, K;
  int in_dtype, out_dtype;
  int round_f16;
  int group_m;
  int swiglu;
  int bias_rope;  // see GemmKernelParams
  int rope_cols;
  int head_dim;
  const void* bias;
  const void* rope_cos;
  const void* rope_sin;
  const float* row_scale;  // see GemmKernelParams
  void* workspace;         // stream-K partial tiles and flags, or null
  size_t workspace_bytes;
};

// Epilogues that need whole 256-column tiles (gate/up block pairs, whole heads).
inline bool gemm_fixed_width(const GemmLaunch& L) { return L.swiglu || L.bias_rope; }

int fa_select_config(int dtype, int D, FaConfigInfo* out);
int fa_forward(const FaLaunch& L, cudaStream_t stream);
int fa_select_split_config(int dtype, int D, FaConfigInfo* out);
int fa_select_one_tile_config(int dtype, int D, FaConfigInfo* out);
int fa_forward_one_tile(const FaLaunch& L, cudaStream_t stream);
// The tile a forward launch of `variant` (0 two tiles, 1 one tile) runs, its
// grid size and how many of its CTAs share an SM; fa_forward_one_tile takes
// its kernel from this.
struct FaPlanInfo {
  FaConfigInfo cfg;
  long long ctas;
  int ctas_per_sm;
  bool split_table;  // the one-tile call runs the split-KV tile as one pass
};
int fa_plan(const FaLaunch& L, int variant, FaPlanInfo* out);
// num_splits <= 0 picks a split count from the SM count (needs a device).
int fa_split_plan(const FaLaunch& L, int num_splits, FaSplitPlan* plan);
// Launches the split kernel and the combine kernel; L carries the plan.
int fa_forward_split(const FaLaunch& L, cudaStream_t stream);
int fa_kernel_attrs(int dtype, int D, int* regs, int* smem, int* threads, bool one_tile = false);
int gemm_forward(const GemmLaunch& L, cudaStream_t stream);
int gemm_plan(const GemmLaunch& L, int* kernel, int* split, int* tile_n);
// Workspace the stream-K schedule would use for L (0 when it is not chosen).
size_t gemm_workspace_bytes(const GemmLaunch& L);
// CTAs in the grid gemm_forward would launch for L.
long long gemm_grid_ctas(const GemmLaunch& L);
// Output tiles of the fused GEMM + all-reduce: tile t belongs to rank t % world.
int gemm_ar_tiles(int M, int N);
int gemm_allreduce(const GemmLaunch& L, const GemmArParams& ar, cudaStream_t stream);
int gemm_kernel_attrs(int in_dtype, int* regs, int* smem, int* threads);
// Reads and clears the GEMM translation unit's device status word.
int gemm_take_device_error(int* code);

// Helpers implemented in capi.cu.
int ensure_smem_attr(const void* kernel, int bytes);
int num_sms();
// 4-D [B, H, S, D] tensor map with unit stride on D, 128-byte swizzle,
// box = {atom, rows, 1, 1}.
int make_bhsd_map(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elt, int D, int S, int H, int B,
                  int64_t s_s, int64_t s_h, int64_t s_b, int box_inner, int box_rows, CUtensorMapSwizzle swizzle);
// 2-D [rows, cols] row-major tensor map, 128-byte swizzle, box = {inner, rows}.
int make_2d_map(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elt, int cols, int rows, int64_t ld,
                int box_inner, int box_rows, CUtensorMapSwizzle swizzle);

}  // namespace fab
