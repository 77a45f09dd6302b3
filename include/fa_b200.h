/*
 * fa_b200.h -- C ABI of the B200 (sm_100a) FlashAttention-forward and matmul
 * kernels that stand in for the Triton kernels of flash-attn-economical-gpu.
 *
 * Every entry point takes plain device pointers, sizes and element strides,
 * launches asynchronously on the given CUDA stream (a cudaStream_t passed as
 * void*; NULL is the legacy default stream) and returns FAB_OK or a FAB_ERR_*
 * code.  Nothing here allocates device memory, synchronises the stream or
 * aborts the process.  All entry points are safe to call from several host
 * threads.
 *
 * Layout rules shared by the attention entry points: tensors are indexed
 * [batch, head, seq, head_dim] with arbitrary element strides for the first
 * three dims, stride 1 along head_dim, 16-byte aligned base pointers and
 * strides that are multiples of 16 bytes (the Tensor Memory Accelerator reads
 * them directly).  Inputs outside these rules return FAB_ERR_INVALID_ARG; the
 * Python layer copies such tensors into conforming ones first.
 */
#ifndef FA_B200_H_
#define FA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes. */
#define FAB_OK 0
#define FAB_ERR_INVALID_ARG 1     /* bad pointer, shape, stride or alignment */
#define FAB_ERR_UNSUPPORTED 2     /* valid request outside the kernels' range (e.g. head_dim > 256) */
#define FAB_ERR_LAUNCH 3          /* the CUDA launch itself failed */
#define FAB_ERR_DEVICE_TIMEOUT 4  /* a kernel gave up on a bounded wait (see fab_get_device_error) */
#define FAB_ERR_CUDA 5            /* another CUDA runtime error */
#define FAB_ERR_WORKSPACE 6       /* split-KV workspace missing, not 256-byte aligned, or too small */

/* Element types. */
#define FAB_DTYPE_F16 0
#define FAB_DTYPE_BF16 1
#define FAB_DTYPE_F32 2 /* computed on the tensor cores as tf32, like Triton's default tl.dot */

/*
 * Replaces `_flash_attn_fwd_kernel_basic[grid](q, k, v, o, lse, strides..., H, M, N, D,
 * sm_scale, causal=, HAS_LSE=, ...)` (flash_atten.py:14-51, launched from
 * flash_atten.py:377 with grid (cdiv(M, BLOCK_M), B*H) built at tuner.py:264-295).
 * o = softmax(sm_scale * q k^T [causal: key n visible to query m iff m >= n]) v,
 * fp32 softmax, P rounded to the input dtype before P*V; lse[b,h,m] (fp32,
 * natural log) is written when has_lse != 0.  sm_scale must be > 0.
 */
int fab_flash_attn_fwd_basic(const void* q, const void* k, const void* v, void* o, float* lse,
                             int64_t stride_qb, int64_t stride_qh, int64_t stride_qm, int64_t stride_qd,
                             int64_t stride_kb, int64_t stride_kh, int64_t stride_kn, int64_t stride_kd,
                             int64_t stride_vb, int64_t stride_vh, int64_t stride_vn, int64_t stride_vd,
                             int64_t stride_ob, int64_t stride_oh, int64_t stride_om, int64_t stride_od,
                             int64_t stride_lb, int64_t stride_lh, int64_t stride_lm, int B, int H, int M, int N,
                             int D, float sm_scale, int causal, int has_lse, int dtype, void* stream);

/*
 * Replaces `_flash_attn_fwd_kernel_optimize_shared_mem[grid](...)` (flash_atten.py:136-173).
 * Same arguments and results as fab_flash_attn_fwd_basic; on sm_100a both
 * variants run the same tcgen05 kernel.
 */
int fab_flash_attn_fwd_optimize_shared_mem(const void* q, const void* k, const void* v, void* o, float* lse,
                                           int64_t stride_qb, int64_t stride_qh, int64_t stride_qm,
                                           int64_t stride_qd, int64_t stride_kb, int64_t stride_kh,
                                           int64_t stride_kn, int64_t stride_kd, int64_t stride_vb,
                                           int64_t stride_vh, int64_t stride_vn, int64_t stride_vd,
                                           int64_t stride_ob, int64_t stride_oh, int64_t stride_om,
                                           int64_t stride_od, int64_t stride_lb, int64_t stride_lh,
                                           int64_t stride_lm, int B, int H, int M, int N, int D, float sm_scale,
                                           int causal, int has_lse, int dtype, void* stream);

/*
 * Replaces `_flash_attn_fwd_kernel_block_d_nomask_contiguous[grid](q, k, v, o, H, M, N, D,
 * sm_scale, ...)` (flash_atten.py:261-276, launch args at tuner.py:639-650): contiguous
 * [B, H, M|N, D] tensors, non-causal, no LSE.  B is grid[1] / H of the Triton
 * launch.  Unlike the Triton kernel, M, N and D need not divide any tile size.
 */
int fab_flash_attn_fwd_block_d_nomask_contiguous(const void* q, const void* k, const void* v, void* o, int B,
                                                 int H, int M, int N, int D, float sm_scale, int dtype,
                                                 void* stream);

/*
 * General attention forward with grouped-query heads mapped in the kernel
 * (query head h reads key/value head h / (Hq / Hkv)).  Replaces the
 * `_repeat_kv_for_gqa` + `_run_block_d_nomask_vanilla` pair behind the SDPA
 * patch (ttft.py:169-219, 299-327), without materialising repeated K/V.
 * Strides are in elements, stride along head_dim must be 1.
 */
typedef struct fab_attention_params {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  float* lse; /* may be NULL */
  int64_t q_stride_b, q_stride_h, q_stride_s;
  int64_t k_stride_b, k_stride_h, k_stride_s;
  int64_t v_stride_b, v_stride_h, v_stride_s;
  int64_t o_stride_b, o_stride_h, o_stride_s;
  int64_t lse_stride_b, lse_stride_h, lse_stride_s;
  int batch;
  int heads_q;
  int heads_kv;
  int seqlen_q;
  int seqlen_k;
  int head_dim;
  int dtype;
  float sm_scale;
  int causal;
} fab_attention_params;

int fab_attention_fwd(const fab_attention_params* params, void* stream);

/*
 * fab_attention_fwd over a packed batch of variable-length sequences: q is
 * [total_q, heads_q, head_dim] with sequence b's queries in rows
 * [cu_seqlens_q[b], cu_seqlens_q[b+1]), k/v are [total_k, heads_kv, head_dim]
 * likewise with cu_seqlens_k (int32 device arrays of batch + 1 offsets), o
 * is laid out like q and lse (fp32, may be NULL) is indexed [head, token].
 * max_seqlen_q / max_seqlen_k bound the per-sequence lengths.  Causal
 * masking is top-left within each sequence, as in the reference (key n of a
 * sequence visible to its query m iff m >= n); a sequence with queries but no
 * keys gets NaN rows and lse -inf.  No counterpart in the reference, whose
 * kernels take one dense [batch, head, seq, head_dim] block (the ragged case
 * of its scope: flash_atten.py:21-39 strides, ttft.py:169-219 SDPA calls).
 */
typedef struct fab_attention_varlen_params {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  float* lse;
  const int32_t* cu_seqlens_q;
  const int32_t* cu_seqlens_k;
  int64_t q_stride_t, q_stride_h;
  int64_t k_stride_t, k_stride_h;
  int64_t v_stride_t, v_stride_h;
  int64_t o_stride_t, o_stride_h;
  int64_t lse_stride_h, lse_stride_t;
  int batch;
  int heads_q;
  int heads_kv;
  int total_q;
  int total_k;
  int max_seqlen_q;
  int max_seqlen_k;
  int head_dim;
  int dtype;
  float sm_scale;
  int causal;
} fab_attention_varlen_params;

int fab_attention_fwd_varlen(const fab_attention_varlen_params* params, void* stream);

/*
 * Split-KV ("flash-decoding") form of fab_attention_fwd for short query blocks
 * against long key ranges, where (batch x heads x query tiles) alone would
 * leave most SMs idle.  No counterpart in the reference: it is the split-KV
 * variant its LSE path allows (an extension of the ttft.py:169-219 SDPA
 * replacement to decode-shaped calls).  Same parameters, same results within
 * fp32 rounding of the merge.
 *
 * The keys are cut into num_splits ranges (num_splits <= 0: as many ranges as
 * keep the CTAs in one wave, at most one per SM).  Each range's attention (normalised O in fp32 and its LSE)
 * goes to the workspace; the last range of each row group to finish merges
 * the group into o (and lse, when not NULL) with weights exp(LSE_split - LSE),
 * inside the same kernel, found through one arrival counter per row group.  When the query heads of a
 * key/value head are evenly spaced in memory (q_stride_h == seqlen_q *
 * q_stride_s, or seqlen_q == 1) they share one query tile, so every K/V tile
 * is read once per key/value head.
 *
 * fab_attention_fwd_splitkv_workspace writes the workspace size the call
 * needs (0 when a single range suffices) and, if splits_used is not NULL, the
 * number of ranges it will use.  The workspace is caller-owned device memory,
 * 256-byte aligned and zero-filled before its first use (its counters must
 * start at zero; each call leaves them zero again, so refill it only after a
 * FAB_ERR_DEVICE_TIMEOUT); calls that share a workspace must be ordered on one
 * stream.  FAB_ERR_WORKSPACE when it is missing, misaligned or too small.
 */
int fab_attention_fwd_splitkv_workspace(const fab_attention_params* params, int num_splits, size_t* bytes,
                                        int* splits_used);
int fab_attention_fwd_splitkv(const fab_attention_params* params, int num_splits, void* workspace,
                              size_t workspace_bytes, void* stream);

/*
 * fab_attention_fwd_splitkv for callers that cannot allocate device memory.
 * No counterpart in the reference.  The split partials live in an 8 MiB
 * array inside the library's device image (looked up once per device with
 * cudaGetSymbolAddress), so the call allocates nothing.  A request whose
 * partials need more than 8 MiB (fab_attention_fwd_splitkv_workspace reports
 * the size) returns FAB_ERR_WORKSPACE; fewer splits make it smaller.  All
 * calls on a device share the array: calls whose executions overlap
 * (different streams, or concurrent host threads) race on it, calls ordered
 * on one stream do not.
 */
int fab_attention_fwd_splitkv_static(const fab_attention_params* params, int num_splits, void* stream);

/*
 * Replaces `_matmul_contiguous_kernel[grid](a, b, c, M, N, K, BLOCK_M=..., ...)`
 * (mma.py:8-21, launched as in test_mma.py:318-332): row-major contiguous
 * A[M,K], B[K,N], C[M,N], fp32 accumulation.  round_f16 != 0 rounds the
 * accumulator to fp16 before storing it in out_dtype, as the Triton kernel's
 * `accumulator.to(tl.float16)` store does (mma.py:51-52).  Unlike the Triton
 * kernel, M, N and K need not divide the tile sizes (K and N must be
 * multiples of 16 bytes' worth of elements).
 */
int fab_matmul_contiguous(const void* a, const void* b, void* c, int M, int N, int K, int in_dtype,
                          int out_dtype, int round_f16, void* stream);

/* General row-major GEMM with leading dimensions (elements); used by the TTFT model. */
typedef struct fab_gemm_params {
  const void* a;
  const void* b;
  void* c;
  int64_t lda, ldb, ldc;
  int M, N, K;
  int in_dtype;
  int out_dtype;
  int round_f16;
  int group_m;  /* tile-row group for L2 reuse, 0 = default (8) */
  int epilogue; /* FAB_GEMM_EPILOGUE_*; 0 = store C */
  /* FAB_GEMM_EPILOGUE_BIAS_ROPE only (ignored otherwise): */
  const void* bias;     /* [N] in the output type, or NULL */
  const void* rope_cos; /* [M][head_dim] in the output type (row r: position r) */
  const void* rope_sin;
  int rope_cols;        /* leading columns that get RoPE (whole heads) */
  int head_dim;         /* 64, 128 or 256 */
  /*
   * NULL, or [M] fp32 (4-byte aligned): row r's accumulator is multiplied by
   * row_scale[r] before any epilogue step or rounding, with every epilogue.
   * This folds an RMSNorm into the GEMM that consumes its rows: A holds the
   * raw rows, B's row k is pre-multiplied by the norm weight w[k], and
   * row_scale holds each row's rsqrt(mean(x^2) + eps) (fab_rmsnorm_rstd).
   * Such GEMMs are never split over K.  No counterpart in the reference,
   * which runs the norm as its own PyTorch op (ttft.py forward).
   */
  const float* row_scale;
  /*
   * NULL, or device memory (256-byte aligned, zero-filled before its first
   * use) for the stream-K schedule of the CTA-pair kernel: when the output
   * tiles leave part of the last wave of SM pairs idle, the K blocks of the
   * tiles past the full waves are split evenly over all pairs, and each such
   * tile's pieces are added through this memory (plain store epilogue only).
   * fab_gemm_workspace_size gives the size; without a workspace (or with a
   * smaller one) the call runs whole tiles.  The kernel leaves the memory's
   * flag words zero again when it completes, so one workspace serves calls
   * ordered on one stream, CUDA graph replays included; calls that overlap
   * in time must not share it.  After a FAB_ERR_DEVICE_TIMEOUT, zero it again.
   * No counterpart in the reference.
   */
  void* workspace;
  size_t workspace_bytes;
} fab_gemm_params;

/*
 * FAB_GEMM_EPILOGUE_SWIGLU (no counterpart in the reference): B's N columns
 * alternate 64 gate and 64 up columns, and C [M, N/2] receives
 * round(round(silu(round(gate))) * round(up)) for each pair -- a SwiGLU MLP's
 * gate/up projection and activation in one kernel, rounding as the PyTorch
 * expression silu(x @ W_gate) * (x @ W_up) does in the 16-bit output type.
 * N a multiple of 128; 16-bit output; round_f16 0.
 */
#define FAB_GEMM_EPILOGUE_STORE 0
#define FAB_GEMM_EPILOGUE_SWIGLU 1

/*
 * FAB_GEMM_EPILOGUE_BIAS_ROPE: the QKV projection's bias add and rotate-half
 * rotary embedding in the GEMM epilogue (no counterpart in the reference,
 * whose model code adds the bias and applies RoPE as separate PyTorch ops;
 * here it replaces fab_gemm followed by fab_bias_rope, with equal bits).
 * Every column gets round(round(acc) + bias); each head of head_dim columns
 * among the first rope_cols becomes [lo*cos - hi*sin, hi*cos + lo*sin] of its
 * halves, every product and sum rounded to the output type, with row r's
 * cos/sin.  16-bit, in type == out type, N a multiple of head_dim, round_f16 0.
 */
#define FAB_GEMM_EPILOGUE_BIAS_ROPE 2

int fab_gemm(const fab_gemm_params* params, void* stream);

/*
 * Which kernel fab_gemm runs for these parameters (no counterpart in the
 * reference; like the launch facts of `_select_2d_contiguous_config`,
 * mma.py:22-81, it only reads the shapes): one CTA per 128 x *tile_n output
 * tile (*tile_n 256, or 128 / 64 for 16-bit problems whose 256-wide tiles
 * would leave over a quarter of the SMs idle), CTA pairs per 256 x *tile_n
 * tile (*tile_n 256 or 224; 16-bit inputs, at least one wave of pairs; with
 * a large enough workspace, the stream-K schedule), or split K, where the
 * *k_split CTAs of a cluster share each 128x256 tile's K and add their
 * partial sums in distributed shared memory (16-bit inputs, few tiles, deep
 * K).  Validates like fab_gemm; pointers are not dereferenced.  Nothing to
 * compute (M, N or K zero) reports SINGLE, 1, 256.
 */
#define FAB_GEMM_KERNEL_SINGLE 0
#define FAB_GEMM_KERNEL_PAIR 1
#define FAB_GEMM_KERNEL_SPLITK 2
#define FAB_GEMM_KERNEL_PAIR_STREAMK 3 /* CTA pairs, stream-K schedule through the caller's workspace */

int fab_gemm_plan(const fab_gemm_params* params, int* kernel, int* k_split, int* tile_n);
/* Stream-K workspace bytes a fab_gemm call with these parameters would use if given one (0: none). */
int fab_gemm_workspace_size(const fab_gemm_params* params, size_t* bytes);
/* CTAs in the grid a fab_gemm call with these parameters launches (0 when nothing is computed). */
int fab_gemm_grid(const fab_gemm_params* params, long long* ctas);

/*
 * GEMM + all-reduce over the ranks of a tensor-parallel group in one kernel,
 * through NVLink peer memory: out = sum over ranks of a_r[M,K] * b_r[K,N],
 * on every rank.  Replaces the o_proj / down_proj matmul followed by an NCCL
 * all-reduce in the tensor-parallel decoder (the reference runs the model on
 * one GPU; ttft.py:401-412 is its forward).  No counterpart in the
 * reference.
 *
 * Each rank owns the 128x256 output tiles t with t % world == rank.  While
 * its MMAs run, a rank stores every partial tile straight into the owner's
 * inbox and counts it there; each owner then sums the world partials in fp32
 * and writes the result into every rank's output.  All waits are bounded: a
 * rank that never joins makes the others return FAB_OK with
 * fab_get_device_error reporting the timeout.
 *
 * Buffers (sizes from fab_gemm_allreduce_layout): per rank an inbox
 * (16-byte aligned), an output [M, ldo] of the input dtype and a counter
 * array (8-byte aligned, zero before the first call; every call leaves it
 * zero again).  inbox[r], out[r] and counters[r] are rank r's buffers as
 * this process sees them (its own, or peers' mapped with fab_ipc_import).
 * Every rank makes the same sequence of calls with the same M and N (K may
 * differ: each rank's GEMM is its own), on one stream each.  After a timeout the counters are left mid-count: replace
 * the buffers.  bf16 or fp16, row-major.
 */
#define FAB_MAX_TP_RANKS 8
typedef struct fab_gemm_allreduce_params {
  const void* a;
  const void* b;
  int64_t lda, ldb, ldo;
  int M, N, K;
  int in_dtype;
  int world;
  int rank;
  void* inbox[FAB_MAX_TP_RANKS];
  void* out[FAB_MAX_TP_RANKS];
  void* counters[FAB_MAX_TP_RANKS];
} fab_gemm_allreduce_params;

int fab_gemm_allreduce_layout(int M, int N, int world, int* tiles_per_owner, size_t* inbox_bytes,
                              size_t* counter_bytes);
int fab_gemm_allreduce(const fab_gemm_allreduce_params* params, void* stream);

/*
 * CUDA IPC for the peer buffers above: fab_ipc_export writes the 64-byte
 * handle of the allocation holding `ptr` and ptr's offset in it;
 * fab_ipc_import maps a peer's handle in this process (base = the mapping,
 * ptr = base + offset); fab_ipc_close unmaps `base`.
 */
int fab_ipc_export(const void* ptr, void* handle, size_t* offset);
int fab_ipc_import(const void* handle, size_t offset, void** base, void** ptr);
int fab_ipc_close(void* base);

/*
 * The memory-bound steps of a Qwen2-style decoder layer between its GEMMs and
 * its attention (the model the reference's TTFT benchmark prefills,
 * ttft.py:401-412), each one pass with 16-byte accesses, rounding where the
 * PyTorch expressions of that model round so bf16 results match them.  No
 * counterpart in the reference (it runs them as PyTorch ops).  bf16 or fp16;
 * leading dims in elements; 16-byte aligned pointers and rows.
 *
 * fab_rmsnorm: h = w * round(x' * rsqrt(mean(x'^2) + eps)) per row, where
 *   x' = x, or round(x + residual) (written to x_out, which may alias x) when
 *   residual is not NULL.  cols a multiple of 8, at most 8192.
 * fab_rmsnorm_rstd: the first half of fab_rmsnorm for a GEMM with the norm
 *   folded into it (fab_gemm_params.row_scale): x' as above (written to
 *   x_out when residual is not NULL), and rstd[row] = rsqrt(mean(x'^2) + eps)
 *   in fp32; h is not formed.
 * fab_bias_rope: in place on y [rows, heads, head_dim] (row stride ld): adds
 *   bias [heads * head_dim] (may be NULL) to every head, then applies
 *   rotate-half rotary embedding (cos/sin [rows, head_dim]) to the first
 *   rot_heads heads: y = round(round(y * cos) + round(rotate_half(y) * sin)).
 * fab_silu_mul: a[:, j] = round(round(silu(g_j)) * u_j) with g_j = gu[:, j],
 *   u_j = gu[:, m + j] (interleave 0), or gu's columns alternating
 *   `interleave` gate and `interleave` up columns (the SwiGLU GEMM layout).
 */
int fab_rmsnorm(const void* x, const void* residual, const void* w, void* h, void* x_out, int rows, int cols,
                int64_t ld_x, int64_t ld_res, int64_t ld_h, int64_t ld_xo, float eps, int dtype, void* stream);
int fab_rmsnorm_rstd(const void* x, const void* residual, void* x_out, float* rstd, int rows, int cols, int64_t ld_x,
                     int64_t ld_res, int64_t ld_xo, float eps, int dtype, void* stream);
int fab_bias_rope(void* y, const void* bias, const void* cos, const void* sin, int rows, int heads, int rot_heads,
                  int head_dim, int64_t ld, int dtype, void* stream);
int fab_silu_mul(const void* gu, void* a, int rows, int m, int64_t ld_gu, int64_t ld_a, int interleave, int dtype,
                 void* stream);

/*
 * Static sm_100a tile table that replaces the reference tuner's compile-and-rank
 * search (tuner.py:414-561): the configuration the attention kernel uses for a
 * dtype and head_dim.
 */
typedef struct fab_fa_config {
  int head_dim_padded; /* head_dim rounded up to whole 128-byte swizzle atoms */
  int q_tiles_per_cta; /* 128-row query tiles per CTA (BLOCK_M = 128 * this) */
  int block_n;         /* keys per KV tile */
  int stages;          /* K/V ring slots: K and V tiles alternate in one ring */
  int threads;
  int smem_bytes;
  int tmem_columns;
  int s_buffers;       /* S/P buffers per query tile in TMEM (2 lets S(j+1) overlap softmax(j)) */
} fab_fa_config;

int fab_flash_attn_config(int dtype, int head_dim, fab_fa_config* out);

/*
 * Tile families for fab_attention_fwd_variant / fab_flash_attn_config_variant.
 * TWO_TILES is the table fab_attention_fwd uses (two 128-row query tiles per
 * CTA where TMEM allows, one S buffer each); ONE_TILE is one 128-row query
 * tile per CTA (more CTAs for the same rows: better for short or few
 * sequences) -- with one S buffer and two CTAs per SM where shared memory
 * allows (16-bit head dim <= 128, fp32 <= 64; the config reports s_buffers 1)
 * and the launch has at least 1.5 CTAs per SM, else two S buffers and one
 * CTA per SM.  Which is faster depends on the shape; the Python tuner
 * picks by measured time (the reference picks the largest tile that fits,
 * tuner.py:503-517).
 */
#define FAB_FA_VARIANT_TWO_TILES 0
#define FAB_FA_VARIANT_ONE_TILE 1

int fab_attention_fwd_variant(const fab_attention_params* params, int variant, void* stream);
int fab_flash_attn_config_variant(int dtype, int head_dim, int variant, fab_fa_config* out);

/*
 * The kernel a fab_attention_fwd_variant call with these arguments would
 * launch, without launching it: its tile, the CTAs of its grid and how many
 * of them share one SM (2 for the one-tile, one-S-buffer kernel; a ONE_TILE
 * call with fewer than 1.5 CTAs per SM runs the two-S-buffer tile instead and
 * reports 1).  Replaces the launch facts the reference's tuner reads back
 * from its chosen config (grid and num_warps, tuner.py:533-561).  A call with
 * no query rows reports all zeros.
 */
typedef struct fab_fa_plan {
  fab_fa_config config;
  long long ctas;
  int ctas_per_sm;
} fab_fa_plan;

int fab_attention_fwd_plan(const fab_attention_params* params, int variant, fab_fa_plan* out);

/*
 * Compiled-kernel facts that replace Triton's `kernel.warmup(...)` metadata
 * (tuner.py:355-368: metadata.shared, metadata.num_warps, n_regs).
 * which: 0 = attention kernel for (dtype, head_dim), 1 = matmul kernel for dtype.
 */
#define FAB_KERNEL_ATTENTION 0
#define FAB_KERNEL_MATMUL 1
#define FAB_KERNEL_ATTENTION_ONE_TILE 2 /* the FAB_FA_VARIANT_ONE_TILE attention family */
typedef struct fab_kernel_attrs {
  int registers_per_thread;
  int shared_bytes;
  int threads;
} fab_kernel_attrs;

int fab_kernel_attrs_query(int which, int dtype, int head_dim, fab_kernel_attrs* out);

/* Device limits that replace exceptions.get_sm_resource_limits() (exceptions.py:760-775). */
typedef struct fab_device_limits {
  int shared_bytes_per_sm;
  int shared_bytes_per_block_optin;
  int registers_per_sm;
  int warp_size;
  int max_threads_per_block;
  int multiprocessor_count;
  int cc_major;
  int cc_minor;
} fab_device_limits;

int fab_device_limits_query(int device, fab_device_limits* out);

/*
 * Reads and clears the device error word of the current device.  *code is 0
 * when no kernel has given up on a bounded wait, else a positive code naming
 * the wait (the first to give up):
 *    1 a Q tile's load            2 a K/V tile's load       3 an S product
 *    4 a softmax's P              5 O's last product        6 a free K/V or stage slot
 *    7 a GEMM accumulator         8 the drain at teardown   9 a peer rank's partial tile
 *   10 a peer owner's reduced tile                          11 a stream-K piece from another pair
 *   12 the CTA-pair GEMM's next tile from its scheduler     13 the split-KV merge's copies
 * Synchronises with the device (call it between launches).
 */
int fab_get_device_error(int* code);

/*
 * Test hooks for the bounded waits of the attention kernels (no counterpart
 * in the reference, which has no device-side waits).  They change device
 * state of the current device and synchronise with it; call them only
 * between launches.
 * fab_debug_set_wait_limit_ns: the time one wait may take before the kernel
 *   records its code in the device error word and unwinds (0 restores the
 *   default of 2 s).
 * fab_debug_starve_kv_load: the producer of every attention CTA skips the
 *   K/V ring load with this index (ring order: K_0, V_0, K_1, V_1, ... with
 *   one S buffer), so the wait for it runs out; -1 restores normal loading.
 */
int fab_debug_set_wait_limit_ns(unsigned long long ns);
int fab_debug_starve_kv_load(int ring_tile);

/* Human-readable text for a FAB_* return code. */
const char* fab_error_string(int rc);

/* ABI version of this header (incremented on incompatible changes). */
int fab_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FA_B200_H_ */
