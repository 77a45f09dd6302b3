// C-ABI entry points of libfa_b200.so (declared in include/fa_b200.h), the
// host helpers the kernels share, and the attention and decoder-op kernels
// (included below).  The GEMM kernels are the library's second translation
// unit (gemm.cu); each unit keeps its own copy of the device status word, so
// neither needs relocatable device code.
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <set>
#include <utility>

#include "fa_b200.h"
#include "fa_internal.h"
#include "ptx.cuh"

#include "fa_fwd_kernel.cuh"
#include "decoder_ops.cuh"

namespace fab {

static_assert(FAB_OK == kOk && FAB_ERR_INVALID_ARG == kErrInvalidArg && FAB_ERR_UNSUPPORTED == kErrUnsupported &&
                  FAB_ERR_LAUNCH == kErrLaunch && FAB_ERR_DEVICE_TIMEOUT == kErrDeviceTimeout &&
                  FAB_ERR_CUDA == kErrCuda,
              "public and internal return codes must agree");
static_assert(FAB_DTYPE_F16 == kDtypeF16 && FAB_DTYPE_BF16 == kDtypeBF16 && FAB_DTYPE_F32 == kDtypeF32,
              "public and internal dtype codes must agree");

static int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}

int ensure_smem_attr(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  const int dev = current_device();
  if (dev < 0) return kErrCuda;
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({kernel, dev})) return kOk;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) {
    cudaGetLastError();
    return kErrLaunch;
  }
  done.insert({kernel, dev});
  return kOk;
}

int num_sms() {
  static std::mutex mu;
  static int cache[64] = {0};
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return -1;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    cache[dev] = n;
  }
  return cache[dev];
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_tiled_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

static bool stride_ok(int64_t stride_bytes) {
  return stride_bytes > 0 && (stride_bytes % 16) == 0 && stride_bytes < (int64_t(1) << 40);
}

static int64_t round16(int64_t x) { return (x + 15) / 16 * 16; }

int make_bhsd_map(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elt, int D, int S, int H, int B,
                  int64_t s_s, int64_t s_h, int64_t s_b, int box_inner, int box_rows, CUtensorMapSwizzle swizzle) {
  auto enc = encode_tiled_fn();
  if (enc == nullptr) return kErrCuda;
  if (base == nullptr || (reinterpret_cast<uintptr_t>(base) & 15u) != 0) return kErrInvalidArg;
  if (D <= 0 || S <= 0 || H <= 0 || B <= 0) return kErrInvalidArg;
  // Strides of size-1 dims are never followed; give them a valid value.
  int64_t bs = S == 1 ? round16(int64_t(D) * elt) : s_s * elt;
  int64_t bh = H == 1 ? round16(bs * S) : s_h * elt;
  int64_t bb = B == 1 ? round16(bh * H) : s_b * elt;
  if (!stride_ok(bs) || !stride_ok(bh) || !stride_ok(bb)) return kErrInvalidArg;
  cuuint64_t dims[4] = {cuuint64_t(D), cuuint64_t(S), cuuint64_t(H), cuuint64_t(B)};
  cuuint64_t strides[3] = {cuuint64_t(bs), cuuint64_t(bh), cuuint64_t(bb)};
  cuuint32_t box[4] = {cuuint32_t(box_inner), cuuint32_t(box_rows), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : kErrInvalidArg;
}

int make_2d_map(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elt, int cols, int rows, int64_t ld,
                int box_inner, int box_rows, CUtensorMapSwizzle swizzle) {
  auto enc = encode_tiled_fn();
  if (enc == nullptr) return kErrCuda;
  if (base == nullptr || (reinterpret_cast<uintptr_t>(base) & 15u) != 0) return kErrInvalidArg;
  if (cols <= 0 || rows <= 0) return kErrInvalidArg;
  const int64_t bs = rows == 1 ? round16(int64_t(cols) * elt) : ld * elt;
  if (!stride_ok(bs)) return kErrInvalidArg;
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(bs)};
  cuuint32_t box[2] = {cuuint32_t(box_inner), cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : kErrInvalidArg;
}

static int elt_size(int dtype) { return dtype == kDtypeF32 ? 4 : 2; }

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Shared validation for every attention entry point.  Returns kOk with
// *empty set when there is nothing to compute (no query rows).
static int attention_validate(FaLaunch& L, bool* empty) {
  *empty = false;
  if (L.dtype != kDtypeF16 && L.dtype != kDtypeBF16 && L.dtype != kDtypeF32) return kErrInvalidArg;
  if (L.B < 0 || L.Hq < 0 || L.Hkv < 0 || L.M < 0 || L.N < 0 || L.D <= 0) return kErrInvalidArg;
  if (L.M == 0 || L.B == 0 || L.Hq == 0) {
    *empty = true;
    return kOk;
  }
  if (L.Hkv <= 0 || L.Hq % L.Hkv != 0) return kErrInvalidArg;
  if (!(L.sm_scale > 0.f) || !std::isfinite(L.sm_scale)) return kErrUnsupported;
  FaConfigInfo cfg;
  int rc = fa_select_config(L.dtype, L.D, &cfg);
  if (rc) return rc;
  if (L.q == nullptr || L.o == nullptr) return kErrInvalidArg;
  const int elt = elt_size(L.dtype);
  // The epilogue stores rows with 16-byte vector stores.
  if (!aligned16(L.o)) return kErrInvalidArg;
  for (int64_t s : {L.o_sb, L.o_sh, L.o_ss})
    if ((s * elt) % 16 != 0) return kErrInvalidArg;
  if (L.lse != nullptr && (reinterpret_cast<uintptr_t>(L.lse) & 3u) != 0) return kErrInvalidArg;
  if (L.N == 0) {
    // No keys: the kernel only writes NaN rows; point the K/V maps at Q.
    L.k = L.q;
    L.v = L.q;
    L.N = 0;
    L.k_sb = L.q_sb;
    L.k_sh = L.q_sh;
    L.k_ss = L.q_ss;
    L.v_sb = L.q_sb;
    L.v_sh = L.q_sh;
    L.v_ss = L.q_ss;
    L.Hkv = L.Hq;
  } else if (L.k == nullptr || L.v == nullptr) {
    return kErrInvalidArg;
  }
  return kOk;
}

static int attention_launch(FaLaunch L, cudaStream_t stream) {
  bool empty = false;
  const int rc = attention_validate(L, &empty);
  if (rc || empty) return rc;
  return fa_forward(L, stream);
}

static FaLaunch launch_from_params(const fab_attention_params* p) {
  FaLaunch L{};
  L.q = p->q;
  L.k = p->k;
  L.v = p->v;
  L.o = p->o;
  L.lse = p->lse;
  L.q_sb = p->q_stride_b;
  L.q_sh = p->q_stride_h;
  L.q_ss = p->q_stride_s;
  L.k_sb = p->k_stride_b;
  L.k_sh = p->k_stride_h;
  L.k_ss = p->k_stride_s;
  L.v_sb = p->v_stride_b;
  L.v_sh = p->v_stride_h;
  L.v_ss = p->v_stride_s;
  L.o_sb = p->o_stride_b;
  L.o_sh = p->o_stride_h;
  L.o_ss = p->o_stride_s;
  L.l_sb = p->lse_stride_b;
  L.l_sh = p->lse_stride_h;
  L.l_ss = p->lse_stride_s;
  L.B = p->batch;
  L.Hq = p->heads_q;
  L.Hkv = p->heads_kv;
  L.M = p->seqlen_q;
  L.N = p->seqlen_k;
  L.D = p->head_dim;
  L.dtype = p->dtype;
  L.sm_scale = p->sm_scale;
  L.causal = p->causal ? 1 : 0;
  return L;
}

// Validated split-KV plan for the given request; *empty as above.
static int splitkv_prepare(const fab_attention_params* p, int num_splits, FaLaunch* L, FaSplitPlan* plan,
                           bool* empty) {
  if (p == nullptr || plan == nullptr) return kErrInvalidArg;
  *L = launch_from_params(p);
  int rc = attention_validate(*L, empty);
  if (rc || *empty) return rc;
  rc = fa_split_plan(*L, num_splits, plan);
  if (rc) return rc;
  L->num_splits = plan->num_splits;
  L->split_len = plan->split_len;
  L->pack_gqa = plan->pack_gqa;
  L->split_dual = plan->dual;
  return kOk;
}

// ---------------------------------------------------------------------------
// Static split-KV scratch, for callers that cannot allocate device memory.
//
// fab_attention_fwd_splitkv_static runs the split-KV path with its partial
// results in this file-scope device array instead of a caller-owned
// workspace.  It is part of the library's device image, so using it needs no
// cudaMalloc, cudaFree or any other allocating call.  Its address is looked
// up with cudaGetSymbolAddress once per device, at the first call on that
// device.  Requests whose partials need more than kStaticScratchBytes are
// rejected with FAB_ERR_WORKSPACE.  Every call on a device uses the same
// array, so two calls whose executions overlap (different streams, or host
// threads launching concurrently) race on it; calls ordered on one stream do
// not.
constexpr size_t kStaticScratchBytes = size_t(8) << 20;  // 8 MiB
static __device__ __align__(256) unsigned char g_splitkv_static_scratch[kStaticScratchBytes];

constexpr int kMaxScratchDevices = 64;

// Device address of the scratch array on `device` (the current device).  Only
// a successful lookup is cached, so a call after a failed one tries again; a
// failed lookup's error is read off the runtime here, so it is not reported
// later by an unrelated launch check.
static void* static_scratch_address(int device) {
  static std::mutex mu;
  static void* addr[kMaxScratchDevices] = {};
  if (device < 0 || device >= kMaxScratchDevices) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[device] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_splitkv_static_scratch) == cudaSuccess)
      addr[device] = p;
    else
      cudaGetLastError();
  }
  return addr[device];
}

}  // namespace fab

using namespace fab;

extern "C" {

int fab_abi_version(void) { return 8; }

const char* fab_error_string(int rc) {
  switch (rc) {
    case FAB_OK:
      return "ok";
    case FAB_ERR_INVALID_ARG:
      return "invalid argument (pointer, shape, stride or alignment)";
    case FAB_ERR_UNSUPPORTED:
      return "unsupported configuration";
    case FAB_ERR_LAUNCH:
      return "kernel launch failed";
    case FAB_ERR_DEVICE_TIMEOUT:
      return "a kernel gave up on a bounded wait";
    case FAB_ERR_CUDA:
      return "CUDA runtime error";
    case FAB_ERR_WORKSPACE:
      return "workspace missing, misaligned or smaller than the split-KV plan needs";
    default:
      return "unknown error";
  }
}

static int fa_basic_common(const void* q, const void* k, const void* v, void* o, float* lse, int64_t sqb,
                           int64_t sqh, int64_t sqm, int64_t sqd, int64_t skb, int64_t skh, int64_t skn,
                           int64_t skd, int64_t svb, int64_t svh, int64_t svn, int64_t svd, int64_t sob,
                           int64_t soh, int64_t som, int64_t sod, int64_t slb, int64_t slh, int64_t slm, int B,
                           int H, int M, int N, int D, float sm_scale, int causal, int has_lse, int dtype,
                           void* stream) {
  if (M > 0 && B > 0 && H > 0 && (sqd != 1 || sod != 1 || (N > 0 && (skd != 1 || svd != 1)))) return kErrInvalidArg;
  if (has_lse && lse == nullptr) return kErrInvalidArg;
  FaLaunch L{};
  L.q = q;
  L.k = k;
  L.v = v;
  L.o = o;
  L.lse = has_lse ? lse : nullptr;
  L.q_sb = sqb;
  L.q_sh = sqh;
  L.q_ss = sqm;
  L.k_sb = skb;
  L.k_sh = skh;
  L.k_ss = skn;
  L.v_sb = svb;
  L.v_sh = svh;
  L.v_ss = svn;
  L.o_sb = sob;
  L.o_sh = soh;
  L.o_ss = som;
  L.l_sb = slb;
  L.l_sh = slh;
  L.l_ss = slm;
  L.B = B;
  L.Hq = H;
  L.Hkv = H;
  L.M = M;
  L.N = N;
  L.D = D;
  L.dtype = dtype;
  L.sm_scale = sm_scale;
  L.causal = causal ? 1 : 0;
  return attention_launch(L, static_cast<cudaStream_t>(stream));
}

int fab_flash_attn_fwd_basic(const void* q, const void* k, const void* v, void* o, float* lse, int64_t stride_qb,
                             int64_t stride_qh, int64_t stride_qm, int64_t stride_qd, int64_t stride_kb,
                             int64_t stride_kh, int64_t stride_kn, int64_t stride_kd, int64_t stride_vb,
                             int64_t stride_vh, int64_t stride_vn, int64_t stride_vd, int64_t stride_ob,
                             int64_t stride_oh, int64_t stride_om, int64_t stride_od, int64_t stride_lb,
                             int64_t stride_lh, int64_t stride_lm, int B, int H, int M, int N, int D,
                             float sm_scale, int causal, int has_lse, int dtype, void* stream) {
  return fa_basic_common(q, k, v, o, lse, stride_qb, stride_qh, stride_qm, stride_qd, stride_kb, stride_kh,
                         stride_kn, stride_kd, stride_vb, stride_vh, stride_vn, stride_vd, stride_ob, stride_oh,
                         stride_om, stride_od, stride_lb, stride_lh, stride_lm, B, H, M, N, D, sm_scale, causal,
                         has_lse, dtype, stream);
}

int fab_flash_attn_fwd_optimize_shared_mem(const void* q, const void* k, const void* v, void* o, float* lse,
                                           int64_t stride_qb, int64_t stride_qh, int64_t stride_qm,
                                           int64_t stride_qd, int64_t stride_kb, int64_t stride_kh,
                                           int64_t stride_kn, int64_t stride_kd, int64_t stride_vb,
                                           int64_t stride_vh, int64_t stride_vn, int64_t stride_vd,
                                           int64_t stride_ob, int64_t stride_oh, int64_t stride_om,
                                           int64_t stride_od, int64_t stride_lb, int64_t stride_lh,
                                           int64_t stride_lm, int B, int H, int M, int N, int D, float sm_scale,
                                           int causal, int has_lse, int dtype, void* stream) {
  return fa_basic_common(q, k, v, o, lse, stride_qb, stride_qh, stride_qm, stride_qd, stride_kb, stride_kh,
                         stride_kn, stride_kd, stride_vb, stride_vh, stride_vn, stride_vd, stride_ob, stride_oh,
                         stride_om, stride_od, stride_lb, stride_lh, stride_lm, B, H, M, N, D, sm_scale, causal,
                         has_lse, dtype, stream);
}

int fab_flash_attn_fwd_block_d_nomask_contiguous(const void* q, const void* k, const void* v, void* o, int B,
                                                 int H, int M, int N, int D, float sm_scale, int dtype,
                                                 void* stream) {
  const int64_t qs = D, qh = int64_t(M) * D, qb = qh * H;
  const int64_t ks = D, kh = int64_t(N) * D, kb = kh * H;
  return fa_basic_common(q, k, v, o, nullptr, qb, qh, qs, 1, kb, kh, ks, 1, kb, kh, ks, 1, qb, qh, qs, 1, 0, 0, 0,
                         B, H, M, N, D, sm_scale, 0, 0, dtype, stream);
}

int fab_attention_fwd(const fab_attention_params* p, void* stream) {
  if (p == nullptr) return kErrInvalidArg;
  return attention_launch(launch_from_params(p), static_cast<cudaStream_t>(stream));
}

int fab_attention_fwd_variant(const fab_attention_params* p, int variant, void* stream) {
  if (p == nullptr) return kErrInvalidArg;
  if (variant == FAB_FA_VARIANT_TWO_TILES) return fab_attention_fwd(p, stream);
  if (variant != FAB_FA_VARIANT_ONE_TILE) return kErrInvalidArg;
  FaLaunch L = launch_from_params(p);
  bool empty = false;
  const int rc = attention_validate(L, &empty);
  if (rc || empty) return rc;
  // One query tile per CTA, one pass over all keys.
  L.num_splits = 1;
  L.split_len = L.N > 0 ? L.N : 1;
  return fa_forward_one_tile(L, static_cast<cudaStream_t>(stream));
}

int fab_attention_fwd_plan(const fab_attention_params* p, int variant, fab_fa_plan* out) {
  if (p == nullptr || out == nullptr) return kErrInvalidArg;
  if (variant != FAB_FA_VARIANT_TWO_TILES && variant != FAB_FA_VARIANT_ONE_TILE) return kErrInvalidArg;
  FaLaunch L = launch_from_params(p);
  bool empty = false;
  int rc = attention_validate(L, &empty);
  if (rc) return rc;
  *out = fab_fa_plan{};
  if (empty) return kOk;  // nothing would launch
  L.num_splits = 1;
  FaPlanInfo plan;
  rc = fa_plan(L, variant, &plan);
  if (rc) return rc;
  const FaConfigInfo& c = plan.cfg;
  out->config = fab_fa_config{c.d_pad, c.nq, c.bn, c.stages, c.threads, c.smem_bytes, c.tmem_cols, c.s_bufs};
  out->ctas = plan.ctas;
  out->ctas_per_sm = plan.ctas_per_sm;
  return kOk;
}

int fab_debug_set_wait_limit_ns(unsigned long long ns) {
  const uint64_t v = ns == 0 ? kWaitLimitNs : static_cast<uint64_t>(ns);
  return cudaMemcpyToSymbol(g_fab_wait_limit_ns, &v, sizeof(v)) == cudaSuccess ? kOk : kErrCuda;
}

int fab_debug_starve_kv_load(int ring_tile) {
  const int v = ring_tile < 0 ? -1 : ring_tile;
  return cudaMemcpyToSymbol(g_fab_starve_kv_load, &v, sizeof(v)) == cudaSuccess ? kOk : kErrCuda;
}

int fab_flash_attn_config_variant(int dtype, int head_dim, int variant, fab_fa_config* out) {
  if (out == nullptr) return kErrInvalidArg;
  if (variant == FAB_FA_VARIANT_TWO_TILES) return fab_flash_attn_config(dtype, head_dim, out);
  if (variant != FAB_FA_VARIANT_ONE_TILE) return kErrInvalidArg;
  FaConfigInfo c;
  const int rc = fa_select_one_tile_config(dtype, head_dim, &c);
  if (rc) return rc;
  out->head_dim_padded = c.d_pad;
  out->q_tiles_per_cta = c.nq;
  out->block_n = c.bn;
  out->stages = c.stages;
  out->threads = c.threads;
  out->smem_bytes = c.smem_bytes;
  out->tmem_columns = c.tmem_cols;
  out->s_buffers = c.s_bufs;
  return kOk;
}

int fab_attention_fwd_varlen(const fab_attention_varlen_params* p, void* stream) {
  if (p == nullptr) return kErrInvalidArg;
  if (p->batch < 0 || p->total_q < 0 || p->total_k < 0 || p->max_seqlen_q < 0 || p->max_seqlen_k < 0)
    return kErrInvalidArg;
  if (p->batch == 0 || p->total_q == 0 || p->max_seqlen_q == 0 || p->heads_q == 0) return kOk;
  if (p->cu_seqlens_q == nullptr || p->cu_seqlens_k == nullptr ||
      (reinterpret_cast<uintptr_t>(p->cu_seqlens_q) & 3u) != 0 || (reinterpret_cast<uintptr_t>(p->cu_seqlens_k) & 3u) != 0)
    return kErrInvalidArg;
  FaLaunch L{};
  L.q = p->q;
  L.k = p->k;
  L.v = p->v;
  L.o = p->o;
  L.lse = p->lse;
  L.q_sh = p->q_stride_h;
  L.q_ss = p->q_stride_t;
  L.k_sh = p->k_stride_h;
  L.k_ss = p->k_stride_t;
  L.v_sh = p->v_stride_h;
  L.v_ss = p->v_stride_t;
  L.o_sh = p->o_stride_h;
  L.o_ss = p->o_stride_t;
  L.l_sh = p->lse_stride_h;
  L.l_ss = p->lse_stride_t;
  L.B = p->batch;
  L.Hq = p->heads_q;
  L.Hkv = p->heads_kv;
  L.M = p->max_seqlen_q;
  L.N = p->max_seqlen_k;
  L.D = p->head_dim;
  L.dtype = p->dtype;
  L.sm_scale = p->sm_scale;
  L.causal = p->causal ? 1 : 0;
  L.cu_q = p->cu_seqlens_q;
  L.cu_k = p->cu_seqlens_k;
  L.total_q = p->total_q;
  L.total_k = p->total_k;
  bool empty = false;
  int rc = attention_validate(L, &empty);
  if (rc || empty) return rc;
  if (p->total_k == 0) {
    // No keys in any sequence: the kernel only writes NaN rows; the K/V maps
    // (never read) point at Q.
    L.k = L.q;
    L.v = L.q;
    L.k_sh = L.v_sh = L.q_sh;
    L.k_ss = L.v_ss = L.q_ss;
    L.Hkv = L.Hq;
    L.total_k = L.total_q;
  }
  return fa_forward(L, static_cast<cudaStream_t>(stream));
}

int fab_attention_fwd_splitkv_workspace(const fab_attention_params* p, int num_splits, size_t* bytes,
                                        int* splits_used) {
  if (bytes == nullptr) return kErrInvalidArg;
  FaLaunch L;
  FaSplitPlan plan{};
  bool empty = false;
  const int rc = splitkv_prepare(p, num_splits, &L, &plan, &empty);
  if (rc) return rc;
  *bytes = empty ? 0 : plan.workspace_bytes;
  if (splits_used != nullptr) *splits_used = empty ? 0 : plan.num_splits;
  return kOk;
}

int fab_attention_fwd_splitkv(const fab_attention_params* p, int num_splits, void* workspace, size_t workspace_bytes,
                              void* stream) {
  FaLaunch L;
  FaSplitPlan plan{};
  bool empty = false;
  int rc = splitkv_prepare(p, num_splits, &L, &plan, &empty);
  if (rc || empty) return rc;
  if (plan.num_splits > 1) {
    if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0 ||
        workspace_bytes < plan.workspace_bytes)
      return kErrWorkspace;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    L.o_part = reinterpret_cast<float*>(ws);
    L.lse_part = reinterpret_cast<float*>(ws + plan.lse_offset);
    L.split_cnt = reinterpret_cast<unsigned int*>(ws + plan.counter_offset);
  }
  return fa_forward_split(L, static_cast<cudaStream_t>(stream));
}

int fab_attention_fwd_splitkv_static(const fab_attention_params* p, int num_splits, void* stream) {
  FaLaunch L;
  FaSplitPlan plan{};
  bool empty = false;
  int rc = splitkv_prepare(p, num_splits, &L, &plan, &empty);
  if (rc || empty) return rc;
  if (plan.num_splits > 1) {
    if (plan.workspace_bytes > kStaticScratchBytes) return kErrWorkspace;
    uint8_t* ws = static_cast<uint8_t*>(static_scratch_address(current_device()));
    if (ws == nullptr) return kErrCuda;
    // Every split writes all of its partial rows (an empty split writes
    // zeros and LSE -inf) before the group's last CTA merges them.  The row
    // groups' arrival counters must start at zero: they are cleared here, on
    // the call's stream, since an earlier call that gave up on a bounded wait
    // may have left them counted.
    L.o_part = reinterpret_cast<float*>(ws);
    L.lse_part = reinterpret_cast<float*>(ws + plan.lse_offset);
    L.split_cnt = reinterpret_cast<unsigned int*>(ws + plan.counter_offset);
    if (cudaMemsetAsync(L.split_cnt, 0, sizeof(unsigned int) * plan.groups, static_cast<cudaStream_t>(stream)) !=
        cudaSuccess)
      return kErrCuda;
  }
  return fa_forward_split(L, static_cast<cudaStream_t>(stream));
}

static int gemm_validate(const fab_gemm_params* p, GemmLaunch* out, bool* nothing, bool* empty_k) {
  *nothing = *empty_k = false;
  if (p == nullptr) return kErrInvalidArg;
  if (p->M < 0 || p->N < 0 || p->K < 0) return kErrInvalidArg;
  if (p->M == 0 || p->N == 0) {
    *nothing = true;
    return kOk;
  }
  for (int dt : {p->in_dtype, p->out_dtype})
    if (dt != kDtypeF16 && dt != kDtypeBF16 && dt != kDtypeF32) return kErrInvalidArg;
  if (p->c == nullptr || !aligned16(p->c)) return kErrInvalidArg;
  const int oe = elt_size(p->out_dtype);
  if (p->epilogue != FAB_GEMM_EPILOGUE_STORE && p->epilogue != FAB_GEMM_EPILOGUE_SWIGLU &&
      p->epilogue != FAB_GEMM_EPILOGUE_BIAS_ROPE)
    return kErrInvalidArg;
  const bool swiglu = p->epilogue == FAB_GEMM_EPILOGUE_SWIGLU;
  if (swiglu && (p->N % 128 != 0 || oe != 2 || p->round_f16)) return kErrInvalidArg;
  const bool rope = p->epilogue == FAB_GEMM_EPILOGUE_BIAS_ROPE;
  if (rope) {
    // Whole heads inside 256-column tiles; bias and tables in the output type.
    const int hd = p->head_dim;
    if ((hd != 64 && hd != 128 && hd != 256) || oe != 2 || p->in_dtype != p->out_dtype || p->round_f16 ||
        p->N % hd != 0 || p->rope_cols < 0 || p->rope_cols > p->N || p->rope_cols % hd != 0)
      return kErrInvalidArg;
    if (p->bias != nullptr && !aligned16(p->bias)) return kErrInvalidArg;
    if (p->rope_cols > 0 && (p->rope_cos == nullptr || p->rope_sin == nullptr || !aligned16(p->rope_cos) ||
                             !aligned16(p->rope_sin)))
      return kErrInvalidArg;
  }
  const int c_cols = swiglu ? p->N / 2 : p->N;
  if ((p->ldc * oe) % 16 != 0 || p->ldc < c_cols) return kErrInvalidArg;
  if (p->row_scale != nullptr && (reinterpret_cast<uintptr_t>(p->row_scale) & 3u) != 0) return kErrInvalidArg;
  if (p->K == 0) {
    *empty_k = true;
    return kOk;
  }
  if (p->lda < p->K || p->ldb < p->N) return kErrInvalidArg;
  GemmLaunch& L = *out;
  L = GemmLaunch{};
  L.a = p->a;
  L.b = p->b;
  L.c = p->c;
  L.lda = p->lda;
  L.ldb = p->ldb;
  L.ldc = p->ldc;
  L.M = p->M;
  L.N = p->N;
  L.K = p->K;
  L.in_dtype = p->in_dtype;
  L.out_dtype = p->out_dtype;
  L.round_f16 = p->round_f16;
  L.group_m = p->group_m;
  L.swiglu = swiglu ? 1 : 0;
  L.row_scale = p->row_scale;
  L.workspace = p->workspace;
  L.workspace_bytes = p->workspace_bytes;
  if (rope) {
    L.bias_rope = 1;
    L.rope_cols = p->rope_cols;
    L.head_dim = p->head_dim;
    L.bias = p->bias;
    L.rope_cos = p->rope_cos;
    L.rope_sin = p->rope_sin;
  }
  return kOk;
}

int fab_gemm(const fab_gemm_params* p, void* stream) {
  GemmLaunch L;
  bool nothing, empty_k;
  const int rc = gemm_validate(p, &L, &nothing, &empty_k);
  if (rc || nothing) return rc;
  if (empty_k) {
    // Empty contraction: C = 0 (also under SwiGLU: silu(0) * 0 = 0); with
    // bias + RoPE, then the epilogue on the zeros, as the two-pass path does.
    const int oe = elt_size(p->out_dtype);
    const int c_cols = p->epilogue == FAB_GEMM_EPILOGUE_SWIGLU ? p->N / 2 : p->N;
    cudaError_t e = cudaMemset2DAsync(p->c, size_t(p->ldc) * oe, 0, size_t(c_cols) * oe, size_t(p->M),
                                      static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return kErrCuda;
    if (p->epilogue == FAB_GEMM_EPILOGUE_BIAS_ROPE)
      return fab_bias_rope(p->c, p->bias, p->rope_cos, p->rope_sin, p->M, p->N / p->head_dim,
                           p->rope_cols / p->head_dim, p->head_dim, p->ldc, p->out_dtype, stream);
    return kOk;
  }
  return gemm_forward(L, static_cast<cudaStream_t>(stream));
}

int fab_gemm_workspace_size(const fab_gemm_params* p, size_t* bytes) {
  if (bytes == nullptr) return kErrInvalidArg;
  *bytes = 0;
  GemmLaunch L;
  bool nothing, empty_k;
  const int rc = gemm_validate(p, &L, &nothing, &empty_k);
  if (rc || nothing || empty_k) return rc;
  *bytes = gemm_workspace_bytes(L);
  return kOk;
}

int fab_gemm_grid(const fab_gemm_params* p, long long* ctas) {
  if (ctas == nullptr) return kErrInvalidArg;
  *ctas = 0;
  GemmLaunch L;
  bool nothing, empty_k;
  const int rc = gemm_validate(p, &L, &nothing, &empty_k);
  if (rc || nothing || empty_k) return rc;
  *ctas = gemm_grid_ctas(L);
  return kOk;
}

int fab_gemm_plan(const fab_gemm_params* p, int* kernel, int* k_split, int* tile_n) {
  if (kernel == nullptr || k_split == nullptr || tile_n == nullptr) return kErrInvalidArg;
  *kernel = FAB_GEMM_KERNEL_SINGLE;
  *k_split = 1;
  *tile_n = 256;
  GemmLaunch L;
  bool nothing, empty_k;
  const int rc = gemm_validate(p, &L, &nothing, &empty_k);
  if (rc || nothing || empty_k) return rc;
  return gemm_plan(L, kernel, k_split, tile_n);
}

int fab_gemm_allreduce_layout(int M, int N, int world, int* tiles_per_owner, size_t* inbox_bytes,
                              size_t* counter_bytes) {
  if (M <= 0 || N <= 0 || world < 1 || world > kMaxTpRanks || tiles_per_owner == nullptr || inbox_bytes == nullptr ||
      counter_bytes == nullptr)
    return kErrInvalidArg;
  const int tiles = gemm_ar_tiles(M, N);
  const int per_owner = (tiles + world - 1) / world;
  *tiles_per_owner = per_owner;
  *inbox_bytes = static_cast<size_t>(world) * per_owner * 128 * 256 * 2;
  *counter_bytes = (static_cast<size_t>(per_owner) + 1) * sizeof(unsigned long long);
  return kOk;
}

int fab_gemm_allreduce(const fab_gemm_allreduce_params* p, void* stream) {
  if (p == nullptr) return kErrInvalidArg;
  if (p->world < 1 || p->world > kMaxTpRanks || p->rank < 0 || p->rank >= p->world) return kErrInvalidArg;
  if (p->in_dtype != FAB_DTYPE_BF16 && p->in_dtype != FAB_DTYPE_F16) return kErrUnsupported;
  if (p->M <= 0 || p->N <= 0 || p->K <= 0 || p->lda < p->K || p->ldb < p->N || p->ldo < p->N) return kErrInvalidArg;
  if ((p->N * 2) % 16 != 0 || (p->ldo * 2) % 16 != 0) return kErrInvalidArg;
  int per_owner = 0;
  size_t inbox_bytes = 0, counter_bytes = 0;
  int rc = fab_gemm_allreduce_layout(p->M, p->N, p->world, &per_owner, &inbox_bytes, &counter_bytes);
  if (rc) return rc;
  GemmArParams ar{};
  for (int r = 0; r < p->world; ++r) {
    if (p->inbox[r] == nullptr || p->out[r] == nullptr || p->counters[r] == nullptr) return kErrInvalidArg;
    if ((reinterpret_cast<uintptr_t>(p->inbox[r]) & 15u) || (reinterpret_cast<uintptr_t>(p->out[r]) & 15u) ||
        (reinterpret_cast<uintptr_t>(p->counters[r]) & 7u))
      return kErrInvalidArg;
    ar.inbox[r] = p->inbox[r];
    ar.out[r] = p->out[r];
    // counters: [tiles_per_owner] arrivals, then the done counter
    ar.arrive[r] = static_cast<unsigned long long*>(p->counters[r]);
    ar.done[r] = static_cast<unsigned long long*>(p->counters[r]) + per_owner;
  }
  ar.ldo = p->ldo;
  ar.world = p->world;
  ar.rank = p->rank;
  ar.tiles_per_owner = per_owner;
  GemmLaunch L{};
  L.a = p->a;
  L.b = p->b;
  L.c = p->out[p->rank];
  L.lda = p->lda;
  L.ldb = p->ldb;
  L.ldc = p->ldo;
  L.M = p->M;
  L.N = p->N;
  L.K = p->K;
  L.in_dtype = L.out_dtype = p->in_dtype;
  L.group_m = 8;
  return gemm_allreduce(L, ar, static_cast<cudaStream_t>(stream));
}

// Peer memory: export a device pointer so another process can map it, and
// map / unmap what a peer exported.  Handles are cudaIpcMemHandle_t bytes.
static int ipc_base(const void* ptr, void** base, size_t* offset) {
  static PFN_cuMemGetAddressRange_v3020 get_range = [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &fn, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      fn = nullptr;
    return reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
  }();
  if (get_range == nullptr) return kErrCuda;
  CUdeviceptr b = 0;
  size_t size = 0;
  if (get_range(&b, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return kErrInvalidArg;
  *base = reinterpret_cast<void*>(b);
  *offset = static_cast<size_t>(reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(b));
  return kOk;
}

int fab_ipc_export(const void* ptr, void* handle, size_t* offset) {
  if (ptr == nullptr || handle == nullptr || offset == nullptr) return kErrInvalidArg;
  void* base = nullptr;
  int rc = ipc_base(ptr, &base, offset);
  if (rc) return rc;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, base) != cudaSuccess) return kErrCuda;
  memcpy(handle, &h, sizeof(h));
  return kOk;
}

int fab_ipc_import(const void* handle, size_t offset, void** base, void** ptr) {
  if (handle == nullptr || base == nullptr || ptr == nullptr) return kErrInvalidArg;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* b = nullptr;
  if (cudaIpcOpenMemHandle(&b, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return kErrCuda;
  *base = b;
  *ptr = static_cast<uint8_t*>(b) + offset;
  return kOk;
}

int fab_ipc_close(void* base) {
  if (base == nullptr) return kErrInvalidArg;
  return cudaIpcCloseMemHandle(base) == cudaSuccess ? kOk : kErrCuda;
}

static bool al16(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
static bool ld16(int64_t ld) { return (ld * 2) % 16 == 0; }

int fab_rmsnorm(const void* x, const void* residual, const void* w, void* h, void* x_out, int rows, int cols,
                int64_t ld_x, int64_t ld_res, int64_t ld_h, int64_t ld_xo, float eps, int dtype, void* stream) {
  if (rows < 0 || cols <= 0 || cols % 8 != 0 || cols > 8192) return kErrInvalidArg;
  if (x == nullptr || w == nullptr || h == nullptr || (residual != nullptr && x_out == nullptr)) return kErrInvalidArg;
  if (!al16(x) || !al16(residual) || !al16(w) || !al16(h) || !al16(x_out)) return kErrInvalidArg;
  if (!ld16(ld_x) || !ld16(ld_h) || (residual != nullptr && (!ld16(ld_res) || !ld16(ld_xo)))) return kErrInvalidArg;
  if (dtype != kDtypeBF16 && dtype != kDtypeF16) return kErrUnsupported;
  if (rows == 0) return kOk;
  auto st = static_cast<cudaStream_t>(stream);
  if (dtype == kDtypeBF16) {
    using T = __nv_bfloat16;
    rmsnorm_kernel<T><<<rows, 256, 0, st>>>(static_cast<const T*>(x), static_cast<const T*>(residual),
                                            static_cast<const T*>(w), static_cast<T*>(h), static_cast<T*>(x_out), cols,
                                            ld_x, ld_res, ld_h, ld_xo, eps, nullptr);
  } else {
    using T = __half;
    rmsnorm_kernel<T><<<rows, 256, 0, st>>>(static_cast<const T*>(x), static_cast<const T*>(residual),
                                            static_cast<const T*>(w), static_cast<T*>(h), static_cast<T*>(x_out), cols,
                                            ld_x, ld_res, ld_h, ld_xo, eps, nullptr);
  }
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int fab_rmsnorm_rstd(const void* x, const void* residual, void* x_out, float* rstd, int rows, int cols, int64_t ld_x,
                     int64_t ld_res, int64_t ld_xo, float eps, int dtype, void* stream) {
  if (rows < 0 || cols <= 0 || cols % 8 != 0 || cols > 8192) return kErrInvalidArg;
  if (x == nullptr || rstd == nullptr || (residual != nullptr && x_out == nullptr)) return kErrInvalidArg;
  if (!al16(x) || !al16(residual) || !al16(x_out) || (reinterpret_cast<uintptr_t>(rstd) & 3u) != 0)
    return kErrInvalidArg;
  if (!ld16(ld_x) || (residual != nullptr && (!ld16(ld_res) || !ld16(ld_xo)))) return kErrInvalidArg;
  if (dtype != kDtypeBF16 && dtype != kDtypeF16) return kErrUnsupported;
  if (rows == 0) return kOk;
  auto st = static_cast<cudaStream_t>(stream);
  if (dtype == kDtypeBF16) {
    using T = __nv_bfloat16;
    rmsnorm_kernel<T><<<rows, 256, 0, st>>>(static_cast<const T*>(x), static_cast<const T*>(residual), nullptr,
                                            nullptr, static_cast<T*>(x_out), cols, ld_x, ld_res, 0, ld_xo, eps, rstd);
  } else {
    using T = __half;
    rmsnorm_kernel<T><<<rows, 256, 0, st>>>(static_cast<const T*>(x), static_cast<const T*>(residual), nullptr,
                                            nullptr, static_cast<T*>(x_out), cols, ld_x, ld_res, 0, ld_xo, eps, rstd);
  }
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int fab_bias_rope(void* y, const void* bias, const void* cos, const void* sin, int rows, int heads, int rot_heads,
                  int head_dim, int64_t ld, int dtype, void* stream) {
  if (rows < 0 || heads <= 0 || rot_heads < 0 || rot_heads > heads || head_dim <= 0 || head_dim % 16 != 0)
    return kErrInvalidArg;
  if (y == nullptr || (rot_heads > 0 && (cos == nullptr || sin == nullptr))) return kErrInvalidArg;
  if (!al16(y) || !al16(bias) || !al16(cos) || !al16(sin) || !ld16(ld) || ld < static_cast<int64_t>(heads) * head_dim)
    return kErrInvalidArg;
  if (dtype != kDtypeBF16 && dtype != kDtypeF16) return kErrUnsupported;
  const int64_t threads = static_cast<int64_t>(rows) * heads * (head_dim / 16);
  if (threads == 0) return kOk;
  const unsigned blocks = static_cast<unsigned>((threads + 255) / 256);
  auto st = static_cast<cudaStream_t>(stream);
  if (dtype == kDtypeBF16) {
    using T = __nv_bfloat16;
    bias_rope_kernel<T><<<blocks, 256, 0, st>>>(static_cast<T*>(y), static_cast<const T*>(bias),
                                                static_cast<const T*>(cos), static_cast<const T*>(sin), rows, heads,
                                                rot_heads, head_dim, ld);
  } else {
    using T = __half;
    bias_rope_kernel<T><<<blocks, 256, 0, st>>>(static_cast<T*>(y), static_cast<const T*>(bias),
                                                static_cast<const T*>(cos), static_cast<const T*>(sin), rows, heads,
                                                rot_heads, head_dim, ld);
  }
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int fab_silu_mul(const void* gu, void* a, int rows, int m, int64_t ld_gu, int64_t ld_a, int interleave, int dtype,
                 void* stream) {
  if (rows < 0 || m <= 0 || m % 8 != 0 || gu == nullptr || a == nullptr) return kErrInvalidArg;
  if (interleave != 0 && (interleave % 8 != 0 || m % interleave != 0)) return kErrInvalidArg;
  if (!al16(gu) || !al16(a) || !ld16(ld_gu) || !ld16(ld_a) || ld_gu < 2LL * m || ld_a < m) return kErrInvalidArg;
  if (dtype != kDtypeBF16 && dtype != kDtypeF16) return kErrUnsupported;
  const int64_t threads = static_cast<int64_t>(rows) * (m / 8);
  if (threads == 0) return kOk;
  const unsigned blocks = static_cast<unsigned>((threads + 255) / 256);
  auto st = static_cast<cudaStream_t>(stream);
  if (dtype == kDtypeBF16) {
    using T = __nv_bfloat16;
    silu_mul_kernel<T><<<blocks, 256, 0, st>>>(static_cast<const T*>(gu), static_cast<T*>(a), rows, m, ld_gu, ld_a,
                                               interleave);
  } else {
    using T = __half;
    silu_mul_kernel<T><<<blocks, 256, 0, st>>>(static_cast<const T*>(gu), static_cast<T*>(a), rows, m, ld_gu, ld_a,
                                               interleave);
  }
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int fab_matmul_contiguous(const void* a, const void* b, void* c, int M, int N, int K, int in_dtype, int out_dtype,
                          int round_f16, void* stream) {
  fab_gemm_params p{};
  p.a = a;
  p.b = b;
  p.c = c;
  p.lda = K;
  p.ldb = N;
  p.ldc = N;
  p.M = M;
  p.N = N;
  p.K = K;
  p.in_dtype = in_dtype;
  p.out_dtype = out_dtype;
  p.round_f16 = round_f16;
  p.group_m = 8;
  return fab_gemm(&p, stream);
}

int fab_flash_attn_config(int dtype, int head_dim, fab_fa_config* out) {
  if (out == nullptr) return kErrInvalidArg;
  FaConfigInfo c;
  int rc = fa_select_config(dtype, head_dim, &c);
  if (rc) return rc;
  out->head_dim_padded = c.d_pad;
  out->q_tiles_per_cta = c.nq;
  out->block_n = c.bn;
  out->stages = c.stages;
  out->threads = c.threads;
  out->smem_bytes = c.smem_bytes;
  out->tmem_columns = c.tmem_cols;
  out->s_buffers = c.s_bufs;
  return kOk;
}

int fab_kernel_attrs_query(int which, int dtype, int head_dim, fab_kernel_attrs* out) {
  if (out == nullptr) return kErrInvalidArg;
  int regs = 0, smem = 0, threads = 0, rc;
  if (which == FAB_KERNEL_ATTENTION)
    rc = fa_kernel_attrs(dtype, head_dim, &regs, &smem, &threads);
  else if (which == FAB_KERNEL_ATTENTION_ONE_TILE)
    rc = fa_kernel_attrs(dtype, head_dim, &regs, &smem, &threads, true);
  else if (which == FAB_KERNEL_MATMUL)
    rc = gemm_kernel_attrs(dtype, &regs, &smem, &threads);
  else
    return kErrInvalidArg;
  if (rc) return rc;
  out->registers_per_thread = regs;
  out->shared_bytes = smem;
  out->threads = threads;
  return kOk;
}

int fab_device_limits_query(int device, fab_device_limits* out) {
  if (out == nullptr) return kErrInvalidArg;
  struct {
    cudaDeviceAttr attr;
    int* dst;
  } q[] = {
      {cudaDevAttrMaxSharedMemoryPerMultiprocessor, &out->shared_bytes_per_sm},
      {cudaDevAttrMaxSharedMemoryPerBlockOptin, &out->shared_bytes_per_block_optin},
      {cudaDevAttrMaxRegistersPerMultiprocessor, &out->registers_per_sm},
      {cudaDevAttrWarpSize, &out->warp_size},
      {cudaDevAttrMaxThreadsPerBlock, &out->max_threads_per_block},
      {cudaDevAttrMultiProcessorCount, &out->multiprocessor_count},
      {cudaDevAttrComputeCapabilityMajor, &out->cc_major},
      {cudaDevAttrComputeCapabilityMinor, &out->cc_minor},
  };
  for (auto& e : q)
    if (cudaDeviceGetAttribute(e.dst, e.attr, device) != cudaSuccess) {
      cudaGetLastError();
      return kErrCuda;
    }
  return kOk;
}

int fab_get_device_error(int* code) {
  if (code == nullptr) return kErrInvalidArg;
  // This unit's status word (attention, decoder ops), then the GEMM unit's;
  // both are cleared, the first code recorded is reported.
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_fab_device_error, sizeof(int)) != cudaSuccess) return kErrCuda;
  if (v != 0) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_fab_device_error, &zero, sizeof(int)) != cudaSuccess) return kErrCuda;
  }
  int g = 0;
  const int rc = gemm_take_device_error(&g);
  if (rc) return rc;
  *code = v != 0 ? v : g;
  return kOk;
}

}  // extern "C"
