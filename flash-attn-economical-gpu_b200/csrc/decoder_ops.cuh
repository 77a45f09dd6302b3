// Memory-bound decoder-layer operations around the GEMMs and the attention of
// the tensor-parallel prefill (Qwen2-style decoder, the model the reference's
// TTFT benchmark runs: ttft.py:401-412).  Each is one pass over its tensors
// with 16-byte accesses, and each rounds where the reference's PyTorch
// expressions round, so the bf16 results match them:
//   residual + RMSNorm   x' = x + r (bf16);  h = w * bf16(x' * rsqrt(mean(x'^2) + eps))
//   bias + RoPE          y = y + b (bf16);   y = bf16(bf16(y * cos) + bf16(rotate_half(y) * sin))
//   SwiGLU               a = bf16(bf16(silu(g)) * u)
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "fa_internal.h"

namespace fab {

template <typename T>
struct Elem;
template <>
struct Elem<__nv_bfloat16> {
  __device__ static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ static __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};
template <>
struct Elem<__half> {
  __device__ static float to_f(__half x) { return __half2float(x); }
  __device__ static __half from_f(float x) { return __float2half_rn(x); }
};

template <typename T>
__device__ __forceinline__ float rnd(float x) {  // round to T and back
  return Elem<T>::to_f(Elem<T>::from_f(x));
}

// 8 values of T in one 16-byte word.
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& w, float (&f)[8]) {
  const T* e = reinterpret_cast<const T*>(&w);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = Elem<T>::to_f(e[i]);
}
template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 w;
  T* e = reinterpret_cast<T*>(&w);
#pragma unroll
  for (int i = 0; i < 8; ++i) e[i] = Elem<T>::from_f(f[i]);
  return w;
}

// One CTA per row; `cols` a multiple of 8.  With `res` != nullptr the row is
// x + res, written to x_out (may alias x) before the norm.  With h ==
// nullptr only the row's rsqrt(mean(x^2) + eps) is written, to rstd[row]
// (the scale a GEMM with the norm folded into it applies).
template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const T* __restrict__ x, const T* __restrict__ res,
                                                      const T* __restrict__ w, T* __restrict__ h, T* x_out, int cols,
                                                      int64_t ld_x, int64_t ld_res, int64_t ld_h, int64_t ld_xo,
                                                      float eps, float* __restrict__ rstd) {
  constexpr int kMaxVec = 4;  // 8 columns per vector, 256 threads: up to 8192 columns
  const int64_t row = blockIdx.x;
  const int nvec = cols / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ld_x);
  float v[kMaxVec][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxVec; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) {
      unpack8<T>(xr[i], v[k]);
      if (res != nullptr) {
        float r[8];
        unpack8<T>(reinterpret_cast<const uint4*>(res + row * ld_res)[i], r);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[k][e] = rnd<T>(v[k][e] + r[e]);
        reinterpret_cast<uint4*>(x_out + row * ld_xo)[i] = pack8<T>(v[k]);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(v[k][e], v[k][e], ss);
    }
  }
  __shared__ float red[8];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float inv = rsqrtf(tot / static_cast<float>(cols) + eps);
  if (h == nullptr) {
    if (threadIdx.x == 0) rstd[row] = inv;
    return;
  }
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* hr = reinterpret_cast<uint4*>(h + row * ld_h);
#pragma unroll
  for (int k = 0; k < kMaxVec; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) {
      float wf[8], o[8];
      unpack8<T>(wr[i], wf);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = wf[e] * rnd<T>(v[k][e] * inv);
      hr[i] = pack8<T>(o);
    }
  }
}

// In place on y [rows, heads, D] (row stride ld): bias add on every head,
// rotate-half RoPE on the first rot_heads; cos/sin [rows, D].  One thread per
// 8 columns of the first half of a head (it also owns the matching 8 of the
// second half).
template <typename T>
__global__ void __launch_bounds__(256) bias_rope_kernel(T* y, const T* __restrict__ bias, const T* __restrict__ cs,
                                                        const T* __restrict__ sn, int rows, int heads, int rot_heads,
                                                        int D, int64_t ld) {
  const int half_vec = D / 16;  // 8-column vectors in half a head
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = static_cast<int64_t>(rows) * heads * half_vec;
  if (idx >= total) return;
  const int vi = static_cast<int>(idx % half_vec);
  const int hd = static_cast<int>((idx / half_vec) % heads);
  const int64_t s = idx / (static_cast<int64_t>(half_vec) * heads);
  T* base = y + s * ld + static_cast<int64_t>(hd) * D;
  uint4* lo_p = reinterpret_cast<uint4*>(base) + vi;
  uint4* hi_p = reinterpret_cast<uint4*>(base + D / 2) + vi;
  float lo[8], hi[8];
  unpack8<T>(*lo_p, lo);
  unpack8<T>(*hi_p, hi);
  if (bias != nullptr) {
    float bl[8], bh[8];
    unpack8<T>(reinterpret_cast<const uint4*>(bias + static_cast<int64_t>(hd) * D)[vi], bl);
    unpack8<T>(reinterpret_cast<const uint4*>(bias + static_cast<int64_t>(hd) * D + D / 2)[vi], bh);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      lo[e] = rnd<T>(lo[e] + bl[e]);
      hi[e] = rnd<T>(hi[e] + bh[e]);
    }
  }
  if (hd < rot_heads) {
    // rotate_half(y) = [-y_hi, y_lo]; cos/sin repeat over the two halves
    float cl[8], ch[8], sl[8], sh[8];
    unpack8<T>(reinterpret_cast<const uint4*>(cs + s * D)[vi], cl);
    unpack8<T>(reinterpret_cast<const uint4*>(cs + s * D + D / 2)[vi], ch);
    unpack8<T>(reinterpret_cast<const uint4*>(sn + s * D)[vi], sl);
    unpack8<T>(reinterpret_cast<const uint4*>(sn + s * D + D / 2)[vi], sh);
    float nlo[8], nhi[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      nlo[e] = rnd<T>(rnd<T>(lo[e] * cl[e]) + rnd<T>(-hi[e] * sl[e]));
      nhi[e] = rnd<T>(rnd<T>(hi[e] * ch[e]) + rnd<T>(lo[e] * sh[e]));
    }
    *lo_p = pack8<T>(nlo);
    *hi_p = pack8<T>(nhi);
  } else if (bias != nullptr) {
    *lo_p = pack8<T>(lo);
    *hi_p = pack8<T>(hi);
  }
}

// a[s, j] = bf16(bf16(silu(g)) * u).  interleave 0: g = gu[s, j], u = gu[s, m + j];
// interleave b: gu's columns alternate b gate and b up columns.
template <typename T>
__global__ void __launch_bounds__(256) silu_mul_kernel(const T* __restrict__ gu, T* __restrict__ a, int rows, int m,
                                                       int64_t ld_gu, int64_t ld_a, int interleave) {
  const int mv = m / 8;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(rows) * mv) return;
  const int64_t s = idx / mv;
  const int j = static_cast<int>(idx % mv);
  const int col = j * 8;
  const int gcol = interleave ? (col / interleave) * 2 * interleave + col % interleave : col;
  const int ucol = interleave ? gcol + interleave : m + col;
  float g[8], u[8], o[8];
  unpack8<T>(*reinterpret_cast<const uint4*>(gu + s * ld_gu + gcol), g);
  unpack8<T>(*reinterpret_cast<const uint4*>(gu + s * ld_gu + ucol), u);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float sg = rnd<T>(g[e] / (1.0f + expf(-g[e])));
    o[e] = sg * u[e];
  }
  reinterpret_cast<uint4*>(a + s * ld_a)[j] = pack8<T>(o);
}

}  // namespace fab
