// The GEMM kernels' translation unit of libfa_b200.so: one CTA per tile,
// CTA pairs (tcgen05 cta_group::2) and the fused GEMM + all-reduce.  It is
// compiled apart from capi.cu (attention, decoder ops, the C ABI): built in
// one unit with them, the CTA-pair kernel's instantiation changed the
// attention kernels' register allocation (a small spill; measured on B200,
// 2.5 % of attention throughput).  Each unit has its own copy of the device
// status word; fab_get_device_error reads both.
#include <cudaTypedefs.h>

#include <cstdint>

#include "fa_internal.h"
#include "ptx.cuh"

#include "gemm_kernel.cuh"

namespace fab {

int gemm_take_device_error(int* code) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_fab_device_error, sizeof(int)) != cudaSuccess) return kErrCuda;
  if (v != 0) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_fab_device_error, &zero, sizeof(int)) != cudaSuccess) return kErrCuda;
  }
  *code = v;
  return kOk;
}

}  // namespace fab
