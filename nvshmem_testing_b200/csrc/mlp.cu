// The expert MLP's activation (the full expert MLP of the step after the
// reference's single GEMM, baseline.py:50): h = silu(gate) * up, with
// a = [gate | up] the first GEMM's output rows (a [rows, 2F] bf16, gate in
// columns [0, F), up in [F, 2F)).  silu(g) = g / (1 + exp(-g)) in fp32, the
// product rounded to bf16.  HBM-bound: reads 4F bytes and writes 2F bytes per
// row; 16-byte vectors (8 features) per thread, grid-stride.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "moe_ep.h"
#include "moe_ep_internal.h"
#include "ptx.cuh"

namespace moe {
namespace {

constexpr int kSwigluThreads = 256;

__global__ void __launch_bounds__(kSwigluThreads)
    swiglu_kernel(const __nv_bfloat16* __restrict__ a, int64_t rows, int F, __nv_bfloat16* __restrict__ h) {
  const int vec = F / 8;
  const int64_t total = rows * vec;
  for (int64_t i = int64_t(blockIdx.x) * kSwigluThreads + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * kSwigluThreads) {
    const int64_t r = i / vec;
    const int f = int(i - r * vec) * 8;
    const __nv_bfloat16* row = a + r * int64_t(2 * F);
    const uint4 gv = ld_nc_v4(row + f);
    const uint4 uv = ld_nc_v4(row + F + f);
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv);
    const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(&uv);
    uint4 ov;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&ov);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 g = __bfloat1622float2(g2[j]);
      const float2 u = __bfloat1622float2(u2[j]);
      const float s0 = g.x / (1.f + expf(-g.x));
      const float s1 = g.y / (1.f + expf(-g.y));
      o2[j] = __floats2bfloat162_rn(s0 * u.x, s1 * u.y);
    }
    st_v4(h + r * int64_t(F) + f, ov);
  }
}

}  // namespace
}  // namespace moe

using namespace moe;

extern "C" int moe_swiglu(const void* a, int64_t rows, int32_t F, void* h, void* stream) {
  if (rows < 0 || F <= 0 || F % 8) return kBadArg;
  if (rows == 0) return kOk;
  if (!a || !h || ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(h)) & 15)) return kBadArg;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kCudaErr;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return kCudaErr;
  const int64_t total = rows * (F / 8);
  int64_t blocks = (total + kSwigluThreads - 1) / kSwigluThreads;
  const int64_t cap = int64_t(sms) * 8;
  if (blocks > cap) blocks = cap;
  swiglu_kernel<<<unsigned(blocks), kSwigluThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(a), rows, F, static_cast<__nv_bfloat16*>(h));
  return cudaGetLastError() == cudaSuccess ? kOk : kCudaErr;
}
