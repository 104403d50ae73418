// Router: the step before the path (utils.py:17-25 of the reference:
// logits = einsum('bh,he->be', tokens, router) in bf16, softmax over the
// experts, top-k).
//
// The logits GEMM runs on the fused kernel's tcgen05 GEMM as a one-rank,
// one-expert layer (tokens = x [T, H], weights = router [H, E], out = logits
// [T, E] bf16: fp32 accumulation rounded once, like the reference's bf16
// einsum).  Its control words (a one-entry peer table, the count matrix,
// flags, counters and the status word) and its one count word live in a
// fixed array of this file, so the router needs no workspace and allocates
// nothing; the first call on a device looks the array's address up with
// cudaGetSymbolAddress.  A second kernel then takes one token per warp: the
// fp32 softmax of the bf16 logits, rounded to bf16 (the reference's softmax
// output dtype), and the K largest probabilities in descending order, equal
// probabilities by ascending expert id (torch.topk leaves their order
// unspecified).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <climits>
#include <mutex>

#include "moe_ep.h"
#include "moe_ep_internal.h"

namespace moe {
namespace {

constexpr size_t kRouterScratchBytes = 2048;
constexpr size_t kPeerTable = 256;                          // [0, 256): control base of the one rank
constexpr size_t kCountOffset = kRouterScratchBytes - 16;   // int32 rows of the one (rank, expert) cell
constexpr int kMaxDevices = 64;
constexpr int kTopkThreads = 256;
constexpr int kTopkWarps = kTopkThreads / 32;

__device__ __align__(256) unsigned char g_router_scratch[kRouterScratchBytes];

uint64_t g_router_addr[kMaxDevices];
std::mutex g_router_setup;

// Once per device, with `dev` current: the array's device address, and the
// control base stored in its peer-table slot.
int router_scratch(int dev, uint64_t* out) {
  std::lock_guard<std::mutex> lock(g_router_setup);
  if (g_router_addr[dev] == 0) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_router_scratch) != cudaSuccess || ptr == nullptr) return kCudaErr;
    const uint64_t control_base = reinterpret_cast<uint64_t>(ptr) + kPeerTable;
    if (cudaMemcpyToSymbol(g_router_scratch, &control_base, sizeof(control_base), 0, cudaMemcpyHostToDevice) !=
        cudaSuccess)
      return kCudaErr;
    g_router_addr[dev] = reinterpret_cast<uint64_t>(ptr);
  }
  *out = g_router_addr[dev];
  return kOk;
}

__global__ void set_count_kernel(int32_t* p, int32_t v) { *p = v; }

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// PER = probabilities held per lane (E <= 32 * PER).
template <typename IdT, int PER>
__global__ void __launch_bounds__(kTopkThreads)
    router_topk_kernel(const __nv_bfloat16* __restrict__ logits, int64_t T, int E, int K, IdT* __restrict__ ids,
                       float* __restrict__ vals) {
  const int lane = threadIdx.x & 31;
  const int64_t stride = int64_t(gridDim.x) * kTopkWarps;
  for (int64_t t = int64_t(blockIdx.x) * kTopkWarps + (threadIdx.x >> 5); t < T; t += stride) {
    const __nv_bfloat16* row = logits + t * E;
    float v[PER];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int e = lane + 32 * j;
      v[j] = e < E ? __bfloat162float(row[e]) : -INFINITY;
      m = fmaxf(m, v[j]);
    }
    m = warp_max(m);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      v[j] = (lane + 32 * j) < E ? expf(v[j] - m) : 0.f;
      sum += v[j];
    }
    sum = warp_sum(sum);
    // Probabilities are >= 0; -1 marks a slot past E, -2 a slot already taken.
#pragma unroll
    for (int j = 0; j < PER; ++j)
      v[j] = (lane + 32 * j) < E ? __bfloat162float(__float2bfloat16_rn(v[j] / sum)) : -1.f;
    for (int k = 0; k < K; ++k) {
      float best = -3.f;
      int be = INT_MAX;
#pragma unroll
      for (int j = 0; j < PER; ++j) {  // ids ascend with j: a strict > keeps the lowest id of equal values
        if (v[j] > best) {
          best = v[j];
          be = lane + 32 * j;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oe = __shfl_xor_sync(0xffffffffu, be, o);
        if (ob > best || (ob == best && oe < be)) {
          best = ob;
          be = oe;
        }
      }
#pragma unroll
      for (int j = 0; j < PER; ++j)
        if (lane + 32 * j == be) v[j] = -2.f;
      if (lane == 0) {
        ids[t * K + k] = static_cast<IdT>(be);
        vals[t * K + k] = best;
      }
    }
  }
}

template <typename IdT>
int launch_topk(const __nv_bfloat16* logits, int64_t T, int E, int K, void* ids, float* vals, cudaStream_t s) {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kCudaErr;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return kCudaErr;
  int64_t blocks = (T + kTopkWarps - 1) / kTopkWarps;
  const int64_t cap = int64_t(sms) * 8;
  if (blocks > cap) blocks = cap;
  IdT* out = static_cast<IdT*>(ids);
  const unsigned g = unsigned(blocks);
  if (E <= 32) router_topk_kernel<IdT, 1><<<g, kTopkThreads, 0, s>>>(logits, T, E, K, out, vals);
  else if (E <= 64) router_topk_kernel<IdT, 2><<<g, kTopkThreads, 0, s>>>(logits, T, E, K, out, vals);
  else if (E <= 128) router_topk_kernel<IdT, 4><<<g, kTopkThreads, 0, s>>>(logits, T, E, K, out, vals);
  else if (E <= 256) router_topk_kernel<IdT, 8><<<g, kTopkThreads, 0, s>>>(logits, T, E, K, out, vals);
  else if (E <= 512) router_topk_kernel<IdT, 16><<<g, kTopkThreads, 0, s>>>(logits, T, E, K, out, vals);
  else router_topk_kernel<IdT, 32><<<g, kTopkThreads, 0, s>>>(logits, T, E, K, out, vals);
  return cudaGetLastError() == cudaSuccess ? kOk : kCudaErr;
}

}  // namespace
}  // namespace moe

using namespace moe;

extern "C" int moe_router(const void* x, int64_t T, int32_t H, const void* router_w, int32_t E, int32_t K,
                          void* logits, void* top_idxs, int32_t ids_are_int64, float* top_vals, void* stream) {
  if (T < 0 || T > (int64_t(1) << 30) || H <= 0 || H % 8 || E < 8 || E % 8 || E > kMaxExperts || K < 1 ||
      K > kMaxRouteK || K > E)
    return kBadArg;
  if (T == 0) return kOk;
  if (!x || !router_w || !logits || !top_idxs || !top_vals) return kBadArg;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(router_w) | reinterpret_cast<uintptr_t>(logits)) &
      15)
    return kBadArg;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);

  moe_ep_layout L;
  if (workspace_layout(1, 1, H, 2, 0, 1, 0, 0, &L) != kOk) return kBadArg;
  if (kPeerTable + L.ctrl_bytes > kCountOffset) return kBadArg;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return kCudaErr;
  uint64_t base = 0;
  if (router_scratch(dev, &base) != kOk) return kCudaErr;
  // The array keeps the previous call's words: zero the control region and
  // set this call's row count, in stream order.
  if (cudaMemsetAsync(reinterpret_cast<void*>(base + kPeerTable), 0, L.ctrl_bytes, s) != cudaSuccess) return kCudaErr;
  int32_t* count = reinterpret_cast<int32_t*>(base + kCountOffset);
  set_count_kernel<<<1, 1, 0, s>>>(count, int32_t(T));
  if (cudaGetLastError() != cudaSuccess) return kCudaErr;

  moe_ep_run_params p = {};
  p.world_size = 1;
  p.rank = 0;
  p.local_experts = 1;
  p.hidden = H;
  p.out_dim = E;
  p.elem_bytes = 2;
  p.gm = T;
  p.tokens = x;
  p.weights = router_w;
  p.recv_counts = count;
  p.out = logits;
  p.peer_bases = reinterpret_cast<const uint64_t*>(base);
  p.local_base = base + kPeerTable;
  p.cap_rows = 0;
  p.push_rows = int32_t(T);
  p.max_chunks = 1;
  p.epoch = 1;
  p.timeout_ns = 1000000000ull;  // one rank: it only waits for itself
  // One expert and few features: spread the rows over every CTA pair
  // (tiles of 16..256 rows, at least one per pair where T allows).
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return kCudaErr;
  const int64_t pairs = sms / 2 > 0 ? sms / 2 : 1;
  const int64_t feat_slices = (E + 255) / 256;
  int64_t cap = (T * feat_slices + pairs - 1) / pairs;
  cap = (cap + 15) / 16 * 16;
  FusedMode m;
  m.tile_cap = int(cap < 16 ? 16 : (cap > 256 ? 256 : cap));
  // Every tile reads the same router matrix: start each one at a different
  // k-block so the CTAs do not all request the same lines at once.
  m.kstagger = 1;
  const int rc = launch_fused(&p, m, s);
  if (rc != kOk) return rc;
  const auto* lg = static_cast<const __nv_bfloat16*>(logits);
  return ids_are_int64 ? launch_topk<long long>(lg, T, E, K, top_idxs, top_vals, s)
                       : launch_topk<int32_t>(lg, T, E, K, top_idxs, top_vals, s);
}
