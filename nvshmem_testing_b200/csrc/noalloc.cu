// moe_ep_run_noalloc: the single-rank fused layer for callers that cannot
// allocate device memory.
//
// moe_ep_run keeps its control words (published counts, arrival flags, work
// counters, status) in a workspace that the caller allocates with
// moe_symm_alloc.  Some callers have no way to do that: a host program that
// reaches this library only through the C ABI and owns no CUDA allocator, a
// serving process whose device memory is planned up front and may not grow
// after start-up, or a single-GPU user who does not want the exportable cuMem
// allocation (2 MB granularity, a file descriptor) that the multi-GPU
// workspace needs.  For one rank those control words are tiny, so this entry
// point keeps them in a fixed array that lives in the library itself.
//
// The array is a file-scope __device__ variable: every GPU that loads the
// library holds a copy until the process exits.  Host code cannot use its
// name as a device address, so the first call on each device looks the
// address up with cudaGetSymbolAddress (with that device current) and
// records it; make that first call before any stream capture.  Every call
// then prepares the array in stream order with a one-block kernel (the
// one-entry peer table and zeroed control words) before the layer kernel.
#include <cuda_runtime.h>

#include <mutex>

#include "moe_ep.h"
#include "moe_ep_internal.h"

using namespace moe;

namespace {

// [0, 256): one-entry peer table (this rank's control base);
// [256, 256 + ctrl_bytes): the control region for <= MOE_EP_NOALLOC_MAX_EXPERTS experts.
constexpr size_t kPeerTableBytes = 256;
constexpr size_t kScratchBytes = MOE_EP_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

uint64_t g_scratch_addr[kMaxDevices];  // device address of the array per device; 0 = not yet looked up
std::mutex g_setup;

// Once per device, with `dev` current: the array's device address.
int scratch_address(int dev, uint64_t* out) {
  std::lock_guard<std::mutex> lock(g_setup);
  if (g_scratch_addr[dev] == 0) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) return kCudaErr;
    g_scratch_addr[dev] = reinterpret_cast<uint64_t>(ptr);
  }
  *out = g_scratch_addr[dev];
  return kOk;
}

// In stream order before each layer kernel: the peer-table slot holds the
// control base, and the control words the previous call left start at zero.
__global__ void prepare_scratch_kernel(uint32_t ctrl_words) {
  if (threadIdx.x == 0)
    *reinterpret_cast<uint64_t*>(g_noalloc_scratch) = reinterpret_cast<uint64_t>(g_noalloc_scratch + kPeerTableBytes);
  uint32_t* ctrl = reinterpret_cast<uint32_t*>(g_noalloc_scratch + kPeerTableBytes);
  for (uint32_t i = threadIdx.x; i < ctrl_words; i += blockDim.x) ctrl[i] = 0u;
}

}  // namespace

extern "C" int moe_ep_run_noalloc(const moe_ep_run_params* params, void* stream) {
  if (!params) return kBadArg;
  if (params->world_size != 1 || params->rank != 0 || params->local_experts < 1) return kBadArg;
  if (params->local_experts > MOE_EP_NOALLOC_MAX_EXPERTS) return MOE_EP_SCRATCH_LIMIT;
  // The control words are cleared by the next call, so a device-side error
  // can only be read through the caller's mapped status word: require it.
  if (!params->status_host) return kBadArg;
  if (params->gm < 0 || params->gm > (int64_t(1) << 30)) return kBadArg;

  // One flag slot per expert: a chunk of gm rows covers every valid count.
  const int push_rows = params->gm > 0 ? int(params->gm) : 1;
  moe_ep_layout L;
  if (workspace_layout(1, params->local_experts, params->hidden, params->elem_bytes, 0, 1, 0, 0, &L) != kOk)
    return kBadArg;
  if (kPeerTableBytes + L.ctrl_bytes > kScratchBytes) return MOE_EP_SCRATCH_LIMIT;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return kCudaErr;
  uint64_t scratch = 0;
  if (scratch_address(dev, &scratch) != kOk) return kCudaErr;

  // The array keeps whatever the previous call left there; the kernel needs
  // zeroed counters and epochs, so clear the control region in stream order.
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  prepare_scratch_kernel<<<1, 256, 0, s>>>(uint32_t(L.ctrl_bytes / 4));
  if (cudaGetLastError() != cudaSuccess) return kCudaErr;

  moe_ep_run_params q = *params;
  q.peer_bases = reinterpret_cast<const uint64_t*>(scratch);
  q.local_base = scratch + kPeerTableBytes;
  q.cap_rows = 0;
  q.push_rows = push_rows;
  q.max_chunks = 1;
  q.epoch = 1;
  q.push_ctas = 0;
  q.local_first = 0;
  return launch_fused(&q, FusedMode{}, s);
}
