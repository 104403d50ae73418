// Internal declarations shared by the .cu files of the extension.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

#include "moe_ep.h"

namespace moe {

// Status codes; identical to the MOE_EP_* values of include/moe_ep.h.
enum : int {
  kOk = 0,
  kBadArg = 1,
  kCudaErr = 2,
  kTimeout = 3,
  kCapacity = 4,
  kBadRoute = 5,
};

// Status-word sites shared by the kernels (the "site" byte of a latched error).
enum Site : int {
  kSiteCounts = 1,
  kSiteTable = 2,
  kSiteTileFlag = 3,
  kSiteFree = 4,
  kSitePipe = 5,
  kSiteDrain = 6,
  kSiteReturn = 7,
};

constexpr int kMaxExperts = 1024;  // routing kernel: experts per call
constexpr int kMaxRouteK = 32;     // routing kernel: ids per token (top-k width)

// ---- routing (route.cu)
size_t route_smem_bytes(int E);
int launch_route(const void* ids, int ids_are_int64, int64_t T, int K, int E, int32_t* counts, int32_t* offsets,
                 int32_t* perm, int32_t* slots, int32_t* max_count, cudaStream_t stream);
// Words at the workspace's off_local (never accessed by peers).
struct LocalWords {
  uint32_t push_ctr[2];
  uint32_t done_ctr[2];
  uint32_t status;
  uint32_t tile_ctr[2];
  uint32_t pad;
  uint32_t zero_ctr[2];
  uint32_t local_ctr[2];
};

int launch_publish_i32(const int32_t* src, int64_t n, int32_t* dst, cudaStream_t stream);
int launch_pack_compact(const void* tokens, int64_t H, int elem_bytes, const int32_t* perm, int64_t rows, void* out,
                        int num_sms, cudaStream_t stream);
int launch_pack_padded(const void* tokens, int64_t H, int elem_bytes, const int32_t* counts, const int32_t* offsets,
                       const int32_t* perm, int E, int64_t gm, void* out, int num_sms, cudaStream_t stream);

// ---- driver entry points (driver.cu), resolved at first use through the runtime
struct Driver {
  CUresult (*cuMemGetAllocationGranularity)(size_t*, const CUmemAllocationProp*, CUmemAllocationGranularity_flags);
  CUresult (*cuMemCreate)(CUmemGenericAllocationHandle*, size_t, const CUmemAllocationProp*, unsigned long long);
  CUresult (*cuMemAddressReserve)(CUdeviceptr*, size_t, size_t, CUdeviceptr, unsigned long long);
  CUresult (*cuMemMap)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long);
  CUresult (*cuMemSetAccess)(CUdeviceptr, size_t, const CUmemAccessDesc*, size_t);
  CUresult (*cuMemExportToShareableHandle)(void*, CUmemGenericAllocationHandle, CUmemAllocationHandleType,
                                           unsigned long long);
  CUresult (*cuMemImportFromShareableHandle)(CUmemGenericAllocationHandle*, void*, CUmemAllocationHandleType);
  CUresult (*cuMemUnmap)(CUdeviceptr, size_t);
  CUresult (*cuMemRelease)(CUmemGenericAllocationHandle);
  CUresult (*cuMemAddressFree)(CUdeviceptr, size_t);
  CUresult (*cuTensorMapEncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                     const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                     CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  bool ok;
};
const Driver& driver();

// ---- fused dispatch + grouped GEMM (fused.cu)
int workspace_layout(int W, int El, int64_t H, int elem_bytes, int64_t cap_rows, int max_chunks, int64_t ret_rows,
                     int64_t ret_cols, moe_ep_layout* L);
struct FusedMode {
  int64_t ret_rows = 0;   // > 0: return mode (combine path)
  int general = 0;        // compact (unpadded) send buffer and output
  int64_t send_rows = 0;  // compact mode: rows of tokens
  int64_t out_rows = 0;   // compact mode: rows of out
  int tile_cap = 0;       // most rows per GEMM tile (multiple of 16); 0 = 256
  int kstagger = 0;       // stagger each tile's first k-block (tiles that share weights)
  int glu = 0;            // compact mode only: SwiGLU epilogue (out has out_dim / 2 columns)
};
int launch_fused(const moe_ep_run_params* a, const FusedMode& m, cudaStream_t stream);

// ---- return path: top-k weighted combine (combine.cu)
int launch_combine(const moe_ep_run_params* run, const moe_ep_combine_params* c, const moe_ep_layout& L,
                   cudaStream_t stream);
}  // namespace moe
