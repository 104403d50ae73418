// extern "C" entry points of libmoe_ep.so (declared in include/moe_ep.h).
#include <cuda_runtime.h>

#include "moe_ep.h"
#include "moe_ep_internal.h"

using namespace moe;

static int set_device(int device) {
  if (cudaSetDevice(device) != cudaSuccess) return kCudaErr;
  if (cudaFree(nullptr) != cudaSuccess) return kCudaErr;  // make the primary context current
  return kOk;
}

extern "C" {

int moe_ep_abi_version(void) { return MOE_EP_ABI_VERSION; }

const char* moe_ep_status_string(int code) {
  switch (code) {
    case MOE_EP_OK: return "ok";
    case MOE_EP_BAD_ARG: return "bad argument";
    case MOE_EP_CUDA_ERR: return "CUDA error";
    case MOE_EP_TIMEOUT: return "timed out waiting for a peer";
    case MOE_EP_CAPACITY: return "receive capacity exceeded";
    case MOE_EP_BAD_ROUTE: return "bad routing input";
    case MOE_EP_SCRATCH_LIMIT: return "size exceeds the fixed scratch of moe_ep_run_noalloc";
    default: return "unknown status";
  }
}

int moe_ep_num_sms(int device, int* out) {
  if (!out) return kBadArg;
  return cudaDeviceGetAttribute(out, cudaDevAttrMultiProcessorCount, device) == cudaSuccess ? kOk : kCudaErr;
}

int moe_route(const void* top_idxs, int ids_are_int64, int64_t T, int K, int E, int32_t* counts, int32_t* offsets,
              int32_t* perm, int32_t* max_count, void* stream) {
  if (T < 0 || K < 1 || K > kMaxRouteK || E < 1 || E > kMaxExperts || (T > 0 && !top_idxs) || !counts || !offsets || !max_count ||
      (T > 0 && !perm))
    return kBadArg;
  if (T * int64_t(K) >= (int64_t(1) << 31)) return kBadArg;
  return launch_route(top_idxs, ids_are_int64, T, K, E, counts, offsets, perm, nullptr, max_count,
                      static_cast<cudaStream_t>(stream));
}

int moe_route_slots(const void* top_idxs, int ids_are_int64, int64_t T, int K, int E, int32_t* counts,
                    int32_t* offsets, int32_t* perm, int32_t* slots, int32_t* max_count, void* stream) {
  if (T < 0 || K < 1 || K > kMaxRouteK || E < 1 || E > kMaxExperts || (T > 0 && (!top_idxs || !perm || !slots)) ||
      !counts || !offsets || !max_count)
    return kBadArg;
  if (T * int64_t(K) >= (int64_t(1) << 31)) return kBadArg;
  return launch_route(top_idxs, ids_are_int64, T, K, E, counts, offsets, perm, slots, max_count,
                      static_cast<cudaStream_t>(stream));
}

int moe_publish_i32(const int32_t* src, int64_t n, int32_t* dst, void* stream) {
  if (n < 0 || (n > 0 && (!src || !dst)) || n > (int64_t(1) << 20)) return kBadArg;
  return launch_publish_i32(src, n, dst, static_cast<cudaStream_t>(stream));
}

int moe_pack_padded(const void* tokens, int64_t H, int elem_bytes, const int32_t* counts, const int32_t* offsets,
                    const int32_t* perm, int E, int64_t gm, void* out, void* stream) {
  if (H <= 0 || elem_bytes <= 0 || (H * elem_bytes) % 16 || E < 1 || gm < 0 || !counts || !offsets || !out)
    return kBadArg;
  if ((reinterpret_cast<uintptr_t>(tokens) | reinterpret_cast<uintptr_t>(out)) & 15) return kBadArg;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kCudaErr;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return kCudaErr;
  return launch_pack_padded(tokens, H, elem_bytes, counts, offsets, perm, E, gm, out, sms,
                            static_cast<cudaStream_t>(stream));
}

int moe_pack_compact(const void* tokens, int64_t H, int elem_bytes, const int32_t* perm, int64_t rows, void* out,
                     void* stream) {
  if (H <= 0 || elem_bytes <= 0 || (H * elem_bytes) % 16 || rows < 0 || (rows > 0 && (!tokens || !perm || !out)))
    return kBadArg;
  if ((reinterpret_cast<uintptr_t>(tokens) | reinterpret_cast<uintptr_t>(out)) & 15) return kBadArg;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kCudaErr;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return kCudaErr;
  return launch_pack_compact(tokens, H, elem_bytes, perm, rows, out, sms, static_cast<cudaStream_t>(stream));
}

int moe_symm_alloc(int device, size_t bytes, size_t* mapped_bytes, uint64_t* ptr, int* fd, uint64_t* handle) {
  if (bytes == 0 || !mapped_bytes || !ptr || !fd || !handle) return kBadArg;
  if (set_device(device) != kOk) return kCudaErr;
  const Driver& d = driver();
  if (!d.ok) return kCudaErr;
  CUmemAllocationProp prop = {};
  prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  prop.location.id = device;
  prop.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  size_t gran = 0;
  if (d.cuMemGetAllocationGranularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED) != CUDA_SUCCESS)
    return kCudaErr;
  const size_t size = (bytes + gran - 1) / gran * gran;
  CUmemGenericAllocationHandle h;
  if (d.cuMemCreate(&h, size, &prop, 0) != CUDA_SUCCESS) return kCudaErr;
  CUdeviceptr va = 0;
  if (d.cuMemAddressReserve(&va, size, gran, 0, 0) != CUDA_SUCCESS) {
    d.cuMemRelease(h);
    return kCudaErr;
  }
  if (d.cuMemMap(va, size, 0, h, 0) != CUDA_SUCCESS) {
    d.cuMemAddressFree(va, size);
    d.cuMemRelease(h);
    return kCudaErr;
  }
  CUmemAccessDesc acc = {};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = device;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  int shared_fd = -1;
  if (d.cuMemSetAccess(va, size, &acc, 1) != CUDA_SUCCESS ||
      d.cuMemExportToShareableHandle(&shared_fd, h, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0) != CUDA_SUCCESS) {
    d.cuMemUnmap(va, size);
    d.cuMemAddressFree(va, size);
    d.cuMemRelease(h);
    return kCudaErr;
  }
  *mapped_bytes = size;
  *ptr = uint64_t(va);
  *fd = shared_fd;
  *handle = uint64_t(h);
  return kOk;
}

int moe_symm_import(int device, int fd, size_t bytes, uint64_t* ptr, uint64_t* handle) {
  if (fd < 0 || bytes == 0 || !ptr || !handle) return kBadArg;
  if (set_device(device) != kOk) return kCudaErr;
  const Driver& d = driver();
  if (!d.ok) return kCudaErr;
  CUmemGenericAllocationHandle h;
  if (d.cuMemImportFromShareableHandle(&h, reinterpret_cast<void*>(static_cast<uintptr_t>(fd)),
                                       CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR) != CUDA_SUCCESS)
    return kCudaErr;
  CUmemAllocationProp prop = {};
  prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  prop.location.id = device;
  size_t gran = 0;
  if (d.cuMemGetAllocationGranularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED) != CUDA_SUCCESS) {
    d.cuMemRelease(h);
    return kCudaErr;
  }
  CUdeviceptr va = 0;
  if (d.cuMemAddressReserve(&va, bytes, gran, 0, 0) != CUDA_SUCCESS) {
    d.cuMemRelease(h);
    return kCudaErr;
  }
  if (d.cuMemMap(va, bytes, 0, h, 0) != CUDA_SUCCESS) {
    d.cuMemAddressFree(va, bytes);
    d.cuMemRelease(h);
    return kCudaErr;
  }
  CUmemAccessDesc acc = {};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = device;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  if (d.cuMemSetAccess(va, bytes, &acc, 1) != CUDA_SUCCESS) {
    d.cuMemUnmap(va, bytes);
    d.cuMemAddressFree(va, bytes);
    d.cuMemRelease(h);
    return kCudaErr;
  }
  *ptr = uint64_t(va);
  *handle = uint64_t(h);
  return kOk;
}

int moe_symm_free(uint64_t ptr, size_t bytes, uint64_t handle) {
  const Driver& d = driver();
  if (!d.ok) return kCudaErr;
  if (ptr == 0 || bytes == 0) return kBadArg;
  if (cudaDeviceSynchronize() != cudaSuccess) return kCudaErr;
  int rc = kOk;
  if (d.cuMemUnmap(CUdeviceptr(ptr), bytes) != CUDA_SUCCESS) rc = kCudaErr;
  if (d.cuMemAddressFree(CUdeviceptr(ptr), bytes) != CUDA_SUCCESS) rc = kCudaErr;
  if (d.cuMemRelease(CUmemGenericAllocationHandle(handle)) != CUDA_SUCCESS) rc = kCudaErr;
  return rc;
}

int moe_ep_workspace_layout(int W, int El, int64_t H, int elem_bytes, int64_t cap_rows, int max_chunks,
                            moe_ep_layout* out) {
  if (W < 1 || El < 1 || H < 1 || elem_bytes < 1 || cap_rows < 0 || max_chunks < 1 || !out) return kBadArg;
  return workspace_layout(W, El, H, elem_bytes, cap_rows, max_chunks, 0, 0, out);
}

int moe_ep_workspace_layout_ret(int W, int El, int64_t H, int elem_bytes, int64_t cap_rows, int max_chunks,
                                int64_t ret_rows, int64_t ret_cols, moe_ep_layout* out) {
  if (W < 1 || El < 1 || H < 1 || elem_bytes < 1 || cap_rows < 0 || max_chunks < 1 || ret_rows < 0 || ret_cols < 0 ||
      !out)
    return kBadArg;
  return workspace_layout(W, El, H, elem_bytes, cap_rows, max_chunks, ret_rows, ret_cols, out);
}

int moe_ep_run(const moe_ep_run_params* params, void* stream) {
  if (!params) return kBadArg;
  return launch_fused(params, FusedMode{}, static_cast<cudaStream_t>(stream));
}

int moe_ep_run_compact_swiglu(const moe_ep_run_params* params, int64_t send_rows, int64_t out_rows, void* stream) {
  if (!params || send_rows < 0 || out_rows < 0) return kBadArg;
  FusedMode m;
  m.general = 1;
  m.glu = 1;
  m.send_rows = send_rows;
  m.out_rows = out_rows;
  return launch_fused(params, m, static_cast<cudaStream_t>(stream));
}

int moe_ep_run_compact(const moe_ep_run_params* params, int64_t send_rows, int64_t out_rows, void* stream) {
  if (!params || send_rows < 0 || out_rows < 0) return kBadArg;
  FusedMode m;
  m.general = 1;
  m.send_rows = send_rows;
  m.out_rows = out_rows;
  return launch_fused(params, m, static_cast<cudaStream_t>(stream));
}

int moe_ep_run_combine(const moe_ep_run_params* run, const moe_ep_combine_params* c, void* stream) {
  if (!run || !c) return kBadArg;
  if (c->T < 0 || c->K < 1 || c->K > kMaxRouteK || c->ret_rows <= 0 || (c->T > 0 && (!c->top_idxs || !c->top_vals ||
      !c->slots || !c->y)))
    return kBadArg;
  if (reinterpret_cast<uintptr_t>(c->y) & 15) return kBadArg;
  if (int64_t(run->world_size) * run->local_experts * run->gm > c->ret_rows) return kBadArg;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  moe_ep_layout L;
  if (workspace_layout(run->world_size, run->local_experts, run->hidden, run->elem_bytes, run->cap_rows,
                       run->max_chunks, c->ret_rows, run->out_dim, &L) != kOk)
    return kBadArg;
  FusedMode m;
  m.ret_rows = c->ret_rows;
  const int rc = launch_fused(run, m, s);
  if (rc != kOk) return rc;
  return launch_combine(run, c, L, s);
}

int moe_ep_workspace_reset(uint64_t local_base, const moe_ep_layout* layout, void* stream) {
  if (!local_base || !layout) return kBadArg;
  return cudaMemsetAsync(reinterpret_cast<void*>(local_base), 0, layout->ctrl_bytes,
                         static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? kOk
             : kCudaErr;
}

int moe_ep_read_status(uint64_t local_base, const moe_ep_layout* layout, uint32_t* out) {
  if (!local_base || !layout || !out) return kBadArg;
  // LocalWords: push_ctr[2], done_ctr[2], status
  const void* src = reinterpret_cast<const unsigned char*>(local_base) + layout->off_local + 4 * sizeof(uint32_t);
  return cudaMemcpy(out, src, sizeof(uint32_t), cudaMemcpyDeviceToHost) == cudaSuccess ? kOk : kCudaErr;
}

}  // extern "C"
