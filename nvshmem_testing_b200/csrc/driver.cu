// Driver API entry points resolved through the CUDA runtime, so the shared
// library carries no link-time dependency on libcuda and loads on hosts
// without a GPU driver (the functions then report kCudaErr).
#include <mutex>

#include "moe_ep_internal.h"

namespace moe {

template <typename F>
static bool resolve(const char* name, F& fn) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess ||
      p == nullptr)
    return false;
  fn = reinterpret_cast<F>(p);
  return true;
}

const Driver& driver() {
  static Driver d{};
  static std::once_flag once;
  std::call_once(once, [] {
    bool ok = true;
    ok &= resolve("cuMemGetAllocationGranularity", d.cuMemGetAllocationGranularity);
    ok &= resolve("cuMemCreate", d.cuMemCreate);
    ok &= resolve("cuMemAddressReserve", d.cuMemAddressReserve);
    ok &= resolve("cuMemMap", d.cuMemMap);
    ok &= resolve("cuMemSetAccess", d.cuMemSetAccess);
    ok &= resolve("cuMemExportToShareableHandle", d.cuMemExportToShareableHandle);
    ok &= resolve("cuMemImportFromShareableHandle", d.cuMemImportFromShareableHandle);
    ok &= resolve("cuMemUnmap", d.cuMemUnmap);
    ok &= resolve("cuMemRelease", d.cuMemRelease);
    ok &= resolve("cuMemAddressFree", d.cuMemAddressFree);
    ok &= resolve("cuTensorMapEncodeTiled", d.cuTensorMapEncodeTiled);
    d.ok = ok;
  });
  return d;
}

}  // namespace moe
