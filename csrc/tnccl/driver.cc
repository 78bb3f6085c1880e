#include "driver.h"

#include <cuda_runtime_api.h>

#include <mutex>

#include "common.h"

namespace tnccl {

namespace {

template <typename Fn>
bool resolve(const char* name, Fn* fn) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
  cudaError_t e = cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr) {
    (void)cudaGetLastError();
    TN_INFO("driver entry point %s unavailable", name);
    return false;
  }
  *fn = reinterpret_cast<Fn>(p);
  return true;
}

}  // namespace

const DriverApi* driverApi() {
  static DriverApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    bool ok = true;
    ok &= resolve("cuGetErrorString", &api.cuGetErrorString);
    ok &= resolve("cuDeviceGet", &api.cuDeviceGet);
    ok &= resolve("cuDeviceGetAttribute", &api.cuDeviceGetAttribute);
    ok &= resolve("cuMemGetAllocationGranularity", &api.cuMemGetAllocationGranularity);
    ok &= resolve("cuMemCreate", &api.cuMemCreate);
    ok &= resolve("cuMemRelease", &api.cuMemRelease);
    ok &= resolve("cuMemExportToShareableHandle", &api.cuMemExportToShareableHandle);
    ok &= resolve("cuMemImportFromShareableHandle", &api.cuMemImportFromShareableHandle);
    ok &= resolve("cuMemAddressReserve", &api.cuMemAddressReserve);
    ok &= resolve("cuMemAddressFree", &api.cuMemAddressFree);
    ok &= resolve("cuMemMap", &api.cuMemMap);
    ok &= resolve("cuMemUnmap", &api.cuMemUnmap);
    ok &= resolve("cuMemSetAccess", &api.cuMemSetAccess);
    // Multicast entry points are optional: without them NVLS stays off.
    resolve("cuMulticastCreate", &api.cuMulticastCreate);
    resolve("cuMulticastAddDevice", &api.cuMulticastAddDevice);
    resolve("cuMulticastBindMem", &api.cuMulticastBindMem);
    resolve("cuMulticastUnbind", &api.cuMulticastUnbind);
    resolve("cuMulticastGetGranularity", &api.cuMulticastGetGranularity);
    api.loaded = ok;
  });
  return api.loaded ? &api : nullptr;
}

const char* cuErrorName(CUresult r) {
  const DriverApi* api = driverApi();
  const char* s = nullptr;
  if (api && api->cuGetErrorString && api->cuGetErrorString(r, &s) == CUDA_SUCCESS && s) {
    return s;
  }
  return "unknown CUDA driver error";
}

}  // namespace tnccl
