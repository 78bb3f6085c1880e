// transport.cc - mailbox export/import and the NVLS multicast object.
//
// tiny-nccl allocates its inbox with cudaMalloc, exports a legacy CUDA IPC
// handle and opens only the next rank's inbox (src/comm.cc:13-38, :62-85).
// On an NVSwitch system every peer is one hop away, so here every rank maps
// every peer's mailbox. The default export is a cuMem (VMM) allocation shared
// as a POSIX file descriptor over the bootstrap socket (SCM_RIGHTS); this is
// also the memory kind that can be bound to an NVLS multicast object. The
// legacy cudaIpc path remains as a fallback (TNCCL_CUMEM_ENABLE=0 or a driver
// that refuses POSIX-fd export).
#include <string.h>
#include <unistd.h>

#include <vector>

#include "comm.h"
#include "driver.h"

namespace tnccl {

CUmemAllocationProp deviceProp(int device, bool exportable) {
  CUmemAllocationProp prop{};
  prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  prop.location.id = device;
  prop.requestedHandleTypes =
      exportable ? CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR : CU_MEM_HANDLE_TYPE_NONE;
  return prop;
}

bool cuOk(CUresult r, const char* what) {
  if (r == CUDA_SUCCESS) return true;
  TN_WARN("%s failed: %s (%d)", what, cuErrorName(r), (int)r);
  return false;
}

// Maps handle at a fresh VA range of `bytes` with read/write access for
// `device`.
bool mapHandle(const DriverApi* api, CUmemGenericAllocationHandle h, size_t bytes,
               size_t align, int device, CUdeviceptr* va, bool* reserved,
               bool* mapped) {
  if (!cuOk(api->cuMemAddressReserve(va, bytes, align, 0, 0), "cuMemAddressReserve"))
    return false;
  *reserved = true;
  if (!cuOk(api->cuMemMap(*va, bytes, 0, h, 0), "cuMemMap")) return false;
  *mapped = true;
  CUmemAccessDesc acc{};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = device;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  return cuOk(api->cuMemSetAccess(*va, bytes, &acc, 1), "cuMemSetAccess");
}

tncclResult allocLocalMailbox(tncclComm* comm, size_t bytes, bool tryCuMem) {
  LocalMailbox& m = comm->local;
  const DriverApi* api = tryCuMem ? driverApi() : nullptr;
  int fdSupported = 0;
  if (api) {
    api->cuDeviceGetAttribute(&fdSupported,
                              CU_DEVICE_ATTRIBUTE_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR_SUPPORTED,
                              comm->cuDevice);
  }
  if (api && fdSupported) {
    CUmemAllocationProp prop = deviceProp(comm->device, true);
    size_t gran = 0;
    bool ok = cuOk(api->cuMemGetAllocationGranularity(&gran, &prop,
                                                      CU_MEM_ALLOC_GRANULARITY_MINIMUM),
                   "cuMemGetAllocationGranularity");
    if (ok) {
      m.bytes = (bytes + gran - 1) / gran * gran;
      ok = cuOk(api->cuMemCreate(&m.handle, m.bytes, &prop, 0), "cuMemCreate");
      m.created = ok;
    }
    CUdeviceptr va = 0;
    if (ok) ok = mapHandle(api, m.handle, m.bytes, gran, comm->device, &va,
                           &m.reserved, &m.mapped);
    if (ok) {
      m.base = reinterpret_cast<char*>(va);
      int fd = -1;
      ok = cuOk(api->cuMemExportToShareableHandle(&fd, m.handle,
                                                  CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0),
                "cuMemExportToShareableHandle");
      m.exportFd = ok ? fd : -1;
    }
    if (ok) {
      comm->ipcMode = kIpcCuMem;
      TN_INFO("rank %d: cuMem mailbox %zu bytes at %p", comm->rank, m.bytes, m.base);
      return TNCCL_SUCCESS;
    }
    tncclResult ignored = TNCCL_SUCCESS;
    freeLocalMailbox(comm, &ignored);
    TN_WARN("rank %d: cuMem export unavailable, using legacy CUDA IPC", comm->rank);
  }
  // Legacy CUDA IPC.
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return TNCCL_CUDA_ERROR;
  m.base = static_cast<char*>(p);
  m.bytes = bytes;
  m.legacyAlloc = true;
  if (cudaIpcGetMemHandle(&m.ipcHandle, p) != cudaSuccess) {
    tncclResult ignored = TNCCL_SUCCESS;
    freeLocalMailbox(comm, &ignored);
    return TNCCL_CUDA_ERROR;
  }
  comm->ipcMode = kIpcLegacy;
  return TNCCL_SUCCESS;
}

tncclResult importPeerMailbox(tncclComm* comm, int peer, int fd,
                              const PeerMeta& meta) {
  PeerMailbox& pm = comm->peers[peer];
  if (comm->ipcMode == kIpcLegacy) {
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, meta.ipcHandle, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      TN_WARN("rank %d: cudaIpcOpenMemHandle(peer %d): %s", comm->rank, peer,
              cudaGetErrorString(e));
      return TNCCL_CUDA_ERROR;
    }
    pm.base = static_cast<char*>(p);
    pm.bytes = meta.mailboxBytes;
    pm.legacyOpened = true;
    return TNCCL_SUCCESS;
  }
  const DriverApi* api = driverApi();
  if (api == nullptr || fd < 0) return TNCCL_SYSTEM_ERROR;
  CUmemAllocationProp prop = deviceProp(comm->device, true);
  size_t gran = 0;
  if (!cuOk(api->cuMemGetAllocationGranularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_MINIMUM),
            "cuMemGetAllocationGranularity"))
    return TNCCL_CUDA_ERROR;
  if (!cuOk(api->cuMemImportFromShareableHandle(&pm.handle, (void*)(uintptr_t)fd,
                                                CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
            "cuMemImportFromShareableHandle"))
    return TNCCL_CUDA_ERROR;
  pm.imported = true;
  pm.bytes = meta.mailboxBytes;
  CUdeviceptr va = 0;
  if (!mapHandle(api, pm.handle, pm.bytes, gran, comm->device, &va, &pm.reserved,
                 &pm.mapped)) {
    return TNCCL_CUDA_ERROR;
  }
  pm.base = reinterpret_cast<char*>(va);
  return TNCCL_SUCCESS;
}

void closePeerMailboxes(tncclComm* comm, tncclResult* result) {
  const DriverApi* api = driverApi();
  for (int r = 0; r < kMaxRanks; ++r) {
    PeerMailbox& pm = comm->peers[r];
    if (pm.legacyOpened) {
      if (cudaIpcCloseMemHandle(pm.base) != cudaSuccess && *result == TNCCL_SUCCESS)
        *result = TNCCL_CUDA_ERROR;
    }
    if (api) {
      CUdeviceptr va = reinterpret_cast<CUdeviceptr>(pm.base);
      if (pm.mapped && api->cuMemUnmap(va, pm.bytes) != CUDA_SUCCESS &&
          *result == TNCCL_SUCCESS)
        *result = TNCCL_CUDA_ERROR;
      if (pm.reserved && va) api->cuMemAddressFree(va, pm.bytes);
      if (pm.imported) api->cuMemRelease(pm.handle);
    }
    pm = PeerMailbox{};
  }
  for (int r = 0; r < kMaxRanks; ++r) comm->dev.peers[r] = nullptr;
}

void freeLocalMailbox(tncclComm* comm, tncclResult* result) {
  LocalMailbox& m = comm->local;
  if (m.exportFd >= 0) close(m.exportFd);
  m.exportFd = -1;
  if (m.legacyAlloc) {
    if (cudaFree(m.base) != cudaSuccess && *result == TNCCL_SUCCESS) *result = TNCCL_CUDA_ERROR;
  } else {
    const DriverApi* api = driverApi();
    if (api) {
      CUdeviceptr va = reinterpret_cast<CUdeviceptr>(m.base);
      if (m.mapped && api->cuMemUnmap(va, m.bytes) != CUDA_SUCCESS && *result == TNCCL_SUCCESS)
        *result = TNCCL_CUDA_ERROR;
      if (m.reserved && va) api->cuMemAddressFree(va, m.bytes);
      if (m.created) api->cuMemRelease(m.handle);
    }
  }
  m = LocalMailbox{};
}

bool nvlsLocallyCapable(const tncclComm* comm) {
  if (!comm->cfg.nvlsEnable || comm->ipcMode != kIpcCuMem || comm->nranks < 2) return false;
  const DriverApi* api = driverApi();
  if (api == nullptr || !api->cuMulticastCreate || !api->cuMulticastAddDevice ||
      !api->cuMulticastBindMem || !api->cuMulticastUnbind || !api->cuMulticastGetGranularity)
    return false;
  int mc = 0;
  if (api->cuDeviceGetAttribute(&mc, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED,
                                comm->cuDevice) != CUDA_SUCCESS)
    return false;
  return mc != 0;
}

// Collective: every rank calls it when every rank reported NVLS capability.
// Any failure disables NVLS on all ranks (statuses are all-gathered after
// each stage), so ranks never disagree on whether the path exists.
tncclResult setupNvls(tncclComm* comm) {
  const DriverApi* api = driverApi();
  NvlsState& n = comm->nvls;
  n.channels = comm->cfg.nvlsChannels;
  n.tileBytes = (uint64_t)comm->cfg.nvlsTileBytes;
  const size_t want = (size_t)nvlsRegionBytes(n.tileBytes, n.channels);
  std::vector<int32_t> statuses((size_t)comm->nranks);

  auto agree = [&](int32_t mine) -> tncclResult {
    tncclResult r = bootstrapAllGather(&comm->bootstrap, &mine, statuses.data(), sizeof(mine));
    if (r != TNCCL_SUCCESS) return r;
    for (int32_t s : statuses)
      if (s != TNCCL_SUCCESS) return TNCCL_UNSUPPORTED;
    return TNCCL_SUCCESS;
  };

  CUmulticastObjectProp mprop{};
  mprop.numDevices = (unsigned)comm->nranks;
  mprop.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  mprop.size = want;
  size_t mgran = 0;
  int32_t st = cuOk(api->cuMulticastGetGranularity(&mgran, &mprop, CU_MULTICAST_GRANULARITY_MINIMUM),
                    "cuMulticastGetGranularity")
                   ? TNCCL_SUCCESS
                   : TNCCL_UNSUPPORTED;
  CUmemAllocationProp uprop = deviceProp(comm->device, true);
  size_t ugran = 0;
  if (st == TNCCL_SUCCESS &&
      !cuOk(api->cuMemGetAllocationGranularity(&ugran, &uprop, CU_MEM_ALLOC_GRANULARITY_MINIMUM),
            "cuMemGetAllocationGranularity"))
    st = TNCCL_UNSUPPORTED;
  size_t gran = mgran > ugran ? mgran : ugran;
  if (gran == 0) gran = 2u << 20;
  n.bytes = (want + gran - 1) / gran * gran;
  mprop.size = n.bytes;
  // Every rank must agree on the size; the granularities are per device but
  // equal on a homogeneous node. Gather the size and insist on equality.
  std::vector<uint64_t> sizes((size_t)comm->nranks);
  uint64_t mine = n.bytes;
  tncclResult r = bootstrapAllGather(&comm->bootstrap, &mine, sizes.data(), sizeof(mine));
  if (r != TNCCL_SUCCESS) return r;
  for (uint64_t s : sizes)
    if (s != mine) st = TNCCL_UNSUPPORTED;

  // Stage 1: rank 0 creates the multicast object and shares it.
  int fd = -1;
  if (comm->rank == 0 && st == TNCCL_SUCCESS) {
    if (cuOk(api->cuMulticastCreate(&n.mc, &mprop), "cuMulticastCreate")) {
      n.mcValid = true;
      if (!cuOk(api->cuMemExportToShareableHandle(&fd, n.mc,
                                                  CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0),
                "cuMemExportToShareableHandle(multicast)"))
        fd = -1;
    }
  }
  if ((r = agree(st)) != TNCCL_SUCCESS) {
    if (fd >= 0) close(fd);
    nvlsRelease(comm, &r);
    return r == TNCCL_UNSUPPORTED ? TNCCL_UNSUPPORTED : r;
  }
  int got = -1;
  r = bootstrapBroadcastFd(&comm->bootstrap, comm->rank == 0 ? fd : -1, &got);
  if (fd >= 0) close(fd);
  if (r != TNCCL_SUCCESS) {
    if (got >= 0) close(got);
    tncclResult ignored = TNCCL_SUCCESS;
    nvlsRelease(comm, &ignored);
    return r;
  }
  st = TNCCL_SUCCESS;
  if (comm->rank != 0) {
    if (cuOk(api->cuMemImportFromShareableHandle(&n.mc, (void*)(uintptr_t)got,
                                                 CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
             "cuMemImportFromShareableHandle(multicast)"))
      n.mcValid = true;
    else
      st = TNCCL_UNSUPPORTED;
  }
  if (got >= 0) close(got);
  // Stage 2: every rank adds its device.
  if (st == TNCCL_SUCCESS) {
    if (cuOk(api->cuMulticastAddDevice(n.mc, comm->cuDevice), "cuMulticastAddDevice"))
      n.deviceAdded = true;
    else
      st = TNCCL_UNSUPPORTED;
  }
  if ((r = agree(st)) != TNCCL_SUCCESS) {
    tncclResult ignored = TNCCL_SUCCESS;
    nvlsRelease(comm, &ignored);
    return r;
  }
  // Stage 3: allocate, bind and map (after all devices were added).
  st = TNCCL_SUCCESS;
  if (cuOk(api->cuMemCreate(&n.uc, n.bytes, &uprop, 0), "cuMemCreate(nvls)")) {
    n.ucCreated = true;
    if (cuOk(api->cuMulticastBindMem(n.mc, 0, n.uc, 0, n.bytes, 0), "cuMulticastBindMem")) {
      n.bound = true;
    } else {
      st = TNCCL_UNSUPPORTED;
    }
  } else {
    st = TNCCL_UNSUPPORTED;
  }
  if (st == TNCCL_SUCCESS &&
      !mapHandle(api, n.uc, n.bytes, gran, comm->device, &n.ucVa, &n.ucReserved, &n.ucMapped))
    st = TNCCL_UNSUPPORTED;
  if (st == TNCCL_SUCCESS &&
      !mapHandle(api, n.mc, n.bytes, gran, comm->device, &n.mcVa, &n.mcReserved, &n.mcMapped))
    st = TNCCL_UNSUPPORTED;
  // Zero the region (its barrier counters start at 0) and wait for it: no
  // rank may add to a counter before every rank finished zeroing its copy.
  if (st == TNCCL_SUCCESS &&
      (cudaMemset(reinterpret_cast<void*>(n.ucVa), 0, n.bytes) != cudaSuccess ||
       cudaDeviceSynchronize() != cudaSuccess))
    st = TNCCL_UNSUPPORTED;
  if ((r = agree(st)) != TNCCL_SUCCESS) {
    // Nobody has used the object yet; unmap and unbind in step on all ranks.
    tncclResult ignored = TNCCL_SUCCESS;
    nvlsUnmap(comm, &ignored);
    tncclResult b = bootstrapBarrier(&comm->bootstrap);
    nvlsRelease(comm, &ignored);
    return b != TNCCL_SUCCESS ? b : r;
  }
  n.enabled = true;
  TN_INFO("rank %d: NVLS enabled, %zu bytes, %d channels x %llu-byte tiles", comm->rank,
          n.bytes, n.channels, (unsigned long long)n.tileBytes);
  return TNCCL_SUCCESS;
}

// Unmaps both views and unbinds this device's memory. Peers must have
// stopped using the object (destroy calls it after barrier #1).
void nvlsUnmap(tncclComm* comm, tncclResult* result) {
  const DriverApi* api = driverApi();
  NvlsState& n = comm->nvls;
  if (api == nullptr) return;
  if (n.mcMapped && api->cuMemUnmap(n.mcVa, n.bytes) != CUDA_SUCCESS && *result == TNCCL_SUCCESS)
    *result = TNCCL_CUDA_ERROR;
  n.mcMapped = false;
  if (n.mcReserved) api->cuMemAddressFree(n.mcVa, n.bytes);
  n.mcReserved = false;
  if (n.ucMapped && api->cuMemUnmap(n.ucVa, n.bytes) != CUDA_SUCCESS && *result == TNCCL_SUCCESS)
    *result = TNCCL_CUDA_ERROR;
  n.ucMapped = false;
  if (n.ucReserved) api->cuMemAddressFree(n.ucVa, n.bytes);
  n.ucReserved = false;
  if (n.bound &&
      api->cuMulticastUnbind(n.mc, comm->cuDevice, 0, n.bytes) != CUDA_SUCCESS &&
      *result == TNCCL_SUCCESS)
    *result = TNCCL_CUDA_ERROR;
  n.bound = false;
  n.enabled = false;
}

void nvlsRelease(tncclComm* comm, tncclResult* result) {
  const DriverApi* api = driverApi();
  NvlsState& n = comm->nvls;
  if (api == nullptr) return;
  nvlsUnmap(comm, result);
  if (n.ucCreated) api->cuMemRelease(n.uc);
  n.ucCreated = false;
  if (n.mcValid) api->cuMemRelease(n.mc);
  n.mcValid = false;
  n.deviceAdded = false;
}

}  // namespace tnccl
