// register.cc - memory that the NVSwitch can reduce in place: tncclMemAlloc /
// tncclMemFree and the collective tncclCommRegister / tncclCommDeregister.
//
// The staged NVLS kernel copies every tile into the communicator's own
// multicast-bound region and the result back out. A buffer allocated with
// tncclMemAlloc is a cuMem (VMM) allocation, which, unlike cudaMalloc memory,
// can be bound to a multicast object. Registering it binds it, on every rank,
// to a multicast object of its own; an NVLS all-reduce whose send and recv
// both lie in registered buffers then reduces straight from the senders'
// memory and stores straight into every receiver's (nvlsZeroCopyKernel).
// tiny-nccl has no counterpart (its data always goes through the mailbox
// FIFOs, src/device.cuh:164-238).
//
// Registration follows the staged set-up of the communicator's own NVLS
// region (transport.cc setupNvls): statuses are all-gathered after every
// stage, so a failure anywhere leaves every rank unregistered. Deregistration
// and destroy follow tiny-nccl's two-phase teardown (src/comm.cc:218-290):
// barrier once every kernel of every rank is done, unbind, barrier, release.
#include <string.h>
#include <unistd.h>

#include <mutex>
#include <vector>

#include "comm.h"
#include "driver.h"

namespace tnccl {
namespace {

// One tncclMemAlloc allocation.
struct MemAllocation {
  char* va = nullptr;
  size_t bytes = 0;  // mapped (granularity-rounded)
  size_t gran = 0;   // alignment of its VA range and of binding offsets
  int device = -1;
  CUmemGenericAllocationHandle handle = 0;
  int registrations = 0;  // live bindings to multicast objects
};

std::mutex gMemMu;
std::vector<MemAllocation> gMem;

// Index of the allocation holding [p, p + bytes), or -1. Caller holds gMemMu.
int findAllocation(const void* p, size_t bytes) {
  const char* c = static_cast<const char*>(p);
  for (size_t i = 0; i < gMem.size(); ++i) {
    const MemAllocation& m = gMem[i];
    if (c >= m.va && c < m.va + m.bytes && bytes <= (size_t)(m.va + m.bytes - c)) return (int)i;
  }
  return -1;
}

bool multicastApi(const DriverApi* api) {
  return api != nullptr && api->cuMulticastCreate && api->cuMulticastAddDevice &&
         api->cuMulticastBindMem && api->cuMulticastUnbind && api->cuMulticastGetGranularity;
}

// Minimum (or, with recommended, the driver's recommended) multicast
// granularity for `numDevices` devices (0 if unknown).
size_t multicastGranularity(const DriverApi* api, unsigned numDevices, size_t bytes,
                            bool recommended = false) {
  if (!multicastApi(api)) return 0;
  CUmulticastObjectProp mp{};
  mp.numDevices = numDevices;
  mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  mp.size = bytes;
  size_t g = 0;
  if (api->cuMulticastGetGranularity(&g, &mp,
                                     recommended ? CU_MULTICAST_GRANULARITY_RECOMMENDED
                                                 : CU_MULTICAST_GRANULARITY_MINIMUM) !=
      CUDA_SUCCESS)
    return 0;
  return g;
}

void unbindOne(tncclComm* comm, Registration& g, tncclResult* result) {
  const DriverApi* api = driverApi();
  if (api == nullptr) return;
  if (g.mapped && api->cuMemUnmap(g.mcVa, g.bytes) != CUDA_SUCCESS && *result == TNCCL_SUCCESS)
    *result = TNCCL_CUDA_ERROR;
  g.mapped = false;
  if (g.reserved) api->cuMemAddressFree(g.mcVa, g.bytes);
  g.reserved = false;
  if (g.bound) {
    if (api->cuMulticastUnbind(g.mc, comm->cuDevice, 0, g.bytes) != CUDA_SUCCESS &&
        *result == TNCCL_SUCCESS)
      *result = TNCCL_CUDA_ERROR;
    std::lock_guard<std::mutex> lock(gMemMu);
    const int i = findAllocation(g.allocation, 1);
    if (i >= 0 && gMem[(size_t)i].registrations > 0) --gMem[(size_t)i].registrations;
  }
  g.bound = false;
}

void releaseOne(Registration& g) {
  const DriverApi* api = driverApi();
  if (api != nullptr && g.mcValid) api->cuMemRelease(g.mc);
  g = Registration{};
}

}  // namespace

const Registration* findRegistration(const tncclComm* comm, const void* p, size_t bytes) {
  const char* c = static_cast<const char*>(p);
  for (const Registration& g : comm->regs) {
    if (!g.used || !g.bound || !g.mapped) continue;
    if (c >= g.base && c < g.base + g.userBytes && bytes <= (size_t)(g.base + g.userBytes - c))
      return &g;
  }
  return nullptr;
}

void registrationsUnmap(tncclComm* comm, tncclResult* result) {
  for (Registration& g : comm->regs)
    if (g.used) unbindOne(comm, g, result);
}

void registrationsRelease(tncclComm* comm, tncclResult* result) {
  for (Registration& g : comm->regs) {
    if (!g.used) continue;
    unbindOne(comm, g, result);
    releaseOne(g);
  }
}

}  // namespace tnccl

using namespace tnccl;

extern "C" tncclResult tncclMemAlloc(void** ptr, size_t size) {
  if (ptr == nullptr || size == 0) return TNCCL_INVALID_ARGUMENT;
  *ptr = nullptr;
  const DriverApi* api = driverApi();
  if (api == nullptr) return TNCCL_UNSUPPORTED;
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess) return TNCCL_CUDA_ERROR;
  CUmemAllocationProp prop = deviceProp(device, true);
  size_t gran = 0;
  if (!cuOk(api->cuMemGetAllocationGranularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_MINIMUM),
            "cuMemGetAllocationGranularity") ||
      gran == 0)
    return TNCCL_CUDA_ERROR;
  // Binding offsets into the allocation are multiples of the multicast
  // granularity, so the VA range and the size are aligned to it as well.
  const size_t mgran = multicastGranularity(api, 1, size);
  if (mgran > gran) gran = (mgran + gran - 1) / gran * gran;
  if (size > SIZE_MAX - gran) return TNCCL_INVALID_ARGUMENT;
  MemAllocation m;
  m.bytes = (size + gran - 1) / gran * gran;
  m.gran = gran;
  m.device = device;
  if (!cuOk(api->cuMemCreate(&m.handle, m.bytes, &prop, 0), "cuMemCreate(tncclMemAlloc)"))
    return TNCCL_CUDA_ERROR;
  CUdeviceptr va = 0;
  bool reserved = false, mapped = false;
  if (!mapHandle(api, m.handle, m.bytes, gran, device, &va, &reserved, &mapped)) {
    if (mapped) api->cuMemUnmap(va, m.bytes);
    if (reserved) api->cuMemAddressFree(va, m.bytes);
    api->cuMemRelease(m.handle);
    return TNCCL_CUDA_ERROR;
  }
  m.va = reinterpret_cast<char*>(va);
  {
    std::lock_guard<std::mutex> lock(gMemMu);
    gMem.push_back(m);
  }
  *ptr = m.va;
  return TNCCL_SUCCESS;
}

extern "C" tncclResult tncclMemFree(void* ptr) {
  if (ptr == nullptr) return TNCCL_SUCCESS;
  MemAllocation m;
  {
    std::lock_guard<std::mutex> lock(gMemMu);
    size_t i = 0;
    while (i < gMem.size() && gMem[i].va != ptr) ++i;
    if (i == gMem.size()) return TNCCL_INVALID_ARGUMENT;  // not a tncclMemAlloc base
    if (gMem[i].registrations > 0) return TNCCL_INVALID_ARGUMENT;  // deregister first
    m = gMem[i];
    gMem.erase(gMem.begin() + (long)i);
  }
  const DriverApi* api = driverApi();
  if (api == nullptr) return TNCCL_SYSTEM_ERROR;
  // Like cudaFree: work queued on the device may still use the memory.
  int original = -1;
  if (cudaGetDevice(&original) != cudaSuccess) original = -1;
  if (original != m.device) cudaSetDevice(m.device);
  tncclResult r = cudaDeviceSynchronize() == cudaSuccess ? TNCCL_SUCCESS : TNCCL_CUDA_ERROR;
  const CUdeviceptr va = reinterpret_cast<CUdeviceptr>(m.va);
  if (api->cuMemUnmap(va, m.bytes) != CUDA_SUCCESS) r = TNCCL_CUDA_ERROR;
  api->cuMemAddressFree(va, m.bytes);
  api->cuMemRelease(m.handle);
  if (original >= 0 && original != m.device) cudaSetDevice(original);
  return r;
}

// Collective over the communicator: every rank calls it in the same order
// with a buffer of the same size. Bad arguments on one rank still take part
// in every status round, so no rank waits for a stage that others skipped.
extern "C" tncclResult tncclCommRegister(tncclComm_t comm, void* buff, size_t size,
                                         void** handle) {
  if (comm == nullptr) return TNCCL_INVALID_ARGUMENT;
  if (!comm->nvls.enabled) return TNCCL_UNSUPPORTED;  // agreed on every rank at init
  if (handle != nullptr) *handle = nullptr;
  const DriverApi* api = driverApi();
  int32_t st = TNCCL_SUCCESS;
  int device = -1;
  if (handle == nullptr || buff == nullptr || size == 0) st = TNCCL_INVALID_ARGUMENT;
  if (st == TNCCL_SUCCESS && (cudaGetDevice(&device) != cudaSuccess || device != comm->device))
    st = TNCCL_INVALID_ARGUMENT;
  if (st == TNCCL_SUCCESS && comm->aborted) st = TNCCL_ABORTED;
  // Where the buffer lies: a tncclMemAlloc allocation, at an offset that
  // the multicast binding accepts, with room for the rounded size.
  size_t offset = 0, bytes = 0;
  void* allocation = nullptr;
  CUmemGenericAllocationHandle memHandle = 0;
  size_t gran = 0;
  if (st == TNCCL_SUCCESS) {
    std::lock_guard<std::mutex> lock(gMemMu);
    const int i = findAllocation(buff, size);
    if (i < 0) {
      st = TNCCL_INVALID_ARGUMENT;
    } else {
      const MemAllocation& m = gMem[(size_t)i];
      offset = (size_t)(static_cast<char*>(buff) - m.va);
      gran = m.gran;
      const size_t mg = multicastGranularity(api, (unsigned)comm->nranks, size);
      if (mg > gran) gran = (mg + gran - 1) / gran * gran;
      bytes = (size + gran - 1) / gran * gran;
      allocation = m.va;
      memHandle = m.handle;
      if (m.device != comm->device || offset % gran != 0 || bytes > m.bytes - offset)
        st = TNCCL_INVALID_ARGUMENT;
    }
  }
  int slot = -1;
  for (int k = 0; k < kMaxRegistrations && slot < 0; ++k)
    if (!comm->regs[k].used) slot = k;
  if (st == TNCCL_SUCCESS && slot < 0) st = TNCCL_SYSTEM_ERROR;

  // First status exchange: statuses and bound sizes must agree.
  struct Status {
    int32_t st;
    int32_t pad;
    uint64_t bytes;
  };
  std::vector<Status> all((size_t)comm->nranks);
  auto agree = [&](int32_t mine, uint64_t b, tncclResult* out) -> bool {
    Status s{mine, 0, b};
    tncclResult r = bootstrapAllGather(&comm->bootstrap, &s, all.data(), sizeof(s));
    if (r != TNCCL_SUCCESS) {
      *out = r;
      return false;
    }
    for (const Status& o : all)
      if (o.st != TNCCL_SUCCESS) {
        *out = mine != TNCCL_SUCCESS ? (tncclResult)mine : (tncclResult)o.st;
        return false;
      }
    for (const Status& o : all)
      if (o.bytes != b) {
        *out = TNCCL_INVALID_ARGUMENT;  // buffers of different sizes
        return false;
      }
    return true;
  };
  tncclResult r = TNCCL_SUCCESS;
  if (!agree(st, bytes, &r)) return r;

  Registration& g = comm->regs[slot];
  g = Registration{};
  g.used = true;
  g.base = static_cast<char*>(buff);
  g.userBytes = size;
  g.bytes = bytes;
  g.allocation = allocation;
  auto fail = [&](tncclResult why) {
    tncclResult ignored = TNCCL_SUCCESS;
    unbindOne(comm, g, &ignored);
    releaseOne(g);
    return why;
  };

  // Stage 1: rank 0 creates the multicast object and passes it on.
  CUmulticastObjectProp mp{};
  mp.numDevices = (unsigned)comm->nranks;
  mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  mp.size = bytes;
  st = TNCCL_SUCCESS;
  int fd = -1;
  if (comm->rank == 0) {
    if (cuOk(api->cuMulticastCreate(&g.mc, &mp), "cuMulticastCreate(register)")) {
      g.mcValid = true;
      if (!cuOk(api->cuMemExportToShareableHandle(&fd, g.mc,
                                                  CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0),
                "cuMemExportToShareableHandle(register)"))
        fd = -1;
    }
    if (fd < 0) st = TNCCL_CUDA_ERROR;
  }
  if (!agree(st, bytes, &r)) {
    if (fd >= 0) close(fd);
    return fail(r);
  }
  int got = -1;
  r = bootstrapBroadcastFd(&comm->bootstrap, comm->rank == 0 ? fd : -1, &got);
  if (fd >= 0) close(fd);
  if (r != TNCCL_SUCCESS) {
    if (got >= 0) close(got);
    return fail(r);
  }
  if (comm->rank != 0) {
    if (cuOk(api->cuMemImportFromShareableHandle(&g.mc, (void*)(uintptr_t)got,
                                                 CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
             "cuMemImportFromShareableHandle(register)"))
      g.mcValid = true;
    else
      st = TNCCL_CUDA_ERROR;
  }
  if (got >= 0) close(got);
  // Stage 2: every rank adds its device (before any rank binds memory).
  if (st == TNCCL_SUCCESS) {
    if (cuOk(api->cuMulticastAddDevice(g.mc, comm->cuDevice), "cuMulticastAddDevice(register)"))
      g.deviceAdded = true;
    else
      st = TNCCL_CUDA_ERROR;
  }
  if (!agree(st, bytes, &r)) return fail(r);
  // Stage 3: bind this rank's buffer and map the multicast view.
  if (cuOk(api->cuMulticastBindMem(g.mc, 0, memHandle, offset, bytes, 0),
           "cuMulticastBindMem(register)")) {
    g.bound = true;
    std::lock_guard<std::mutex> lock(gMemMu);
    const int i = findAllocation(allocation, 1);
    if (i >= 0) ++gMem[(size_t)i].registrations;
  } else {
    st = TNCCL_CUDA_ERROR;
  }
  if (st == TNCCL_SUCCESS &&
      !mapHandle(api, g.mc, bytes, gran, comm->device, &g.mcVa, &g.reserved, &g.mapped))
    st = TNCCL_CUDA_ERROR;
  if (!agree(st, bytes, &r)) {
    // Nobody has used the object: unbind on every rank before any releases.
    tncclResult ignored = TNCCL_SUCCESS;
    unbindOne(comm, g, &ignored);
    tncclResult b = bootstrapBarrier(&comm->bootstrap);
    fail(r);
    return b != TNCCL_SUCCESS ? b : r;
  }
  *handle = &g;
  TN_INFO("rank %d: registered %zu bytes at %p for zero-copy NVLS (%zu bound; multicast "
          "granularity %zu, recommended %zu)", comm->rank, size, buff, bytes, gran,
          multicastGranularity(api, (unsigned)comm->nranks, size, true));
  return TNCCL_SUCCESS;
}

// Collective: waits for the bound stream, then a barrier (no rank's kernel
// can still reach the object), unbinds, a second barrier, releases.
extern "C" tncclResult tncclCommDeregister(tncclComm_t comm, void* handle) {
  if (comm == nullptr) return TNCCL_INVALID_ARGUMENT;
  if (!comm->nvls.enabled) return TNCCL_UNSUPPORTED;
  Registration* g = nullptr;
  for (Registration& k : comm->regs)
    if (&k == handle && k.used) g = &k;
  tncclResult r = g != nullptr ? TNCCL_SUCCESS : TNCCL_INVALID_ARGUMENT;
  int original = -1;
  if (cudaGetDevice(&original) != cudaSuccess) original = -1;
  if (original != comm->device) cudaSetDevice(comm->device);
  if (comm->streamBound && cudaStreamSynchronize(comm->boundStream) != cudaSuccess &&
      r == TNCCL_SUCCESS)
    r = TNCCL_CUDA_ERROR;
  // A rank whose stream failed keeps its binding: a kernel may still run.
  const bool idle = r == TNCCL_SUCCESS;
  tncclResult b1 = bootstrapBarrier(&comm->bootstrap);
  if (idle && b1 == TNCCL_SUCCESS) unbindOne(comm, *g, &r);
  tncclResult b2 = bootstrapBarrier(&comm->bootstrap);
  if (idle && b1 == TNCCL_SUCCESS && b2 == TNCCL_SUCCESS) releaseOne(*g);
  if (original >= 0 && original != comm->device) cudaSetDevice(original);
  if (b1 != TNCCL_SUCCESS) return b1;
  if (b2 != TNCCL_SUCCESS) return b2;
  return r;
}
