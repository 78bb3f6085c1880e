// register_test.cc - CPU test of the registered-buffer control plane
// (csrc/tnccl/register.cc) with forked ranks over the real AF_UNIX
// bootstrap and a fake CUDA driver: tncclMemAlloc / tncclMemFree, the
// collective tncclCommRegister (all-gathered statuses after every stage) and
// tncclCommDeregister / the destroy halves. The fake driver counts live
// handles, mappings and bindings per process, so every path must leave them
// balanced; failures are injected on one rank at each stage and every rank
// must fail the registration, in step, without waiting for a deadline.
//
// The same binary checks the enqueue side (csrc/tnccl/enqueue.cc): which
// all-reduces take the zero-copy NVLS kernel and the multicast addresses,
// vector count and channel count they launch with, through a launcher that
// records its arguments.
//
// Built from sources without the CUDA runtime: this file provides the few
// runtime calls register.cc and enqueue.cc make, the transport helpers and
// the kernel launchers.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/wait.h>
#include <unistd.h>

#include <chrono>
#include <functional>
#include <map>
#include <set>
#include <vector>

#include "comm.h"
#include "driver.h"
#include "launch.h"

using namespace tnccl;

// ---------------------------------------------------------------------------
// Fake CUDA runtime (only what register.cc calls).
// ---------------------------------------------------------------------------
extern "C" {
cudaError_t cudaGetDevice(int* d) {
  *d = 0;
  return cudaSuccess;
}
cudaError_t cudaSetDevice(int) { return cudaSuccess; }
cudaError_t cudaStreamSynchronize(cudaStream_t) { return cudaSuccess; }
cudaError_t cudaDeviceSynchronize() { return cudaSuccess; }
cudaError_t cudaGetLastError() { return cudaSuccess; }
cudaError_t cudaMemcpyAsync(void*, const void*, size_t, cudaMemcpyKind, cudaStream_t) {
  return cudaSuccess;
}
const char* tncclAlgoName(tncclAlgo_t) { return "fake"; }
}

// Kernel launchers: record the last all-reduce launch.
namespace {
struct Launch {
  int count = 0;
  int algo = -1;
  AllReduceArgs args{};
} gLast;
}  // namespace
namespace tnccl {
cudaError_t launchAllReduceKernel(const DevComm&, const AllReduceArgs& a, int algo, int,
                                  cudaStream_t) {
  ++gLast.count;
  gLast.algo = algo;
  gLast.args = a;
  return cudaSuccess;
}
cudaError_t launchScale(const void*, void*, uint64_t, int, float, int, cudaStream_t) {
  return cudaSuccess;
}
}  // namespace tnccl

namespace {

// Failure injection: the stage that fails, on which rank (-1: none).
enum Stage { kNone, kCreate, kImport, kAddDevice, kBind, kMap };
Stage gFailStage = kNone;
int gFailRank = -1;
int gRank = 0;
bool failHere(Stage s) { return gFailStage == s && gFailRank == gRank; }

uint64_t gNextHandle = 100;
std::set<uint64_t> gHandles;                     // live allocation / multicast handles
std::set<uint64_t> gMcHandles;                   // the multicast ones among them
std::set<uint64_t> gMapped;                      // live VA mappings
std::set<uint64_t> gReserved;                    // live VA reservations
std::map<uint64_t, int> gBindings;               // multicast handle -> bound ranges
uint64_t gNextVa = 0x7f0000000000ull;
constexpr size_t kGran = 2u << 20;

CUresult fGran(size_t* g, const CUmemAllocationProp*, CUmemAllocationGranularity_flags) {
  *g = kGran;
  return CUDA_SUCCESS;
}
CUresult fMcGran(size_t* g, const CUmulticastObjectProp*, CUmulticastGranularity_flags) {
  *g = kGran;
  return CUDA_SUCCESS;
}
CUresult fCreate(CUmemGenericAllocationHandle* h, size_t, const CUmemAllocationProp*,
                 unsigned long long) {
  *h = gNextHandle++;
  gHandles.insert(*h);
  return CUDA_SUCCESS;
}
CUresult fRelease(CUmemGenericAllocationHandle h) {
  return gHandles.erase(h) ? CUDA_SUCCESS : CUDA_ERROR_INVALID_VALUE;
}
CUresult fMcCreate(CUmemGenericAllocationHandle* h, const CUmulticastObjectProp* p) {
  if (failHere(kCreate) || p->size % kGran != 0) return CUDA_ERROR_OUT_OF_MEMORY;
  *h = gNextHandle++;
  gHandles.insert(*h);
  gMcHandles.insert(*h);
  return CUDA_SUCCESS;
}
CUresult fExport(void* out, CUmemGenericAllocationHandle h, CUmemAllocationHandleType,
                 unsigned long long) {
  if (!gHandles.count(h)) return CUDA_ERROR_INVALID_VALUE;
  int fd = memfd_create("fake-mc", MFD_CLOEXEC);
  *static_cast<int*>(out) = fd;
  return fd >= 0 ? CUDA_SUCCESS : CUDA_ERROR_OPERATING_SYSTEM;
}
CUresult fImport(CUmemGenericAllocationHandle* h, void* fd, CUmemAllocationHandleType) {
  if (failHere(kImport) || (int)(uintptr_t)fd < 0) return CUDA_ERROR_INVALID_VALUE;
  *h = gNextHandle++;
  gHandles.insert(*h);
  gMcHandles.insert(*h);
  return CUDA_SUCCESS;
}
CUresult fAddDevice(CUmemGenericAllocationHandle h, CUdevice) {
  if (failHere(kAddDevice) || !gHandles.count(h)) return CUDA_ERROR_INVALID_VALUE;
  return CUDA_SUCCESS;
}
CUresult fBind(CUmemGenericAllocationHandle mc, size_t mcOff, CUmemGenericAllocationHandle mem,
               size_t memOff, size_t size, unsigned long long) {
  if (failHere(kBind) || !gHandles.count(mc) || !gHandles.count(mem) || mcOff != 0 ||
      memOff % kGran != 0 || size % kGran != 0)
    return CUDA_ERROR_INVALID_VALUE;
  ++gBindings[mc];
  return CUDA_SUCCESS;
}
CUresult fUnbind(CUmemGenericAllocationHandle mc, CUdevice, size_t, size_t) {
  auto it = gBindings.find(mc);
  if (it == gBindings.end() || it->second == 0) return CUDA_ERROR_INVALID_VALUE;
  if (--it->second == 0) gBindings.erase(it);
  return CUDA_SUCCESS;
}
CUresult fUnmap(CUdeviceptr va, size_t) {
  return gMapped.erase(va) ? CUDA_SUCCESS : CUDA_ERROR_INVALID_VALUE;
}
CUresult fAddressFree(CUdeviceptr va, size_t) {
  return gReserved.erase(va) ? CUDA_SUCCESS : CUDA_ERROR_INVALID_VALUE;
}

DriverApi makeFake() {
  DriverApi a{};
  a.loaded = true;
  a.cuMemGetAllocationGranularity = fGran;
  a.cuMulticastGetGranularity = fMcGran;
  a.cuMemCreate = fCreate;
  a.cuMemRelease = fRelease;
  a.cuMulticastCreate = fMcCreate;
  a.cuMemExportToShareableHandle = fExport;
  a.cuMemImportFromShareableHandle = fImport;
  a.cuMulticastAddDevice = fAddDevice;
  a.cuMulticastBindMem = fBind;
  a.cuMulticastUnbind = fUnbind;
  a.cuMemUnmap = fUnmap;
  a.cuMemAddressFree = fAddressFree;
  return a;
}
DriverApi gFake = makeFake();

bool balanced() {
  return gHandles.empty() && gMapped.empty() && gReserved.empty() && gBindings.empty();
}

}  // namespace

// The driver and transport entry points register.cc links against.
namespace tnccl {
const DriverApi* driverApi() { return &gFake; }
const char* cuErrorName(CUresult) { return "fake"; }
CUmemAllocationProp deviceProp(int device, bool) {
  CUmemAllocationProp p{};
  p.location.id = device;
  return p;
}
bool cuOk(CUresult r, const char*) { return r == CUDA_SUCCESS; }
bool mapHandle(const DriverApi*, CUmemGenericAllocationHandle h, size_t bytes, size_t,
               int, CUdeviceptr* va, bool* reserved, bool* mapped) {
  *va = gNextVa;
  gNextVa += bytes + kGran;
  gReserved.insert(*va);
  *reserved = true;
  if (failHere(kMap) && gMcHandles.count(h)) return false;
  gMapped.insert(*va);
  *mapped = true;
  return true;
}
}  // namespace tnccl

namespace {

int gFailed = 0;

void report(const char* name, bool ok) {
  printf("%-58s %s\n", name, ok ? "ok" : "FAILED");
  fflush(stdout);
  if (!ok) ++gFailed;
}

std::vector<int> forkRanks(int n, const std::function<int(int)>& fn) {
  std::vector<pid_t> kids;
  for (int i = 0; i < n; ++i) {
    pid_t p = fork();
    if (p == 0) {
      fflush(stdout);
      _exit(fn(i));
    }
    kids.push_back(p);
  }
  std::vector<int> codes;
  for (pid_t k : kids) {
    int st = 0;
    waitpid(k, &st, 0);
    codes.push_back(WIFEXITED(st) ? WEXITSTATUS(st) : 255);
  }
  return codes;
}

bool allZero(const std::vector<int>& codes) {
  for (int c : codes)
    if (c != 0) return false;
  return true;
}

// One rank: a communicator with NVLS "on" over a real bootstrap, then `body`.
int withComm(int r, int P, const tncclUniqueId& id, const std::function<int(tncclComm*)>& body) {
  gRank = r;
  tncclComm comm;
  comm.rank = r;
  comm.nranks = P;
  comm.device = 0;
  comm.nvls.enabled = true;
  if (bootstrapOpen(&comm.bootstrap, id, P, r, 7, 5000) != TNCCL_SUCCESS) return 90;
  const int rc = body(&comm);
  bootstrapClose(&comm.bootstrap);
  return rc;
}

void allocAndFree() {
  gRank = 0;
  void* p = nullptr;
  bool ok = tncclMemAlloc(&p, 3u << 20) == TNCCL_SUCCESS && p != nullptr;
  ok = ok && gHandles.size() == 1 && gMapped.size() == 1;
  ok = ok && tncclMemFree(static_cast<char*>(p) + 16) == TNCCL_INVALID_ARGUMENT;  // not a base
  ok = ok && tncclMemFree(p) == TNCCL_SUCCESS && balanced();
  ok = ok && tncclMemFree(p) == TNCCL_INVALID_ARGUMENT;  // twice
  report("tncclMemAlloc / tncclMemFree balance handles and mappings", ok);
}

void registerAndDeregister() {
  const int P = 3;
  tncclUniqueId id;
  bootstrapNewId(&id);
  auto codes = forkRanks(P, [&](int r) {
    return withComm(r, P, id, [&](tncclComm* comm) -> int {
      void* a = nullptr;
      void* b = nullptr;
      if (tncclMemAlloc(&a, 5u << 20) != TNCCL_SUCCESS) return 1;
      if (tncclMemAlloc(&b, 1u << 20) != TNCCL_SUCCESS) return 1;
      void* ha = nullptr;
      void* hb = nullptr;
      if (tncclCommRegister(comm, a, 5u << 20, &ha) != TNCCL_SUCCESS || ha == nullptr) return 2;
      // A sub-range at a granularity offset, and a second buffer.
      void* hs = nullptr;
      if (tncclCommRegister(comm, static_cast<char*>(a) + kGran, kGran, &hs) != TNCCL_SUCCESS)
        return 3;
      if (tncclCommRegister(comm, b, 1u << 20, &hb) != TNCCL_SUCCESS) return 4;
      // Lookups: inside, at the edges, past the end.
      const char* ca = static_cast<const char*>(a);
      if (findRegistration(comm, ca + 4096, 4096) == nullptr) return 5;
      if (findRegistration(comm, ca, 5u << 20) == nullptr) return 5;
      if (findRegistration(comm, ca + (5u << 20) - 16, 32) != nullptr) return 5;
      if (findRegistration(comm, b, (1u << 20) + 16) != nullptr) return 5;
      if (gBindings.size() != 3) return 6;
      // Registered memory cannot be freed.
      if (tncclMemFree(a) != TNCCL_INVALID_ARGUMENT) return 7;
      if (tncclCommDeregister(comm, hs) != TNCCL_SUCCESS) return 8;
      if (tncclCommDeregister(comm, hs) != TNCCL_INVALID_ARGUMENT) return 8;  // stale handle
      if (tncclCommDeregister(comm, ha) != TNCCL_SUCCESS) return 8;
      if (tncclMemFree(a) != TNCCL_SUCCESS) return 9;
      // hb is left to the destroy halves.
      tncclResult res = TNCCL_SUCCESS;
      registrationsUnmap(comm, &res);
      registrationsRelease(comm, &res);
      if (res != TNCCL_SUCCESS) return 10;
      if (tncclMemFree(b) != TNCCL_SUCCESS) return 11;
      return balanced() ? 0 : 12;
    });
  });
  report("register, look up, deregister, destroy halves (3 ranks)", allZero(codes));
}

void argumentErrors() {
  const int P = 2;
  tncclUniqueId id;
  bootstrapNewId(&id);
  auto codes = forkRanks(P, [&](int r) {
    return withComm(r, P, id, [&](tncclComm* comm) -> int {
      void* a = nullptr;
      if (tncclMemAlloc(&a, 4u << 20) != TNCCL_SUCCESS) return 1;
      void* h = nullptr;
      // Rank 1 passes memory that is not from tncclMemAlloc: both fail.
      char local[64];
      tncclResult res = tncclCommRegister(comm, r == 1 ? (void*)local : a, 4u << 20, &h);
      if (res != TNCCL_INVALID_ARGUMENT || h != nullptr) return 2;
      // Sizes that differ across ranks: both fail.
      res = tncclCommRegister(comm, a, r == 0 ? (2u << 20) : (4u << 20), &h);
      if (res != TNCCL_INVALID_ARGUMENT || h != nullptr) return 3;
      // An offset that is not a multiple of the granularity: both fail.
      res = tncclCommRegister(comm, static_cast<char*>(a) + 4096, 1u << 20, &h);
      if (res != TNCCL_INVALID_ARGUMENT) return 4;
      // After the failures the communicator still registers in step.
      if (tncclCommRegister(comm, a, 4u << 20, &h) != TNCCL_SUCCESS) return 5;
      // Rank 1 deregisters a bogus handle: it fails, rank 0 succeeds, no hang.
      res = tncclCommDeregister(comm, r == 1 ? (void*)local : h);
      if (r == 0 && res != TNCCL_SUCCESS) return 6;
      if (r == 1 && res != TNCCL_INVALID_ARGUMENT) return 6;
      tncclResult ignored = TNCCL_SUCCESS;
      registrationsRelease(comm, &ignored);
      if (tncclMemFree(a) != TNCCL_SUCCESS) return 7;
      return balanced() ? 0 : 8;
    });
  });
  report("mismatched or bad arguments fail every rank in step", allZero(codes));
  tncclComm off;
  off.nvls.enabled = false;
  void* h = nullptr;
  report("no NVLS: registration unsupported without a collective",
         tncclCommRegister(&off, &off, 64, &h) == TNCCL_UNSUPPORTED &&
             tncclCommDeregister(&off, nullptr) == TNCCL_UNSUPPORTED &&
             tncclCommRegister(nullptr, &off, 64, &h) == TNCCL_INVALID_ARGUMENT);
}

void injectedFailures() {
  const int P = 3;
  const struct {
    Stage stage;
    int rank;
    const char* name;
  } cases[] = {{kCreate, 0, "multicast create fails on rank 0"},
               {kImport, 2, "multicast import fails on rank 2"},
               {kAddDevice, 1, "add device fails on rank 1"},
               {kBind, 2, "bind fails on rank 2"},
               {kMap, 1, "map fails on rank 1"}};
  for (const auto& c : cases) {
    tncclUniqueId id;
    bootstrapNewId(&id);
    const auto t0 = std::chrono::steady_clock::now();
    auto codes = forkRanks(P, [&](int r) {
      gFailStage = c.stage;
      gFailRank = c.rank;
      return withComm(r, P, id, [&](tncclComm* comm) -> int {
        void* a = nullptr;
        if (tncclMemAlloc(&a, 2u << 20) != TNCCL_SUCCESS) return 1;
        void* h = nullptr;
        tncclResult res = tncclCommRegister(comm, a, 2u << 20, &h);
        if (res == TNCCL_SUCCESS || h != nullptr) return 2;
        for (const Registration& g : comm->regs)
          if (g.used) return 3;
        // The failure is over: the next registration succeeds everywhere.
        gFailStage = kNone;
        if (tncclCommRegister(comm, a, 2u << 20, &h) != TNCCL_SUCCESS) return 4;
        if (tncclCommDeregister(comm, h) != TNCCL_SUCCESS) return 5;
        if (tncclMemFree(a) != TNCCL_SUCCESS) return 6;
        return balanced() ? 0 : 7;
      });
    });
    const double s =
        std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    char name[96];
    snprintf(name, sizeof(name), "%s: all fail, then recover", c.name);
    report(name, allZero(codes) && s < 4.0);
  }
}

// Enqueue: registrations filled in directly (one process), launches recorded.
void zeroCopySelection() {
  setenv("TNCCL_NVLS_ZERO_COPY", "1", 1);
  tncclComm comm;
  comm.rank = 0;
  comm.nranks = 4;
  comm.device = 0;
  comm.cfg = loadConfig();
  comm.cfg.nvlsZcMinBytes = 1 << 20;  // what TNCCL_NVLS_ZC_MIN_BYTES=1048576 sets
  comm.nvls.enabled = true;
  comm.nvls.channels = comm.cfg.nvlsChannels;
  comm.nvls.tileBytes = (uint64_t)comm.cfg.nvlsTileBytes;
  comm.oneShotMaxBytes = 1 << 20;
  comm.nvlsMinBytes = ~0ull;  // the staged NVLS kernel is never AUTO's choice
  alignas(16) static char bufA[8 << 20], bufB[8 << 20], plain[8 << 20];
  auto reg = [&](int k, char* base, size_t bytes, uint64_t mcVa) {
    Registration& g = comm.regs[k];
    g.used = g.bound = g.mapped = true;
    g.base = base;
    g.userBytes = bytes;
    g.bytes = bytes;
    g.mcVa = mcVa;
  };
  reg(0, bufA, sizeof(bufA), 0x100000000ull);
  reg(1, bufB, sizeof(bufB), 0x200000000ull);
  auto run = [&](const void* s, void* r, size_t count, tncclDataType_t t, tncclAlgo_t algo) {
    gLast = Launch{};
    return tncclAllReduceEx(s, r, count, t, tncclSum, 1.0f, algo, &comm, nullptr) ==
           TNCCL_SUCCESS;
  };
  const size_t n4m = (4u << 20) / 4;
  bool ok = true;
  // Registered in place, AUTO, 4 MiB fp32: zero copy with the mc addresses.
  ok = ok && run(bufA + 4096, bufA + 4096, n4m, tncclFloat32, TNCCL_ALGO_AUTO);
  ok = ok && gLast.algo == TNCCL_ALGO_NVLS &&
       gLast.args.mcSend == reinterpret_cast<const char*>(0x100000000ull + 4096) &&
       gLast.args.mcRecv == reinterpret_cast<char*>(0x100000000ull + 4096) &&
       gLast.args.zcVecs == (4u << 20) / 16 && gLast.args.zcChannels >= 1 &&
       gLast.args.zcChannels <= comm.cfg.nvlsZcChannels && comm.zeroCopyLaunches == 1;
  report("zero copy: registered, AUTO, 4 MiB", ok);
  // Send in one registration, recv in another.
  ok = run(bufA, bufB + (1 << 20), n4m, tncclBfloat16, TNCCL_ALGO_AUTO) &&
       gLast.args.mcSend == reinterpret_cast<const char*>(0x100000000ull) &&
       gLast.args.mcRecv == reinterpret_cast<char*>(0x200000000ull + (1 << 20)) &&
       gLast.args.zcVecs == n4m * 2 / 16;
  report("zero copy: send and recv in different registrations", ok);
  // Not zero copy: unregistered recv, unaligned, not whole vectors, below the
  // AUTO minimum (but zero copy when NVLS is asked for), past the end.
  ok = run(bufA, plain, n4m, tncclFloat32, TNCCL_ALGO_AUTO) && gLast.args.mcSend == nullptr &&
       gLast.algo != TNCCL_ALGO_NVLS;
  ok = ok && run(bufA + 4, bufA + 4, n4m, tncclFloat32, TNCCL_ALGO_AUTO) &&
       gLast.args.mcSend == nullptr;
  ok = ok && run(bufA, bufA, n4m + 1, tncclFloat32, TNCCL_ALGO_AUTO) &&
       gLast.args.mcSend == nullptr;
  ok = ok && run(bufA, bufA, 1024, tncclFloat32, TNCCL_ALGO_AUTO) &&
       gLast.args.mcSend == nullptr;
  ok = ok && run(bufA, bufA, 1024, tncclFloat32, TNCCL_ALGO_NVLS) &&
       gLast.args.mcSend != nullptr && gLast.args.zcChannels == 1;
  ok = ok && run(bufA + (6 << 20), bufA + (6 << 20), n4m, tncclFloat32, TNCCL_ALGO_AUTO) &&
       gLast.args.mcSend == nullptr;
  ok = ok && run(bufA, bufA, n4m, tncclFloat32, TNCCL_ALGO_TWOSHOT) &&
       gLast.args.mcSend == nullptr && gLast.algo == TNCCL_ALGO_TWOSHOT;
  report("not zero copy: unregistered, unaligned, ragged, small, past end, other algo", ok);
  // TNCCL_ALGO=nvls (forced) counts like an explicit NVLS request; another
  // forced algorithm keeps AUTO calls off the zero-copy kernel.
  comm.cfg.forcedAlgo = TNCCL_ALGO_NVLS;
  ok = run(bufA, bufA, 1024, tncclFloat32, TNCCL_ALGO_AUTO) && gLast.args.mcSend != nullptr;
  comm.cfg.forcedAlgo = TNCCL_ALGO_TWOSHOT;
  ok = ok && run(bufA, bufA, n4m, tncclFloat32, TNCCL_ALGO_AUTO) &&
       gLast.args.mcSend == nullptr && gLast.algo == TNCCL_ALGO_TWOSHOT;
  comm.cfg.forcedAlgo = TNCCL_ALGO_AUTO;
  report("zero copy: TNCCL_ALGO=nvls yes, TNCCL_ALGO=twoshot no", ok);
  // The channel cap applies to the zero-copy kernel too.
  comm.maxChannels = 3;  // what tncclCommSetMaxChannels(comm, 3) sets
  ok = run(bufA, bufA, 2 * n4m, tncclFloat32, TNCCL_ALGO_AUTO) && gLast.args.mcSend != nullptr &&
       gLast.args.zcChannels == 3;
  comm.maxChannels = 0;
  // Off by default: without TNCCL_NVLS_ZERO_COPY the staged paths run.
  comm.cfg.nvlsZeroCopy = 0;
  ok = ok && run(bufA, bufA, n4m, tncclFloat32, TNCCL_ALGO_NVLS) && gLast.args.mcSend == nullptr &&
       gLast.algo == TNCCL_ALGO_NVLS;
  report("zero copy: channel cap, and off without TNCCL_NVLS_ZERO_COPY", ok);
  unsetenv("TNCCL_NVLS_ZERO_COPY");
}

}  // namespace

int main() {
  zeroCopySelection();
  allocAndFree();
  registerAndDeregister();
  argumentErrors();
  injectedFailures();
  printf("register_test: %s\n", gFailed ? "FAIL" : "PASS");
  return gFailed ? 1 : 0;
}
