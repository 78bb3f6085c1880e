// comm.h - the host-side communicator object and transport helpers.
#pragma once

#include <cuda.h>
#include <cuda_runtime_api.h>

#include <atomic>

#include "bootstrap.h"
#include "common.h"
#include "devcomm.h"
#include "driver.h"
#include "net.h"
#include "tnccl.h"

namespace tnccl {

enum IpcMode : int { kIpcNone = 0, kIpcCuMem = 1, kIpcLegacy = 2 };

// This rank's exported mailbox.
struct LocalMailbox {
  char* base = nullptr;
  size_t bytes = 0;  // mapped size (granularity-rounded)
  // cuMem mode
  CUmemGenericAllocationHandle handle = 0;
  bool created = false;
  bool reserved = false;
  bool mapped = false;
  int exportFd = -1;
  // legacy mode
  bool legacyAlloc = false;
  cudaIpcMemHandle_t ipcHandle{};
};

// A peer's mailbox mapped into this process.
struct PeerMailbox {
  char* base = nullptr;
  size_t bytes = 0;
  CUmemGenericAllocationHandle handle = 0;
  bool imported = false;
  bool reserved = false;
  bool mapped = false;
  bool legacyOpened = false;
};

struct NvlsState {
  bool enabled = false;
  size_t bytes = 0;
  int channels = 0;
  uint64_t tileBytes = 0;
  CUmemGenericAllocationHandle mc = 0;
  bool mcValid = false;
  bool deviceAdded = false;
  CUmemGenericAllocationHandle uc = 0;
  bool ucCreated = false;
  bool bound = false;
  CUdeviceptr ucVa = 0;
  bool ucReserved = false;
  bool ucMapped = false;
  CUdeviceptr mcVa = 0;
  bool mcReserved = false;
  bool mcMapped = false;
};

// A buffer registered with tncclCommRegister: a range of a tncclMemAlloc
// allocation bound to a multicast object of its own on every rank, for the
// zero-copy NVLS all-reduce.
constexpr int kMaxRegistrations = 32;
struct Registration {
  bool used = false;
  char* base = nullptr;     // the caller's pointer (this process's unicast view)
  size_t userBytes = 0;     // bytes the caller registered
  size_t bytes = 0;         // bytes bound (multicast granularity)
  void* allocation = nullptr;  // base of the tncclMemAlloc allocation it lies in
  CUmemGenericAllocationHandle mc = 0;
  bool mcValid = false;
  bool deviceAdded = false;
  bool bound = false;
  CUdeviceptr mcVa = 0;
  bool reserved = false;
  bool mapped = false;
};

// Exchanged through the bootstrap all-gather at init.
struct PeerMeta {
  int32_t status;
  int32_t device;       // ordinal in the sender's process
  int32_t ipcMode;
  int32_t nvlsCapable;
  uint64_t mailboxBytes;
  char uuid[16];
  char busId[32];
  cudaIpcMemHandle_t ipcHandle;
  uint64_t hostId;      // ranks with equal ids share a host (NVLink / IPC reach)
  uint64_t nonce;       // rank 0's random communicator nonce (socket hellos)
};

// This rank's socket ring edges (TNCCL_NET) and their proxy.
struct NetState {
  bool any = false;   // some ring edge of the communicator is a socket edge
  bool send = false;  // this rank's edge to rank + 1
  bool recv = false;  // this rank's edge from rank - 1
  NetFifoLayout layout{};
  char* sendHost = nullptr;  // cudaHostAlloc'd FIFOs (host views)
  char* recvHost = nullptr;
  char* sendDev = nullptr;   // their device views
  char* recvDev = nullptr;
  NetRing ring;
  NetProxy* proxy = nullptr;
};

}  // namespace tnccl

struct tncclComm {
  int rank = -1;
  int nranks = 0;
  int device = -1;
  CUdevice cuDevice = 0;
  tnccl::Config cfg{};
  tnccl::Bootstrap bootstrap;
  int ipcMode = tnccl::kIpcNone;
  tnccl::MailboxLayout layout{};
  tnccl::LocalMailbox local;
  tnccl::PeerMailbox peers[tnccl::kMaxRanks];
  tnccl::NvlsState nvls;
  tnccl::Registration regs[tnccl::kMaxRegistrations];
  tnccl::NetState net;
  bool allPeersMapped = true;  // every peer is on this host and mapped
  tnccl::DevComm dev{};
  uint64_t* counters = nullptr;
  uint64_t* diagWord = nullptr;  // device word that nothing writes (self tests)
  uint64_t* trace = nullptr;      // TNCCL_TRACE records (devcomm.h)
  uint32_t* traceCount = nullptr;
  tnccl::DevStatus* hostStatus = nullptr;
  tnccl::DevStatus* devStatus = nullptr;
  cudaStream_t boundStream = nullptr;
  bool streamBound = false;
  bool aborted = false;
  bool deviceErrorReported = false;  // the warning below is printed once
  uint64_t oneShotMaxBytes = 0;
  uint64_t nvlsMinBytes = 0;
  int maxChannels = 0;  // tncclCommSetMaxChannels cap (0: none)
  uint64_t zeroCopyLaunches = 0;  // launches of the zero-copy NVLS kernel
};

namespace tnccl {

// transport.cc
CUmemAllocationProp deviceProp(int device, bool exportable);
// Logs a failed driver call; true on CUDA_SUCCESS.
bool cuOk(CUresult r, const char* what);
// Maps handle at a fresh VA range of `bytes` with read/write access for
// `device`.
bool mapHandle(const DriverApi* api, CUmemGenericAllocationHandle h, size_t bytes, size_t align,
               int device, CUdeviceptr* va, bool* reserved, bool* mapped);
tncclResult allocLocalMailbox(tncclComm* comm, size_t bytes, bool tryCuMem);
tncclResult importPeerMailbox(tncclComm* comm, int peer, int fd,
                              const PeerMeta& meta);
void closePeerMailboxes(tncclComm* comm, tncclResult* result);
void freeLocalMailbox(tncclComm* comm, tncclResult* result);
bool nvlsLocallyCapable(const tncclComm* comm);
tncclResult setupNvls(tncclComm* comm);
void nvlsUnmap(tncclComm* comm, tncclResult* result);
void nvlsRelease(tncclComm* comm, tncclResult* result);

// register.cc: the registration holding [p, p + bytes), or nullptr.
const Registration* findRegistration(const tncclComm* comm, const void* p, size_t bytes);
// Destroy's halves: unmap and unbind every registration (after barrier 1),
// release the multicast objects (after barrier 2).
void registrationsUnmap(tncclComm* comm, tncclResult* result);
void registrationsRelease(tncclComm* comm, tncclResult* result);

// enqueue.cc
tncclAlgo_t selectAlgo(const tncclComm* comm, uint64_t bytes);

// comm.cc: mailbox canary regions that were overwritten.
tncclResult countBadCanaries(tncclComm* comm, int* corrupted);

// net_setup.cc: socket ring edges of a communicator.
// Hash of this host's identity (hostname and kernel boot id; TNCCL_HOST_ID
// overrides it, which lets one machine act as several hosts).
uint64_t hostIdentity();
// Sets the socket FIFO layout (every rank of a communicator with socket
// edges: it caps the ring's channels) and allocates and initialises the
// host-mapped FIFOs of this rank's own socket edges (local; before the
// connection status round).
tncclResult netAllocFifos(tncclComm* comm);
// Connects the socket edges (collective) and starts the proxy.
tncclResult netStart(tncclComm* comm, uint64_t nonce);
// Stops and joins the proxy (close frames first when `graceful`; a proxy
// failure then lands in *result).
void netStopProxy(tncclComm* comm, bool graceful, tncclResult* result);
// Closes the connections; frees the FIFOs when `freeFifos` (no kernel of
// this rank can touch them any more).
void netRelease(tncclComm* comm, bool freeFifos);

// Launch counter shared by every kernel launch in the library.
extern std::atomic<unsigned long long> gLaunchCount;

}  // namespace tnccl
