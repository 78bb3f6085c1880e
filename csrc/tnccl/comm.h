// comm.h - the host-side communicator object and transport helpers.
#pragma once

#include <cuda.h>
#include <cuda_runtime_api.h>

#include <atomic>

#include "bootstrap.h"
#include "common.h"
#include "devcomm.h"
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
  uint64_t oneShotMaxBytes = 0;
  uint64_t nvlsMinBytes = 0;
  int maxChannels = 0;  // tncclCommSetMaxChannels cap (0: none)
};

namespace tnccl {

// transport.cc
tncclResult allocLocalMailbox(tncclComm* comm, size_t bytes, bool tryCuMem);
tncclResult importPeerMailbox(tncclComm* comm, int peer, int fd,
                              const PeerMeta& meta);
void closePeerMailboxes(tncclComm* comm, tncclResult* result);
void freeLocalMailbox(tncclComm* comm, tncclResult* result);
bool nvlsLocallyCapable(const tncclComm* comm);
tncclResult setupNvls(tncclComm* comm);
void nvlsUnmap(tncclComm* comm, tncclResult* result);
void nvlsRelease(tncclComm* comm, tncclResult* result);

// enqueue.cc
tncclAlgo_t selectAlgo(const tncclComm* comm, uint64_t bytes);

// comm.cc: mailbox canary regions that were overwritten.
tncclResult countBadCanaries(tncclComm* comm, int* corrupted);

// Launch counter shared by every kernel launch in the library.
extern std::atomic<unsigned long long> gLaunchCount;

}  // namespace tnccl
