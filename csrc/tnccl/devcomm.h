// devcomm.h - the plain-old-data structures handed to every kernel launch.
//
// tiny-nccl passes DevComm{rank, nranks, inbox, outbox} and DevWork{comm,
// send, recv, count, baseTicket, tilesPerSegment} by value
// (src/internal.h:24-40). Here the communicator view holds every peer's
// mailbox (NVSwitch makes every peer one hop away), the NVLS multicast view,
// device-resident FIFO counters (so launches replay correctly from CUDA
// graphs) and a host-mapped status block for bounded waits.
#pragma once

#include <stdint.h>

#include "protocol.h"

namespace tnccl {

// Host-mapped (cudaHostAllocMapped) status block polled by device waits.
struct DevStatus {
  volatile int32_t error;   // first tncclResult recorded by device code
  volatile int32_t abort;   // set by tncclCommAbort; every wait polls it
  volatile int32_t where;   // (family << 24) | (channel << 8) | phase
  volatile int32_t pad;
  volatile uint64_t expectedSeq;  // flag value the failed wait expected
  volatile uint64_t observedSeq;  // flag value it last observed
};

struct DevComm {
  int rank;
  int nranks;
  MailboxLayout layout;
  char* peers[kMaxRanks];  // mailbox base of every rank (peers[rank] = local)
  uint64_t* counters;      // device memory [kNumCounterFamilies][kMaxChannels]
  DevStatus* status;       // device pointer of the host-mapped status block
  uint64_t timeoutNs;      // bound for every device-side wait
  // NVLS (valid when nvlsEnabled != 0)
  int nvlsEnabled;
  int nvlsChannels;
  uint64_t nvlsTileBytes;
  char* nvlsUc;  // this rank's unicast view of the multicast-bound region
  char* nvlsMc;  // multicast view (multimem.* operations)
  // Phase tracer (TNCCL_TRACE=1): per channel a ring of traceEvents records
  // {globaltimer ns, tag}; traceCount[c] counts records written. Null when off.
  uint64_t* trace;
  uint32_t* traceCount;
  uint32_t traceEvents;
  // Warp split (eighths, a | b << 4) of the two-shot and NVLS teams.
  int tsSplit;
  int nvlsSplit;
  int acquireMode;  // 1: ld.acquire.sys on the flag, 0: fence.acq_rel.sys
  // Two-shot shared-memory staging: stages per team, push stage bytes,
  // reduce stage bytes (all sources together).
  int tsStages;
  uint32_t tsPushStage;
  uint32_t tsRedStage;
  // NVLS copy-in / copy-out staging: stages per team, bytes per stage.
  int nvlsStages;
  uint32_t nvlsStage;
  // Copies of fewer bytes per source than this go through registers.
  uint32_t stageMinBytes;
  // Socket ring edges (TNCCL_NET): device views of the host-mapped FIFOs
  // this rank's ring kernel shares with its proxy thread (layout netLayout);
  // null where the edge to rank + 1 / from rank - 1 is an NVLink edge.
  char* netSend;
  char* netRecv;
  NetFifoLayout netLayout;
};

// Tag of one trace record: algorithm family, phase, tile index (low 16 bits).
constexpr uint64_t traceTag(int family, int phase, uint64_t tile) {
  return ((uint64_t)family << 24) | ((uint64_t)phase << 16) | (tile & 0xffffu);
}

enum DataType : int { kF32 = 0, kBF16 = 1, kF16 = 2 };

struct AllReduceArgs {
  const void* send;
  void* recv;
  uint64_t count;
  float scale;
  int dtype;
  int vectorized;  // 1 when send/recv are 16-byte aligned
  // partition (ring / two-shot use chunk, one-shot / NVLS use block)
  ChunkPlan chunk;
  BlockPlan block;
  // Zero-copy NVLS (set only for buffers registered with tncclCommRegister):
  // multicast views of send and recv, the message in 16-byte vectors and the
  // channel count (protocol.h nvlsZcSpan). Null mcSend: the staged kernels.
  const char* mcSend;
  char* mcRecv;
  uint64_t zcVecs;
  int zcChannels;
};

// One cooperative launch that emulates `nranks` ranks on one GPU (tests and
// profiling of the multi-rank kernels without peers).
constexpr int kMaxEmulatedRanks = 8;
struct EmulatedLaunch {
  int nranks;
  int algo;
  int dtype;
  DevComm comm[kMaxEmulatedRanks];
  AllReduceArgs args[kMaxEmulatedRanks];
};

}  // namespace tnccl
