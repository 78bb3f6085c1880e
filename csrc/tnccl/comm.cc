// comm.cc - communicator init (blocking collective) and two-phase destroy.
//
// Same contract as tiny-nccl src/comm.cc:118-290: capture the current device;
// nranks == 1 needs no bootstrap; statuses are all-gathered so that every
// rank sees a peer's failure; a failed init closes its imports, passes a
// cleanup barrier and only then frees its export; destroy synchronizes the
// bound stream, passes barrier #1 (all kernels done), closes every import,
// passes barrier #2 (all importers closed) and only then frees; destroy always
// consumes the handle and retains exported memory when teardown cannot be
// proven safe.
//
// Differences: every peer (not only the next rank) is mapped and checked for
// P2P access and native peer atomics; devices are compared by UUID rather
// than by per-process ordinal; an NVLS multicast object is created when every
// rank supports it; the host-mapped status block and the device-resident FIFO
// counters are allocated here. Ranks on other hosts (compared by host
// identity) are not mapped: the ring edges that reach them are socket edges
// (net_setup.cc), and such a communicator runs the ring only.
#include <string.h>
#include <unistd.h>

#include <memory>
#include <new>
#include <vector>

#include "comm.h"
#include "driver.h"
#include "nvtx.h"
#include "sockio.h"

namespace tnccl {
namespace {

tncclResult firstFailure(const std::vector<PeerMeta>& metas) {
  for (const PeerMeta& m : metas) {
    if (m.status < TNCCL_SUCCESS || m.status >= TNCCL_NUM_RESULTS) return TNCCL_SYSTEM_ERROR;
    if (m.status != TNCCL_SUCCESS) return (tncclResult)m.status;
  }
  return TNCCL_SUCCESS;
}

bool devicesUnique(const std::vector<PeerMeta>& metas) {
  for (size_t i = 0; i < metas.size(); ++i)
    for (size_t j = 0; j < i; ++j)
      if (memcmp(metas[i].uuid, metas[j].uuid, sizeof(metas[i].uuid)) == 0) return false;
  return true;
}

// Checks P2P reachability and native atomics to a peer whose device is
// visible in this process. A peer hidden by CUDA_VISIBLE_DEVICES cannot be
// queried; its mapping is then validated by cuMemSetAccess during import.
tncclResult checkPeer(const tncclComm* comm, const PeerMeta& m) {
  int peerDev = -1;
  if (cudaDeviceGetByPCIBusId(&peerDev, m.busId) != cudaSuccess) {
    (void)cudaGetLastError();
    TN_INFO("rank %d: peer device %s not visible; skipping P2P attribute query",
            comm->rank, m.busId);
    return TNCCL_SUCCESS;
  }
  if (peerDev == comm->device) return TNCCL_UNSUPPORTED;
  int can = 0, atomics = 0;
  if (cudaDeviceCanAccessPeer(&can, comm->device, peerDev) != cudaSuccess) return TNCCL_CUDA_ERROR;
  if (!can) {
    TN_WARN("rank %d: no P2P access from device %d to %d", comm->rank, comm->device, peerDev);
    return TNCCL_UNSUPPORTED;
  }
  if (cudaDeviceGetP2PAttribute(&atomics, cudaDevP2PAttrNativeAtomicSupported, comm->device,
                                peerDev) != cudaSuccess)
    return TNCCL_CUDA_ERROR;
  if (!atomics) {
    TN_WARN("rank %d: no native peer atomics from device %d to %d", comm->rank, comm->device,
            peerDev);
    return TNCCL_UNSUPPORTED;
  }
  return TNCCL_SUCCESS;
}

// Initial FIFO state: zero everywhere except the ring credits, which start
// at the slot index (slot s may carry ticket s first).
tncclResult initMailboxContents(tncclComm* comm) {
  const MailboxLayout& L = comm->layout;
  if (cudaMemset(comm->local.base, 0, comm->local.bytes) != cudaSuccess) return TNCCL_CUDA_ERROR;
  std::vector<uint64_t> credits((size_t)L.channels * (size_t)L.ringSlots);
  for (int c = 0; c < L.channels; ++c)
    for (int s = 0; s < L.ringSlots; ++s) credits[(size_t)c * L.ringSlots + s] = (uint64_t)s;
  if (cudaMemcpy(comm->local.base + L.ringCreditOff, credits.data(),
                 credits.size() * sizeof(uint64_t), cudaMemcpyHostToDevice) != cudaSuccess)
    return TNCCL_CUDA_ERROR;
  for (int k = 0; k < kNumCanaries; ++k)
    if (cudaMemset(comm->local.base + L.canaryOff[k], kCanaryByte, kCanaryBytes) != cudaSuccess)
      return TNCCL_CUDA_ERROR;
  return cudaDeviceSynchronize() == cudaSuccess ? TNCCL_SUCCESS : TNCCL_CUDA_ERROR;
}

}  // namespace

// Counts the canary regions of this rank's mailbox that no longer hold
// kCanaryByte (the caller has synchronised the bound stream).
tncclResult countBadCanaries(tncclComm* comm, int* corrupted) {
  *corrupted = 0;
  if (comm->local.base == nullptr) return TNCCL_SUCCESS;
  unsigned char buf[kCanaryBytes];
  for (int k = 0; k < kNumCanaries; ++k) {
    if (cudaMemcpy(buf, comm->local.base + comm->layout.canaryOff[k], kCanaryBytes,
                   cudaMemcpyDeviceToHost) != cudaSuccess)
      return TNCCL_CUDA_ERROR;
    for (uint64_t i = 0; i < kCanaryBytes; ++i)
      if (buf[i] != kCanaryByte) {
        ++*corrupted;
        break;
      }
  }
  return TNCCL_SUCCESS;
}

namespace {

tncclResult allocDeviceState(tncclComm* comm) {
  void* h = nullptr;
  if (cudaHostAlloc(&h, sizeof(DevStatus), cudaHostAllocMapped | cudaHostAllocPortable) !=
      cudaSuccess)
    return TNCCL_CUDA_ERROR;
  memset(h, 0, sizeof(DevStatus));
  comm->hostStatus = static_cast<DevStatus*>(h);
  void* d = nullptr;
  if (cudaHostGetDevicePointer(&d, h, 0) != cudaSuccess) return TNCCL_CUDA_ERROR;
  comm->devStatus = static_cast<DevStatus*>(d);
  const size_t cbytes = sizeof(uint64_t) * kNumCounterFamilies * kMaxChannels;
  if (cudaMalloc(reinterpret_cast<void**>(&comm->counters), cbytes) != cudaSuccess)
    return TNCCL_CUDA_ERROR;
  if (cudaMemset(comm->counters, 0, cbytes) != cudaSuccess) return TNCCL_CUDA_ERROR;
  if (cudaMalloc(reinterpret_cast<void**>(&comm->diagWord), sizeof(uint64_t)) != cudaSuccess)
    return TNCCL_CUDA_ERROR;
  if (cudaMemset(comm->diagWord, 0, sizeof(uint64_t)) != cudaSuccess) return TNCCL_CUDA_ERROR;
  if (comm->cfg.traceEvents > 0) {
    const size_t tb = (size_t)kMaxChannels * comm->cfg.traceEvents * 2 * sizeof(uint64_t);
    if (cudaMalloc(reinterpret_cast<void**>(&comm->trace), tb) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void**>(&comm->traceCount), kMaxChannels * sizeof(uint32_t)) !=
            cudaSuccess)
      return TNCCL_CUDA_ERROR;
    cudaMemset(comm->trace, 0, tb);
    cudaMemset(comm->traceCount, 0, kMaxChannels * sizeof(uint32_t));
  }
  return TNCCL_SUCCESS;
}

void freeDeviceState(tncclComm* comm) {
  if (comm->counters) cudaFree(comm->counters);
  comm->counters = nullptr;
  if (comm->diagWord) cudaFree(comm->diagWord);
  comm->diagWord = nullptr;
  if (comm->trace) cudaFree(comm->trace);
  if (comm->traceCount) cudaFree(comm->traceCount);
  comm->trace = nullptr;
  comm->traceCount = nullptr;
  if (comm->hostStatus) cudaFreeHost(comm->hostStatus);
  comm->hostStatus = nullptr;
  comm->devStatus = nullptr;
}

void fillDevComm(tncclComm* comm) {
  DevComm& d = comm->dev;
  d.rank = comm->rank;
  d.nranks = comm->nranks;
  d.layout = comm->layout;
  for (int r = 0; r < kMaxRanks; ++r) d.peers[r] = nullptr;
  for (int r = 0; r < comm->nranks; ++r)
    d.peers[r] = r == comm->rank ? comm->local.base : comm->peers[r].base;
  d.counters = comm->counters;
  d.status = comm->devStatus;
  d.timeoutNs = (uint64_t)comm->cfg.timeoutMs * 1000000ull;
  d.nvlsEnabled = comm->nvls.enabled ? 1 : 0;
  d.nvlsChannels = comm->nvls.channels;
  d.nvlsTileBytes = comm->nvls.tileBytes;
  d.nvlsUc = reinterpret_cast<char*>(comm->nvls.ucVa);
  d.nvlsMc = reinterpret_cast<char*>(comm->nvls.mcVa);
  d.trace = comm->trace;
  d.traceCount = comm->traceCount;
  d.traceEvents = (uint32_t)comm->cfg.traceEvents;
  d.tsSplit = comm->cfg.tsSplit;
  d.nvlsSplit = comm->cfg.nvlsSplit;
  d.acquireMode = comm->cfg.acquireMode;
  d.tsStages = comm->cfg.tsStages;
  d.tsPushStage = (uint32_t)comm->cfg.tsPushStage;
  d.tsRedStage = (uint32_t)comm->cfg.tsRedStage;
  d.nvlsStages = comm->cfg.nvlsStages;
  d.nvlsStage = (uint32_t)comm->cfg.nvlsStage;
  d.stageMinBytes = (uint32_t)comm->cfg.stageMinBytes;
  d.netSend = comm->net.sendDev;
  d.netRecv = comm->net.recvDev;
  d.netLayout = comm->net.layout;
}

void deriveThresholds(tncclComm* comm) {
  const int P = comm->nranks;
  // Defaults from the measured sweeps on 2, 4 and 8 B200 (benchmarks/
  // allreduce_sweep.py, tune_allreduce.py): one-shot (64 channels) moves
  // (P-1) x the message per link direction but needs one flag round trip
  // instead of two, so it wins up to 2 MiB on 2 GPUs (112 vs 104 GB/s) and
  // up to 1 MiB on 4 and 8 (61 vs 56 GB/s at 1 MiB on 8); the
  // warp-specialised two-shot above (it also beats the NVLS kernel at every
  // size measured, so AUTO picks NVLS only when TNCCL_NVLS_MIN_BYTES asks
  // for it). TNCCL_ONESHOT_MAX_BYTES / TNCCL_NVLS_MIN_BYTES override them.
  uint64_t os = P <= 2 ? (2u << 20) : (1u << 20);
  uint64_t nv = ~0ull;
  if (comm->cfg.oneShotMaxBytes > 0) os = (uint64_t)comm->cfg.oneShotMaxBytes;
  if (comm->cfg.nvlsMinBytes > 0) nv = (uint64_t)comm->cfg.nvlsMinBytes;
  comm->oneShotMaxBytes = os;
  comm->nvlsMinBytes = nv;
}

// Gives up on a communicator whose export may already be mapped by peers:
// close our imports and the control connection, keep the export alive.
void abandonPublished(tncclComm* comm) {
  tncclResult ignored = TNCCL_SUCCESS;
  netStopProxy(comm, false, &ignored);
  netRelease(comm, true);  // host FIFOs: no kernel has run
  closePeerMailboxes(comm, &ignored);
  bootstrapClose(&comm->bootstrap);
}

}  // namespace
}  // namespace tnccl

using namespace tnccl;

extern "C" tncclResult tncclCommInitRank(tncclComm_t* out, int nranks, tncclUniqueId id,
                                         int rank) {
  if (out == nullptr || nranks <= 0 || rank < 0 || rank >= nranks) return TNCCL_INVALID_ARGUMENT;
  *out = nullptr;
  NvtxRange range("tncclCommInitRank %d/%d", rank, nranks);
  if (nranks > kMaxRanks) return TNCCL_UNSUPPORTED;
  std::unique_ptr<tncclComm> comm(new (std::nothrow) tncclComm);
  if (!comm) return TNCCL_SYSTEM_ERROR;
  comm->rank = rank;
  comm->nranks = nranks;
  comm->cfg = loadConfig();
  adaptConfig(comm->cfg, nranks);
  if (cudaGetDevice(&comm->device) != cudaSuccess) {
    (void)cudaGetLastError();
    return TNCCL_CUDA_ERROR;
  }
  deriveThresholds(comm.get());
  if (tncclResult r = allocDeviceState(comm.get()); r != TNCCL_SUCCESS) {
    freeDeviceState(comm.get());
    return r;
  }
  if (nranks == 1) {
    fillDevComm(comm.get());
    *out = comm.release();
    return TNCCL_SUCCESS;
  }
  const DriverApi* api = driverApi();
  if (api) api->cuDeviceGet(&comm->cuDevice, comm->device);

  tncclResult r = bootstrapOpen(&comm->bootstrap, id, nranks, rank, configHash(comm->cfg),
                                (int)comm->cfg.bootstrapTimeoutMs);
  if (r != TNCCL_SUCCESS) {
    freeDeviceState(comm.get());
    return r;
  }

  LayoutConfig lc{};
  lc.nranks = nranks;
  lc.channels = comm->cfg.channels;
  lc.osChannels = comm->cfg.osChannels;
  lc.ringSlots = comm->cfg.ringSlots;
  lc.ringChunkBytes = (uint64_t)comm->cfg.ringChunkBytes;
  lc.tsChunkBytes = (uint64_t)comm->cfg.tsChunkBytes;
  lc.osSlots = comm->cfg.osSlots;
  lc.osTileBytes = (uint64_t)comm->cfg.osTileBytes;
  comm->layout = makeLayout(lc);

  PeerMeta me{};
  me.device = comm->device;
  me.hostId = hostIdentity();
  if (rank == 0 && !randomBytes(&me.nonce, sizeof(me.nonce))) me.status = TNCCL_SYSTEM_ERROR;
  cudaDeviceProp prop{};
  if (cudaGetDeviceProperties(&prop, comm->device) == cudaSuccess) {
    memcpy(me.uuid, &prop.uuid, sizeof(me.uuid));
  } else {
    me.status = TNCCL_CUDA_ERROR;
  }
  if (cudaDeviceGetPCIBusId(me.busId, sizeof(me.busId), comm->device) != cudaSuccess)
    me.status = TNCCL_CUDA_ERROR;
  // A TCP bootstrap cannot pass descriptors: mailboxes are shared as cudaIpc
  // handles inside PeerMeta instead.
  if (me.status == TNCCL_SUCCESS)
    me.status = allocLocalMailbox(comm.get(), comm->layout.totalBytes,
                                  comm->cfg.useCuMem != 0 && !comm->bootstrap.tcp);
  if (me.status == TNCCL_SUCCESS) me.status = initMailboxContents(comm.get());
  me.ipcMode = comm->ipcMode;
  me.mailboxBytes = comm->local.bytes;
  me.ipcHandle = comm->local.ipcHandle;
  me.nvlsCapable = me.status == TNCCL_SUCCESS && nvlsLocallyCapable(comm.get()) ? 1 : 0;

  std::vector<PeerMeta> metas((size_t)nranks);
  r = bootstrapAllGather(&comm->bootstrap, &me, metas.data(), sizeof(me));
  if (r != TNCCL_SUCCESS) {
    abandonPublished(comm.get());
    return r;
  }
  tncclResult status = firstFailure(metas);
  if (status == TNCCL_SUCCESS && !devicesUnique(metas)) status = TNCCL_UNSUPPORTED;
  for (const PeerMeta& m : metas)
    if (status == TNCCL_SUCCESS && m.ipcMode != metas[0].ipcMode) status = TNCCL_UNSUPPORTED;

  // Locality. Peers on this host are mapped; a ring edge between hosts (every
  // ring edge with TNCCL_NET=force) is a socket edge. All inputs are
  // all-gathered or hashed into the configuration, so every rank decides
  // alike.
  std::vector<char> local((size_t)nranks);
  comm->allPeersMapped = true;
  for (int p = 0; p < nranks; ++p) {
    local[(size_t)p] = metas[(size_t)p].hostId == metas[(size_t)rank].hostId;
    comm->allPeersMapped = comm->allPeersMapped && local[(size_t)p];
  }
  const int netMode = comm->cfg.netMode;
  auto socketEdge = [&](int a) {
    const int b = (a + 1) % nranks;
    return netMode == 2 || (netMode == 1 && metas[(size_t)a].hostId != metas[(size_t)b].hostId);
  };
  for (int q = 0; q < nranks; ++q) comm->net.any = comm->net.any || socketEdge(q);
  comm->net.send = socketEdge(rank);
  comm->net.recv = socketEdge((rank + nranks - 1) % nranks);
  if (status == TNCCL_SUCCESS && !comm->allPeersMapped && netMode == 0) {
    TN_WARN("rank %d: ranks on several hosts need socket edges (TNCCL_NET=auto)", rank);
    status = TNCCL_UNSUPPORTED;
  }
  for (int p = 0; p < nranks && status == TNCCL_SUCCESS; ++p)
    if (p != rank && local[(size_t)p]) status = checkPeer(comm.get(), metas[(size_t)p]);

  // Every rank takes part in the descriptor all-gather (cuMem mode) even
  // after a local failure, so the collective sequence stays aligned.
  std::vector<int> fds((size_t)nranks, -1);
  bool allCuMem = true;
  for (const PeerMeta& m : metas) allCuMem = allCuMem && m.ipcMode == kIpcCuMem;
  if (allCuMem && firstFailure(metas) == TNCCL_SUCCESS) {
    r = bootstrapAllGatherFds(&comm->bootstrap, comm->local.exportFd, fds.data());
    if (r != TNCCL_SUCCESS) {
      abandonPublished(comm.get());
      return r;
    }
  }
  for (int p = 0; p < nranks && status == TNCCL_SUCCESS; ++p) {
    if (p == rank || !local[(size_t)p]) continue;
    status = importPeerMailbox(comm.get(), p, fds[(size_t)p], metas[(size_t)p]);
  }
  for (int fd : fds)
    if (fd >= 0) close(fd);
  if (status == TNCCL_SUCCESS && comm->net.any) status = netAllocFifos(comm.get());

  // Connection status round, then the ready barrier (tiny-nccl
  // src/comm.cc:173-196).
  PeerMeta conn{};
  conn.status = status;
  std::vector<PeerMeta> conns((size_t)nranks);
  r = bootstrapAllGather(&comm->bootstrap, &conn, conns.data(), sizeof(conn));
  if (r != TNCCL_SUCCESS) {
    abandonPublished(comm.get());
    return r;
  }
  status = firstFailure(conns);

  // NVLS only when every rank is connected, on this host and capable (the
  // multicast handle travels as a descriptor, so not over a TCP bootstrap).
  bool allNvls = status == TNCCL_SUCCESS && comm->allPeersMapped && !comm->bootstrap.tcp;
  for (const PeerMeta& m : metas) allNvls = allNvls && m.nvlsCapable;
  if (allNvls) {
    r = setupNvls(comm.get());
    if (r != TNCCL_SUCCESS && r != TNCCL_UNSUPPORTED) {
      abandonPublished(comm.get());
      return r;
    }
    if (r == TNCCL_UNSUPPORTED) TN_INFO("rank %d: NVLS unavailable; using P2P algorithms", rank);
  }

  // Socket edges: connections and proxy (collective; `status` is the same on
  // every rank here).
  if (status == TNCCL_SUCCESS && comm->net.any) {
    r = netStart(comm.get(), metas[0].nonce);
    if (r != TNCCL_SUCCESS) status = r;
  }

  r = bootstrapBarrier(&comm->bootstrap);
  if (r != TNCCL_SUCCESS) {
    abandonPublished(comm.get());
    return r;
  }
  if (status != TNCCL_SUCCESS) {
    tncclResult ignored = TNCCL_SUCCESS;
    netStopProxy(comm.get(), false, &ignored);
    netRelease(comm.get(), true);  // host FIFOs: no kernel has run
    nvlsUnmap(comm.get(), &ignored);
    closePeerMailboxes(comm.get(), &ignored);
    tncclResult cleanup = bootstrapBarrier(&comm->bootstrap);
    if (cleanup == TNCCL_SUCCESS) {
      nvlsRelease(comm.get(), &ignored);
      freeLocalMailbox(comm.get(), &ignored);
      freeDeviceState(comm.get());
    }
    bootstrapClose(&comm->bootstrap);
    return cleanup == TNCCL_SUCCESS ? status : cleanup;
  }
  fillDevComm(comm.get());
  TN_INFO("rank %d/%d: device %d, ipc %s, mailbox %zu bytes, NVLS %s, socket edges %s", rank,
          nranks, comm->device, comm->ipcMode == kIpcCuMem ? "cuMem" : "legacy",
          comm->local.bytes, comm->nvls.enabled ? "on" : "off", comm->net.any ? "yes" : "no");
  *out = comm.release();
  return TNCCL_SUCCESS;
}

extern "C" tncclResult tncclCommDestroy(tncclComm_t comm) {
  if (comm == nullptr) return TNCCL_INVALID_ARGUMENT;
  NvtxRange range("tncclCommDestroy %d/%d", comm->rank, comm->nranks);
  int original = -1;
  if (cudaGetDevice(&original) != cudaSuccess) {
    bootstrapClose(&comm->bootstrap);
    delete comm;
    return TNCCL_CUDA_ERROR;
  }
  if (original != comm->device && cudaSetDevice(comm->device) != cudaSuccess) {
    bootstrapClose(&comm->bootstrap);
    delete comm;
    return TNCCL_CUDA_ERROR;
  }
  tncclResult result = TNCCL_SUCCESS;
  if (comm->streamBound && cudaStreamSynchronize(comm->boundStream) != cudaSuccess) {
    // A kernel may still own the mappings: break the control connection so
    // peers take their bounded error paths; retain device memory and the
    // socket FIFOs.
    tncclResult ignored = TNCCL_SUCCESS;
    netStopProxy(comm, false, &ignored);
    netRelease(comm, false);
    bootstrapClose(&comm->bootstrap);
    delete comm;
    return TNCCL_CUDA_ERROR;
  }
  if (comm->nranks == 1) {
    freeDeviceState(comm);
    if (original != comm->device) cudaSetDevice(original);
    delete comm;
    return TNCCL_SUCCESS;
  }
  int corrupted = 0;
  if (countBadCanaries(comm, &corrupted) == TNCCL_SUCCESS && corrupted > 0)
    TN_WARN("rank %d: %d mailbox canary region(s) overwritten; a kernel wrote past an area",
            comm->rank, corrupted);
  tncclResult b1 = bootstrapBarrier(&comm->bootstrap);  // every kernel has finished
  if (b1 != TNCCL_SUCCESS) result = b1;
  netStopProxy(comm, b1 == TNCCL_SUCCESS, &result);  // no frame is in flight any more
  nvlsUnmap(comm, &result);
  registrationsUnmap(comm, &result);
  closePeerMailboxes(comm, &result);
  tncclResult b2 = bootstrapBarrier(&comm->bootstrap);  // every importer has closed
  if (b2 != TNCCL_SUCCESS && result == TNCCL_SUCCESS) result = b2;
  // This rank's stream is idle and its proxy stopped: nothing touches its
  // socket FIFOs whatever the barriers returned.
  netRelease(comm, true);
  if (b1 == TNCCL_SUCCESS && b2 == TNCCL_SUCCESS) {
    registrationsRelease(comm, &result);
    nvlsRelease(comm, &result);
    freeLocalMailbox(comm, &result);
    freeDeviceState(comm);
  }
  bootstrapClose(&comm->bootstrap);
  if (original != comm->device && cudaSetDevice(original) != cudaSuccess &&
      result == TNCCL_SUCCESS)
    result = TNCCL_CUDA_ERROR;
  delete comm;
  return result;
}
