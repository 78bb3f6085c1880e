// emulate.cc - single-GPU emulation of a multi-rank communicator.
//
// tncclEmuCreate builds `nranks` virtual ranks on the current device: one
// mailbox, one set of FIFO sequence counters and one DevComm per rank, with
// every rank's "peer" pointers aimed at the other virtual ranks' mailboxes in
// the same GPU memory. tncclEmuAllReduce runs all ranks' channels as one
// cooperative launch (grid = channels x nranks), so CTAs that wait on one
// another are guaranteed to be resident together. The device code is the
// same ring / one-shot / two-shot bodies that the real communicator launches;
// only the memory the peer stores land in differs (local HBM instead of a
// peer over NVLink). It serves single-GPU tests of the multi-rank algorithms
// and ncu profiles of their kernels. NVLS needs a multicast object spanning
// several GPUs and is not emulated.
//
// With TNCCL_NET=force the virtual ranks' ring edges are socket edges: each
// virtual rank gets host-mapped send / receive FIFOs and a proxy thread, and
// the edges are loopback TCP connections inside this process; the ring then
// runs through the same socket path (ringBody<T, true>) as ranks on
// different hosts. TNCCL_EMU_HOSTS=<id>,<id>,... (one per virtual rank)
// instead makes only the edges between different ids socket edges, so NVLink
// and socket edges mix in one ring.
#include <string.h>
#include <unistd.h>

#include <algorithm>
#include <new>
#include <vector>

#include "comm.h"
#include "diag.h"
#include "launch.h"
#include "net.h"
#include "sockio.h"

struct tncclEmu {
  int nranks = 0;
  int device = -1;
  tnccl::Config cfg{};
  tnccl::MailboxLayout layout{};
  std::vector<char*> mailbox;
  uint64_t* counters = nullptr;
  tnccl::DevStatus* hostStatus = nullptr;
  tnccl::DevStatus* devStatus = nullptr;
  tnccl::DevComm dev[tnccl::kMaxEmulatedRanks];
  // socket edges (TNCCL_NET=force)
  bool net = false;
  tnccl::NetFifoLayout netLayout{};
  std::vector<char*> netSend, netRecv;  // host FIFOs per virtual rank
  std::vector<tnccl::NetRing> rings;
  std::vector<tnccl::NetProxy*> proxies;
};

using namespace tnccl;

namespace {

void freeEmu(tncclEmu* e) {
  for (tnccl::NetProxy*& p : e->proxies) {
    if (p) netProxyStop(p, false);
    delete p;
    p = nullptr;
  }
  for (tnccl::NetRing& r : e->rings) netCloseRing(&r);
  for (char* f : e->netSend)
    if (f) cudaFreeHost(f);
  for (char* f : e->netRecv)
    if (f) cudaFreeHost(f);
  e->netSend.clear();
  e->netRecv.clear();
  for (char* m : e->mailbox)
    if (m) cudaFree(m);
  e->mailbox.clear();
  if (e->counters) cudaFree(e->counters);
  if (e->hostStatus) cudaFreeHost(e->hostStatus);
  e->counters = nullptr;
  e->hostStatus = nullptr;
}

size_t elemSize(tncclDataType_t t) {
  return t == tncclFloat32 ? 4 : (t == tncclBfloat16 || t == tncclFloat16) ? 2 : 0;
}

void emuNetFailure(void* arg, tncclResult code) {
  auto* e = static_cast<tncclEmu*>(arg);
  auto* err = const_cast<int32_t*>(&e->hostStatus->error);
  int32_t expected = 0;
  __atomic_compare_exchange_n(err, &expected, (int32_t)code, false, __ATOMIC_SEQ_CST,
                              __ATOMIC_SEQ_CST);
}

// Socket edges between the virtual ranks (edge k -> k+1 where socket[k]):
// FIFOs, loopback connections (each edge is connected, accepted and
// acknowledged in turn; the listen backlog holds the connections meanwhile)
// and one proxy per virtual rank that has a socket edge.
tncclResult setupEmuNet(tncclEmu* e, const std::vector<char>& socket) {
  const int P = e->nranks;
  NetOptions o;
  o.channels = e->cfg.netChannels;
  o.sndBuf = o.rcvBuf = e->cfg.netSockBuf;
  o.spinUs = e->cfg.netSpinUs;
  o.timeoutMs = (int)e->cfg.bootstrapTimeoutMs;
  const NetFifoLayout L =
      makeNetFifoLayout(o.channels, e->cfg.ringSlots, (uint64_t)e->cfg.ringChunkBytes);
  e->netLayout = L;
  e->netSend.assign((size_t)P, nullptr);
  e->netRecv.assign((size_t)P, nullptr);
  e->rings.assign((size_t)P, NetRing{});
  e->proxies.assign((size_t)P, nullptr);
  auto alloc = [&](char** host, char** dev) -> bool {
    void* h = nullptr;
    void* d = nullptr;
    if (cudaHostAlloc(&h, L.totalBytes, cudaHostAllocMapped | cudaHostAllocPortable) !=
        cudaSuccess)
      return false;
    *host = static_cast<char*>(h);
    netFifoInit(*host, L);
    if (cudaHostGetDevicePointer(&d, h, 0) != cudaSuccess) return false;
    *dev = static_cast<char*>(d);
    return true;
  };
  uint64_t nonce = 0;
  if (!randomBytes(&nonce, sizeof(nonce))) return TNCCL_SYSTEM_ERROR;
  uint32_t ip = 0;
  parseIpv4("127.0.0.1", &ip);
  for (int k = 0; k < P; ++k) {
    const bool sendSock = socket[(size_t)k] != 0, recvSock = socket[(size_t)((k + P - 1) % P)] != 0;
    char* sendDev = nullptr;
    char* recvDev = nullptr;
    if ((sendSock && !alloc(&e->netSend[(size_t)k], &sendDev)) ||
        (recvSock && !alloc(&e->netRecv[(size_t)k], &recvDev)))
      return TNCCL_CUDA_ERROR;
    e->dev[k].netSend = sendDev;
    e->dev[k].netRecv = recvDev;
    e->dev[k].netLayout = L;
  }
  for (int k = 0; k < P; ++k) {
    if (!socket[(size_t)k]) continue;
    const int next = (k + 1) % P;
    int port = 0;
    const int lfd = tcpListen("127.0.0.1", 0, o.channels + 4, &port);
    if (lfd < 0) return TNCCL_SYSTEM_ERROR;
    NetHello h{kNetHelloMagic, kNetVersion, 0, k, next, nonce, L.chunkBytes, L.slots,
               o.channels};
    tncclResult r = netConnectEdge(ip, port, h, o, e->rings[(size_t)k].sendFds, o.timeoutMs);
    if (r == TNCCL_SUCCESS)
      r = netAcceptEdge(lfd, h, o, e->rings[(size_t)next].recvFds, o.timeoutMs);
    if (r == TNCCL_SUCCESS) r = netWaitAcks(e->rings[(size_t)k].sendFds, o.channels, o.timeoutMs);
    close(lfd);
    if (r != TNCCL_SUCCESS) return r;
  }
  for (int k = 0; k < P; ++k) {
    if (e->netSend[(size_t)k] == nullptr && e->netRecv[(size_t)k] == nullptr) continue;
    e->rings[(size_t)k].channels = o.channels;
    e->proxies[(size_t)k] = new (std::nothrow) NetProxy;
    if (e->proxies[(size_t)k] == nullptr) return TNCCL_SYSTEM_ERROR;
    tncclResult r = netProxyStart(e->proxies[(size_t)k], o, L, e->netSend[(size_t)k],
                                  e->netRecv[(size_t)k], &e->rings[(size_t)k], emuNetFailure, e);
    if (r != TNCCL_SUCCESS) return r;
  }
  e->net = true;
  return TNCCL_SUCCESS;
}

}  // namespace

extern "C" tncclResult tncclEmuCreate(tncclEmu_t* out, int nranks) {
  if (out == nullptr || nranks < 2 || nranks > kMaxEmulatedRanks) return TNCCL_INVALID_ARGUMENT;
  *out = nullptr;
  auto* e = new (std::nothrow) tncclEmu;
  if (e == nullptr) return TNCCL_SYSTEM_ERROR;
  e->nranks = nranks;
  e->cfg = loadConfig();
  adaptConfig(e->cfg, nranks);
  if (cudaGetDevice(&e->device) != cudaSuccess) {
    delete e;
    return TNCCL_CUDA_ERROR;
  }
  // Every CTA of every emulated rank must be resident at once.
  const int maxCtas = emulatedMaxCtas(e->cfg.threads);
  const int perRank = maxCtas / nranks;
  if (perRank < 1) {
    delete e;
    return TNCCL_UNSUPPORTED;
  }
  e->cfg.channels = std::min(e->cfg.channels, perRank);
  e->cfg.osChannels = std::min(e->cfg.osChannels, perRank);
  LayoutConfig lc{};
  lc.nranks = nranks;
  lc.channels = e->cfg.channels;
  lc.osChannels = e->cfg.osChannels;
  lc.ringSlots = e->cfg.ringSlots;
  lc.ringChunkBytes = (uint64_t)e->cfg.ringChunkBytes;
  lc.tsChunkBytes = (uint64_t)e->cfg.tsChunkBytes;
  lc.osSlots = e->cfg.osSlots;
  lc.osTileBytes = (uint64_t)e->cfg.osTileBytes;
  e->layout = makeLayout(lc);
  tncclResult r = TNCCL_SUCCESS;
  e->mailbox.assign((size_t)nranks, nullptr);
  std::vector<uint64_t> credits((size_t)e->layout.channels * e->layout.ringSlots);
  for (int c = 0; c < e->layout.channels; ++c)
    for (int s = 0; s < e->layout.ringSlots; ++s)
      credits[(size_t)c * e->layout.ringSlots + s] = (uint64_t)s;
  for (int k = 0; k < nranks && r == TNCCL_SUCCESS; ++k) {
    void* p = nullptr;
    if (cudaMalloc(&p, e->layout.totalBytes) != cudaSuccess ||
        cudaMemset(p, 0, e->layout.totalBytes) != cudaSuccess ||
        cudaMemcpy(static_cast<char*>(p) + e->layout.ringCreditOff, credits.data(),
                   credits.size() * 8, cudaMemcpyHostToDevice) != cudaSuccess)
      r = TNCCL_CUDA_ERROR;
    e->mailbox[(size_t)k] = static_cast<char*>(p);
  }
  const size_t cbytes = sizeof(uint64_t) * kNumCounterFamilies * kMaxChannels * (size_t)nranks;
  void* h = nullptr;
  void* d = nullptr;
  if (r == TNCCL_SUCCESS &&
      (cudaMalloc(reinterpret_cast<void**>(&e->counters), cbytes) != cudaSuccess ||
       cudaMemset(e->counters, 0, cbytes) != cudaSuccess ||
       cudaHostAlloc(&h, sizeof(DevStatus), cudaHostAllocMapped) != cudaSuccess ||
       cudaHostGetDevicePointer(&d, h, 0) != cudaSuccess))
    r = TNCCL_CUDA_ERROR;
  if (h) {
    memset(h, 0, sizeof(DevStatus));
    e->hostStatus = static_cast<DevStatus*>(h);
    e->devStatus = static_cast<DevStatus*>(d);
  }
  if (r != TNCCL_SUCCESS || cudaDeviceSynchronize() != cudaSuccess) {
    freeEmu(e);
    delete e;
    return r != TNCCL_SUCCESS ? r : TNCCL_CUDA_ERROR;
  }
  for (int k = 0; k < nranks; ++k) {
    DevComm& dc = e->dev[k];
    dc = DevComm{};
    dc.rank = k;
    dc.nranks = nranks;
    dc.layout = e->layout;
    for (int q = 0; q < nranks; ++q) dc.peers[q] = e->mailbox[(size_t)q];
    dc.counters = e->counters + (size_t)k * kNumCounterFamilies * kMaxChannels;
    dc.status = e->devStatus;
    dc.timeoutNs = (uint64_t)e->cfg.timeoutMs * 1000000ull;
    dc.tsSplit = e->cfg.tsSplit;
    dc.nvlsSplit = e->cfg.nvlsSplit;
    dc.acquireMode = e->cfg.acquireMode;
    dc.tsStages = e->cfg.tsStages;
    dc.tsPushStage = (uint32_t)e->cfg.tsPushStage;
    dc.tsRedStage = (uint32_t)e->cfg.tsRedStage;
    dc.nvlsStages = e->cfg.nvlsStages;
    dc.nvlsStage = (uint32_t)e->cfg.nvlsStage;
    dc.stageMinBytes = (uint32_t)e->cfg.stageMinBytes;
  }
  // Which ring edges are socket edges (edge k -> k+1).
  std::vector<char> socket((size_t)nranks, e->cfg.netMode == 2 ? 1 : 0);
  const std::string hosts = envStr("TNCCL_EMU_HOSTS", "");
  if (!hosts.empty()) {
    std::vector<long> ids;
    for (size_t pos = 0; pos <= hosts.size();) {
      const size_t comma = std::min(hosts.find(',', pos), hosts.size());
      ids.push_back(strtol(hosts.substr(pos, comma - pos).c_str(), nullptr, 10));
      pos = comma + 1;
    }
    if ((int)ids.size() != nranks) {
      freeEmu(e);
      delete e;
      return TNCCL_INVALID_ARGUMENT;
    }
    for (int k = 0; k < nranks; ++k)
      socket[(size_t)k] = ids[(size_t)k] != ids[(size_t)((k + 1) % nranks)] ? 1 : 0;
  }
  bool anySocket = false;
  for (char c : socket) anySocket = anySocket || c;
  if (anySocket) {
    r = setupEmuNet(e, socket);
    if (r != TNCCL_SUCCESS) {
      freeEmu(e);
      delete e;
      return r;
    }
  }
  *out = e;
  return TNCCL_SUCCESS;
}

extern "C" tncclResult tncclEmuAllReduce(tncclEmu_t e, const void* const* send,
                                         void* const* recv, size_t count, tncclDataType_t dtype,
                                         tncclRedOp_t op, float preScale, tncclAlgo_t algo,
                                         cudaStream_t stream) {
  const size_t es = elemSize(dtype);
  if (e == nullptr || send == nullptr || recv == nullptr || es == 0 || op < tncclSum ||
      op >= tncclNumOps)
    return TNCCL_INVALID_ARGUMENT;
  if (e->hostStatus->error != 0) return (tncclResult)e->hostStatus->error;
  if (algo == TNCCL_ALGO_AUTO) algo = TNCCL_ALGO_TWOSHOT;
  if (algo == TNCCL_ALGO_NVLS) return TNCCL_UNSUPPORTED;
  if (count == 0) return TNCCL_SUCCESS;
  const int P = e->nranks;
  EmulatedLaunch L{};
  L.nranks = P;
  L.algo = (int)algo;
  L.dtype = (int)dtype;
  const uint64_t V = kVectorBytes / es;
  const float scale = op == tncclAvg ? preScale / (float)P : preScale;
  int channels = 1;
  for (int k = 0; k < P; ++k) {
    if (send[k] == nullptr || recv[k] == nullptr) return TNCCL_INVALID_ARGUMENT;
    AllReduceArgs& a = L.args[k];
    a.send = send[k];
    a.recv = recv[k];
    a.count = count;
    a.scale = scale;
    a.dtype = (int)dtype;
    a.vectorized = (reinterpret_cast<uintptr_t>(send[k]) % kVectorBytes == 0 &&
                    reinterpret_cast<uintptr_t>(recv[k]) % kVectorBytes == 0)
                       ? 1
                       : 0;
    if (algo == TNCCL_ALGO_ONESHOT) {
      a.block = makeBlockPlan(count, e->cfg.osChannels, (uint64_t)e->cfg.osTileBytes / es,
                              kOneShotMinTileBytes / es, V);
      channels = a.block.channels;
    } else {
      const uint64_t maxChunk = (uint64_t)(algo == TNCCL_ALGO_RING ? e->cfg.ringChunkBytes
                                                                   : e->cfg.tsChunkBytes) / es;
      const uint64_t minChunk =
          (algo == TNCCL_ALGO_RING ? kRingMinChunkBytes : kTwoShotMinChunkBytes) / es;
      // Socket edges carry the first netLayout.channels ring channels only.
      const int ch = algo == TNCCL_ALGO_RING && e->net
                         ? std::min(e->cfg.channels, e->netLayout.channels)
                         : e->cfg.channels;
      a.chunk = makeChunkPlan(count, P, ch, maxChunk, minChunk, V);
      channels = a.chunk.channels;
    }
    L.comm[k] = e->dev[k];
  }
  // Every emulated rank must see the same vectorization choice (their tile
  // plans are identical); mixed alignment falls back to the scalar path.
  int vec = 1;
  for (int k = 0; k < P; ++k) vec &= L.args[k].vectorized;
  for (int k = 0; k < P; ++k) L.args[k].vectorized = vec;
  if (launchEmulated(L, channels, e->cfg.threads, stream) != cudaSuccess) return TNCCL_CUDA_ERROR;
  gLaunchCount.fetch_add(1, std::memory_order_relaxed);
  return TNCCL_SUCCESS;
}

extern "C" tncclResult tncclEmuGetAsyncError(tncclEmu_t e, tncclResult* err) {
  if (e == nullptr || err == nullptr) return TNCCL_INVALID_ARGUMENT;
  const int v = e->hostStatus->error;
  *err = v == 0 ? TNCCL_SUCCESS : v < TNCCL_NUM_RESULTS ? (tncclResult)v : TNCCL_SYSTEM_ERROR;
  return TNCCL_SUCCESS;
}

extern "C" tncclResult tncclEmuDestroy(tncclEmu_t e) {
  if (e == nullptr) return TNCCL_INVALID_ARGUMENT;
  const bool ok = cudaDeviceSynchronize() == cudaSuccess;
  freeEmu(e);
  delete e;
  return ok ? TNCCL_SUCCESS : TNCCL_CUDA_ERROR;
}
