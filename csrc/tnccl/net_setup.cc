// net_setup.cc - a communicator's socket ring edges: host identity, the
// host-mapped FIFOs the ring kernel shares with the proxy thread, connection
// set-up and the proxy's lifetime (the data path itself is net.cc).
//
// Lifetime follows tiny-nccl's socket design (docs/design-v0.2.md:143-147):
// the FIFOs are allocated before the connection status round of init; the
// proxy stops after destroy's first barrier (every kernel of every rank has
// finished), and the connections close and the FIFOs are freed after the
// second.
#include <arpa/inet.h>
#include <netinet/in.h>
#include <stdio.h>
#include <string.h>
#include <sys/socket.h>
#include <unistd.h>

#include <new>
#include <vector>

#include "comm.h"
#include "sockio.h"

namespace tnccl {
namespace {

void mixBytes(uint64_t& h, const void* p, size_t n) {
  const auto* b = static_cast<const unsigned char*>(p);
  for (size_t i = 0; i < n; ++i) {
    h ^= b[i];
    h *= 1099511628211ull;
  }
}

// Proxy failure: record it in the host-mapped status block that every device
// wait polls (first error wins), so waiting kernels return.
void onNetFailure(void* arg, tncclResult code) {
  auto* comm = static_cast<tncclComm*>(arg);
  auto* err = const_cast<int32_t*>(&comm->hostStatus->error);
  int32_t expected = 0;
  if (__atomic_compare_exchange_n(err, &expected, (int32_t)code, false, __ATOMIC_SEQ_CST,
                                  __ATOMIC_SEQ_CST))
    TN_WARN("rank %d: socket ring edge failed; collectives on this communicator now fail",
            comm->rank);
}

// The IPv4 address this rank listens on: TNCCL_NET_IF, else the local
// address that routes to rank 0's bootstrap address (TCP bootstrap), else
// loopback (one host).
bool listenAddress(const tncclComm* comm, char (&out)[64]) {
  if (!comm->cfg.netIf.empty()) {
    snprintf(out, sizeof(out), "%s", comm->cfg.netIf.c_str());
    return true;
  }
  snprintf(out, sizeof(out), "127.0.0.1");
  if (!comm->bootstrap.tcp) return true;
  int fd = socket(AF_INET, SOCK_DGRAM | SOCK_CLOEXEC, 0);
  if (fd < 0) return false;
  sockaddr_in a{};
  a.sin_family = AF_INET;
  a.sin_addr.s_addr = comm->bootstrap.hubIpv4;
  a.sin_port = htons(9);  // a UDP connect only selects the route
  bool ok = connect(fd, reinterpret_cast<sockaddr*>(&a), sizeof(a)) == 0;
  socklen_t len = sizeof(a);
  ok = ok && getsockname(fd, reinterpret_cast<sockaddr*>(&a), &len) == 0;
  close(fd);
  if (!ok) return false;
  return inet_ntop(AF_INET, &a.sin_addr, out, sizeof(out)) != nullptr;
}

}  // namespace

uint64_t hostIdentity() {
  uint64_t h = 1469598103934665603ull;
  const std::string forced = envStr("TNCCL_HOST_ID", "");
  if (!forced.empty()) {
    mixBytes(h, "id:", 3);
    mixBytes(h, forced.data(), forced.size());
    return h;
  }
  char host[256] = {};
  gethostname(host, sizeof(host) - 1);
  mixBytes(h, host, strlen(host));
  FILE* f = fopen("/proc/sys/kernel/random/boot_id", "r");
  if (f) {
    char boot[64] = {};
    const size_t n = fread(boot, 1, sizeof(boot) - 1, f);
    fclose(f);
    mixBytes(h, boot, n);
  }
  return h;
}

tncclResult netAllocFifos(tncclComm* comm) {
  NetState& n = comm->net;
  n.layout = makeNetFifoLayout(comm->cfg.netChannels, comm->cfg.ringSlots,
                               (uint64_t)comm->cfg.ringChunkBytes);
  auto alloc = [&](char** host, char** dev) -> tncclResult {
    void* h = nullptr;
    if (cudaHostAlloc(&h, n.layout.totalBytes, cudaHostAllocMapped | cudaHostAllocPortable) !=
        cudaSuccess) {
      (void)cudaGetLastError();
      return TNCCL_CUDA_ERROR;
    }
    netFifoInit(static_cast<char*>(h), n.layout);
    void* d = nullptr;
    if (cudaHostGetDevicePointer(&d, h, 0) != cudaSuccess) {
      (void)cudaGetLastError();
      cudaFreeHost(h);
      return TNCCL_CUDA_ERROR;
    }
    *host = static_cast<char*>(h);
    *dev = static_cast<char*>(d);
    return TNCCL_SUCCESS;
  };
  tncclResult r = TNCCL_SUCCESS;
  if (n.send) r = alloc(&n.sendHost, &n.sendDev);
  if (r == TNCCL_SUCCESS && n.recv) r = alloc(&n.recvHost, &n.recvDev);
  return r;
}

tncclResult netStart(tncclComm* comm, uint64_t nonce) {
  NetState& n = comm->net;
  NetOptions o;
  o.channels = comm->cfg.netChannels;
  o.sndBuf = o.rcvBuf = comm->cfg.netSockBuf;
  o.spinUs = comm->cfg.netSpinUs;
  o.timeoutMs = (int)comm->cfg.bootstrapTimeoutMs;
  if ((n.send || n.recv) && !listenAddress(comm, o.ifAddr)) {
    // An empty address fails this rank's entry of the address all-gather,
    // so every rank's netConnectRing returns the error.
    TN_WARN("rank %d: no local address routes to rank 0; set TNCCL_NET_IF", comm->rank);
    o.ifAddr[0] = '\0';
  }
  tncclResult r = netConnectRing(&comm->bootstrap, o, n.layout, n.send, n.recv, nonce, &n.ring);
  if (r != TNCCL_SUCCESS) return r;
  int32_t st = TNCCL_SUCCESS;
  if (n.send || n.recv) {
    n.proxy = new (std::nothrow) NetProxy;
    st = n.proxy == nullptr ? TNCCL_SYSTEM_ERROR
                            : netProxyStart(n.proxy, o, n.layout, n.sendHost, n.recvHost,
                                            &n.ring, onNetFailure, comm);
  }
  std::vector<int32_t> all((size_t)comm->nranks);
  r = bootstrapAllGather(&comm->bootstrap, &st, all.data(), sizeof(st));
  if (r != TNCCL_SUCCESS) return r;
  for (int32_t s : all)
    if (s != TNCCL_SUCCESS)
      return s > 0 && s < TNCCL_NUM_RESULTS ? (tncclResult)s : TNCCL_SYSTEM_ERROR;
  TN_INFO("rank %d: socket ring edges: send %s, recv %s, %d channel(s), listen %s", comm->rank,
          n.send ? "socket" : "nvlink", n.recv ? "socket" : "nvlink", o.channels, o.ifAddr);
  return TNCCL_SUCCESS;
}

void netStopProxy(tncclComm* comm, bool graceful, tncclResult* result) {
  NetState& n = comm->net;
  if (n.proxy == nullptr) return;
  tncclResult st = netProxyStop(n.proxy, graceful);
  if (graceful && st != TNCCL_SUCCESS && result && *result == TNCCL_SUCCESS) *result = st;
  delete n.proxy;
  n.proxy = nullptr;
}

void netRelease(tncclComm* comm, bool freeFifos) {
  NetState& n = comm->net;
  netCloseRing(&n.ring);
  if (!freeFifos) return;  // a kernel may still use them: retained
  if (n.sendHost) cudaFreeHost(n.sendHost);
  if (n.recvHost) cudaFreeHost(n.recvHost);
  n.sendHost = n.recvHost = n.sendDev = n.recvDev = nullptr;
}

}  // namespace tnccl
