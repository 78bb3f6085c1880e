// net.cc - socket ring edges and the proxy thread (see net.h).
#ifndef _GNU_SOURCE
#define _GNU_SOURCE
#endif

#include "net.h"

#include <errno.h>
#include <fcntl.h>
#include <poll.h>
#include <sched.h>
#include <string.h>
#include <sys/socket.h>
#include <sys/uio.h>
#include <time.h>
#include <unistd.h>

#include <algorithm>
#include <vector>

#include "common.h"
#include "sockio.h"

namespace tnccl {
namespace {

constexpr uint64_t H = kNetFrameHeaderBytes;

// The FIFO words are shared with the kernel (over PCIe / C2C for the GPU) or
// with the test's consumer threads: acquire / release on the flag words,
// relaxed on the size word, which the ready word orders.
uint64_t ldAcquire(const uint64_t* p) { return __atomic_load_n(p, __ATOMIC_ACQUIRE); }
uint64_t ldRelaxed(const uint64_t* p) { return __atomic_load_n(p, __ATOMIC_RELAXED); }
void stRelease(uint64_t* p, uint64_t v) { __atomic_store_n(p, v, __ATOMIC_RELEASE); }
void stRelaxed(uint64_t* p, uint64_t v) { __atomic_store_n(p, v, __ATOMIC_RELAXED); }

void fail(NetProxy* p, tncclResult code, int c, const char* what, uint64_t a = 0,
          uint64_t b = 0) {
  int expected = 0;
  if (p->error.compare_exchange_strong(expected, (int)code)) {
    TN_WARN("net proxy: channel %d: %s (%llu, %llu)", c, what, (unsigned long long)a,
            (unsigned long long)b);
    if (p->hook) p->hook(p->hookArg, code);
  }
}

// Send edge, one channel: wait for the kernel's next ready slot, write the
// frame (resuming partial writes), then credit the slot back.
bool stepSend(NetProxy* p, int c) {
  NetProxy::SendCh& s = p->send[c];
  const RingFifo& f = p->sendFifo;
  const int fd = p->ring->sendFds[c];
  const uint64_t i = ringFifoIndex(f, c, s.ticket);
  if (s.phase == 0) {
    if (ldAcquire(f.ready + i) < s.ticket + 1) return false;
    const uint64_t n = ldRelaxed(f.bytes + i);
    if (n > f.chunkBytes) {
      fail(p, TNCCL_SYSTEM_ERROR, c, "slot payload larger than the chunk", n, f.chunkBytes);
      return false;
    }
    netEncodeHeader(s.hdr, s.ticket, (uint32_t)n);
    s.bytes = n;
    s.off = 0;
    s.partial = false;
    s.phase = 1;
  }
  const uint64_t total = H + s.bytes;
  bool moved = false;
  while (s.off < total) {
    iovec iov[2];
    int k = 0;
    if (s.off < H) iov[k++] = iovec{s.hdr + s.off, (size_t)(H - s.off)};
    const uint64_t poff = s.off > H ? s.off - H : 0;
    if (s.bytes > poff)
      iov[k++] = iovec{ringFifoData(f, c, s.ticket) + poff, (size_t)(s.bytes - poff)};
    msghdr m{};
    m.msg_iov = iov;
    m.msg_iovlen = (size_t)k;
    ssize_t rc = sendmsg(fd, &m, MSG_NOSIGNAL | MSG_DONTWAIT);
    if (rc > 0) {
      if ((uint64_t)rc < total - s.off) s.partial = true;
      s.off += (uint64_t)rc;
      moved = true;
      continue;
    }
    if (rc < 0 && errno == EINTR) continue;
    if (rc < 0 && (errno == EAGAIN || errno == EWOULDBLOCK)) {
      s.partial = true;
      break;
    }
    fail(p, TNCCL_SYSTEM_ERROR, c, "send failed (errno, ticket)", (uint64_t)errno, s.ticket);
    return moved;
  }
  if (s.off < total) return moved;
  if (s.partial) p->partialWrites.fetch_add(1, std::memory_order_relaxed);
  stRelease(f.credit + i, s.ticket + (uint64_t)f.slots);
  p->framesSent.fetch_add(1, std::memory_order_relaxed);
  p->bytesSent.fetch_add(s.bytes, std::memory_order_relaxed);
  ++s.ticket;
  s.phase = 0;
  return true;
}

// Input on a send connection: only a close frame from downstream may arrive.
void readSendControl(NetProxy* p, int c) {
  NetProxy::SendCh& s = p->send[c];
  const int fd = p->ring->sendFds[c];
  for (;;) {
    ssize_t rc = recv(fd, s.ctl + s.ctlHave, H - (uint64_t)s.ctlHave, MSG_DONTWAIT);
    if (rc > 0) {
      s.ctlHave += (int)rc;
      if ((uint64_t)s.ctlHave < H) continue;
      uint64_t t;
      uint32_t n;
      netDecodeHeader(s.ctl, &t, &n);
      s.ctlHave = 0;
      if (t != kNetCloseTicket || n != 0 || s.peerClosed) {
        fail(p, TNCCL_SYSTEM_ERROR, c, "unexpected data on a send connection", t, n);
        return;
      }
      s.peerClosed = true;
      continue;
    }
    if (rc == 0) {
      if (!s.peerClosed || s.ctlHave != 0)
        fail(p, TNCCL_SYSTEM_ERROR, c, "downstream rank closed without a close frame", s.ticket);
      s.ctlEof = true;
      return;
    }
    if (errno == EINTR) continue;
    if (errno != EAGAIN && errno != EWOULDBLOCK)
      fail(p, TNCCL_SYSTEM_ERROR, c, "send connection failed (errno)", (uint64_t)errno);
    return;
  }
}

// Receive edge, one channel: read a header, wait until the kernel credited
// the slot, read the payload into it, publish size and ready.
bool stepRecv(NetProxy* p, int c) {
  NetProxy::RecvCh& s = p->recv[c];
  const RingFifo& f = p->recvFifo;
  const int fd = p->ring->recvFds[c];
  bool moved = false;
  for (;;) {
    if (s.phase == 0) {
      if (s.peerEof) return moved;
      ssize_t rc = recv(fd, s.hdr + s.hoff, H - s.hoff, MSG_DONTWAIT);
      if (rc > 0) {
        s.hoff += (uint64_t)rc;
        moved = true;
        if (s.hoff < H) continue;
        uint64_t t;
        uint32_t n;
        netDecodeHeader(s.hdr, &t, &n);
        s.hoff = 0;
        if (t == kNetCloseTicket && n == 0 && !s.peerClosed) {
          s.peerClosed = true;
          continue;
        }
        if (s.peerClosed) {
          fail(p, TNCCL_SYSTEM_ERROR, c, "frame after the close frame", t, n);
          return moved;
        }
        if (t != s.ticket) {
          fail(p, TNCCL_SYSTEM_ERROR, c, "unexpected ticket (got, expected)", t, s.ticket);
          return moved;
        }
        if (n > f.chunkBytes) {
          fail(p, TNCCL_SYSTEM_ERROR, c, "frame larger than a slot (bytes, chunk)", n,
               f.chunkBytes);
          return moved;
        }
        s.bytes = n;
        s.off = 0;
        s.partial = false;
        s.stalled = false;
        s.phase = 1;
        continue;
      }
      if (rc == 0) {
        if (s.peerClosed && s.hoff == 0) {
          s.peerEof = true;
          return moved;
        }
        fail(p, TNCCL_SYSTEM_ERROR, c, "upstream rank closed without a close frame", s.ticket);
        return moved;
      }
      if (errno == EINTR) continue;
      if (errno == EAGAIN || errno == EWOULDBLOCK) return moved;
      fail(p, TNCCL_SYSTEM_ERROR, c, "receive failed (errno)", (uint64_t)errno);
      return moved;
    }
    const uint64_t i = ringFifoIndex(f, c, s.ticket);
    if (s.phase == 1) {
      if (ldAcquire(f.credit + i) < s.ticket) {
        if (!s.stalled) {
          s.stalled = true;
          p->creditStalls.fetch_add(1, std::memory_order_relaxed);
        }
        return moved;
      }
      s.phase = 2;
    }
    char* dst = ringFifoData(f, c, s.ticket);
    while (s.off < s.bytes) {
      ssize_t rc = recv(fd, dst + s.off, s.bytes - s.off, MSG_DONTWAIT);
      if (rc > 0) {
        if ((uint64_t)rc < s.bytes - s.off) s.partial = true;
        s.off += (uint64_t)rc;
        moved = true;
        continue;
      }
      if (rc == 0) {
        fail(p, TNCCL_SYSTEM_ERROR, c, "upstream rank closed inside a frame", s.ticket);
        return moved;
      }
      if (errno == EINTR) continue;
      if (errno == EAGAIN || errno == EWOULDBLOCK) {
        s.partial = true;
        return moved;
      }
      fail(p, TNCCL_SYSTEM_ERROR, c, "receive failed (errno)", (uint64_t)errno);
      return moved;
    }
    stRelaxed(f.bytes + i, s.bytes);
    stRelease(f.ready + i, s.ticket + 1);
    p->framesReceived.fetch_add(1, std::memory_order_relaxed);
    p->bytesReceived.fetch_add(s.bytes, std::memory_order_relaxed);
    if (s.partial) p->partialReads.fetch_add(1, std::memory_order_relaxed);
    ++s.ticket;
    s.phase = 0;
    return true;  // one frame per call keeps the channels fair
  }
}

void proxyMain(NetProxy* p) {
  const int C = p->ring->channels;
  const bool hasSend = p->sendFifo.data != nullptr;
  const bool hasRecv = p->recvFifo.data != nullptr;
  auto last = Clock::now();
  std::vector<pollfd> pfds;
  std::vector<int> sendOf;  // pfds index -> send channel, or -1
  pfds.reserve(1 + 2 * (size_t)C);
  sendOf.reserve(1 + 2 * (size_t)C);
  while (!p->stop.load(std::memory_order_acquire) && p->error.load() == 0) {
    bool moved = false;
    for (int c = 0; c < C; ++c) {
      if (hasSend) moved |= stepSend(p, c);
      if (hasRecv) moved |= stepRecv(p, c);
    }
    if (p->error.load() != 0) break;
    const auto now = Clock::now();
    if (moved) {
      last = now;
      continue;
    }
    const int64_t idleUs =
        std::chrono::duration_cast<std::chrono::microseconds>(now - last).count();
    if (idleUs < p->opts.spinUs) {
      sched_yield();
      continue;
    }
    // Idle: sleep until a socket is ready or the stop pipe is written; while
    // a channel waits on a FIFO word that the kernel writes, wake up every
    // 50 us (every 1 ms after 10 ms without progress) to poll it.
    pfds.clear();
    sendOf.clear();
    pfds.push_back(pollfd{p->wakeFds[0], POLLIN, 0});
    sendOf.push_back(-1);
    bool flagWait = false;
    for (int c = 0; c < C; ++c) {
      if (hasSend) {
        const NetProxy::SendCh& s = p->send[c];
        short ev = 0;
        if (s.phase == 1) ev |= POLLOUT;
        else flagWait = true;
        if (!s.ctlEof) ev |= POLLIN | POLLRDHUP;
        if (ev) {
          pfds.push_back(pollfd{p->ring->sendFds[c], ev, 0});
          sendOf.push_back(c);
        }
      }
      if (hasRecv) {
        const NetProxy::RecvCh& s = p->recv[c];
        if (s.phase == 1) {
          flagWait = true;
        } else if (!s.peerEof) {
          pfds.push_back(pollfd{p->ring->recvFds[c], (short)(POLLIN | POLLRDHUP), 0});
          sendOf.push_back(-1);
        }
      }
    }
    const long waitNs = flagWait ? (idleUs < 10000 ? 50000L : 1000000L) : 100000000L;
    timespec ts{0, waitNs};
    int rc = ppoll(pfds.data(), (nfds_t)pfds.size(), &ts, nullptr);
    if (rc <= 0) continue;
    if (pfds[0].revents) {
      char buf[64];
      while (read(p->wakeFds[0], buf, sizeof(buf)) > 0) {
      }
    }
    for (size_t k = 1; k < pfds.size(); ++k) {
      if (sendOf[k] >= 0 && (pfds[k].revents & (POLLIN | POLLRDHUP | POLLHUP | POLLERR)))
        readSendControl(p, sendOf[k]);
    }
  }
}

void closeFds(int* fds, int n) {
  for (int c = 0; c < n; ++c) {
    if (fds[c] >= 0) close(fds[c]);
    fds[c] = -1;
  }
}

}  // namespace

void netFifoInit(char* base, const NetFifoLayout& L) {
  memset(base, 0, L.totalBytes);
  auto* credit = reinterpret_cast<uint64_t*>(base + L.creditOff);
  for (int c = 0; c < L.channels; ++c)
    for (int s = 0; s < L.slots; ++s) credit[(size_t)c * L.slots + s] = (uint64_t)s;
}

tncclResult netConnectEdge(uint32_t ipv4, int port, const NetHello& hello, const NetOptions& o,
                           int* fds, int timeoutMs) {
  const int C = hello.channels;
  if (C < 1 || C > kMaxNetChannels) return TNCCL_INVALID_ARGUMENT;
  for (int c = 0; c < C; ++c) fds[c] = -1;
  Deadline d = deadlineIn(timeoutMs);
  for (int c = 0; c < C; ++c) {
    Io why = Io::kOk;
    int fd = tcpConnect(ipv4, port, d, &why);
    if (fd < 0) {
      closeFds(fds, C);
      return toResult(why);
    }
    tcpTune(fd, o.sndBuf, o.rcvBuf);
    NetHello h = hello;
    h.channel = c;
    Io io = writeAll(fd, &h, sizeof(h), d);
    fds[c] = fd;
    if (io != Io::kOk) {
      closeFds(fds, C);
      return toResult(io);
    }
  }
  return TNCCL_SUCCESS;
}

tncclResult netAcceptEdge(int listenFd, const NetHello& expect, const NetOptions& o, int* fds,
                          int timeoutMs) {
  const int C = expect.channels;
  if (C < 1 || C > kMaxNetChannels) return TNCCL_INVALID_ARGUMENT;
  for (int c = 0; c < C; ++c) fds[c] = -1;
  Deadline d = deadlineIn(timeoutMs);
  int got = 0;
  tncclResult st = TNCCL_SUCCESS;
  while (got < C && st == TNCCL_SUCCESS) {
    Io why = Io::kOk;
    int fd = acceptOne(listenFd, d, &why);
    if (fd < 0) {
      TN_WARN("net: accepted %d of %d connections from rank %d", got, C, expect.src);
      st = toResult(why);
      break;
    }
    NetHello h{};
    // A connection gets one second for its hello, so a silent stray one
    // cannot use up the whole deadline.
    Io io = readAll(fd, &h, sizeof(h), std::min(d, deadlineIn(1000)));
    if (io != Io::kOk) {
      // Not one of ours (or it gave up): drop it and keep waiting.
      close(fd);
      continue;
    }
    NetHelloAck ack{kNetHelloMagic, TNCCL_SUCCESS, 0};
    if (h.magic != kNetHelloMagic || h.version != kNetVersion || h.nonce != expect.nonce) {
      // Another communicator's (or a stray) connection: refuse it, keep waiting.
      ack.status = TNCCL_INVALID_ARGUMENT;
      (void)writeAll(fd, &ack, sizeof(ack), d);
      close(fd);
      TN_INFO("net: refused a connection with a foreign hello");
      continue;
    }
    if (h.src != expect.src || h.dst != expect.dst || h.chunkBytes != expect.chunkBytes ||
        h.slots != expect.slots || h.channels != expect.channels || h.channel < 0 ||
        h.channel >= C || fds[h.channel] != -1) {
      ack.status = TNCCL_INVALID_ARGUMENT;
      (void)writeAll(fd, &ack, sizeof(ack), d);
      close(fd);
      TN_WARN("net: rank %d's hello does not match (src %d dst %d channel %d)", expect.src,
              h.src, h.dst, h.channel);
      st = TNCCL_INVALID_ARGUMENT;
      break;
    }
    io = writeAll(fd, &ack, sizeof(ack), d);
    if (io != Io::kOk) {
      close(fd);
      st = toResult(io);
      break;
    }
    tcpTune(fd, o.sndBuf, o.rcvBuf);
    fds[h.channel] = fd;
    ++got;
  }
  if (st != TNCCL_SUCCESS) closeFds(fds, C);
  return st;
}

tncclResult netWaitAcks(const int* fds, int channels, int timeoutMs) {
  Deadline d = deadlineIn(timeoutMs);
  for (int c = 0; c < channels; ++c) {
    NetHelloAck a{};
    Io io = readAll(fds[c], &a, sizeof(a), d);
    if (io != Io::kOk) return toResult(io);
    if (a.magic != kNetHelloMagic) return TNCCL_SYSTEM_ERROR;
    if (a.status != TNCCL_SUCCESS)
      return a.status > 0 && a.status < TNCCL_NUM_RESULTS ? (tncclResult)a.status
                                                          : TNCCL_SYSTEM_ERROR;
  }
  return TNCCL_SUCCESS;
}

tncclResult netConnectRing(Bootstrap* b, const NetOptions& o, const NetFifoLayout& L,
                           bool sendRemote, bool recvRemote, uint64_t nonce, NetRing* ring) {
  if (b == nullptr || !b->active || ring == nullptr) return TNCCL_INVALID_ARGUMENT;
  const int P = b->nranks, r = b->rank;
  const int next = (r + 1) % P, prev = (r + P - 1) % P;
  const int C = o.channels;
  struct Addr {
    uint32_t ip;
    int32_t port;
    int32_t status;
    int32_t listening;
  };
  Addr mine{0, 0, TNCCL_SUCCESS, 0};
  int lfd = -1;
  if (C < 1 || C > kMaxNetChannels || C > L.channels) {
    mine.status = TNCCL_INVALID_ARGUMENT;
  } else if (recvRemote) {
    uint32_t ip = 0;
    int port = 0;
    if (!parseIpv4(o.ifAddr, &ip)) {
      TN_WARN("net: TNCCL_NET_IF '%s' is not an IPv4 address", o.ifAddr);
      mine.status = TNCCL_INVALID_ARGUMENT;
    } else if ((lfd = tcpListen(o.ifAddr, 0, C + 8, &port)) < 0) {
      TN_WARN("net: cannot listen on %s: %s", o.ifAddr, strerror(errno));
      mine.status = TNCCL_SYSTEM_ERROR;
    } else {
      mine.ip = ip;
      mine.port = port;
      mine.listening = 1;
    }
  }
  std::vector<Addr> all((size_t)P);
  tncclResult res = bootstrapAllGather(b, &mine, all.data(), sizeof(Addr));
  if (res != TNCCL_SUCCESS) {
    if (lfd >= 0) close(lfd);
    return res;
  }
  tncclResult st = TNCCL_SUCCESS;
  for (const Addr& a : all)
    if (a.status != TNCCL_SUCCESS && st == TNCCL_SUCCESS) st = (tncclResult)a.status;
  ring->channels = C;
  NetHello base{kNetHelloMagic, kNetVersion, 0, 0, 0, nonce, L.chunkBytes, L.slots, C};
  if (st == TNCCL_SUCCESS && sendRemote) {
    if (!all[(size_t)next].listening) {
      st = TNCCL_INVALID_ARGUMENT;  // the ranks disagree about the edge
    } else {
      NetHello h = base;
      h.src = r;
      h.dst = next;
      st = netConnectEdge(all[(size_t)next].ip, all[(size_t)next].port, h, o, ring->sendFds,
                          o.timeoutMs);
    }
  }
  if (st == TNCCL_SUCCESS && recvRemote) {
    NetHello e = base;
    e.src = prev;
    e.dst = r;
    st = netAcceptEdge(lfd, e, o, ring->recvFds, o.timeoutMs);
  }
  if (st == TNCCL_SUCCESS && sendRemote) st = netWaitAcks(ring->sendFds, C, o.timeoutMs);
  if (lfd >= 0) close(lfd);
  int32_t mySt = st;
  std::vector<int32_t> sts((size_t)P);
  res = bootstrapAllGather(b, &mySt, sts.data(), sizeof(int32_t));
  if (res == TNCCL_SUCCESS)
    for (int32_t s : sts)
      if (s != TNCCL_SUCCESS && res == TNCCL_SUCCESS)
        res = s > 0 && s < TNCCL_NUM_RESULTS ? (tncclResult)s : TNCCL_SYSTEM_ERROR;
  if (res != TNCCL_SUCCESS) netCloseRing(ring);
  return res;
}

void netCloseRing(NetRing* ring) {
  if (ring == nullptr) return;
  closeFds(ring->sendFds, kMaxNetChannels);
  closeFds(ring->recvFds, kMaxNetChannels);
  ring->channels = 0;
}

tncclResult netProxyStart(NetProxy* p, const NetOptions& o, const NetFifoLayout& L,
                          char* sendFifo, char* recvFifo, NetRing* ring, NetFailureHook hook,
                          void* hookArg) {
  if (p == nullptr || p->running || ring == nullptr || ring->channels < 1 ||
      ring->channels > kMaxNetChannels || ring->channels > L.channels ||
      (sendFifo == nullptr && recvFifo == nullptr))
    return TNCCL_INVALID_ARGUMENT;
  for (int c = 0; c < ring->channels; ++c)
    if ((sendFifo && ring->sendFds[c] < 0) || (recvFifo && ring->recvFds[c] < 0))
      return TNCCL_INVALID_ARGUMENT;
  p->opts = o;
  p->layout = L;
  p->sendFifo = sendFifo ? netRingFifo(sendFifo, L) : RingFifo{};
  p->recvFifo = recvFifo ? netRingFifo(recvFifo, L) : RingFifo{};
  p->ring = ring;
  p->hook = hook;
  p->hookArg = hookArg;
  for (int c = 0; c < kMaxNetChannels; ++c) {
    p->send[c] = NetProxy::SendCh{};
    p->recv[c] = NetProxy::RecvCh{};
  }
  p->stop.store(0);
  p->error.store(0);
  p->framesSent = p->framesReceived = p->bytesSent = p->bytesReceived = 0;
  p->partialWrites = p->partialReads = p->creditStalls = 0;
  if (pipe2(p->wakeFds, O_NONBLOCK | O_CLOEXEC) != 0) return TNCCL_SYSTEM_ERROR;
  try {
    p->thread = std::thread(proxyMain, p);
  } catch (...) {
    close(p->wakeFds[0]);
    close(p->wakeFds[1]);
    p->wakeFds[0] = p->wakeFds[1] = -1;
    return TNCCL_SYSTEM_ERROR;
  }
  p->running = true;
  return TNCCL_SUCCESS;
}

tncclResult netProxyStop(NetProxy* p, bool graceful) {
  if (p == nullptr) return TNCCL_INVALID_ARGUMENT;
  if (!p->running) return (tncclResult)p->error.load();
  p->stop.store(1, std::memory_order_release);
  const char x = 1;
  (void)!write(p->wakeFds[1], &x, 1);
  p->thread.join();
  p->running = false;
  close(p->wakeFds[0]);
  close(p->wakeFds[1]);
  p->wakeFds[0] = p->wakeFds[1] = -1;
  const int err = p->error.load();
  if (graceful && err == 0) {
    unsigned char h[H];
    netEncodeHeader(h, kNetCloseTicket, 0);
    Deadline d = deadlineIn(std::min(p->opts.timeoutMs, 5000));
    for (int c = 0; c < p->ring->channels; ++c) {
      // A frame cut off in the middle cannot be followed by a close frame;
      // the peer then sees the connection end inside the stream.
      if (p->sendFifo.data && p->send[c].phase == 0) (void)writeAll(p->ring->sendFds[c], h, H, d);
      if (p->recvFifo.data) (void)writeAll(p->ring->recvFds[c], h, H, d);
    }
  }
  return (tncclResult)err;
}

}  // namespace tnccl
