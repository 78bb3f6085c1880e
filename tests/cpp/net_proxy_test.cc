// net_proxy_test.cc - CPU tests of the socket ring edges (csrc/tnccl/net.cc):
// TCP connection set-up over the real bootstrap, the proxy thread, and the
// ring protocol of the GPU ring kernel run by host threads over
// RingFifo views, so NVLink edges (shared memory) and socket edges (host
// FIFO + proxy + loopback TCP) mix in one ring.
//
// Checks (the completion criteria of tiny-nccl's socket data-plane design,
// docs/design-v0.2.md:198-207, without a GPU):
//  * frame header codec; FIFO layout; NVLink-edge RingFifo addresses equal
//    the mailbox layout's ring offsets (the kernel's local path);
//  * one edge, 1-3 channels, random payload sizes (0 .. chunk), small socket
//    buffers and a slow consumer: every byte in order, partial reads and
//    writes and credit stalls observed, FIFOs bounded, clean close;
//  * ring all-reduce on P = 2, 3, 4 ranks with every edge a socket edge and
//    with mixed edges, tiny-nccl's count matrix plus 1,000,003 elements,
//    several collectives in a row, bit-exact against the ring oracle;
//  * failures, all made on the host: a downstream or upstream peer that
//    closes without a close frame, an out-of-order ticket, an oversized
//    frame, a foreign hello (refused, the edge still connects), a mismatched
//    hello (edge fails), a rank that dies inside a collective (the others'
//    waits end through the failure hook, long before their timeout), random
//    bytes on a receive connection (a recorded failure, nothing written
//    past the FIFO);
//  * no descriptor leaks.
#include <dirent.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <functional>
#include <memory>
#include <random>
#include <thread>
#include <vector>

#include "bootstrap.h"
#include "net.h"
#include "oracle.h"
#include "protocol.h"
#include "sockio.h"

using namespace tnccl;

namespace {

int gFailed = 0;
auto gLast = std::chrono::steady_clock::now();
void report(const char* what, bool ok) {
  const auto now = std::chrono::steady_clock::now();
  printf("%-60s %s (%.2f s)\n", what, ok ? "ok" : "FAILED",
         std::chrono::duration<double>(now - gLast).count());
  gLast = now;
  fflush(stdout);
  if (!ok) ++gFailed;
}

int countFds() {
  int n = 0;
  DIR* d = opendir("/proc/self/fd");
  if (!d) return -1;
  while (readdir(d)) ++n;
  closedir(d);
  return n;
}

using Ms = std::chrono::milliseconds;
using std::chrono::steady_clock;

// Host buffer of 8-byte words (FIFO words must be 8-byte aligned).
struct Buf {
  std::vector<uint64_t> w;
  explicit Buf(uint64_t bytes = 0) : w((size_t)((bytes + 7) / 8), 0) {}
  char* p() { return reinterpret_cast<char*>(w.data()); }
};

// Bounded wait on a FIFO word; gives up on `error` or after `ms`.
bool waitWord(const uint64_t* word, uint64_t want, const std::atomic<int>& error, int ms) {
  auto start = steady_clock::now();
  uint64_t spins = 0;
  while (__atomic_load_n(word, __ATOMIC_ACQUIRE) < want) {
    if ((++spins & 255) == 0) {
      if (error.load()) return false;
      if (steady_clock::now() - start > Ms(ms)) return false;
      std::this_thread::yield();
    }
  }
  return true;
}

void hookSetError(void* arg, tncclResult code) {
  static_cast<std::atomic<int>*>(arg)->store((int)code);
}

// ---------------------------------------------------------------------------
void testCodecAndLayout() {
  bool ok = true;
  const uint64_t tickets[] = {0, 1, 255, 256, 0x0123456789abcdefull, kNetCloseTicket};
  const uint32_t sizes[] = {0, 1, 65535, 65536, 0xfedcba98u};
  for (uint64_t t : tickets)
    for (uint32_t n : sizes) {
      unsigned char h[kNetFrameHeaderBytes];
      netEncodeHeader(h, t, n);
      uint64_t t2;
      uint32_t n2;
      netDecodeHeader(h, &t2, &n2);
      ok = ok && t2 == t && n2 == n;
    }
  unsigned char h[kNetFrameHeaderBytes];
  netEncodeHeader(h, 0x0102030405060708ull, 0x0a0b0c0du);
  ok = ok && h[0] == 1 && h[7] == 8 && h[8] == 0x0a && h[11] == 0x0d;  // big-endian
  report("frame header codec (big-endian)", ok);

  ok = true;
  for (int C : {1, 2, 3, 8})
    for (int S : {1, 2, 4, 8})
      for (uint64_t chunk : {16ull, 4096ull, 262144ull}) {
        NetFifoLayout L = makeNetFifoLayout(C, S, chunk);
        const uint64_t n = (uint64_t)C * S;
        ok = ok && L.readyOff >= n * chunk && L.readyOff % 128 == 0 &&
             L.creditOff >= L.readyOff + n * 8 && L.creditOff % 128 == 0 &&
             L.bytesOff >= L.creditOff + n * 8 && L.bytesOff % 128 == 0 &&
             L.totalBytes >= L.bytesOff + n * 8 && L.totalBytes % 4096 == 0;
        Buf b(L.totalBytes);
        netFifoInit(b.p(), L);
        RingFifo f = netRingFifo(b.p(), L);
        for (int c = 0; c < C; ++c)
          for (int s = 0; s < S; ++s) {
            const uint64_t i = ringFifoIndex(f, c, (uint64_t)s + 7ull * S);
            ok = ok && i == (uint64_t)c * S + s && f.credit[i] == (uint64_t)s && f.ready[i] == 0;
            ok = ok && ringFifoData(f, c, (uint64_t)s) + chunk <= b.p() + L.readyOff;
          }
      }
  report("socket FIFO layout and initial credits", ok);

  // The kernel's NVLink edge goes through nvlinkRingFifo: its addresses must
  // be the mailbox layout's ring offsets.
  ok = true;
  std::mt19937_64 g(7);
  for (int it = 0; it < 200; ++it) {
    LayoutConfig lc{};
    lc.nranks = 2 + (int)(g() % 7);
    lc.channels = 1 + (int)(g() % 128);
    lc.osChannels = 1 + (int)(g() % 64);
    lc.ringSlots = 1 + (int)(g() % 8);
    lc.ringChunkBytes = 16 * (1 + g() % 16384);
    lc.tsChunkBytes = 16 * (1 + g() % 4096);
    lc.osSlots = 1 + (int)(g() % 4);
    lc.osTileBytes = 16 * (1 + g() % 2048);
    MailboxLayout L = makeLayout(lc);
    char* cons = reinterpret_cast<char*>(0x100000000ull);
    char* prod = reinterpret_cast<char*>(0x900000000ull);
    RingFifo f = nvlinkRingFifo(cons, prod, L);
    for (int k = 0; k < 20; ++k) {
      const int c = (int)(g() % (uint64_t)lc.channels);
      const uint64_t t = g() % 100000;
      const int s = (int)(t % (uint64_t)lc.ringSlots);
      const uint64_t i = ringFifoIndex(f, c, t);
      ok = ok && ringFifoData(f, c, t) == cons + ringDataAt(L, c, s);
      ok = ok && reinterpret_cast<char*>(f.ready + i) == cons + ringReadyAt(L, c, s);
      ok = ok && reinterpret_cast<char*>(f.credit + i) == prod + ringCreditAt(L, c, s);
      ok = ok && f.bytes == nullptr;
    }
  }
  report("NVLink-edge RingFifo == mailbox ring offsets", ok);
}

// ---------------------------------------------------------------------------
// One socket edge A -> B set up by hand (no bootstrap).
struct Edge {
  NetRing a, b;  // a: send side, b: receive side
  bool ok = false;
};

Edge connectEdge(int C, const NetOptions& o, uint64_t nonce = 42) {
  Edge e;
  int port = 0;
  int lfd = tcpListen("127.0.0.1", 0, 16, &port);
  if (lfd < 0) return e;
  uint32_t ip = 0;
  parseIpv4("127.0.0.1", &ip);
  NetFifoLayout L = makeNetFifoLayout(C, 4, 4096);
  NetHello h{kNetHelloMagic, kNetVersion, 0, 0, 1, nonce, L.chunkBytes, L.slots, C};
  tncclResult r1 = netConnectEdge(ip, port, h, o, e.a.sendFds, 5000);
  tncclResult r2 = r1 == TNCCL_SUCCESS ? netAcceptEdge(lfd, h, o, e.b.recvFds, 5000) : r1;
  tncclResult r3 = r2 == TNCCL_SUCCESS ? netWaitAcks(e.a.sendFds, C, 5000) : r2;
  close(lfd);
  e.a.channels = e.b.channels = C;
  e.ok = r3 == TNCCL_SUCCESS;
  return e;
}

uint8_t pattern(uint64_t t, int c, uint64_t i) { return (uint8_t)(t * 131 + (uint64_t)c * 7 + i); }

void testStream() {
  for (int C : {1, 3}) {
    NetOptions o;
    o.channels = C;
    // Frames up to 4x the socket buffers force partial writes and reads.
    // (Buffers below a few loopback MSS (64 KiB) stall TCP's window updates
    // for the persist timer, which tests nothing of ours.)
    o.sndBuf = 256 << 10;
    o.rcvBuf = 256 << 10;
    o.spinUs = 50;
    const int S = 4;
    const uint64_t chunk = 1 << 20;
    const uint64_t N = 64;  // frames per channel
    NetFifoLayout L = makeNetFifoLayout(C, S, chunk);
    // The hello carries the layout, so connect with this one.
    Edge e;
    {
      int port = 0;
      int lfd = tcpListen("127.0.0.1", 0, 16, &port);
      uint32_t ip = 0;
      parseIpv4("127.0.0.1", &ip);
      NetHello h{kNetHelloMagic, kNetVersion, 0, 0, 1, 99, chunk, S, C};
      bool ok = lfd >= 0 && netConnectEdge(ip, port, h, o, e.a.sendFds, 5000) == TNCCL_SUCCESS &&
                netAcceptEdge(lfd, h, o, e.b.recvFds, 5000) == TNCCL_SUCCESS &&
                netWaitAcks(e.a.sendFds, C, 5000) == TNCCL_SUCCESS;
      if (lfd >= 0) close(lfd);
      e.a.channels = e.b.channels = C;
      e.ok = ok;
    }
    Buf sendBuf(L.totalBytes), recvBuf(L.totalBytes);
    netFifoInit(sendBuf.p(), L);
    netFifoInit(recvBuf.p(), L);
    std::atomic<int> errA{0}, errB{0};
    NetProxy pa, pb;
    bool ok = e.ok &&
              netProxyStart(&pa, o, L, sendBuf.p(), nullptr, &e.a, hookSetError, &errA) ==
                  TNCCL_SUCCESS &&
              netProxyStart(&pb, o, L, nullptr, recvBuf.p(), &e.b, hookSetError, &errB) ==
                  TNCCL_SUCCESS;
    RingFifo out = netRingFifo(sendBuf.p(), L), in = netRingFifo(recvBuf.p(), L);
    std::atomic<int> bad{0};
    std::atomic<uint64_t> maxAhead{0};
    std::atomic<uint64_t> consumed{0};
    std::vector<uint64_t> sizes((size_t)C * N);
    std::mt19937_64 g(1234 + C);
    for (auto& s : sizes) {
      const uint64_t k = g() % 8;
      s = k == 0 ? 0 : k == 1 ? chunk : g() % (chunk + 1);
    }
    std::thread producer([&] {
      for (uint64_t t = 0; t < N && ok && !bad.load(); ++t)
        for (int c = 0; c < C; ++c) {
          const uint64_t i = ringFifoIndex(out, c, t);
          if (!waitWord(out.credit + i, t, errA, 10000)) {
            bad = 1;
            return;
          }
          const uint64_t n = sizes[(size_t)c * N + t];
          char* d = ringFifoData(out, c, t);
          for (uint64_t k = 0; k < n; ++k) d[k] = (char)pattern(t, c, k);
          __atomic_store_n(out.bytes + i, n, __ATOMIC_RELAXED);
          __atomic_store_n(out.ready + i, t + 1, __ATOMIC_RELEASE);
          const uint64_t ahead = (t + 1) * C - consumed.load();
          if (ahead > maxAhead.load()) maxAhead = ahead;
        }
    });
    std::thread consumer([&] {
      std::mt19937_64 r(99);
      for (uint64_t t = 0; t < N && ok && !bad.load(); ++t)
        for (int c = 0; c < C; ++c) {
          const uint64_t i = ringFifoIndex(in, c, t);
          if (!waitWord(in.ready + i, t + 1, errB, 10000)) {
            bad = 2;
            return;
          }
          const uint64_t n = __atomic_load_n(in.bytes + i, __ATOMIC_RELAXED);
          if (n != sizes[(size_t)c * N + t]) bad = 3;
          const char* d = ringFifoData(in, c, t);
          for (uint64_t k = 0; k < n && !bad.load(); ++k)
            if ((uint8_t)d[k] != pattern(t, c, k)) bad = 4;
          if (r() % 16 == 0) std::this_thread::sleep_for(std::chrono::microseconds(300));
          __atomic_store_n(in.credit + i, t + (uint64_t)S, __ATOMIC_RELEASE);
          consumed.fetch_add(1);
        }
    });
    producer.join();
    consumer.join();
    tncclResult sa = netProxyStop(&pa, true), sb = netProxyStop(&pb, true);
    const uint64_t frames = (uint64_t)C * N;
    char name[96];
    snprintf(name, sizeof(name), "stream %d channel(s): %llu frames intact, in order", C,
             (unsigned long long)frames);
    report(name, ok && bad.load() == 0 && sa == TNCCL_SUCCESS && sb == TNCCL_SUCCESS &&
                     errA.load() == 0 && errB.load() == 0 && pa.framesSent == frames &&
                     pb.framesReceived == frames);
    snprintf(name, sizeof(name), "stream %d channel(s): partial I/O + credit stalls seen", C);
    report(name, pa.partialWrites.load() + pb.partialReads.load() > 0 &&
                     pb.creditStalls.load() > 0);
    // Bounded: at most S slots in the send FIFO, S in the receive FIFO and
    // what the two socket buffers hold (frames are >= 12 bytes) per channel.
    snprintf(name, sizeof(name), "stream %d channel(s): producer lead bounded (%llu)", C,
             (unsigned long long)maxAhead.load());
    const uint64_t sockFrames = 4 * (uint64_t)(o.sndBuf + o.rcvBuf) / kNetFrameHeaderBytes;  // 4x: kernel overhead
    report(name, maxAhead.load() <= (uint64_t)C * (2 * S + sockFrames));
    netCloseRing(&e.a);
    netCloseRing(&e.b);
  }
}

// Throughput of one socket edge over loopback TCP: full frames of `chunk`
// bytes on C channels through both proxies, host-memory FIFOs, no payload
// writes or checks (the producer only publishes sizes). Returns GB/s of
// payload, or a negative value on failure.
double measureStream(int C, uint64_t chunk, uint64_t totalBytes) {
  NetOptions o;
  o.channels = C;
  o.spinUs = 200;
  const int S = 4;
  const uint64_t N = totalBytes / (chunk * (uint64_t)C);  // frames per channel
  NetFifoLayout L = makeNetFifoLayout(C, S, chunk);
  Edge e;
  {
    int port = 0;
    int lfd = tcpListen("127.0.0.1", 0, 16, &port);
    uint32_t ip = 0;
    parseIpv4("127.0.0.1", &ip);
    NetHello h{kNetHelloMagic, kNetVersion, 0, 0, 1, 77, chunk, S, C};
    e.ok = lfd >= 0 && netConnectEdge(ip, port, h, o, e.a.sendFds, 5000) == TNCCL_SUCCESS &&
           netAcceptEdge(lfd, h, o, e.b.recvFds, 5000) == TNCCL_SUCCESS &&
           netWaitAcks(e.a.sendFds, C, 5000) == TNCCL_SUCCESS;
    if (lfd >= 0) close(lfd);
    e.a.channels = e.b.channels = C;
  }
  Buf sendBuf(L.totalBytes), recvBuf(L.totalBytes);
  netFifoInit(sendBuf.p(), L);
  netFifoInit(recvBuf.p(), L);
  std::atomic<int> errA{0}, errB{0}, bad{0};
  NetProxy pa, pb;
  const bool ok = e.ok &&
                  netProxyStart(&pa, o, L, sendBuf.p(), nullptr, &e.a, hookSetError, &errA) ==
                      TNCCL_SUCCESS &&
                  netProxyStart(&pb, o, L, nullptr, recvBuf.p(), &e.b, hookSetError, &errB) ==
                      TNCCL_SUCCESS;
  RingFifo out = netRingFifo(sendBuf.p(), L), in = netRingFifo(recvBuf.p(), L);
  const auto t0 = steady_clock::now();
  std::thread producer([&] {
    for (uint64_t t = 0; t < N && ok && !bad.load(); ++t)
      for (int c = 0; c < C; ++c) {
        const uint64_t i = ringFifoIndex(out, c, t);
        if (!waitWord(out.credit + i, t, errA, 20000)) {
          bad = 1;
          return;
        }
        __atomic_store_n(out.bytes + i, chunk, __ATOMIC_RELAXED);
        __atomic_store_n(out.ready + i, t + 1, __ATOMIC_RELEASE);
      }
  });
  std::thread consumer([&] {
    for (uint64_t t = 0; t < N && ok && !bad.load(); ++t)
      for (int c = 0; c < C; ++c) {
        const uint64_t i = ringFifoIndex(in, c, t);
        if (!waitWord(in.ready + i, t + 1, errB, 20000)) {
          bad = 2;
          return;
        }
        if (__atomic_load_n(in.bytes + i, __ATOMIC_RELAXED) != chunk) bad = 3;
        __atomic_store_n(in.credit + i, t + (uint64_t)S, __ATOMIC_RELEASE);
      }
  });
  producer.join();
  consumer.join();
  const double sec = std::chrono::duration<double>(steady_clock::now() - t0).count();
  const tncclResult sa = netProxyStop(&pa, true), sb = netProxyStop(&pb, true);
  netCloseRing(&e.a);
  netCloseRing(&e.b);
  if (!ok || bad.load() || sa != TNCCL_SUCCESS || sb != TNCCL_SUCCESS) return -1.0;
  return (double)(N * (uint64_t)C * chunk) / sec / 1e9;
}

// ---------------------------------------------------------------------------
// Failure paths of one edge.
void testEdgeFailures() {
  NetOptions o;
  o.channels = 1;
  o.spinUs = 20;
  const NetFifoLayout L = makeNetFifoLayout(1, 4, 4096);

  // Downstream closes without a close frame while upstream has traffic.
  {
    Edge e = connectEdge(1, o);
    Buf sb(L.totalBytes);
    netFifoInit(sb.p(), L);
    std::atomic<int> err{0};
    NetProxy pa;
    bool ok = e.ok && netProxyStart(&pa, o, L, sb.p(), nullptr, &e.a, hookSetError, &err) ==
                          TNCCL_SUCCESS;
    netCloseRing(&e.b);  // the receiving rank dies
    RingFifo out = netRingFifo(sb.p(), L);
    auto t0 = steady_clock::now();
    for (uint64_t t = 0; t < 64 && ok && !err.load(); ++t) {
      const uint64_t i = ringFifoIndex(out, 0, t);
      if (!waitWord(out.credit + i, t, err, 3000)) break;
      __atomic_store_n(out.bytes + i, 4096, __ATOMIC_RELAXED);
      __atomic_store_n(out.ready + i, t + 1, __ATOMIC_RELEASE);
    }
    while (ok && !err.load() && steady_clock::now() - t0 < Ms(3000))
      std::this_thread::sleep_for(Ms(1));
    const double ms = std::chrono::duration<double, std::milli>(steady_clock::now() - t0).count();
    netProxyStop(&pa, false);
    netCloseRing(&e.a);
    report("downstream closes without close frame -> failure", ok && err.load() != 0 && ms < 3000);
  }

  // Upstream sends two frames, then closes without a close frame.
  {
    Edge e = connectEdge(1, o);
    Buf rb(L.totalBytes);
    netFifoInit(rb.p(), L);
    std::atomic<int> err{0};
    NetProxy pb;
    bool ok = e.ok && netProxyStart(&pb, o, L, nullptr, rb.p(), &e.b, hookSetError, &err) ==
                          TNCCL_SUCCESS;
    unsigned char frame[kNetFrameHeaderBytes + 8] = {};
    Deadline d = deadlineIn(2000);
    for (uint64_t t = 0; t < 2 && ok; ++t) {
      netEncodeHeader(frame, t, 8);
      ok = writeAll(e.a.sendFds[0], frame, sizeof(frame), d) == Io::kOk;
    }
    RingFifo in = netRingFifo(rb.p(), L);
    std::atomic<int> none{0};
    ok = ok && waitWord(in.ready + ringFifoIndex(in, 0, 1), 2, none, 2000) && err.load() == 0;
    netCloseRing(&e.a);  // the sending rank dies
    auto t0 = steady_clock::now();
    while (ok && !err.load() && steady_clock::now() - t0 < Ms(3000))
      std::this_thread::sleep_for(Ms(1));
    netProxyStop(&pb, false);
    netCloseRing(&e.b);
    report("upstream closes without close frame -> failure", ok && err.load() != 0);
  }

  // Out-of-order ticket, then an oversized frame.
  for (int kind = 0; kind < 2; ++kind) {
    Edge e = connectEdge(1, o);
    Buf rb(L.totalBytes);
    netFifoInit(rb.p(), L);
    std::atomic<int> err{0};
    NetProxy pb;
    bool ok = e.ok && netProxyStart(&pb, o, L, nullptr, rb.p(), &e.b, hookSetError, &err) ==
                          TNCCL_SUCCESS;
    unsigned char hdr[kNetFrameHeaderBytes];
    Deadline d = deadlineIn(2000);
    if (kind == 0) {
      netEncodeHeader(hdr, 0, 0);
      ok = ok && writeAll(e.a.sendFds[0], hdr, sizeof(hdr), d) == Io::kOk;
      netEncodeHeader(hdr, 2, 0);  // ticket 1 expected
    } else {
      netEncodeHeader(hdr, 0, (uint32_t)L.chunkBytes + 1);
    }
    ok = ok && writeAll(e.a.sendFds[0], hdr, sizeof(hdr), d) == Io::kOk;
    auto t0 = steady_clock::now();
    while (ok && !err.load() && steady_clock::now() - t0 < Ms(3000))
      std::this_thread::sleep_for(Ms(1));
    netProxyStop(&pb, false);
    netCloseRing(&e.a);
    netCloseRing(&e.b);
    report(kind == 0 ? "out-of-order ticket -> failure" : "frame larger than a slot -> failure",
           ok && err.load() != 0 && pb.framesReceived.load() == (kind == 0 ? 1u : 0u));
  }

  // A foreign hello is refused and the edge still connects; a hello with the
  // right nonce but the wrong ranks fails the edge.
  for (int kind = 0; kind < 2; ++kind) {
    int port = 0;
    int lfd = tcpListen("127.0.0.1", 0, 16, &port);
    uint32_t ip = 0;
    parseIpv4("127.0.0.1", &ip);
    NetHello good{kNetHelloMagic, kNetVersion, 0, 3, 4, 777, 4096, 4, 1};
    NetHello bad = good;
    if (kind == 0) bad.nonce = 778;
    else bad.src = 5;
    tncclResult acc = TNCCL_SYSTEM_ERROR;
    int fdsB[kMaxNetChannels];
    std::thread acceptor([&] { acc = netAcceptEdge(lfd, good, o, fdsB, 3000); });
    int fdsBad[kMaxNetChannels], fdsGood[kMaxNetChannels];
    tncclResult c1 = netConnectEdge(ip, port, bad, o, fdsBad, 3000);
    tncclResult a1 = c1 == TNCCL_SUCCESS ? netWaitAcks(fdsBad, 1, 3000) : c1;
    tncclResult a2 = TNCCL_SYSTEM_ERROR;
    if (kind == 0) {
      tncclResult c2 = netConnectEdge(ip, port, good, o, fdsGood, 3000);
      a2 = c2 == TNCCL_SUCCESS ? netWaitAcks(fdsGood, 1, 3000) : c2;
    }
    acceptor.join();
    close(lfd);
    if (c1 == TNCCL_SUCCESS) close(fdsBad[0]);
    if (kind == 0) {
      if (a2 == TNCCL_SUCCESS) close(fdsGood[0]);
      if (acc == TNCCL_SUCCESS) close(fdsB[0]);
      report("foreign hello refused, edge still connects",
             a1 == TNCCL_INVALID_ARGUMENT && a2 == TNCCL_SUCCESS && acc == TNCCL_SUCCESS);
    } else {
      report("mismatched hello fails the edge",
             a1 == TNCCL_INVALID_ARGUMENT && acc == TNCCL_INVALID_ARGUMENT);
    }
  }

  // Idle start / graceful stop: no failure, prompt join.
  {
    Edge e = connectEdge(2, o);
    const NetFifoLayout L2 = makeNetFifoLayout(2, 4, 4096);
    Buf sb(L2.totalBytes), rb(L2.totalBytes);
    netFifoInit(sb.p(), L2);
    netFifoInit(rb.p(), L2);
    std::atomic<int> ea{0}, eb{0};
    NetProxy pa, pb;
    NetOptions o2 = o;
    o2.channels = 2;
    bool ok = e.ok &&
              netProxyStart(&pa, o2, L2, sb.p(), nullptr, &e.a, hookSetError, &ea) ==
                  TNCCL_SUCCESS &&
              netProxyStart(&pb, o2, L2, nullptr, rb.p(), &e.b, hookSetError, &eb) ==
                  TNCCL_SUCCESS;
    std::this_thread::sleep_for(Ms(30));
    auto t0 = steady_clock::now();
    tncclResult sa = netProxyStop(&pa, true);
    // pb sees pa's close frames; let it read them before stopping.
    std::this_thread::sleep_for(Ms(20));
    tncclResult sbr = netProxyStop(&pb, true);
    const double ms = std::chrono::duration<double, std::milli>(steady_clock::now() - t0).count();
    netCloseRing(&e.a);
    netCloseRing(&e.b);
    report("idle proxies stop cleanly and promptly",
           ok && sa == TNCCL_SUCCESS && sbr == TNCCL_SUCCESS && ea.load() == 0 &&
               eb.load() == 0 && ms < 1000);
  }
}

// Random bytes on a receive connection (sometimes after valid frames) must
// end in a recorded failure, never in a crash, a hang or a payload written
// past its slot.
void testFuzzedStreams() {
  NetOptions o;
  o.channels = 1;
  o.spinUs = 20;
  const NetFifoLayout L = makeNetFifoLayout(1, 4, 4096);
  bool ok = true;
  for (int seed = 0; seed < 40 && ok; ++seed) {
    std::mt19937 g((unsigned)seed);
    Edge e = connectEdge(1, o);
    Buf rb(L.totalBytes + 4096);  // guard bytes after the FIFO
    netFifoInit(rb.p(), L);
    memset(rb.p() + L.totalBytes, 0x5A, 4096);
    std::atomic<int> err{0};
    NetProxy pb;
    ok = e.ok && netProxyStart(&pb, o, L, nullptr, rb.p(), &e.b, hookSetError, &err) ==
                     TNCCL_SUCCESS;
    std::vector<unsigned char> bytes;
    const int valid = (int)(g() % 3);  // a few well-formed frames first
    for (int t = 0; t < valid; ++t) {
      unsigned char h[kNetFrameHeaderBytes];
      netEncodeHeader(h, (uint64_t)t, 16);
      bytes.insert(bytes.end(), h, h + sizeof(h));
      for (int k = 0; k < 16; ++k) bytes.push_back((unsigned char)g());
    }
    const int junk = 1 + (int)(g() % 300);
    for (int k = 0; k < junk; ++k) bytes.push_back((unsigned char)g());
    Deadline d = deadlineIn(2000);
    if (ok) (void)writeAll(e.a.sendFds[0], bytes.data(), bytes.size(), d);
    netCloseRing(&e.a);  // the sender goes away without a close frame
    auto t0 = steady_clock::now();
    while (ok && !err.load() && steady_clock::now() - t0 < Ms(3000))
      std::this_thread::sleep_for(Ms(1));
    netProxyStop(&pb, false);
    netCloseRing(&e.b);
    bool guard = true;
    for (int k = 0; k < 4096; ++k) guard = guard && (unsigned char)rb.p()[L.totalBytes + k] == 0x5A;
    ok = ok && err.load() != 0 && guard;
  }
  report("40 fuzzed receive streams: failure recorded, FIFO bounds kept", ok);

  // Junk connections to a listening edge (short reads, foreign hellos of
  // random bytes) are dropped; the real connector still gets through.
  ok = true;
  for (int seed = 0; seed < 10 && ok; ++seed) {
    std::mt19937 g((unsigned)(100 + seed));
    int port = 0;
    const int lfd = tcpListen("127.0.0.1", 0, 32, &port);
    uint32_t ip = 0;
    parseIpv4("127.0.0.1", &ip);
    NetHello good{kNetHelloMagic, kNetVersion, 0, 0, 1, 4242, 4096, 4, 1};
    tncclResult acc = TNCCL_SYSTEM_ERROR;
    int fdsB[kMaxNetChannels];
    std::thread acceptor([&] { acc = netAcceptEdge(lfd, good, o, fdsB, 5000); });
    // One stray connection that stays open and silent: it is dropped after
    // its hello's one-second allowance, not at the accept deadline.
    Io whySilent = Io::kOk;
    const int silent = seed == 0 ? tcpConnect(ip, port, deadlineIn(2000), &whySilent) : -1;
    for (int j = 0; j < 4; ++j) {
      Io why = Io::kOk;
      const int fd = tcpConnect(ip, port, deadlineIn(2000), &why);
      if (fd < 0) continue;
      std::vector<unsigned char> junk((size_t)(1 + g() % (2 * sizeof(NetHello))));
      for (auto& c : junk) c = (unsigned char)g();
      (void)writeAll(fd, junk.data(), junk.size(), deadlineIn(1000));
      close(fd);
    }
    int fdsA[kMaxNetChannels];
    const tncclResult c = netConnectEdge(ip, port, good, o, fdsA, 3000);
    const tncclResult w = c == TNCCL_SUCCESS ? netWaitAcks(fdsA, 1, 3000) : c;
    acceptor.join();
    close(lfd);
    if (silent >= 0) close(silent);
    if (c == TNCCL_SUCCESS) close(fdsA[0]);
    if (acc == TNCCL_SUCCESS) close(fdsB[0]);
    ok = w == TNCCL_SUCCESS && acc == TNCCL_SUCCESS;
  }
  report("junk connections to a listening edge are dropped", ok);
}

// ---------------------------------------------------------------------------
// Ring all-reduce: P host threads run the ring kernel's protocol; edges are
// NVLink-like (shared mailboxes) or socket edges (host FIFO + proxy + TCP).
struct RingWorld {
  int P, channels, slots;
  uint64_t chunkElems, vec = 4, minChunk = 4;
  std::vector<int> host;  // host id per rank; an edge between hosts is a socket edge
  bool force = false;     // every edge a socket edge
  MailboxLayout L{};
  NetFifoLayout NL{};
  std::vector<Buf> mailbox, sendFifo, recvFifo;
  std::vector<std::vector<uint64_t>> counters;
  std::vector<std::unique_ptr<std::atomic<int>>> error;  // per rank (the status block)
  int timeoutMs = 20000;

  bool remote(int from, int to) const { return force || host[(size_t)from] != host[(size_t)to]; }
  bool sendRemote(int r) const { return remote(r, (r + 1) % P); }
  bool recvRemote(int r) const { return remote((r + P - 1) % P, r); }

  void init() {
    LayoutConfig lc{};
    lc.nranks = P;
    lc.channels = channels;
    lc.osChannels = 1;
    lc.ringSlots = slots;
    lc.ringChunkBytes = chunkElems * 4;
    lc.tsChunkBytes = 16;
    lc.osSlots = 1;
    lc.osTileBytes = 16;
    L = makeLayout(lc);
    NL = makeNetFifoLayout(channels, slots, chunkElems * 4);
    for (int r = 0; r < P; ++r) {
      mailbox.emplace_back(L.totalBytes);
      auto* credit = reinterpret_cast<uint64_t*>(mailbox.back().p() + L.ringCreditOff);
      for (int c = 0; c < channels; ++c)
        for (int s = 0; s < slots; ++s) credit[(size_t)c * slots + s] = (uint64_t)s;
      sendFifo.emplace_back(sendRemote(r) ? NL.totalBytes : 0);
      recvFifo.emplace_back(recvRemote(r) ? NL.totalBytes : 0);
      if (sendRemote(r)) netFifoInit(sendFifo.back().p(), NL);
      if (recvRemote(r)) netFifoInit(recvFifo.back().p(), NL);
      counters.emplace_back((size_t)kMaxChannels, 0);
      error.emplace_back(new std::atomic<int>(0));
    }
  }
};

// The ring kernel's schedule (csrc/tnccl/ring.cuh) for rank r, fp32 on the
// wire, channels one after another.
bool ringRank(RingWorld& w, int r, const std::vector<std::vector<float>>& x,
              std::vector<float>& y, uint64_t count) {
  const int P = w.P, next = (r + 1) % P, prev = (r + P - 1) % P;
  const ChunkPlan pl = makeChunkPlan(count, P, w.channels, w.chunkElems, w.minChunk, w.vec);
  const RingFifo out = w.sendRemote(r) ? netRingFifo(w.sendFifo[(size_t)r].p(), w.NL)
                                       : nvlinkRingFifo(w.mailbox[(size_t)next].p(),
                                                        w.mailbox[(size_t)r].p(), w.L);
  const RingFifo in = w.recvRemote(r) ? netRingFifo(w.recvFifo[(size_t)r].p(), w.NL)
                                      : nvlinkRingFifo(w.mailbox[(size_t)r].p(),
                                                       w.mailbox[(size_t)prev].p(), w.L);
  std::atomic<int>& err = *w.error[(size_t)r];
  const std::vector<float>& xr = x[(size_t)r];
  for (int ch = 0; ch < pl.channels; ++ch) {
    uint64_t& ticket = w.counters[(size_t)r][(size_t)ch];
    uint64_t sendT = ticket, recvT = ticket;
    auto waitSend = [&] {
      return waitWord(out.credit + ringFifoIndex(out, ch, sendT), sendT, err, w.timeoutMs);
    };
    auto waitRecv = [&](uint64_t expectElems) {
      const uint64_t i = ringFifoIndex(in, ch, recvT);
      if (!waitWord(in.ready + i, recvT + 1, err, w.timeoutMs)) return false;
      if (in.bytes && __atomic_load_n(in.bytes + i, __ATOMIC_RELAXED) != expectElems * 4) {
        err.store(TNCCL_SYSTEM_ERROR);
        return false;
      }
      return true;
    };
    auto outSlot = [&] { return reinterpret_cast<float*>(ringFifoData(out, ch, sendT)); };
    auto inSlot = [&] { return reinterpret_cast<const float*>(ringFifoData(in, ch, recvT)); };
    auto publish = [&](uint64_t elems) {
      const uint64_t i = ringFifoIndex(out, ch, sendT);
      if (out.bytes) __atomic_store_n(out.bytes + i, elems * 4, __ATOMIC_RELAXED);
      __atomic_store_n(out.ready + i, sendT + 1, __ATOMIC_RELEASE);
      ++sendT;
    };
    auto release = [&] {
      __atomic_store_n(in.credit + ringFifoIndex(in, ch, recvT), recvT + (uint64_t)in.slots,
                       __ATOMIC_RELEASE);
      ++recvT;
    };
    for (uint64_t t = 0; t < channelTiles(pl.numTiles, pl.channels, ch); ++t) {
      const uint64_t tile = (uint64_t)ch + t * (uint64_t)pl.channels;
      {
        Span sp = chunkSpan(pl, tile, ringChunkBehind(r, 1, P), w.vec);
        if (!waitSend()) return false;
        float* o = outSlot();
        for (uint64_t e = 0; e < sp.count; ++e) o[e] = xr[sp.offset + e];
        publish(sp.count);
      }
      for (int d = 2; d < P; ++d) {
        Span sp = chunkSpan(pl, tile, ringChunkBehind(r, d, P), w.vec);
        if (!waitRecv(sp.count) || !waitSend()) return false;
        const float* i = inSlot();
        float* o = outSlot();
        for (uint64_t e = 0; e < sp.count; ++e) o[e] = oracle::add(i[e], xr[sp.offset + e]);
        release();
        publish(sp.count);
      }
      {
        Span sp = chunkSpan(pl, tile, r, w.vec);
        if (!waitRecv(sp.count) || !waitSend()) return false;
        const float* i = inSlot();
        float* o = outSlot();
        for (uint64_t e = 0; e < sp.count; ++e) y[sp.offset + e] = o[e] = oracle::add(i[e], xr[sp.offset + e]);
        release();
        publish(sp.count);
      }
      for (int d = 1; d < P - 1; ++d) {
        Span sp = chunkSpan(pl, tile, ringChunkBehind(r, d, P), w.vec);
        if (!waitRecv(sp.count) || !waitSend()) return false;
        const float* i = inSlot();
        float* o = outSlot();
        for (uint64_t e = 0; e < sp.count; ++e) y[sp.offset + e] = o[e] = i[e];
        release();
        publish(sp.count);
      }
      {
        Span sp = chunkSpan(pl, tile, ringChunkBehind(r, P - 1, P), w.vec);
        if (!waitRecv(sp.count)) return false;
        const float* i = inSlot();
        for (uint64_t e = 0; e < sp.count; ++e) y[sp.offset + e] = i[e];
        release();
      }
    }
    ticket = sendT;
    if (sendT != recvT) return false;
  }
  return true;
}

// Runs `counts` back to back on a fresh world. dieRank >= 0: that rank
// "crashes" (closes its sockets without close frames) 100 ms into the second
// collective; the others must fail it through their proxies' hooks.
bool runRing(int P, int channels, uint64_t chunkElems, const std::vector<int>& host, bool force,
             const std::vector<uint64_t>& counts, int dieRank = -1, double* failMs = nullptr) {
  RingWorld w;
  w.P = P;
  w.channels = channels;
  w.slots = 4;
  w.chunkElems = chunkElems;
  w.host = host;
  w.force = force;
  w.init();
  tncclUniqueId id;
  if (bootstrapNewId(&id) != TNCCL_SUCCESS) return false;
  std::vector<int> ok((size_t)P, 1);
  std::vector<double> failTimes((size_t)P, 0.0);
  std::vector<std::vector<std::vector<float>>> xs(counts.size());
  std::vector<std::vector<std::vector<float>>> ys(counts.size());
  for (size_t k = 0; k < counts.size(); ++k) {
    xs[k].resize((size_t)P);
    ys[k].assign((size_t)P, std::vector<float>(counts[k], -7.0f));
    std::vector<unsigned char> raw;
    for (int r = 0; r < P; ++r) oracle::fillInput(oracle::kF32, 11 + k, r, counts[k], xs[k][(size_t)r], raw);
  }
  std::vector<std::thread> th;
  for (int r = 0; r < P; ++r) {
    th.emplace_back([&, r] {
      Bootstrap b;
      NetRing ring;
      NetProxy proxy;
      NetOptions o;
      o.channels = channels;
      o.spinUs = 50;
      o.timeoutMs = 10000;
      bool good = bootstrapOpen(&b, id, P, r, 0, 10000) == TNCCL_SUCCESS;
      const bool anyRemote = [&] {
        for (int q = 0; q < P; ++q)
          if (w.sendRemote(q)) return true;
        return false;
      }();
      const bool mine = w.sendRemote(r) || w.recvRemote(r);
      if (good && anyRemote)
        good = netConnectRing(&b, o, w.NL, w.sendRemote(r), w.recvRemote(r), 0xabcdef, &ring) ==
               TNCCL_SUCCESS;
      if (good && mine)
        good = netProxyStart(&proxy, o, w.NL,
                             w.sendRemote(r) ? w.sendFifo[(size_t)r].p() : nullptr,
                             w.recvRemote(r) ? w.recvFifo[(size_t)r].p() : nullptr, &ring,
                             hookSetError, w.error[(size_t)r].get()) == TNCCL_SUCCESS;
      for (size_t k = 0; k < counts.size() && good; ++k) {
        if (dieRank >= 0 && k == 1) {
          if (r == dieRank) {
            // The others are already inside the collective when this rank's
            // sockets close.
            std::this_thread::sleep_for(Ms(100));
            netProxyStop(&proxy, false);
            netCloseRing(&ring);
            bootstrapClose(&b);
            return;
          }
          auto t0 = steady_clock::now();
          const bool res = ringRank(w, r, xs[k], ys[k][(size_t)r], counts[k]);
          failTimes[(size_t)r] =
              std::chrono::duration<double, std::milli>(steady_clock::now() - t0).count();
          ok[(size_t)r] = res ? 2 : (w.error[(size_t)r]->load() != 0 ? 3 : 4);
          good = false;
          break;
        }
        good = ringRank(w, r, xs[k], ys[k][(size_t)r], counts[k]);
      }
      if (dieRank < 0) {
        // Orderly teardown: every rank's traffic is done before any proxy stops.
        if (good) good = bootstrapBarrier(&b) == TNCCL_SUCCESS;
        tncclResult st = mine ? netProxyStop(&proxy, good) : TNCCL_SUCCESS;
        if (good) good = bootstrapBarrier(&b) == TNCCL_SUCCESS && st == TNCCL_SUCCESS &&
                         w.error[(size_t)r]->load() == 0;
        ok[(size_t)r] = good ? 1 : 0;
      } else if (mine) {
        netProxyStop(&proxy, false);
      }
      netCloseRing(&ring);
      bootstrapClose(&b);
    });
  }
  for (auto& t : th) t.join();
  if (dieRank >= 0) {
    // Survivors: every one failed collective 2 through its proxy's hook.
    double worst = 0;
    for (int r = 0; r < P; ++r) {
      if (r == dieRank) continue;
      if (ok[(size_t)r] != 3) return false;
      worst = std::max(worst, failTimes[(size_t)r]);
    }
    if (failMs) *failMs = worst;
    return true;
  }
  for (int v : ok)
    if (v != 1) return false;
  for (size_t k = 0; k < counts.size(); ++k) {
    std::vector<float> want;
    const ChunkPlan pl = makeChunkPlan(counts[k], P, channels, chunkElems, 4, 4);
    oracle::ring(oracle::kF32, xs[k], 1.0f, pl, 4, want);
    for (int r = 0; r < P; ++r)
      if (counts[k] > 0 && memcmp(ys[k][(size_t)r].data(), want.data(), counts[k] * 4) != 0) {
        printf("  count %llu rank %d differs from the ring oracle\n",
               (unsigned long long)counts[k], r);
        return false;
      }
  }
  return true;
}

void testRing() {
  const std::vector<uint64_t> matrix = {0, 1, 2, 5, 8, 31, 113};
  for (int P : {2, 3, 4}) {
    std::vector<int> same((size_t)P, 0);
    char name[96];
    snprintf(name, sizeof(name), "ring P=%d, every edge a socket edge, count matrix", P);
    report(name, runRing(P, 2, 7, same, true, matrix));
  }
  {
    // Hosts {0,0,1,1}: edges 1->2 and 3->0 are socket edges, 0->1 and 2->3 NVLink.
    report("ring P=4, mixed NVLink / socket edges, count matrix",
           runRing(4, 3, 7, {0, 0, 1, 1}, false, matrix));
    report("ring P=3, hosts {0,1,1}, 1,000,003 elements x 3",
           runRing(3, 2, 16384, {0, 1, 1}, false, {1000003, 4096, 1000003}));
    report("ring P=4, all socket edges, 1,000,003 elements, 4 channels",
           runRing(4, 4, 16384, {0, 0, 0, 0}, true, {1000003, 77}));
  }
  {
    double ms = 0;
    const bool ok = runRing(3, 2, 1024, {0, 0, 0}, true, {5000, 5000}, 2, &ms);
    char name[96];
    snprintf(name, sizeof(name), "rank dies mid-collective -> peers fail (%.0f ms)", ms);
    report(name, ok && ms >= 90 && ms < 5000);  // it dies at 100 ms; the wait bound is 20 s
  }
}

}  // namespace

int main(int argc, char** argv) {
  if (argc > 1 && strcmp(argv[1], "--bench") == 0) {
    // net_proxy_test --bench [total MiB]: loopback throughput of one edge.
    const uint64_t total = (argc > 2 ? strtoull(argv[2], nullptr, 10) : 2048) << 20;
    for (int C : {1, 2, 4})
      for (uint64_t chunk : {64ull << 10, 256ull << 10, 1ull << 20}) {
        const double gbs = measureStream(C, chunk, total);
        printf("socket edge loopback: %d channel(s), %4llu KiB frames: %.2f GB/s\n", C,
               (unsigned long long)(chunk >> 10), gbs);
        fflush(stdout);
        if (gbs < 0) return 1;
      }
    return 0;
  }
  const int fds0 = countFds();
  testCodecAndLayout();
  testStream();
  testEdgeFailures();
  testFuzzedStreams();
  testRing();
  const int fds1 = countFds();
  report("no descriptor leaks", fds0 == fds1);
  if (gFailed) {
    printf("net_proxy_test: %d FAILED\n", gFailed);
    return 1;
  }
  printf("net_proxy_test: PASS\n");
  return 0;
}
