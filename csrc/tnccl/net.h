// net.h - socket ring edges: the data plane for ring neighbours that NVLink
// does not connect (ranks on different hosts, or every edge when TNCCL_NET=
// force). Each such edge is a set of TCP connections, one per channel, and a
// proxy thread per rank moves FIFO slots between host-mapped memory, which
// the ring kernel reads and writes directly, and those connections.
//
// tiny-nccl designs this path (docs/design-v0.2.md:34-160) without building
// it. Kept from that design:
//  * a ring edge is either the direct P2P path or a mapped-host FIFO plus a
//    CPU proxy; local edges never pass through the CPU;
//  * a frame is ticket | payload bytes | payload with fixed-size big-endian
//    fields; magic, version and identity are exchanged once per connection;
//  * the send proxy credits a slot back to the kernel only after the socket
//    took the whole frame (partial writes keep their offset), and the receive
//    proxy refills a slot only after the kernel credited it, so network
//    back-pressure ends as "no credit" at the producing kernel and no host
//    buffer grows;
//  * a frame with an unexpected ticket or an oversized payload, and a
//    connection that ends without a close frame, fail the communicator; there
//    is no reconnect;
//  * one proxy thread per rank, non-blocking sockets, poll() when idle.
// Different:
//  * one connection per channel: ring channels are independent pipelines, and
//    a byte stream shared by channels would make a channel that waits on its
//    consumer hold up the others (a cycle around the ring can deadlock);
//  * the kernel writes each slot's payload size next to the ready word, so
//    the proxy needs no knowledge of the collective (it works unchanged for
//    launches replayed from CUDA graphs);
//  * the proxy reports a failure through a hook; the communicator writes it
//    into the host-mapped status block that every device wait polls, so
//    kernels waiting on a dead edge return instead of hanging;
//  * both directions of every connection end with a close frame, so a peer
//    that exits cleanly is told apart from one that died.
#pragma once

#include <stdint.h>

#include <atomic>
#include <thread>

#include "bootstrap.h"
#include "protocol.h"
#include "tnccl.h"

namespace tnccl {

constexpr int kMaxNetChannels = 8;
constexpr uint64_t kNetHelloMagic = 0x30544e4c43434e54ull;  // "TNCCLNT0" little-endian
constexpr uint32_t kNetVersion = 1;

struct NetOptions {
  int channels = 2;               // connections (ring channels) per edge
  char ifAddr[64] = "127.0.0.1";  // IPv4 address this rank listens on
  int sndBuf = 0;                 // SO_SNDBUF / SO_RCVBUF (0: system default)
  int rcvBuf = 0;
  int spinUs = 200;               // busy polling after the last progress
  int timeoutMs = 30000;          // connection set-up deadline
};

// This rank's socket edges of the ring. Descriptors are non-blocking; -1
// where the edge is not a socket edge.
struct NetRing {
  int channels = 0;
  int sendFds[kMaxNetChannels];  // to rank + 1
  int recvFds[kMaxNetChannels];  // from rank - 1
  NetRing() {
    for (int c = 0; c < kMaxNetChannels; ++c) sendFds[c] = recvFds[c] = -1;
  }
};

// First message on every connection (connector -> acceptor); the acceptor
// answers with a NetHelloAck.
struct NetHello {
  uint64_t magic;
  uint32_t version;
  int32_t channel;
  int32_t src;  // connecting rank
  int32_t dst;  // accepting rank
  uint64_t nonce;  // communicator identity (same on every rank)
  uint64_t chunkBytes;
  int32_t slots;
  int32_t channels;
};
struct NetHelloAck {
  uint64_t magic;
  int32_t status;
  int32_t pad;
};

inline void netEncodeHeader(unsigned char* h, uint64_t ticket, uint32_t bytes) {
  for (int i = 0; i < 8; ++i) h[i] = (unsigned char)(ticket >> (56 - 8 * i));
  for (int i = 0; i < 4; ++i) h[8 + i] = (unsigned char)(bytes >> (24 - 8 * i));
}
inline void netDecodeHeader(const unsigned char* h, uint64_t* ticket, uint32_t* bytes) {
  uint64_t t = 0;
  uint32_t b = 0;
  for (int i = 0; i < 8; ++i) t = (t << 8) | h[i];
  for (int i = 0; i < 4; ++i) b = (b << 8) | h[8 + i];
  *ticket = t;
  *bytes = b;
}

// Collective over the bootstrap (every rank calls it, with or without socket
// edges of its own): ranks with a socket receive edge listen on ifAddr, the
// addresses are all-gathered, every rank with a socket send edge opens
// `channels` connections to rank + 1 and sends a NetHello on each, every rank
// with a socket receive edge accepts and validates them, and a final status
// all-gather makes every rank return the same result.
tncclResult netConnectRing(Bootstrap* b, const NetOptions& o, const NetFifoLayout& L,
                           bool sendRemote, bool recvRemote, uint64_t nonce, NetRing* ring);
void netCloseRing(NetRing* ring);

// The halves of netConnectRing for one edge (tests drive them directly).
// netConnectEdge opens the connections of `hello.channels` channels and sends
// the hellos (it does not wait for the acceptor); netAcceptEdge accepts and
// validates them against `expect` (channel ignored) and acknowledges each;
// netWaitAcks reads the acknowledgements on the connector side.
tncclResult netConnectEdge(uint32_t ipv4, int port, const NetHello& hello, const NetOptions& o,
                           int* fds, int timeoutMs);
tncclResult netAcceptEdge(int listenFd, const NetHello& expect, const NetOptions& o, int* fds,
                          int timeoutMs);
tncclResult netWaitAcks(const int* fds, int channels, int timeoutMs);

// Initial FIFO contents: zero, except credit[c][s] = s.
void netFifoInit(char* base, const NetFifoLayout& L);

using NetFailureHook = void (*)(void* arg, tncclResult code);

struct NetProxy {
  // set by netProxyStart
  NetOptions opts;
  NetFifoLayout layout{};
  RingFifo sendFifo{};  // host view; data == nullptr when there is no send edge
  RingFifo recvFifo{};
  NetRing* ring = nullptr;
  NetFailureHook hook = nullptr;
  void* hookArg = nullptr;
  std::thread thread;
  int wakeFds[2] = {-1, -1};
  bool running = false;
  std::atomic<int> stop{0};
  std::atomic<int> error{0};  // first failure (tncclResult), 0 while healthy

  // statistics (read by tests and tncclCommGetInfo-style queries)
  std::atomic<uint64_t> framesSent{0}, framesReceived{0};
  std::atomic<uint64_t> bytesSent{0}, bytesReceived{0};
  std::atomic<uint64_t> partialWrites{0}, partialReads{0};  // frames that took several calls
  std::atomic<uint64_t> creditStalls{0};  // frames that waited for the kernel's credit

  // proxy-thread state per channel
  struct SendCh {
    uint64_t ticket = 0;
    int phase = 0;  // 0: waiting for a ready slot, 1: writing a frame
    unsigned char hdr[kNetFrameHeaderBytes];
    uint64_t bytes = 0, off = 0;
    bool partial = false;     // this frame took several writes
    int ctlHave = 0;  // bytes of a close frame received from downstream
    unsigned char ctl[kNetFrameHeaderBytes];
    bool peerClosed = false;  // downstream sent its close frame
    bool ctlEof = false;      // ... and then closed the connection
  };
  struct RecvCh {
    uint64_t ticket = 0;
    int phase = 0;  // 0: header, 1: waiting for the slot's credit, 2: payload
    unsigned char hdr[kNetFrameHeaderBytes];
    uint64_t hoff = 0, bytes = 0, off = 0;
    bool stalled = false;     // this frame waited for the kernel's credit
    bool partial = false;     // this frame's payload took several reads
    bool peerClosed = false;  // upstream sent its close frame
    bool peerEof = false;     // ... and then closed the connection
  };
  SendCh send[kMaxNetChannels];
  RecvCh recv[kMaxNetChannels];
};

// Starts the proxy thread over `ring`'s connections. sendFifo / recvFifo are
// host pointers of the FIFOs (layout L) of the send and receive edge (null
// for an edge that is not a socket edge). `hook` runs once, on the proxy
// thread, at the first failure.
tncclResult netProxyStart(NetProxy* p, const NetOptions& o, const NetFifoLayout& L,
                          char* sendFifo, char* recvFifo, NetRing* ring, NetFailureHook hook,
                          void* hookArg);
// Stops and joins the proxy thread. With `graceful` (and no failure seen), a
// close frame is then written in both directions of every connection. The
// connections stay open (netCloseRing closes them). Returns the first failure
// the proxy saw, TNCCL_SUCCESS if none.
tncclResult netProxyStop(NetProxy* p, bool graceful);

}  // namespace tnccl
