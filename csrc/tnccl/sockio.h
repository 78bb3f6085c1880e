// sockio.h - deadline-bounded socket I/O shared by the bootstrap (AF_UNIX or
// TCP control plane) and the socket ring edges (TCP data plane).
//
// Every blocking step takes an absolute deadline; sockets are non-blocking
// and waits go through poll(), so EINTR, short reads/writes and peer hang-ups
// are handled in one place (tiny-nccl's src/bootstrap.cc:73-189 keeps the
// same rules for its AF_UNIX socket).
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <chrono>

#include "tnccl.h"

namespace tnccl {

using Clock = std::chrono::steady_clock;
using Deadline = Clock::time_point;

Deadline deadlineIn(int ms);
// Milliseconds until d, rounded up (0 once it has passed).
int msLeft(Deadline d);

// Outcome of a socket step: ok, timed out, or failed otherwise.
enum class Io { kOk, kTimeout, kError };

Io waitFd(int fd, short events, Deadline d);
// Reads / writes exactly n bytes (a peer that closes mid-way is an error).
Io readAll(int fd, void* buf, size_t n, Deadline d);
Io writeAll(int fd, const void* buf, size_t n, Deadline d);
tncclResult toResult(Io io);

// getrandom(2), falling back to /dev/urandom.
bool randomBytes(void* buf, size_t n);

// Accepts one connection on a non-blocking listening socket; the new socket is
// non-blocking and close-on-exec.
int acceptOne(int listenFd, Deadline d, Io* why);

// TCP (IPv4). `addr` is a dotted-quad address. tcpListen binds addr:port
// (port 0: any free port), listens with `backlog` and returns the socket and
// the bound port. tcpConnect retries refused connections every 10 ms until
// the deadline (the listener may not be up yet). Both sockets are
// non-blocking, close-on-exec, with TCP_NODELAY on connected sockets.
bool parseIpv4(const char* addr, uint32_t* out);
int tcpListen(const char* addr, int port, int backlog, int* boundPort);
int tcpConnect(uint32_t ipv4, int port, Deadline d, Io* why);
// TCP_NODELAY, keepalive probes (a silent dead peer fails the socket after
// ~20 s) and, when > 0, SO_SNDBUF / SO_RCVBUF on a connected socket.
void tcpTune(int fd, int sndBuf, int rcvBuf);

}  // namespace tnccl
