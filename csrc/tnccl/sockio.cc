// sockio.cc - deadline-bounded socket I/O (see sockio.h).
#ifndef _GNU_SOURCE
#define _GNU_SOURCE
#endif

#include "sockio.h"

#include <arpa/inet.h>
#include <errno.h>
#include <fcntl.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <string.h>
#include <sys/random.h>
#include <sys/socket.h>
#include <unistd.h>

#include <algorithm>
#include <climits>

namespace tnccl {

Deadline deadlineIn(int ms) { return Clock::now() + std::chrono::milliseconds(ms); }

int msLeft(Deadline d) {
  auto now = Clock::now();
  if (now >= d) return 0;
  auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(d - now).count();
  return (int)std::min<int64_t>(ms + 1, INT_MAX);
}

Io waitFd(int fd, short events, Deadline d) {
  for (;;) {
    int left = msLeft(d);
    if (left == 0) return Io::kTimeout;
    pollfd p{fd, events, 0};
    int rc = poll(&p, 1, left);
    if (rc > 0) {
      if (p.revents & POLLNVAL) return Io::kError;
      if (p.revents & events) return Io::kOk;
      if (p.revents & (POLLERR | POLLHUP)) return Io::kError;
      continue;
    }
    if (rc == 0) return Io::kTimeout;
    if (errno != EINTR) return Io::kError;
  }
}

Io readAll(int fd, void* buf, size_t n, Deadline d) {
  auto* p = static_cast<unsigned char*>(buf);
  size_t done = 0;
  while (done < n) {
    ssize_t rc = recv(fd, p + done, n - done, 0);
    if (rc > 0) {
      done += (size_t)rc;
      continue;
    }
    if (rc == 0) return Io::kError;  // peer closed
    if (errno == EINTR) continue;
    if (errno == EAGAIN || errno == EWOULDBLOCK) {
      Io w = waitFd(fd, POLLIN, d);
      if (w != Io::kOk) return w;
      continue;
    }
    return Io::kError;
  }
  return Io::kOk;
}

Io writeAll(int fd, const void* buf, size_t n, Deadline d) {
  auto* p = static_cast<const unsigned char*>(buf);
  size_t done = 0;
  while (done < n) {
    ssize_t rc = send(fd, p + done, n - done, MSG_NOSIGNAL);
    if (rc > 0) {
      done += (size_t)rc;
      continue;
    }
    if (rc < 0 && errno == EINTR) continue;
    if (rc < 0 && (errno == EAGAIN || errno == EWOULDBLOCK)) {
      Io w = waitFd(fd, POLLOUT, d);
      if (w != Io::kOk) return w;
      continue;
    }
    return Io::kError;
  }
  return Io::kOk;
}

tncclResult toResult(Io io) {
  return io == Io::kOk ? TNCCL_SUCCESS
                       : io == Io::kTimeout ? TNCCL_TIMEOUT : TNCCL_SYSTEM_ERROR;
}

bool randomBytes(void* buf, size_t n) {
  auto* p = static_cast<unsigned char*>(buf);
  size_t done = 0;
  while (done < n) {
    ssize_t rc = getrandom(p + done, n - done, 0);
    if (rc > 0) {
      done += (size_t)rc;
    } else if (rc < 0 && errno == EINTR) {
      continue;
    } else {
      break;
    }
  }
  if (done == n) return true;
  int fd = open("/dev/urandom", O_RDONLY | O_CLOEXEC);
  if (fd < 0) return false;
  while (done < n) {
    ssize_t rc = read(fd, p + done, n - done);
    if (rc > 0) {
      done += (size_t)rc;
    } else if (rc < 0 && errno == EINTR) {
      continue;
    } else {
      close(fd);
      return false;
    }
  }
  close(fd);
  return true;
}

int acceptOne(int listenFd, Deadline d, Io* why) {
  for (;;) {
    int fd = accept4(listenFd, nullptr, nullptr, SOCK_NONBLOCK | SOCK_CLOEXEC);
    if (fd >= 0) return fd;
    if (errno == EINTR) continue;
    if (errno == EAGAIN || errno == EWOULDBLOCK) {
      Io w = waitFd(listenFd, POLLIN, d);
      if (w != Io::kOk) {
        *why = w;
        return -1;
      }
      continue;
    }
    *why = Io::kError;
    return -1;
  }
}

bool parseIpv4(const char* addr, uint32_t* out) {
  in_addr a{};
  if (addr == nullptr || inet_pton(AF_INET, addr, &a) != 1) return false;
  *out = a.s_addr;  // network byte order
  return true;
}

int tcpListen(const char* addr, int port, int backlog, int* boundPort) {
  uint32_t ip = 0;
  if (!parseIpv4(addr, &ip) || port < 0 || port > 65535) return -1;
  int fd = socket(AF_INET, SOCK_STREAM | SOCK_NONBLOCK | SOCK_CLOEXEC, 0);
  if (fd < 0) return -1;
  int one = 1;
  setsockopt(fd, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
  sockaddr_in a{};
  a.sin_family = AF_INET;
  a.sin_addr.s_addr = ip;
  a.sin_port = htons((uint16_t)port);
  if (bind(fd, reinterpret_cast<sockaddr*>(&a), sizeof(a)) != 0 || listen(fd, backlog) != 0) {
    close(fd);
    return -1;
  }
  socklen_t len = sizeof(a);
  if (getsockname(fd, reinterpret_cast<sockaddr*>(&a), &len) != 0) {
    close(fd);
    return -1;
  }
  if (boundPort) *boundPort = ntohs(a.sin_port);
  return fd;
}

void tcpTune(int fd, int sndBuf, int rcvBuf) {
  int one = 1;
  setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
  // A peer host that vanishes without closing its connections shows up as a
  // socket error after ~20 s of silence (10 s idle, then 5 probes 2 s apart).
  int idle = 10, intvl = 2, cnt = 5;
  setsockopt(fd, SOL_SOCKET, SO_KEEPALIVE, &one, sizeof(one));
  setsockopt(fd, IPPROTO_TCP, TCP_KEEPIDLE, &idle, sizeof(idle));
  setsockopt(fd, IPPROTO_TCP, TCP_KEEPINTVL, &intvl, sizeof(intvl));
  setsockopt(fd, IPPROTO_TCP, TCP_KEEPCNT, &cnt, sizeof(cnt));
  if (sndBuf > 0) setsockopt(fd, SOL_SOCKET, SO_SNDBUF, &sndBuf, sizeof(sndBuf));
  if (rcvBuf > 0) setsockopt(fd, SOL_SOCKET, SO_RCVBUF, &rcvBuf, sizeof(rcvBuf));
}

int tcpConnect(uint32_t ipv4, int port, Deadline d, Io* why) {
  sockaddr_in a{};
  a.sin_family = AF_INET;
  a.sin_addr.s_addr = ipv4;
  a.sin_port = htons((uint16_t)port);
  while (msLeft(d) > 0) {
    int fd = socket(AF_INET, SOCK_STREAM | SOCK_NONBLOCK | SOCK_CLOEXEC, 0);
    if (fd < 0) {
      *why = Io::kError;
      return -1;
    }
    int err = 0;
    if (connect(fd, reinterpret_cast<sockaddr*>(&a), sizeof(a)) == 0) {
      tcpTune(fd, 0, 0);
      return fd;
    }
    err = errno;
    if (err == EINPROGRESS) {
      Io w = waitFd(fd, POLLOUT, d);
      if (w == Io::kOk) {
        socklen_t l = sizeof(err);
        if (getsockopt(fd, SOL_SOCKET, SO_ERROR, &err, &l) == 0 && err == 0) {
          tcpTune(fd, 0, 0);
          return fd;
        }
      } else if (w == Io::kTimeout) {
        close(fd);
        break;
      } else {
        socklen_t l = sizeof(err);
        if (getsockopt(fd, SOL_SOCKET, SO_ERROR, &err, &l) != 0) err = ECONNREFUSED;
      }
    }
    close(fd);
    if (err != ECONNREFUSED && err != EINTR && err != EAGAIN && err != ETIMEDOUT &&
        err != ENETUNREACH && err != EHOSTUNREACH) {
      *why = Io::kError;
      return -1;
    }
    int pause = std::min(10, msLeft(d));
    if (pause > 0) poll(nullptr, 0, pause);
  }
  *why = Io::kTimeout;
  return -1;
}

}  // namespace tnccl
