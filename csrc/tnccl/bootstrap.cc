// bootstrap.cc - AF_UNIX or TCP star rendezvous (see bootstrap.h for the
// contract).
#ifndef _GNU_SOURCE
#define _GNU_SOURCE
#endif

#include "bootstrap.h"

#include <arpa/inet.h>
#include <errno.h>
#include <netinet/in.h>
#include <poll.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/socket.h>
#include <sys/stat.h>
#include <sys/un.h>
#include <unistd.h>

#include <algorithm>
#include <string>

#include "common.h"
#include "sockio.h"

namespace tnccl {
namespace {

constexpr uint64_t kIdMagic = 0x3230304242434e54ull;     // "TNCBB002" little-endian
constexpr uint64_t kTcpIdMagic = 0x3330305442434e54ull;  // "TNCBT003" little-endian
constexpr uint32_t kFrameMagic = 0x544e4246u;            // "FBNT"
constexpr uint16_t kWireVersion = 3;
constexpr size_t kMaxGatherBytes = 1u << 20;           // per rank
constexpr char kBaseName[] = "tnccl-b200-";

enum Frame : uint16_t {
  kHello = 1,
  kHelloAck = 2,
  kGather = 3,
  kGatherResult = 4,
  kBarrier = 5,
  kBarrierRelease = 6,
  kFdGather = 7,
  kFdGatherResult = 8,
  kFdBcast = 9,
};

struct IdPayload {
  uint64_t magic;
  uint32_t version;
  uint32_t pathLength;
  char path[104];
  uint64_t reserved;
};
static_assert(sizeof(IdPayload) == sizeof(tncclUniqueId), "id layout");

struct TcpIdPayload {
  uint64_t magic;
  uint32_t version;
  uint32_t ipv4;  // network byte order
  uint32_t port;
  uint32_t pad;
  uint64_t nonce;  // random, never 0
  char reserved[96];
};
static_assert(sizeof(TcpIdPayload) == sizeof(tncclUniqueId), "tcp id layout");

struct FrameHeader {
  uint32_t magic;
  uint16_t version;
  uint16_t type;
  uint32_t op;      // bootstrap collective number (0 = hello)
  uint32_t status;  // sender-side status (tncclResult)
  uint64_t bytes;   // payload bytes that follow
};

struct Hello {
  int32_t rank;
  int32_t nranks;
  int32_t pid;
  int32_t pad;
  uint64_t configHash;
  uint64_t nonce;  // TCP ids: the communicator nonce (0 for AF_UNIX)
};

Io sendFrame(int fd, uint16_t type, uint32_t op, uint32_t status,
             const void* payload, size_t bytes, Deadline d) {
  FrameHeader h{kFrameMagic, kWireVersion, type, op, status, (uint64_t)bytes};
  Io io = writeAll(fd, &h, sizeof(h), d);
  if (io != Io::kOk || bytes == 0) return io;
  return writeAll(fd, payload, bytes, d);
}

// Receives a frame of exactly the expected type/op/size. *status receives the
// sender-side status word.
Io recvFrame(int fd, uint16_t type, uint32_t op, void* payload, size_t bytes,
             uint32_t* status, Deadline d) {
  FrameHeader h{};
  Io io = readAll(fd, &h, sizeof(h), d);
  if (io != Io::kOk) return io;
  if (h.magic != kFrameMagic || h.version != kWireVersion || h.type != type ||
      h.op != op || h.bytes != (uint64_t)bytes) {
    TN_WARN("bootstrap: unexpected frame (type %u op %u bytes %llu; wanted %u %u %zu)",
            h.type, h.op, (unsigned long long)h.bytes, type, op, bytes);
    return Io::kError;
  }
  if (status) *status = h.status;
  if (bytes == 0) return Io::kOk;
  return readAll(fd, payload, bytes, d);
}

// Sends a frame whose payload is `bytes` of data with `nfds` descriptors
// attached to the payload's first byte (SCM_RIGHTS).
Io sendFrameFds(int fd, uint16_t type, uint32_t op, uint32_t status,
                const void* payload, size_t bytes, const int* fds, int nfds,
                Deadline d) {
  FrameHeader h{kFrameMagic, kWireVersion, type, op, status, (uint64_t)bytes};
  Io io = writeAll(fd, &h, sizeof(h), d);
  if (io != Io::kOk) return io;
  if (bytes == 0) return Io::kOk;
  const auto* p = static_cast<const unsigned char*>(payload);
  size_t done = 0;
  if (nfds > 0) {
    alignas(cmsghdr) char ctrl[CMSG_SPACE(sizeof(int) * kMaxRankFds)];
    for (;;) {
      iovec iov{const_cast<unsigned char*>(p), bytes};
      msghdr m{};
      m.msg_iov = &iov;
      m.msg_iovlen = 1;
      memset(ctrl, 0, sizeof(ctrl));
      m.msg_control = ctrl;
      m.msg_controllen = CMSG_SPACE(sizeof(int) * nfds);
      cmsghdr* c = CMSG_FIRSTHDR(&m);
      c->cmsg_level = SOL_SOCKET;
      c->cmsg_type = SCM_RIGHTS;
      c->cmsg_len = CMSG_LEN(sizeof(int) * nfds);
      memcpy(CMSG_DATA(c), fds, sizeof(int) * nfds);
      ssize_t rc = sendmsg(fd, &m, MSG_NOSIGNAL);
      if (rc > 0) {
        done = (size_t)rc;
        break;
      }
      if (rc < 0 && errno == EINTR) continue;
      if (rc < 0 && (errno == EAGAIN || errno == EWOULDBLOCK)) {
        Io w = waitFd(fd, POLLOUT, d);
        if (w != Io::kOk) return w;
        continue;
      }
      return Io::kError;
    }
  }
  return writeAll(fd, p + done, bytes - done, d);
}

// Receives a frame whose payload may carry descriptors. Up to maxFds received
// descriptors are stored in fds; *nfds receives their number.
Io recvFrameFds(int fd, uint16_t type, uint32_t op, void* payload, size_t bytes,
                uint32_t* status, int* fds, int maxFds, int* nfds, Deadline d) {
  *nfds = 0;
  FrameHeader h{};
  Io io = readAll(fd, &h, sizeof(h), d);
  if (io != Io::kOk) return io;
  if (h.magic != kFrameMagic || h.version != kWireVersion || h.type != type ||
      h.op != op || h.bytes != (uint64_t)bytes) {
    TN_WARN("bootstrap: unexpected fd frame (type %u op %u)", h.type, h.op);
    return Io::kError;
  }
  if (status) *status = h.status;
  if (bytes == 0) return Io::kOk;
  auto* p = static_cast<unsigned char*>(payload);
  size_t done = 0;
  alignas(cmsghdr) char ctrl[CMSG_SPACE(sizeof(int) * kMaxRankFds)];
  for (;;) {
    iovec iov{p, bytes};
    msghdr m{};
    m.msg_iov = &iov;
    m.msg_iovlen = 1;
    m.msg_control = ctrl;
    m.msg_controllen = sizeof(ctrl);
    ssize_t rc = recvmsg(fd, &m, MSG_CMSG_CLOEXEC);
    if (rc > 0) {
      done = (size_t)rc;
      for (cmsghdr* c = CMSG_FIRSTHDR(&m); c != nullptr; c = CMSG_NXTHDR(&m, c)) {
        if (c->cmsg_level == SOL_SOCKET && c->cmsg_type == SCM_RIGHTS) {
          int n = (int)((c->cmsg_len - CMSG_LEN(0)) / sizeof(int));
          const int* got = reinterpret_cast<const int*>(CMSG_DATA(c));
          for (int i = 0; i < n; ++i) {
            if (*nfds < maxFds) {
              fds[(*nfds)++] = got[i];
            } else {
              close(got[i]);
            }
          }
        }
      }
      if (m.msg_flags & MSG_CTRUNC) {
        TN_WARN("bootstrap: descriptor message truncated");
        return Io::kError;
      }
      break;
    }
    if (rc == 0) return Io::kError;
    if (errno == EINTR) continue;
    if (errno == EAGAIN || errno == EWOULDBLOCK) {
      Io w = waitFd(fd, POLLIN, d);
      if (w != Io::kOk) return w;
      continue;
    }
    return Io::kError;
  }
  return readAll(fd, p + done, bytes - done, d);
}

sockaddr_un addressOf(const char* path, socklen_t* len) {
  sockaddr_un a{};
  a.sun_family = AF_UNIX;
  const size_t n = strnlen(path, sizeof(a.sun_path) - 1);
  memcpy(a.sun_path, path, n);  // the rest is zero: a{} above
  *len = (socklen_t)(offsetof(sockaddr_un, sun_path) + strlen(a.sun_path) + 1);
  return a;
}

int newSocket() { return socket(AF_UNIX, SOCK_STREAM | SOCK_NONBLOCK | SOCK_CLOEXEC, 0); }

// Connects to rank 0, retrying while the path does not exist yet or refuses.
int connectHub(const char* path, Deadline d, Io* why) {
  socklen_t len;
  sockaddr_un a = addressOf(path, &len);
  while (msLeft(d) > 0) {
    int fd = newSocket();
    if (fd < 0) {
      *why = Io::kError;
      return -1;
    }
    if (connect(fd, reinterpret_cast<sockaddr*>(&a), len) == 0) return fd;
    int err = errno;
    if (err == EINPROGRESS) {
      Io w = waitFd(fd, POLLOUT, d);
      if (w == Io::kOk) {
        socklen_t l = sizeof(err);
        if (getsockopt(fd, SOL_SOCKET, SO_ERROR, &err, &l) == 0 && err == 0) return fd;
      } else if (w == Io::kTimeout) {
        close(fd);
        break;
      }
    }
    close(fd);
    if (err != ENOENT && err != ECONNREFUSED && err != EINTR && err != EAGAIN) {
      *why = Io::kError;
      return -1;
    }
    int pause = std::min(10, msLeft(d));
    if (pause > 0) poll(nullptr, 0, pause);
  }
  *why = Io::kTimeout;
  return -1;
}

bool allowedPathChar(unsigned char ch) {
  return (ch >= 'a' && ch <= 'z') || (ch >= 'A' && ch <= 'Z') ||
         (ch >= '0' && ch <= '9') || ch == '-' || ch == '_' || ch == '.' ||
         ch == '/';
}

}  // namespace

tncclResult bootstrapNewTcpId(tncclUniqueId* id, const char* addr, int port) {
  if (id == nullptr || port <= 0 || port > 65535) return TNCCL_INVALID_ARGUMENT;
  TcpIdPayload p{};
  if (!parseIpv4(addr, &p.ipv4)) return TNCCL_INVALID_ARGUMENT;
  p.magic = kTcpIdMagic;
  p.version = kWireVersion;
  p.port = (uint32_t)port;
  do {
    if (!randomBytes(&p.nonce, sizeof(p.nonce))) return TNCCL_SYSTEM_ERROR;
  } while (p.nonce == 0);
  memcpy(id->bytes, &p, sizeof(p));
  return TNCCL_SUCCESS;
}

bool bootstrapDecodeTcpId(const tncclUniqueId& id, uint32_t* ipv4, int* port, uint64_t* nonce) {
  TcpIdPayload p{};
  memcpy(&p, id.bytes, sizeof(p));
  if (p.magic != kTcpIdMagic || p.version != kWireVersion || p.port == 0 || p.port > 65535 ||
      p.nonce == 0 || p.ipv4 == 0)
    return false;
  *ipv4 = p.ipv4;
  *port = (int)p.port;
  *nonce = p.nonce;
  return true;
}

tncclResult bootstrapNewId(tncclUniqueId* id) {
  if (id == nullptr) return TNCCL_INVALID_ARGUMENT;
  const std::string tcp = envStr("TNCCL_BOOTSTRAP_ADDR", "");
  if (!tcp.empty()) {
    const size_t colon = tcp.rfind(':');
    if (colon == std::string::npos) {
      TN_WARN("TNCCL_BOOTSTRAP_ADDR must be <ipv4>:<port>, got '%s'", tcp.c_str());
      return TNCCL_INVALID_ARGUMENT;
    }
    const std::string host = tcp.substr(0, colon);
    char* end = nullptr;
    const long port = strtol(tcp.c_str() + colon + 1, &end, 10);
    if (end == tcp.c_str() + colon + 1 || *end != '\0') return TNCCL_INVALID_ARGUMENT;
    return bootstrapNewTcpId(id, host.c_str(), (int)port);
  }
  unsigned char rnd[16];
  if (!randomBytes(rnd, sizeof(rnd))) return TNCCL_SYSTEM_ERROR;
  char hex[33];
  static const char kHex[] = "0123456789abcdef";
  for (int i = 0; i < 16; ++i) {
    hex[2 * i] = kHex[rnd[i] >> 4];
    hex[2 * i + 1] = kHex[rnd[i] & 15];
  }
  hex[32] = '\0';
  std::string dir = envStr("TNCCL_SOCKET_DIR", "/tmp");
  while (dir.size() > 1 && dir.back() == '/') dir.pop_back();
  IdPayload p{};
  p.magic = kIdMagic;
  p.version = kWireVersion;
  int n = snprintf(p.path, sizeof(p.path), "%s/%s%lu-%ld-%s.sock", dir.c_str(),
                   kBaseName, (unsigned long)geteuid(), (long)getpid(), hex);
  if (n <= 0 || (size_t)n >= sizeof(p.path)) return TNCCL_SYSTEM_ERROR;
  p.pathLength = (uint32_t)n;
  memcpy(id->bytes, &p, sizeof(p));
  return TNCCL_SUCCESS;
}

bool bootstrapDecodeId(const tncclUniqueId& id, char (&path)[108]) {
  IdPayload p{};
  memcpy(&p, id.bytes, sizeof(p));
  if (p.magic != kIdMagic || p.version != kWireVersion || p.pathLength < 2 ||
      p.pathLength >= sizeof(p.path) || p.path[0] != '/' ||
      memchr(p.path, '\0', p.pathLength) != nullptr) {
    return false;
  }
  for (uint32_t i = 0; i < p.pathLength; ++i) {
    if (!allowedPathChar((unsigned char)p.path[i])) return false;
  }
  // The basename must be one this library generates.
  const char* slash = (const char*)memrchr(p.path, '/', p.pathLength);
  const char* base = slash + 1;
  size_t baseLen = p.pathLength - (size_t)(base - p.path);
  if (baseLen <= sizeof(kBaseName) - 1 ||
      memcmp(base, kBaseName, sizeof(kBaseName) - 1) != 0) {
    return false;
  }
  if (strstr(p.path, "/../") != nullptr) return false;
  memcpy(path, p.path, p.pathLength);
  path[p.pathLength] = '\0';
  return true;
}

tncclResult bootstrapOpen(Bootstrap* b, const tncclUniqueId& id, int nranks,
                          int rank, uint64_t configHash, int timeoutMs) {
  if (b == nullptr || b->active || nranks < 2 || nranks > kMaxRankFds ||
      rank < 0 || rank >= nranks) {
    return TNCCL_INVALID_ARGUMENT;
  }
  char path[108] = {};
  uint32_t ip = 0;
  int port = 0;
  uint64_t nonce = 0;
  const bool tcp = bootstrapDecodeTcpId(id, &ip, &port, &nonce);
  if (!tcp && !bootstrapDecodeId(id, path)) return TNCCL_INVALID_ARGUMENT;
  b->rank = rank;
  b->nranks = nranks;
  b->timeoutMs = timeoutMs;
  b->opSeq = 0;
  b->tcp = tcp;
  b->nonce = nonce;
  b->hubIpv4 = ip;
  Deadline d = deadlineIn(timeoutMs);

  if (rank == 0) {
    b->peerFds.assign((size_t)nranks, -1);
    if (tcp) {
      char addr[INET_ADDRSTRLEN] = {};
      in_addr ia{};
      ia.s_addr = ip;
      inet_ntop(AF_INET, &ia, addr, sizeof(addr));
      b->listenFd = tcpListen(addr, port, nranks, nullptr);
      if (b->listenFd < 0) {
        TN_WARN("bootstrap: cannot listen on %s:%d: %s", addr, port, strerror(errno));
        bootstrapClose(b);
        return TNCCL_SYSTEM_ERROR;
      }
      b->active = true;
    } else {
      b->listenFd = newSocket();
      if (b->listenFd < 0) {
        bootstrapClose(b);
        return TNCCL_SYSTEM_ERROR;
      }
      b->active = true;
      socklen_t len;
      sockaddr_un a = addressOf(path, &len);
      if (bind(b->listenFd, reinterpret_cast<sockaddr*>(&a), len) != 0) {
        TN_WARN("bootstrap: bind(%s) failed: %s", path, strerror(errno));
        bootstrapClose(b);  // path not owned: never unlink another rendezvous
        return TNCCL_SYSTEM_ERROR;
      }
      memcpy(b->path, path, strnlen(path, sizeof(b->path) - 1) + 1);
      b->ownsPath = true;
      if (chmod(path, S_IRUSR | S_IWUSR) != 0 || listen(b->listenFd, nranks) != 0) {
        bootstrapClose(b);
        return TNCCL_SYSTEM_ERROR;
      }
    }
    for (int joined = 1; joined < nranks; ++joined) {
      Io why = Io::kOk;
      int fd = acceptOne(b->listenFd, d, &why);
      if (fd < 0) {
        TN_WARN("bootstrap: rank 0 waited for %d of %d ranks: %s", nranks - joined,
                nranks - 1, why == Io::kTimeout ? "timed out" : "accept failed");
        bootstrapClose(b);
        return toResult(why);
      }
      Hello h{};
      Io io = recvFrame(fd, kHello, 0, &h, sizeof(h), nullptr, d);
      if (io != Io::kOk) {
        close(fd);
        bootstrapClose(b);
        return toResult(io);
      }
      tncclResult st = TNCCL_SUCCESS;
      if (h.nranks != nranks || h.rank <= 0 || h.rank >= nranks ||
          b->peerFds[(size_t)h.rank] != -1) {
        st = TNCCL_INVALID_ARGUMENT;
      } else if (h.nonce != nonce) {
        TN_WARN("bootstrap: a rank of another communicator joined (nonce mismatch)");
        st = TNCCL_INVALID_ARGUMENT;
      } else if (h.configHash != configHash) {
        TN_WARN("bootstrap: rank %d has a different TNCCL_* configuration", h.rank);
        st = TNCCL_INVALID_ARGUMENT;
      }
      io = sendFrame(fd, kHelloAck, 0, (uint32_t)st, nullptr, 0, d);
      if (io != Io::kOk || st != TNCCL_SUCCESS) {
        close(fd);
        bootstrapClose(b);
        return st != TNCCL_SUCCESS ? st : toResult(io);
      }
      b->peerFds[(size_t)h.rank] = fd;
    }
    close(b->listenFd);
    b->listenFd = -1;
    return TNCCL_SUCCESS;
  }

  Io why = Io::kOk;
  b->hubFd = tcp ? tcpConnect(ip, port, d, &why) : connectHub(path, d, &why);
  if (b->hubFd < 0) {
    bootstrapClose(b);
    return toResult(why);
  }
  b->active = true;
  Hello h{rank, nranks, (int32_t)getpid(), 0, configHash, nonce};
  uint32_t st = 0;
  Io io = sendFrame(b->hubFd, kHello, 0, 0, &h, sizeof(h), d);
  if (io == Io::kOk) io = recvFrame(b->hubFd, kHelloAck, 0, nullptr, 0, &st, d);
  if (io != Io::kOk) {
    bootstrapClose(b);
    return toResult(io);
  }
  if (st != TNCCL_SUCCESS) {
    bootstrapClose(b);
    return st < TNCCL_NUM_RESULTS ? (tncclResult)st : TNCCL_SYSTEM_ERROR;
  }
  return TNCCL_SUCCESS;
}

tncclResult bootstrapAllGather(Bootstrap* b, const void* send, void* recv,
                               size_t bytes) {
  if (b == nullptr || !b->active || bytes > kMaxGatherBytes ||
      (bytes != 0 && (send == nullptr || recv == nullptr))) {
    return TNCCL_INVALID_ARGUMENT;
  }
  const uint32_t op = ++b->opSeq;
  const size_t total = bytes * (size_t)b->nranks;
  Deadline d = deadlineIn(b->timeoutMs);
  auto* out = static_cast<unsigned char*>(recv);
  if (b->rank == 0) {
    if (bytes) memcpy(out, send, bytes);
    for (int r = 1; r < b->nranks; ++r) {
      Io io = recvFrame(b->peerFds[(size_t)r], kGather, op,
                        bytes ? out + (size_t)r * bytes : nullptr, bytes, nullptr, d);
      if (io != Io::kOk) return toResult(io);
    }
    for (int r = 1; r < b->nranks; ++r) {
      Io io = sendFrame(b->peerFds[(size_t)r], kGatherResult, op, 0, out, total, d);
      if (io != Io::kOk) return toResult(io);
    }
    return TNCCL_SUCCESS;
  }
  Io io = sendFrame(b->hubFd, kGather, op, 0, send, bytes, d);
  if (io == Io::kOk) io = recvFrame(b->hubFd, kGatherResult, op, out, total, nullptr, d);
  return toResult(io);
}

tncclResult bootstrapBarrier(Bootstrap* b) {
  if (b == nullptr || !b->active) return TNCCL_INVALID_ARGUMENT;
  const uint32_t op = ++b->opSeq;
  Deadline d = deadlineIn(b->timeoutMs);
  if (b->rank == 0) {
    for (int r = 1; r < b->nranks; ++r) {
      Io io = recvFrame(b->peerFds[(size_t)r], kBarrier, op, nullptr, 0, nullptr, d);
      if (io != Io::kOk) return toResult(io);
    }
    for (int r = 1; r < b->nranks; ++r) {
      Io io = sendFrame(b->peerFds[(size_t)r], kBarrierRelease, op, 0, nullptr, 0, d);
      if (io != Io::kOk) return toResult(io);
    }
    return TNCCL_SUCCESS;
  }
  Io io = sendFrame(b->hubFd, kBarrier, op, 0, nullptr, 0, d);
  if (io == Io::kOk) io = recvFrame(b->hubFd, kBarrierRelease, op, nullptr, 0, nullptr, d);
  return toResult(io);
}

tncclResult bootstrapAllGatherFds(Bootstrap* b, int myFd, int* fds) {
  if (b == nullptr || !b->active || fds == nullptr) return TNCCL_INVALID_ARGUMENT;
  if (b->tcp) return TNCCL_UNSUPPORTED;  // same answer on every rank, no message
  const uint32_t op = ++b->opSeq;
  const int P = b->nranks;
  Deadline d = deadlineIn(b->timeoutMs);
  for (int r = 0; r < P; ++r) fds[r] = -1;
  int32_t token = 0x46445321;  // payload byte carrier for the descriptors
  if (b->rank == 0) {
    tncclResult st = myFd >= 0 ? TNCCL_SUCCESS : TNCCL_SYSTEM_ERROR;
    std::vector<int> got((size_t)P, -1);
    Io io = Io::kOk;
    for (int r = 1; r < P && io == Io::kOk; ++r) {
      uint32_t peerSt = 0;
      int n = 0;
      int32_t tk = 0;
      io = recvFrameFds(b->peerFds[(size_t)r], kFdGather, op, &tk, sizeof(tk),
                        &peerSt, &got[(size_t)r], 1, &n, d);
      if (io == Io::kOk && (peerSt != TNCCL_SUCCESS || n != 1) && st == TNCCL_SUCCESS) {
        st = peerSt != TNCCL_SUCCESS ? (tncclResult)peerSt : TNCCL_SYSTEM_ERROR;
      }
    }
    if (io != Io::kOk) {
      for (int fd : got) if (fd >= 0) close(fd);
      return toResult(io);
    }
    got[0] = myFd;
    for (int r = 1; r < P && io == Io::kOk; ++r) {
      if (st == TNCCL_SUCCESS) {
        io = sendFrameFds(b->peerFds[(size_t)r], kFdGatherResult, op, 0, &token,
                          sizeof(token), got.data(), P, d);
      } else {
        io = sendFrameFds(b->peerFds[(size_t)r], kFdGatherResult, op, (uint32_t)st,
                          &token, sizeof(token), nullptr, 0, d);
      }
    }
    for (int r = 1; r < P; ++r) {
      if (st == TNCCL_SUCCESS && io == Io::kOk) {
        fds[r] = got[(size_t)r];
      } else if (got[(size_t)r] >= 0) {
        close(got[(size_t)r]);
      }
    }
    if (io != Io::kOk) return toResult(io);
    if (st != TNCCL_SUCCESS) return st;
    fds[0] = dup(myFd);
    return fds[0] >= 0 ? TNCCL_SUCCESS : TNCCL_SYSTEM_ERROR;
  }
  Io io;
  if (myFd >= 0) {
    io = sendFrameFds(b->hubFd, kFdGather, op, 0, &token, sizeof(token), &myFd, 1, d);
  } else {
    io = sendFrameFds(b->hubFd, kFdGather, op, TNCCL_SYSTEM_ERROR, &token,
                      sizeof(token), nullptr, 0, d);
  }
  if (io != Io::kOk) return toResult(io);
  uint32_t st = 0;
  int n = 0;
  int32_t tk = 0;
  io = recvFrameFds(b->hubFd, kFdGatherResult, op, &tk, sizeof(tk), &st, fds, P, &n, d);
  if (io != Io::kOk || st != TNCCL_SUCCESS || n != P) {
    for (int i = 0; i < n; ++i) {
      if (fds[i] >= 0) close(fds[i]);
      fds[i] = -1;
    }
    if (io != Io::kOk) return toResult(io);
    return st != TNCCL_SUCCESS && st < TNCCL_NUM_RESULTS ? (tncclResult)st
                                                          : TNCCL_SYSTEM_ERROR;
  }
  return TNCCL_SUCCESS;
}

tncclResult bootstrapBroadcastFd(Bootstrap* b, int fd, int* out) {
  if (b == nullptr || !b->active || out == nullptr) return TNCCL_INVALID_ARGUMENT;
  if (b->tcp) return TNCCL_UNSUPPORTED;
  const uint32_t op = ++b->opSeq;
  Deadline d = deadlineIn(b->timeoutMs);
  *out = -1;
  int32_t token = 0x46444243;
  if (b->rank == 0) {
    tncclResult st = fd >= 0 ? TNCCL_SUCCESS : TNCCL_SYSTEM_ERROR;
    for (int r = 1; r < b->nranks; ++r) {
      Io io = sendFrameFds(b->peerFds[(size_t)r], kFdBcast, op, (uint32_t)st, &token,
                           sizeof(token), fd >= 0 ? &fd : nullptr, fd >= 0 ? 1 : 0, d);
      if (io != Io::kOk) return toResult(io);
    }
    if (st != TNCCL_SUCCESS) return st;
    *out = dup(fd);
    return *out >= 0 ? TNCCL_SUCCESS : TNCCL_SYSTEM_ERROR;
  }
  uint32_t st = 0;
  int n = 0;
  int32_t tk = 0;
  Io io = recvFrameFds(b->hubFd, kFdBcast, op, &tk, sizeof(tk), &st, out, 1, &n, d);
  if (io != Io::kOk) return toResult(io);
  if (st != TNCCL_SUCCESS || n != 1) {
    if (n == 1 && *out >= 0) close(*out);
    *out = -1;
    return st != TNCCL_SUCCESS && st < TNCCL_NUM_RESULTS ? (tncclResult)st
                                                          : TNCCL_SYSTEM_ERROR;
  }
  return TNCCL_SUCCESS;
}

void bootstrapClose(Bootstrap* b) {
  if (b == nullptr) return;
  if (b->hubFd >= 0) close(b->hubFd);
  b->hubFd = -1;
  for (int& fd : b->peerFds) {
    if (fd >= 0) close(fd);
    fd = -1;
  }
  b->peerFds.clear();
  if (b->listenFd >= 0) close(b->listenFd);
  b->listenFd = -1;
  if (b->ownsPath && b->path[0] != '\0') unlink(b->path);
  b->ownsPath = false;
  b->path[0] = '\0';
  b->rank = -1;
  b->nranks = 0;
  b->active = false;
  b->tcp = false;
  b->nonce = 0;
  b->hubIpv4 = 0;
}

}  // namespace tnccl
