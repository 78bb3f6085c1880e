// bootstrap_test.cc - CPU-only tests of the AF_UNIX and TCP control plane
// with forked ranks (no GPU): id codecs, rendezvous, all-gather, barrier,
// descriptor passing, and the failure paths (bad id, nranks mismatch,
// duplicate rank, missing rank, peer death, configuration mismatch, ranks
// out of step, a TCP rank of another communicator). Every failure is made on
// the host; every wait is bounded by the bootstrap deadline.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/socket.h>
#include <sys/wait.h>
#include <unistd.h>

#include <functional>
#include <string>
#include <vector>

#include "bootstrap.h"
#include "sockio.h"

using namespace tnccl;

namespace {

int gFailed = 0;

void report(const char* name, bool ok) {
  printf("%-28s %s\n", name, ok ? "ok" : "FAILED");
  fflush(stdout);
  if (!ok) ++gFailed;
}

// Forks one child per entry of `ranks`; child i runs fn(i) and exits with
// its return value. Returns the exit codes (or 255 for abnormal exits).
std::vector<int> forkRanks(int n, const std::function<int(int)>& fn) {
  std::vector<pid_t> kids;
  for (int i = 0; i < n; ++i) {
    pid_t p = fork();
    if (p == 0) {
      fflush(stdout);
      _exit(fn(i));
    }
    kids.push_back(p);
  }
  std::vector<int> codes;
  for (pid_t k : kids) {
    int st = 0;
    waitpid(k, &st, 0);
    codes.push_back(WIFEXITED(st) ? WEXITSTATUS(st) : 255);
  }
  return codes;
}

int memfdWith(const std::string& text) {
  int fd = memfd_create("tnccl-test", MFD_CLOEXEC);
  if (fd < 0) return -1;
  if (write(fd, text.data(), text.size()) != (ssize_t)text.size()) return -1;
  return fd;
}

std::string readFd(int fd) {
  char buf[64] = {};
  ssize_t n = pread(fd, buf, sizeof(buf) - 1, 0);
  return n > 0 ? std::string(buf, (size_t)n) : std::string();
}

void testIdCodec() {
  tncclUniqueId id{};
  bool ok = bootstrapNewId(&id) == TNCCL_SUCCESS;
  char path[108];
  ok = ok && bootstrapDecodeId(id, path) && strstr(path, "tnccl-b200-") != nullptr;
  tncclUniqueId bad = id;
  bad.bytes[0] ^= 0xff;  // magic
  ok = ok && !bootstrapDecodeId(bad, path);
  bad = id;
  bad.bytes[16 + 5] = '!';  // a path character outside the allowed set
  ok = ok && !bootstrapDecodeId(bad, path);
  bad = id;
  uint32_t len = 200;  // longer than the path field
  memcpy(&bad.bytes[12], &len, 4);
  ok = ok && !bootstrapDecodeId(bad, path);
  tncclUniqueId zero{};
  ok = ok && !bootstrapDecodeId(zero, path);
  Bootstrap b;
  ok = ok && bootstrapOpen(&b, zero, 2, 0, 0, 100) == TNCCL_INVALID_ARGUMENT;
  report("id codec / bad id", ok);
}

void testRendezvous(int P) {
  tncclUniqueId id{};
  bootstrapNewId(&id);
  auto codes = forkRanks(P, [&](int r) -> int {
    Bootstrap b;
    if (bootstrapOpen(&b, id, P, r, 42, 5000) != TNCCL_SUCCESS) return 10;
    int64_t mine[2] = {r, 7 * r + 1};
    std::vector<int64_t> all((size_t)P * 2);
    if (bootstrapAllGather(&b, mine, all.data(), sizeof(mine)) != TNCCL_SUCCESS) return 11;
    for (int p = 0; p < P; ++p)
      if (all[(size_t)p * 2] != p || all[(size_t)p * 2 + 1] != 7 * p + 1) return 12;
    for (int i = 0; i < 3; ++i)
      if (bootstrapBarrier(&b) != TNCCL_SUCCESS) return 13;
    // Descriptor all-gather: every rank shares a memfd holding its rank.
    int fd = memfdWith("rank" + std::to_string(r));
    std::vector<int> fds((size_t)P, -1);
    if (bootstrapAllGatherFds(&b, fd, fds.data()) != TNCCL_SUCCESS) return 14;
    for (int p = 0; p < P; ++p) {
      if (readFd(fds[(size_t)p]) != "rank" + std::to_string(p)) return 15;
      close(fds[(size_t)p]);
    }
    close(fd);
    // Broadcast from rank 0.
    int root = r == 0 ? memfdWith("root") : -1;
    int got = -1;
    if (bootstrapBroadcastFd(&b, root, &got) != TNCCL_SUCCESS) return 16;
    if (readFd(got) != "root") return 17;
    close(got);
    if (root >= 0) close(root);
    // Zero-byte all-gather is legal.
    if (bootstrapAllGather(&b, nullptr, nullptr, 0) != TNCCL_SUCCESS) return 18;
    bootstrapClose(&b);
    return 0;
  });
  bool ok = true;
  for (int c : codes) ok = ok && c == 0;
  char path[108];
  bootstrapDecodeId(id, path);
  ok = ok && access(path, F_OK) != 0;  // rank 0 unlinked its socket
  char name[64];
  snprintf(name, sizeof(name), "rendezvous P=%d", P);
  report(name, ok);
  if (!ok)
    for (size_t i = 0; i < codes.size(); ++i) printf("  rank %zu exit %d\n", i, codes[i]);
}

void testNranksMismatch() {
  tncclUniqueId id{};
  bootstrapNewId(&id);
  auto codes = forkRanks(2, [&](int r) -> int {
    Bootstrap b;
    return (int)bootstrapOpen(&b, id, r == 0 ? 2 : 3, r == 0 ? 0 : 1, 1, 2000);
  });
  report("nranks mismatch", codes[0] == TNCCL_INVALID_ARGUMENT &&
                                codes[1] == TNCCL_INVALID_ARGUMENT);
}

void testDuplicateRank() {
  tncclUniqueId id{};
  bootstrapNewId(&id);
  auto codes = forkRanks(3, [&](int r) -> int {
    Bootstrap b;
    tncclResult res = bootstrapOpen(&b, id, 3, r == 0 ? 0 : 1, 1, 2000);
    if (res != TNCCL_SUCCESS || r == 0) return (int)res;
    // The claimant accepted first joined; its next collective must fail
    // because rank 0 gave up on the rendezvous.
    return 50 + (int)bootstrapBarrier(&b);
  });
  // Rank 0 rejects the second hello for rank 1; both claimants fail.
  bool ok = codes[0] == TNCCL_INVALID_ARGUMENT && codes[1] != 0 && codes[2] != 0 &&
            codes[1] != 50 && codes[2] != 50;
  report("duplicate rank", ok);
}

void testConfigMismatch() {
  tncclUniqueId id{};
  bootstrapNewId(&id);
  auto codes = forkRanks(2, [&](int r) -> int {
    Bootstrap b;
    return (int)bootstrapOpen(&b, id, 2, r, r == 0 ? 1 : 2, 2000);
  });
  report("config hash mismatch", codes[0] == TNCCL_INVALID_ARGUMENT &&
                                     codes[1] == TNCCL_INVALID_ARGUMENT);
}

void testMissingRank() {
  tncclUniqueId id{};
  bootstrapNewId(&id);
  // Rank 2 of 3 never starts.
  auto codes = forkRanks(2, [&](int r) -> int {
    Bootstrap b;
    tncclResult res = bootstrapOpen(&b, id, 3, r, 1, 500);
    if (r == 0) return (int)res;
    if (res != TNCCL_SUCCESS) return 100 + (int)res;
    // Rank 1 joined; its next collective must fail within the deadline.
    int x = 1, all[3];
    return 50 + (int)bootstrapAllGather(&b, &x, all, sizeof(x));
  });
  bool ok = codes[0] == TNCCL_TIMEOUT && codes[1] != 50;
  report("missing rank -> timeout", ok);
  if (!ok) printf("  codes %d %d\n", codes[0], codes[1]);
}

void testPeerDeath() {
  tncclUniqueId id{};
  bootstrapNewId(&id);
  auto codes = forkRanks(3, [&](int r) -> int {
    Bootstrap b;
    if (bootstrapOpen(&b, id, 3, r, 1, 1000) != TNCCL_SUCCESS) return 90;
    if (bootstrapBarrier(&b) != TNCCL_SUCCESS) return 91;
    if (r == 2) _exit(0);  // dies without taking part in the gather
    int x = r, all[3];
    return (int)bootstrapAllGather(&b, &x, all, sizeof(x));
  });
  bool ok = codes[0] != 0 && codes[1] != 0 && codes[2] == 0;
  report("peer death mid-gather", ok);
  if (!ok) printf("  codes %d %d %d\n", codes[0], codes[1], codes[2]);
}

void testOutOfStep() {
  tncclUniqueId id{};
  bootstrapNewId(&id);
  auto codes = forkRanks(2, [&](int r) -> int {
    Bootstrap b;
    if (bootstrapOpen(&b, id, 2, r, 1, 1000) != TNCCL_SUCCESS) return 90;
    if (r == 0) return (int)bootstrapBarrier(&b);
    int x = 1, all[2];
    return (int)bootstrapAllGather(&b, &x, all, sizeof(x));
  });
  report("ranks out of step", codes[0] != 0 && codes[1] != 0);
}

// The largest all-gather (1 MiB per rank) moves far more than a socket
// buffer holds, so every frame goes through partial reads and writes.
void testLargeGather(bool tcp) {
  const int P = 4;
  const size_t n = (1u << 20) / sizeof(uint32_t);
  tncclUniqueId id{};
  if (tcp) {
    int port = 0;
    int fd = tcpListen("127.0.0.1", 0, 1, &port);
    if (fd >= 0) close(fd);
    bootstrapNewTcpId(&id, "127.0.0.1", port);
  } else {
    bootstrapNewId(&id);
  }
  auto codes = forkRanks(P, [&](int r) -> int {
    Bootstrap b;
    if (bootstrapOpen(&b, id, P, r, 7, 10000) != TNCCL_SUCCESS) return 10;
    std::vector<uint32_t> mine(n), all(n * P);
    for (size_t i = 0; i < n; ++i) mine[i] = (uint32_t)(r * 2654435761u + i * 40503u);
    for (int rep = 0; rep < 2; ++rep) {
      if (bootstrapAllGather(&b, mine.data(), all.data(), n * sizeof(uint32_t)) != TNCCL_SUCCESS)
        return 11;
      for (int p = 0; p < P; ++p)
        for (size_t i = 0; i < n; i += 997)
          if (all[(size_t)p * n + i] != (uint32_t)(p * 2654435761u + i * 40503u)) return 12;
    }
    // One byte more than the limit is refused on every rank, before any I/O.
    std::vector<char> big((1u << 20) + 1), bigAll(big.size() * P);
    if (bootstrapAllGather(&b, big.data(), bigAll.data(), big.size()) != TNCCL_INVALID_ARGUMENT)
      return 13;
    if (bootstrapBarrier(&b) != TNCCL_SUCCESS) return 14;
    bootstrapClose(&b);
    return 0;
  });
  bool ok = true;
  for (int c : codes) ok = ok && c == 0;
  report(tcp ? "tcp all-gather 1 MiB/rank" : "all-gather 1 MiB/rank", ok);
  if (!ok)
    for (size_t i = 0; i < codes.size(); ++i) printf("  rank %zu exit %d\n", i, codes[i]);
}

// ---- TCP rendezvous --------------------------------------------------------

int freePort() {
  int port = 0;
  int fd = tcpListen("127.0.0.1", 0, 1, &port);
  if (fd >= 0) close(fd);
  return port;
}

void testTcpIdCodec() {
  tncclUniqueId id{};
  bool ok = bootstrapNewTcpId(&id, "127.0.0.1", 29500) == TNCCL_SUCCESS;
  uint32_t ip = 0;
  int port = 0;
  uint64_t nonce = 0, nonce2 = 0;
  char path[108];
  ok = ok && bootstrapDecodeTcpId(id, &ip, &port, &nonce) && port == 29500 && nonce != 0;
  ok = ok && !bootstrapDecodeId(id, path);  // not an AF_UNIX id
  tncclUniqueId id2{};
  ok = ok && bootstrapNewTcpId(&id2, "127.0.0.1", 29500) == TNCCL_SUCCESS &&
       bootstrapDecodeTcpId(id2, &ip, &port, &nonce2) && nonce2 != nonce;
  tncclUniqueId un{};
  ok = ok && bootstrapNewId(&un) == TNCCL_SUCCESS && !bootstrapDecodeTcpId(un, &ip, &port, &nonce);
  ok = ok && bootstrapNewTcpId(&id, "not-an-address", 29500) == TNCCL_INVALID_ARGUMENT;
  ok = ok && bootstrapNewTcpId(&id, "127.0.0.1", 0) == TNCCL_INVALID_ARGUMENT;
  ok = ok && bootstrapNewTcpId(&id, "127.0.0.1", 70000) == TNCCL_INVALID_ARGUMENT;
  // Through the environment, as tncclGetUniqueId does.
  setenv("TNCCL_BOOTSTRAP_ADDR", "127.0.0.1:29501", 1);
  ok = ok && bootstrapNewId(&id) == TNCCL_SUCCESS && bootstrapDecodeTcpId(id, &ip, &port, &nonce) &&
       port == 29501;
  setenv("TNCCL_BOOTSTRAP_ADDR", "127.0.0.1", 1);  // no port
  ok = ok && bootstrapNewId(&id) == TNCCL_INVALID_ARGUMENT;
  unsetenv("TNCCL_BOOTSTRAP_ADDR");
  report("tcp id codec", ok);
}

void testTcpRendezvous(int P) {
  tncclUniqueId id{};
  bootstrapNewTcpId(&id, "127.0.0.1", freePort());
  auto codes = forkRanks(P, [&](int r) -> int {
    Bootstrap b;
    if (bootstrapOpen(&b, id, P, r, 42, 5000) != TNCCL_SUCCESS) return 10;
    if (!b.tcp) return 11;
    int64_t mine[2] = {r, 5 * r + 3};
    std::vector<int64_t> all((size_t)P * 2);
    if (bootstrapAllGather(&b, mine, all.data(), sizeof(mine)) != TNCCL_SUCCESS) return 12;
    for (int p = 0; p < P; ++p)
      if (all[(size_t)p * 2] != p || all[(size_t)p * 2 + 1] != 5 * p + 3) return 13;
    if (bootstrapBarrier(&b) != TNCCL_SUCCESS) return 14;
    // Descriptor passing needs AF_UNIX: every rank gets the same answer and
    // the collective sequence stays aligned.
    std::vector<int> fds((size_t)P, -1);
    if (bootstrapAllGatherFds(&b, 0, fds.data()) != TNCCL_UNSUPPORTED) return 15;
    int got = -1;
    if (bootstrapBroadcastFd(&b, 0, &got) != TNCCL_UNSUPPORTED) return 16;
    if (bootstrapAllGather(&b, mine, all.data(), sizeof(mine)) != TNCCL_SUCCESS) return 17;
    if (bootstrapBarrier(&b) != TNCCL_SUCCESS) return 18;
    bootstrapClose(&b);
    return 0;
  });
  bool ok = true;
  for (int c : codes) ok = ok && c == 0;
  char name[64];
  snprintf(name, sizeof(name), "tcp rendezvous P=%d", P);
  report(name, ok);
  if (!ok)
    for (size_t i = 0; i < codes.size(); ++i) printf("  rank %zu exit %d\n", i, codes[i]);
}

void testTcpNonceMismatch() {
  // Two ids for the same address: a rank holding the other id is refused.
  const int port = freePort();
  tncclUniqueId a{}, b2{};
  bootstrapNewTcpId(&a, "127.0.0.1", port);
  bootstrapNewTcpId(&b2, "127.0.0.1", port);
  auto codes = forkRanks(2, [&](int r) -> int {
    Bootstrap b;
    return (int)bootstrapOpen(&b, r == 0 ? a : b2, 2, r, 1, 3000);
  });
  report("tcp nonce mismatch", codes[0] == TNCCL_INVALID_ARGUMENT &&
                                   codes[1] == TNCCL_INVALID_ARGUMENT);
}

// A peer whose "rank 0" answers its hello with random bytes (or a frame
// header claiming a huge payload) fails the rendezvous instead of crashing,
// hanging past its deadline or allocating what the header claims.
void testFuzzedHub() {
  bool ok = true;
  for (int seed = 0; seed < 20 && ok; ++seed) {
    int port = 0;
    const int lfd = tcpListen("127.0.0.1", 0, 4, &port);
    tncclUniqueId id{};
    bootstrapNewTcpId(&id, "127.0.0.1", port);
    pid_t kid = fork();
    if (kid == 0) {
      Bootstrap b;
      _exit(bootstrapOpen(&b, id, 2, 1, 1, 3000) == TNCCL_SUCCESS ? 0 : 1);
    }
    Io why = Io::kOk;
    const int fd = acceptOne(lfd, deadlineIn(3000), &why);
    if (fd >= 0) {
      unsigned char buf[512];
      (void)recv(fd, buf, sizeof(buf), 0);  // the hello
      uint64_t x = 0x9e3779b97f4a7c15ull * (uint64_t)(seed + 7);
      const size_t n = 1 + (size_t)(x % sizeof(buf));
      for (size_t i = 0; i < n; ++i) {
        x ^= x << 13;
        x ^= x >> 7;
        x ^= x << 17;
        buf[i] = (unsigned char)x;
      }
      if (seed % 2 == 0 && n >= 24) memset(buf + 16, 0xff, 8);  // a huge "payload" length
      (void)writeAll(fd, buf, n, deadlineIn(1000));
      close(fd);
    }
    close(lfd);
    int st = 0;
    waitpid(kid, &st, 0);
    ok = fd >= 0 && WIFEXITED(st) && WEXITSTATUS(st) == 1;
  }
  report("fuzzed answers from rank 0", ok);
}

// Random 128-byte ids decode as neither kind unless their magic matches,
// and never crash the decoders.
void testFuzzedIds() {
  uint64_t x = 88172645463325252ull;
  auto next = [&x] {
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    return x;
  };
  bool ok = true;
  for (int it = 0; it < 20000; ++it) {
    tncclUniqueId id{};
    for (auto& b : id.bytes) b = (unsigned char)next();
    if (it % 4 == 1) memcpy(id.bytes, "TNCBB002", 8);  // right magic, random rest
    if (it % 4 == 2) memcpy(id.bytes, "TNCBT003", 8);
    char path[108];
    uint32_t ip = 0;
    int port = 0;
    uint64_t nonce = 0;
    const bool un = bootstrapDecodeId(id, path);
    const bool tcp = bootstrapDecodeTcpId(id, &ip, &port, &nonce);
    ok = ok && !(un && tcp);
    if (un) ok = ok && path[0] == '/' && strlen(path) < sizeof(path);
    if (tcp) ok = ok && port > 0 && port < 65536 && nonce != 0;
  }
  report("fuzzed ids", ok);
}

// A TCP rendezvous is reachable by anything on the network: random bytes
// instead of a hello must make rank 0 fail the rendezvous, not crash or hang.
void testFuzzedHello() {
  bool ok = true;
  for (int seed = 0; seed < 20 && ok; ++seed) {
    int port = 0;
    int fd0 = tcpListen("127.0.0.1", 0, 1, &port);
    if (fd0 >= 0) close(fd0);
    tncclUniqueId id{};
    bootstrapNewTcpId(&id, "127.0.0.1", port);
    pid_t kid = fork();
    if (kid == 0) {
      Bootstrap b;
      _exit(bootstrapOpen(&b, id, 2, 0, 1, 3000) == TNCCL_SUCCESS ? 0 : 1);
    }
    uint32_t ip = 0;
    parseIpv4("127.0.0.1", &ip);
    Io why = Io::kOk;
    int fd = tcpConnect(ip, port, deadlineIn(3000), &why);
    if (fd >= 0) {
      unsigned char junk[256];
      uint64_t x = 0x9e3779b97f4a7c15ull * (uint64_t)(seed + 1);
      const size_t n = 1 + (size_t)(x % sizeof(junk));
      for (size_t i = 0; i < n; ++i) {
        x ^= x << 13;
        x ^= x >> 7;
        x ^= x << 17;
        junk[i] = (unsigned char)x;
      }
      (void)writeAll(fd, junk, n, deadlineIn(1000));
      close(fd);
    }
    int st = 0;
    waitpid(kid, &st, 0);
    ok = fd >= 0 && WIFEXITED(st) && WEXITSTATUS(st) == 1;
  }
  report("tcp rendezvous: fuzzed hello", ok);
}

}  // namespace

int main() {
  setenv("TNCCL_DEBUG", "NONE", 0);
  testIdCodec();
  for (int P : {2, 3, 4, 8}) testRendezvous(P);
  testNranksMismatch();
  testDuplicateRank();
  testConfigMismatch();
  testMissingRank();
  testPeerDeath();
  testOutOfStep();
  testTcpIdCodec();
  for (int P : {2, 4}) testTcpRendezvous(P);
  testTcpNonceMismatch();
  testLargeGather(false);
  testLargeGather(true);
  testFuzzedHello();
  testFuzzedIds();
  testFuzzedHub();
  printf("bootstrap_test: %s\n", gFailed ? "FAIL" : "PASS");
  return gFailed ? 1 : 0;
}
