// bootstrap.h - host control plane: unique id, AF_UNIX star rendezvous,
// all-gather, barrier and file-descriptor passing.
//
// Behaviour kept from tiny-nccl (src/bootstrap.cc): the unique id names a
// Unix-socket path (tncclGetUniqueId :325, path decoding :221); rank 0 binds
// it (mode 0600), accepts nranks-1 peers and validates their hello (matching
// nranks, rank in range, no duplicate; bootstrapOpen :354); peers retry
// connect until the deadline (:264); every operation has a deadline
// (:73-114); all-gather is gather-to-root then broadcast (:459); barrier is
// collect-then-release (:502); rank 0 unlinks the path only if it bound it
// (:532).
//
// Added here: every frame carries a per-communicator operation number so that
// ranks that drift out of step fail with an error instead of mis-pairing
// messages; the hello carries a configuration hash; SCM_RIGHTS passing of
// POSIX file descriptors (cuMem / multicast handles) as an all-gather and a
// broadcast from rank 0; deadline expiry returns TNCCL_TIMEOUT.
//
// TCP rendezvous for ranks on several hosts (tiny-nccl's socket design,
// docs/design-v0.2.md:78, leaves its encoding open): when
// TNCCL_BOOTSTRAP_ADDR=<ipv4>:<port> is set where the id is created, the id
// carries that address and a random 64-bit communicator nonce instead of a
// socket path; rank 0 listens there, the others connect with retry, and the
// hello must carry the same nonce. Frames, all-gather and barrier are the
// same over both socket kinds; descriptor passing needs AF_UNIX and returns
// TNCCL_UNSUPPORTED on a TCP bootstrap.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <vector>

#include "tnccl.h"

namespace tnccl {

// Largest rank count the bootstrap accepts (descriptor messages carry one
// descriptor per rank).
constexpr int kMaxRankFds = 64;

struct Bootstrap {
  int rank = -1;
  int nranks = 0;
  int listenFd = -1;
  int hubFd = -1;             // non-root: connection to rank 0
  std::vector<int> peerFds;   // root: connection to every rank (index = rank)
  char path[108] = {};
  bool ownsPath = false;
  bool active = false;
  uint32_t opSeq = 0;         // bootstrap collectives issued so far
  int timeoutMs = 30000;
  bool tcp = false;           // TCP rendezvous (no descriptor passing)
  uint64_t nonce = 0;         // communicator nonce of a TCP id (0 for AF_UNIX)
  uint32_t hubIpv4 = 0;       // TCP: rank 0's address (network byte order)
};

// Encodes a fresh rendezvous into id: a TCP id when TNCCL_BOOTSTRAP_ADDR is
// set, else an AF_UNIX path with a random 128-bit suffix.
tncclResult bootstrapNewId(tncclUniqueId* id);
// A TCP id for rank 0 at addr:port (dotted quad, port 1..65535).
tncclResult bootstrapNewTcpId(tncclUniqueId* id, const char* addr, int port);

// Validates an AF_UNIX id and returns the socket path it names.
bool bootstrapDecodeId(const tncclUniqueId& id, char (&path)[108]);
// Validates a TCP id and returns rank 0's address (network byte order), port
// and the communicator nonce.
bool bootstrapDecodeTcpId(const tncclUniqueId& id, uint32_t* ipv4, int* port, uint64_t* nonce);

tncclResult bootstrapOpen(Bootstrap* b, const tncclUniqueId& id, int nranks,
                          int rank, uint64_t configHash, int timeoutMs);
tncclResult bootstrapAllGather(Bootstrap* b, const void* send, void* recv,
                               size_t bytes);
tncclResult bootstrapBarrier(Bootstrap* b);

// Every rank contributes one descriptor (or -1 when it has none, which makes
// the collective fail on every rank). TNCCL_UNSUPPORTED on every rank of a
// TCP bootstrap (the same for bootstrapBroadcastFd). On success fds[r] holds a descriptor
// for rank r's object, owned by the caller (fds[rank] is a duplicate of the
// caller's own descriptor).
tncclResult bootstrapAllGatherFds(Bootstrap* b, int myFd, int* fds);

// Rank 0 passes fd (or -1 to signal failure); every other rank receives a
// duplicate in *out (owned by the caller).
tncclResult bootstrapBroadcastFd(Bootstrap* b, int fd, int* out);

void bootstrapClose(Bootstrap* b);

}  // namespace tnccl
