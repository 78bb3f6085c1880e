// allreduce.cc - fork one process per GPU, run one FP32 SUM all-reduce and
// check the result on the host.
//
// Usage:
//   tnccl_allreduce <nranks> <count>
//       every rank on this host (AF_UNIX rendezvous).
//   tnccl_allreduce --make-id <ipv4>:<port>
//       prints a TCP rendezvous id (hex) for a run across hosts; rank 0 will
//       listen at that address.
//   tnccl_allreduce <nranks> <count> --ranks <first>:<last> --id <hex>
//       this host's ranks first..last of a run across hosts (device =
//       rank - first); every host is given the same id. Ring edges between
//       hosts use the socket data plane (TNCCL_NET=auto).
//
// TNCCL_EXAMPLE_REGISTERED=1 allocates the buffers with tncclMemAlloc and
// registers them with the communicator (tncclCommRegister), so that an NVLS
// all-reduce runs the zero-copy kernel on them (explicitly with
// TNCCL_ALGO=nvls, or chosen by AUTO from TNCCL_NVLS_ZC_MIN_BYTES: 16 MiB on
// 8 ranks); without NVLS the registration is refused and the buffers are
// used unregistered.
//
// Same contract as tiny-nccl's examples/allreduce.cc:22-127: rank r
// contributes r + 1 everywhere, and every element must equal n(n+1)/2; the
// parent waits for every child and exits 0 only if all passed.
#include <cuda_runtime_api.h>
#include <sys/wait.h>
#include <unistd.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "tnccl.h"

namespace {

bool check(cudaError_t e, const char* what, int rank) {
  if (e == cudaSuccess) return true;
  fprintf(stderr, "rank %d: %s: %s\n", rank, what, cudaGetErrorString(e));
  return false;
}

int runRank(int rank, int device, int nranks, size_t count, tncclUniqueId id) {
  if (!check(cudaSetDevice(device), "cudaSetDevice", rank)) return 1;
  tncclComm_t comm = nullptr;
  tncclResult r = tncclCommInitRank(&comm, nranks, id, rank);
  if (r != TNCCL_SUCCESS) {
    fprintf(stderr, "rank %d: init: %s\n", rank, tncclGetErrorString(r));
    return 1;
  }
  cudaStream_t stream = nullptr;
  float* buf = nullptr;
  float* out = nullptr;
  std::vector<float> host(count, (float)(rank + 1));
  const char* regEnv = getenv("TNCCL_EXAMPLE_REGISTERED");
  const bool registered = regEnv != nullptr && atoi(regEnv) != 0 && count != 0;
  void* handles[2] = {nullptr, nullptr};
  bool ok = check(cudaStreamCreate(&stream), "cudaStreamCreate", rank);
  if (ok && registered) {
    // Registration is collective: every rank makes both calls, in this order.
    ok = tncclMemAlloc(reinterpret_cast<void**>(&buf), count * sizeof(float)) == TNCCL_SUCCESS &&
         tncclMemAlloc(reinterpret_cast<void**>(&out), count * sizeof(float)) == TNCCL_SUCCESS;
    if (!ok) fprintf(stderr, "rank %d: tncclMemAlloc failed\n", rank);
    for (int k = 0; ok && k < 2; ++k) {
      r = tncclCommRegister(comm, k == 0 ? (void*)buf : (void*)out, count * sizeof(float),
                            &handles[k]);
      if (r == TNCCL_UNSUPPORTED) {
        if (rank == 0 && k == 0) printf("no NVLS: buffers stay unregistered\n");
      } else if (r != TNCCL_SUCCESS) {
        fprintf(stderr, "rank %d: register: %s\n", rank, tncclGetErrorString(r));
        ok = false;
      }
    }
  } else if (ok && count) {
    ok = check(cudaMalloc(reinterpret_cast<void**>(&buf), count * sizeof(float)), "cudaMalloc",
               rank) &&
         check(cudaMalloc(reinterpret_cast<void**>(&out), count * sizeof(float)), "cudaMalloc",
               rank);
  }
  if (ok && count)
    ok = check(cudaMemcpyAsync(buf, host.data(), count * sizeof(float), cudaMemcpyHostToDevice,
                               stream),
               "copy in", rank);
  if (ok) {
    r = tncclAllReduceSumF32(buf, out, count, comm, stream);
    if (r != TNCCL_SUCCESS) {
      fprintf(stderr, "rank %d: all-reduce: %s\n", rank, tncclGetErrorString(r));
      ok = false;
    }
  }
  if (ok && count)
    ok = check(cudaMemcpyAsync(host.data(), out, count * sizeof(float), cudaMemcpyDeviceToHost,
                               stream),
               "copy out", rank);
  if (ok) ok = check(cudaStreamSynchronize(stream), "synchronize", rank);
  const float expected = (float)(nranks * (nranks + 1) / 2);
  for (size_t i = 0; ok && i < count; ++i) {
    if (std::fabs(host[i] - expected) > 1e-5f) {
      fprintf(stderr, "rank %d: mismatch at %zu: %g != %g\n", rank, i, host[i], expected);
      ok = false;
    }
  }
  for (void* h : handles)
    if (h != nullptr && tncclCommDeregister(comm, h) != TNCCL_SUCCESS) ok = false;
  if (tncclCommDestroy(comm) != TNCCL_SUCCESS) ok = false;
  if (registered) {
    tncclMemFree(buf);
    tncclMemFree(out);
  } else {
    if (buf) cudaFree(buf);
    if (out) cudaFree(out);
  }
  if (stream) cudaStreamDestroy(stream);
  return ok ? 0 : 1;
}

std::string toHex(const tncclUniqueId& id) {
  static const char kHex[] = "0123456789abcdef";
  std::string s;
  for (unsigned char b : id.bytes) {
    s += kHex[b >> 4];
    s += kHex[b & 15];
  }
  return s;
}

bool fromHex(const char* s, tncclUniqueId* id) {
  if (strlen(s) != 2 * sizeof(id->bytes)) return false;
  auto nib = [](char c) {
    return c >= '0' && c <= '9' ? c - '0' : c >= 'a' && c <= 'f' ? c - 'a' + 10 : -1;
  };
  for (size_t i = 0; i < sizeof(id->bytes); ++i) {
    const int hi = nib(s[2 * i]), lo = nib(s[2 * i + 1]);
    if (hi < 0 || lo < 0) return false;
    id->bytes[i] = (unsigned char)(hi * 16 + lo);
  }
  return true;
}

int usage(const char* prog) {
  fprintf(stderr,
          "usage: %s <nranks> <count> [--ranks <first>:<last> --id <hex>]\n"
          "       %s --make-id <ipv4>:<port>\n",
          prog, prog);
  return 2;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc == 3 && strcmp(argv[1], "--make-id") == 0) {
    const char* colon = strrchr(argv[2], ':');
    if (colon == nullptr) return usage(argv[0]);
    const std::string host(argv[2], (size_t)(colon - argv[2]));
    tncclUniqueId id{};
    if (tncclGetUniqueIdTcp(&id, host.c_str(), atoi(colon + 1)) != TNCCL_SUCCESS) {
      fprintf(stderr, "bad address %s\n", argv[2]);
      return 2;
    }
    printf("%s\n", toHex(id).c_str());
    return 0;
  }
  if (argc != 3 && argc != 7) return usage(argv[0]);
  const int nranks = atoi(argv[1]);
  const size_t count = strtoull(argv[2], nullptr, 10);
  if (nranks < 1) {
    fprintf(stderr, "nranks must be positive\n");
    return 2;
  }
  int first = 0, last = nranks - 1;
  tncclUniqueId id{};
  if (argc == 7) {
    if (strcmp(argv[3], "--ranks") != 0 || strcmp(argv[5], "--id") != 0 ||
        sscanf(argv[4], "%d:%d", &first, &last) != 2 || first < 0 || last < first ||
        last >= nranks || !fromHex(argv[6], &id))
      return usage(argv[0]);
  } else if (tncclGetUniqueId(&id) != TNCCL_SUCCESS) {
    return 1;
  }
  std::vector<pid_t> kids;
  for (int r = first; r <= last; ++r) {
    pid_t pid = fork();
    if (pid == 0) _exit(runRank(r, r - first, nranks, count, id));
    if (pid < 0) {
      perror("fork");
      return 1;
    }
    kids.push_back(pid);
  }
  bool ok = true;
  for (pid_t k : kids) {
    int st = 0;
    if (waitpid(k, &st, 0) < 0 || !WIFEXITED(st) || WEXITSTATUS(st) != 0) ok = false;
  }
  if (ok) printf("all ranks: ok\n");
  return ok ? 0 : 1;
}
