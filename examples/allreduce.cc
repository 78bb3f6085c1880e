// allreduce.cc - fork one process per GPU, run one FP32 SUM all-reduce and
// check the result on the host.
//
// Usage: tnccl_allreduce <nranks> <count>
//
// Same contract as tiny-nccl's examples/allreduce.cc:22-127: rank r uses CUDA
// device r, contributes r + 1 everywhere, and every element must equal
// n(n+1)/2; the parent waits for every child and exits 0 only if all passed.
#include <cuda_runtime_api.h>
#include <sys/wait.h>
#include <unistd.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "tnccl.h"

namespace {

bool check(cudaError_t e, const char* what, int rank) {
  if (e == cudaSuccess) return true;
  fprintf(stderr, "rank %d: %s: %s\n", rank, what, cudaGetErrorString(e));
  return false;
}

int runRank(int rank, int nranks, size_t count, tncclUniqueId id) {
  if (!check(cudaSetDevice(rank), "cudaSetDevice", rank)) return 1;
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
  bool ok = check(cudaStreamCreate(&stream), "cudaStreamCreate", rank);
  if (ok && count) {
    ok = check(cudaMalloc(reinterpret_cast<void**>(&buf), count * sizeof(float)), "cudaMalloc", rank) &&
         check(cudaMalloc(reinterpret_cast<void**>(&out), count * sizeof(float)), "cudaMalloc",
               rank) &&
         check(cudaMemcpyAsync(buf, host.data(), count * sizeof(float), cudaMemcpyHostToDevice,
                               stream),
               "copy in", rank);
  }
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
  if (tncclCommDestroy(comm) != TNCCL_SUCCESS) ok = false;
  if (buf) cudaFree(buf);
  if (out) cudaFree(out);
  if (stream) cudaStreamDestroy(stream);
  return ok ? 0 : 1;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 3) {
    fprintf(stderr, "usage: %s <nranks> <count>\n", argv[0]);
    return 2;
  }
  const int nranks = atoi(argv[1]);
  const size_t count = strtoull(argv[2], nullptr, 10);
  if (nranks < 1) {
    fprintf(stderr, "nranks must be positive\n");
    return 2;
  }
  tncclUniqueId id{};
  if (tncclGetUniqueId(&id) != TNCCL_SUCCESS) return 1;
  std::vector<pid_t> kids;
  for (int r = 0; r < nranks; ++r) {
    pid_t pid = fork();
    if (pid == 0) _exit(runRank(r, nranks, count, id));
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
