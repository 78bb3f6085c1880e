// allreduce_gpu_test.cc - multi-process all-reduce correctness on real GPUs.
//
// Usage: allreduce_gpu_test <nranks> [quick|full|stress|nvls_order] [algo,...]
//
// Forks one process per GPU (rank r uses device r). Every rank generates all
// ranks' seeded Uniform[-1,1) inputs on the host, so each rank can compute the
// algorithm-aware oracle (oracle.h) for its own output and compare bit for
// bit. NVLS reduces inside the switch in an order the hardware picks; for
// more than two ranks it is checked against a tolerance and the report says
// whether it happened to be bit-exact.
//
// "stress" is BASELINE config 2: count = 1,048,576 fp32, 100 iterations with
// fresh inputs on one bound stream, every iteration checked. The other modes
// end by checking that device memory did not grow across collectives of 4 to
// 64 MiB and that the mailbox guard lines are intact.
//
// "nvls_order" studies the switch's fp32 reduction: the same inputs are
// reduced 5 times by the NVLS kernel (run-to-run stability must be exact),
// and the result is compared element by element with candidate summation
// orders (rank order 0..P-1, its reverse, a balanced pairwise tree, and the
// P rotations that start at rank k); rank 0 prints the fraction of elements
// each candidate reproduces.
#include <cuda_runtime_api.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/wait.h>
#include <unistd.h>

#include <cmath>
#include <utility>
#include <string>
#include <vector>

#include "oracle.h"
#include "tnccl.h"

namespace {

struct Case {
  tncclAlgo_t algo;
  int dtype;
  size_t count;
  bool inPlace;
  bool avg;
  size_t misalign;  // elements of offset applied to send/recv
};

const char* typeName(int t) { return t == 0 ? "f32" : t == 1 ? "bf16" : "f16"; }

bool cudaOk(cudaError_t e, int rank, const char* what) {
  if (e == cudaSuccess) return true;
  fprintf(stderr, "rank %d: %s: %s\n", rank, what, cudaGetErrorString(e));
  return false;
}

struct Runner {
  int rank, P;
  tncclComm_t comm = nullptr;
  cudaStream_t stream = nullptr;
  tncclCommInfo info{};
  void* dsend = nullptr;
  void* drecv = nullptr;
  size_t cap = 0;
  int failures = 0;
  int passes = 0;
  int nvlsInexact = 0;

  bool ensure(size_t bytes) {
    if (bytes <= cap) return true;
    if (dsend) cudaFree(dsend);
    if (drecv) cudaFree(drecv);
    cap = bytes;
    return cudaOk(cudaMalloc(&dsend, cap), rank, "cudaMalloc") &&
           cudaOk(cudaMalloc(&drecv, cap), rank, "cudaMalloc");
  }

  // Runs one case; returns false on a hard error (API/CUDA failure).
  bool run(const Case& c, uint64_t seed) {
    const size_t es = oracle::typeSize(c.dtype);
    const size_t off = c.misalign * es;
    if (!ensure(c.count * es + off + 64)) return false;
    std::vector<std::vector<float>> x((size_t)P);
    std::vector<unsigned char> raw, mine;
    for (int r = 0; r < P; ++r) {
      oracle::fillInput(c.dtype, seed, r, c.count, x[(size_t)r], raw);
      if (r == rank) mine = raw;
    }
    const float alpha = c.avg ? 1.0f / (float)P : 1.0f;
    tncclAlgo_t algo = c.algo;
    if (algo == TNCCL_ALGO_AUTO) tncclCommSelectAlgo(comm, c.count, (tncclDataType_t)c.dtype, &algo);
    std::vector<float> want;
    if (algo == TNCCL_ALGO_RING) {
      const uint64_t V = 16 / es;
      tnccl::ChunkPlan pl = tnccl::makeChunkPlan(c.count, P, info.channels,
                                                 info.ringChunkBytes / es,
                                                 info.ringMinChunkBytes / es, V);
      oracle::ring(c.dtype, x, alpha, pl, V, want);
    } else {
      oracle::canonical(c.dtype, x, alpha, want);
    }
    char* s = static_cast<char*>(dsend) + off;
    char* d = c.inPlace ? s : static_cast<char*>(drecv) + off;
    if (c.count &&
        !cudaOk(cudaMemcpyAsync(s, mine.data(), mine.size(), cudaMemcpyHostToDevice, stream), rank,
                "H2D"))
      return false;
    tncclResult r = tncclAllReduceEx(s, d, c.count, (tncclDataType_t)c.dtype,
                                     c.avg ? tncclAvg : tncclSum, 1.0f, c.algo, comm, stream);
    if (r != TNCCL_SUCCESS) {
      fprintf(stderr, "rank %d: allreduce(%s) failed: %s\n", rank, tncclAlgoName(c.algo),
              tncclGetErrorString(r));
      return false;
    }
    std::vector<unsigned char> got(c.count * es);
    if (c.count &&
        !cudaOk(cudaMemcpyAsync(got.data(), d, got.size(), cudaMemcpyDeviceToHost, stream), rank,
                "D2H"))
      return false;
    if (!cudaOk(cudaStreamSynchronize(stream), rank, "sync")) return false;
    tncclResult async = TNCCL_SUCCESS;
    tncclCommGetAsyncError(comm, &async);
    if (async != TNCCL_SUCCESS) {
      fprintf(stderr, "rank %d: async error %s\n", rank, tncclGetErrorString(async));
      return false;
    }
    // The switch's reduction order is its own for P > 2, and its bf16/fp16 rounding
    // is not round-to-nearest-even (measured: 1-ulp differences), so NVLS is
    // checked against a tolerance in those cases.
    const bool tolerant = algo == TNCCL_ALGO_NVLS && (P > 2 || c.dtype != oracle::kF32);
    size_t bad = 0, firstBad = 0;
    bool exact = true;
    for (size_t i = 0; i < c.count; ++i) {
      const float g = oracle::rawToFloat(c.dtype, &got[i * es]);
      const float w = want[i];
      if (g == w || (std::isnan(g) && std::isnan(w))) continue;
      exact = false;
      bool okTol = false;
      if (tolerant) {
        const float ulp = c.dtype == 0 ? 6e-7f : c.dtype == 1 ? 8e-3f : 1e-3f;
        okTol = std::fabs(g - w) <= ulp * (float)P * (1.0f + std::fabs(w));
      }
      if (!okTol) {
        if (bad++ == 0) firstBad = i;
      }
    }
    if (tolerant && !exact) ++nvlsInexact;
    if (bad) {
      ++failures;
      const float g = oracle::rawToFloat(c.dtype, &got[firstBad * es]);
      fprintf(stderr,
              "rank %d: FAIL %s %s count=%zu inplace=%d avg=%d misalign=%zu: %zu bad, first at "
              "%zu: got %.9g want %.9g\n",
              rank, tncclAlgoName(c.algo), typeName(c.dtype), c.count, (int)c.inPlace,
              (int)c.avg, c.misalign, bad, firstBad, g, want[firstBad]);
    } else {
      ++passes;
    }
    return true;
  }
};

int nvlsOrderStudy(struct Runner& R);

int runRank(int rank, int P, const std::string& mode, const std::vector<tncclAlgo_t>& algosIn,
            tncclUniqueId id) {
  if (!cudaOk(cudaSetDevice(rank), rank, "cudaSetDevice")) return 1;
  Runner R;
  R.rank = rank;
  R.P = P;
  tncclResult r = tncclCommInitRank(&R.comm, P, id, rank);
  if (r != TNCCL_SUCCESS) {
    fprintf(stderr, "rank %d: init failed: %s\n", rank, tncclGetErrorString(r));
    return 1;
  }
  tncclCommGetInfo(R.comm, &R.info);
  if (!cudaOk(cudaStreamCreateWithFlags(&R.stream, cudaStreamNonBlocking), rank, "stream"))
    return 1;
  std::vector<tncclAlgo_t> algos;
  for (tncclAlgo_t a : algosIn)
    if (a != TNCCL_ALGO_NVLS || R.info.nvlsEnabled) algos.push_back(a);
  bool hard = false;
  uint64_t seed = 1;
  if (mode == "nvls_order") {
    hard = nvlsOrderStudy(R) != 0;
  } else if (mode == "stress") {
    for (int it = 0; it < 100 && !hard; ++it)
      hard = !R.run(Case{TNCCL_ALGO_AUTO, 0, 1048576, false, false, 0}, 1000 + (uint64_t)it);
  } else {
    std::vector<size_t> counts = {1, 3, 8, 1000, 4097, 65539, 262144, 1048581};
    if (mode == "full") {
      counts.push_back(4194304 + 1000);
      counts.push_back(16u << 20);
    }
    for (tncclAlgo_t a : algos) {
      for (int t = 0; t < 3 && !hard; ++t) {
        for (size_t n : counts) {
          if (hard) break;
          hard = !R.run(Case{a, t, n, false, false, 0}, seed++);
          if (!hard && (n == 4097 || n == 262144))
            hard = !R.run(Case{a, t, n, true, false, 0}, seed++);
          if (!hard && (n == 65539 || n == 1048581))
            hard = !R.run(Case{a, t, n, false, true, 0}, seed++);
          if (!hard && n == 4097) hard = !R.run(Case{a, t, n, false, false, 1}, seed++);
        }
      }
    }
    // AUTO across sizes, then count = 0 between non-empty collectives.
    for (size_t n : {(size_t)0, (size_t)4096, (size_t)0, (size_t)3 << 20, (size_t)0})
      if (!hard) hard = !R.run(Case{TNCCL_ALGO_AUTO, 0, n, false, false, 0}, seed++);
  }
  if (!hard && mode != "stress" && mode != "nvls_order") {
    // Communication memory is constant: no device allocation grows with the
    // message (the buffers of this test are freed around the measurement),
    // and the guard lines after every mailbox area are intact.
    auto dropBuffers = [&R]() {
      cudaFree(R.dsend);
      cudaFree(R.drecv);
      R.dsend = R.drecv = nullptr;
      R.cap = 0;
      cudaDeviceSynchronize();
    };
    dropBuffers();
    size_t free0 = 0, free1 = 0, total = 0;
    cudaMemGetInfo(&free0, &total);
    for (size_t n : {(size_t)1 << 20, (size_t)4 << 20, (size_t)16 << 20})
      if (!hard) hard = !R.run(Case{TNCCL_ALGO_AUTO, 0, n, false, false, 0}, seed++);
    dropBuffers();
    cudaMemGetInfo(&free1, &total);
    const long long grew = (long long)free0 - (long long)free1;
    if (grew > (32ll << 20)) {
      fprintf(stderr, "rank %d: device memory grew by %lld bytes across collectives\n", rank,
              grew);
      hard = true;
    }
    int corrupted = 0;
    if (tncclCommValidate(R.comm, &corrupted) != TNCCL_SUCCESS || corrupted != 0) {
      fprintf(stderr, "rank %d: %d mailbox guard line(s) overwritten\n", rank, corrupted);
      hard = true;
    }
  }
  printf("rank %d: nvls=%d passed=%d failed=%d nvls_inexact=%d hard=%d\n", rank,
         R.info.nvlsEnabled, R.passes, R.failures, R.nvlsInexact, (int)hard);
  fflush(stdout);
  if (tncclCommDestroy(R.comm) != TNCCL_SUCCESS) hard = true;
  cudaFree(R.dsend);
  cudaFree(R.drecv);
  cudaStreamDestroy(R.stream);
  return (hard || R.failures) ? 1 : 0;
}

// fp32 sums of P values in the candidate orders of the nvls_order study.
float sumOrder(const std::vector<float>& v, const std::vector<int>& order) {
  float a = v[(size_t)order[0]];
  for (size_t i = 1; i < order.size(); ++i) a = oracle::add(a, v[(size_t)order[i]]);
  return a;
}
float sumTree(const std::vector<float>& v, int lo, int hi) {
  if (hi - lo == 1) return v[(size_t)lo];
  const int mid = lo + (hi - lo + 1) / 2;
  return oracle::add(sumTree(v, lo, mid), sumTree(v, mid, hi));
}

// Returns 0 when the NVLS results are stable run to run; prints the order study.
int nvlsOrderStudy(Runner& R) {
  const int P = R.P;
  if (!R.info.nvlsEnabled) {
    if (R.rank == 0) printf("nvls_order: NVLS not enabled on this communicator (skipped)\n");
    return 0;
  }
  const size_t n = 1 << 20;
  if (!R.ensure(n * 4 + 64)) return 1;
  std::vector<std::vector<float>> x((size_t)P);
  std::vector<unsigned char> raw, mine;
  for (int r = 0; r < P; ++r) {
    oracle::fillInput(oracle::kF32, 77, r, n, x[(size_t)r], raw);
    // Spread the magnitudes so that different orders round differently.
    for (size_t i = 0; i < n; ++i) x[(size_t)r][i] *= (float)(1u << ((i + (size_t)r * 7) % 23));
    if (r == R.rank) {
      mine.resize(n * 4);
      memcpy(mine.data(), x[(size_t)r].data(), n * 4);
    }
  }
  std::vector<float> first(n), got(n);
  int unstable = 0;
  for (int run = 0; run < 5; ++run) {
    if (!cudaOk(cudaMemcpyAsync(R.dsend, mine.data(), n * 4, cudaMemcpyHostToDevice, R.stream),
                R.rank, "H2D"))
      return 1;
    if (tncclAllReduceEx(R.dsend, R.drecv, n, tncclFloat32, tncclSum, 1.0f, TNCCL_ALGO_NVLS,
                         R.comm, R.stream) != TNCCL_SUCCESS)
      return 1;
    if (!cudaOk(cudaMemcpyAsync(got.data(), R.drecv, n * 4, cudaMemcpyDeviceToHost, R.stream),
                R.rank, "D2H") ||
        !cudaOk(cudaStreamSynchronize(R.stream), R.rank, "sync"))
      return 1;
    if (run == 0)
      first = got;
    else if (memcmp(first.data(), got.data(), n * 4) != 0)
      ++unstable;
  }
  std::vector<std::pair<std::string, std::vector<int>>> orders;
  std::vector<int> seq((size_t)P);
  for (int r = 0; r < P; ++r) seq[(size_t)r] = r;
  orders.push_back({"rank order 0..P-1", seq});
  orders.push_back({"reverse", std::vector<int>(seq.rbegin(), seq.rend())});
  for (int k = 1; k < P; ++k) {
    std::vector<int> rot((size_t)P);
    for (int r = 0; r < P; ++r) rot[(size_t)r] = (k + r) % P;
    orders.push_back({"rotation from rank " + std::to_string(k), rot});
  }
  std::vector<size_t> match(orders.size() + 1, 0);
  std::vector<float> v((size_t)P);
  for (size_t i = 0; i < n; ++i) {
    for (int r = 0; r < P; ++r) v[(size_t)r] = x[(size_t)r][i];
    for (size_t o = 0; o < orders.size(); ++o)
      if (sumOrder(v, orders[o].second) == first[i]) ++match[o];
    if (sumTree(v, 0, P) == first[i]) ++match[orders.size()];
  }
  if (R.rank == 0) {
    printf("nvls_order: P=%d, %zu fp32 elements, runs bit-identical: %s\n", P, n,
           unstable ? "NO" : "yes");
    for (size_t o = 0; o < orders.size(); ++o)
      printf("nvls_order:   %-26s matches %6.2f %%\n", orders[o].first.c_str(),
             100.0 * (double)match[o] / (double)n);
    printf("nvls_order:   %-26s matches %6.2f %%\n", "balanced pairwise tree",
           100.0 * (double)match[orders.size()] / (double)n);
    fflush(stdout);
  }
  return unstable ? 1 : 0;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2) {
    fprintf(stderr, "usage: %s <nranks> [quick|full|stress] [algo,...]\n", argv[0]);
    return 2;
  }
  const int P = atoi(argv[1]);
  const std::string mode = argc > 2 ? argv[2] : "quick";
  std::vector<tncclAlgo_t> algos = {TNCCL_ALGO_ONESHOT, TNCCL_ALGO_TWOSHOT, TNCCL_ALGO_RING,
                                    TNCCL_ALGO_NVLS};
  if (argc > 3) {
    algos.clear();
    std::string list = argv[3];
    size_t pos = 0;
    while (pos <= list.size()) {
      size_t e = list.find(',', pos);
      std::string a = list.substr(pos, e == std::string::npos ? std::string::npos : e - pos);
      if (a == "ring") algos.push_back(TNCCL_ALGO_RING);
      if (a == "oneshot") algos.push_back(TNCCL_ALGO_ONESHOT);
      if (a == "twoshot") algos.push_back(TNCCL_ALGO_TWOSHOT);
      if (a == "nvls") algos.push_back(TNCCL_ALGO_NVLS);
      if (e == std::string::npos) break;
      pos = e + 1;
    }
  }
  // No CUDA call in the parent: a driver initialised before fork() is not
  // usable in the children.
  tncclUniqueId id{};
  if (tncclGetUniqueId(&id) != TNCCL_SUCCESS) return 1;
  std::vector<pid_t> kids;
  for (int r = 0; r < P; ++r) {
    pid_t pid = fork();
    if (pid == 0) _exit(runRank(r, P, mode, algos, id));
    kids.push_back(pid);
  }
  int ok = 1;
  for (pid_t k : kids) {
    int st = 0;
    if (waitpid(k, &st, 0) < 0 || !WIFEXITED(st) || WEXITSTATUS(st) != 0) ok = 0;
  }
  printf("allreduce_gpu_test: %s\n", ok ? "PASS" : "FAIL");
  return ok ? 0 : 1;
}
