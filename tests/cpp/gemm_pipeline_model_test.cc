// gemm_pipeline_model_test.cc - threaded CPU model of the synchronisation of
// the tcgen05 GEMM kernels (csrc/ops/gemm_tcgen05.cu): one CTA per tile, the
// persistent kernel with two TMEM accumulators, and the persistent CTA pair
// (cta_group::2: the even CTA's full barrier armed for both CTAs' bytes and
// completed by both CTAs' loads, commits multicast to both CTAs' empty and
// accFull barriers, accEmpty collecting both CTAs' epilogue warps).
//
// The roles run as threads with the kernels' loop structure and parity
// formulas: the TMA producer, the MMA issuer and eight epilogue warps. An
// mbarrier is modelled with the PTX semantics the kernels rely on (a pending
// arrival count and a transaction count; a phase completes when both reach
// zero; try_wait.parity(p) succeeds once the phase with parity p completed,
// so a fresh barrier already "completed" parity 1). The asynchronous units
// are threads too: a TMA engine completes each load's transaction bytes after
// a random delay, and an MMA engine runs issued MMAs in order and performs
// each tcgen05.commit's arrival once every MMA issued before it finished.
//
// Checks: every stage the MMA reads holds the (tile, K block) the producer
// loaded for it (no stage reused too early), every accumulator the epilogue
// reads holds its own tile's complete sum (no accumulator reused too early),
// every tile is stored exactly once, no role waits longer than the bound,
// and the abort path (a producer that stops) ends every role.
#include <stdio.h>

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <deque>
#include <functional>
#include <mutex>
#include <random>
#include <thread>
#include <vector>

namespace {

int gFailed = 0;
void report(const char* what, bool ok) {
  printf("%-60s %s\n", what, ok ? "ok" : "FAILED");
  fflush(stdout);
  if (!ok) ++gFailed;
}

void jitter(std::mt19937& g, int maxUs) {
  const int us = (int)(g() % (unsigned)(maxUs + 1));
  if (us) std::this_thread::sleep_for(std::chrono::microseconds(us));
}

struct MBarrier {
  std::mutex mu;
  int count = 1, pending = 1;
  long tx = 0;
  unsigned phase = 0;  // completed phases

  void init(int c) {
    std::lock_guard<std::mutex> l(mu);
    count = pending = c;
    tx = 0;
    phase = 0;
  }
  void maybeComplete() {
    if (pending == 0 && tx == 0) {
      ++phase;
      pending = count;
    }
  }
  void arrive() {
    std::lock_guard<std::mutex> l(mu);
    --pending;
    maybeComplete();
  }
  void arriveExpectTx(long bytes) {
    std::lock_guard<std::mutex> l(mu);
    tx += bytes;
    --pending;
    maybeComplete();
  }
  void completeTx(long bytes) {
    std::lock_guard<std::mutex> l(mu);
    tx -= bytes;
    maybeComplete();
  }
  bool tryWait(unsigned parity) {
    std::lock_guard<std::mutex> l(mu);
    return (phase & 1u) != parity;
  }
};

// Bounded wait (the kernels' mbarWait): false on abort or after the bound.
bool waitBar(MBarrier& b, unsigned parity, std::atomic<int>& abort, bool ignoreAbort = false) {
  const auto t0 = std::chrono::steady_clock::now();
  while (!b.tryWait(parity)) {
    if (!ignoreAbort && abort.load()) return false;
    if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(5)) {
      abort.store(1);
      return false;
    }
    std::this_thread::yield();
  }
  return true;
}

// An asynchronous unit: runs queued jobs in order on its own thread.
struct Engine {
  std::mutex mu;
  std::condition_variable cv;
  std::deque<std::function<void()>> q;
  bool stop = false;
  std::thread th;
  explicit Engine(int seed, int maxUs) {
    th = std::thread([this, seed, maxUs] {
      std::mt19937 g((unsigned)seed);
      for (;;) {
        std::function<void()> job;
        {
          std::unique_lock<std::mutex> l(mu);
          cv.wait(l, [this] { return stop || !q.empty(); });
          if (q.empty()) return;
          job = std::move(q.front());
          q.pop_front();
        }
        jitter(g, maxUs);
        job();
      }
    });
  }
  void push(std::function<void()> f) {
    {
      std::lock_guard<std::mutex> l(mu);
      q.push_back(std::move(f));
    }
    cv.notify_one();
  }
  ~Engine() {
    {
      std::lock_guard<std::mutex> l(mu);
      stop = true;
    }
    cv.notify_one();
    th.join();
  }
};

constexpr int kStages = 4;
constexpr int kEpiWarps = 8;  // two per TMEM lane quarter, one column half each

struct Result {
  bool ok = true;
  int stored = 0;
  bool aborted = false;
};

// The persistent kernel (gemmBiasActPersistentKernel) for one CTA that owns
// `tiles` tiles of kBlocks K blocks each. stopAt >= 0: the producer stops
// after that many K blocks (a stuck load), which must end every role.
Result runPersistent(int tiles, int kBlocks, int seed, int stopAt = -1) {
  MBarrier full[kStages], empty[kStages], accFull[2], accEmpty[2], done;
  for (int s = 0; s < kStages; ++s) {
    full[s].init(1);
    empty[s].init(1);
  }
  for (int b = 0; b < 2; ++b) {
    accFull[b].init(1);
    accEmpty[b].init(kEpiWarps);
  }
  done.init(1);
  std::atomic<int> abort{0};
  // Contents: what each stage and accumulator currently holds.
  std::atomic<long> stage[kStages];
  std::atomic<long> accTile[2], accBlocks[2];
  for (auto& x : stage) x = -1;
  for (int b = 0; b < 2; ++b) accTile[b] = accBlocks[b] = -1;
  std::atomic<bool> bad{false};
  std::vector<std::atomic<int>> storedCount((size_t)tiles);
  for (auto& c : storedCount) c = 0;
  constexpr long kBytes = 48 * 1024;
  Result res;
  {
    Engine tma(seed * 7 + 1, 30), mmaUnit(seed * 7 + 2, 20);
    std::thread producer([&] {
      std::mt19937 g((unsigned)seed);
      unsigned gk = 0;
      for (int t = 0; t < tiles && !abort.load(); ++t) {
        for (int kb = 0; kb < kBlocks; ++kb, ++gk) {
          if (stopAt >= 0 && (int)gk == stopAt) {
            // A load that never lands: its waiters give up through abort.
            abort.store(1);
            break;
          }
          const unsigned s = gk % kStages, round = gk / kStages;
          if (!waitBar(empty[s], (round & 1u) ^ 1u, abort)) break;
          full[s].arriveExpectTx(kBytes);
          const long tag = (long)t * 1000 + kb;
          tma.push([&, s, tag] {
            stage[s].store(tag);
            full[s].completeTx(kBytes);
          });
          jitter(g, 5);
        }
      }
    });
    std::thread mma([&] {
      std::mt19937 g((unsigned)seed + 1);
      unsigned gk = 0, local = 0;
      for (int t = 0; t < tiles && !abort.load(); ++t, ++local) {
        const unsigned b = local & 1u, use = local >> 1;
        if (!waitBar(accEmpty[b], (use & 1u) ^ 1u, abort)) break;
        bool ok = true;
        for (int kb = 0; kb < kBlocks; ++kb, ++gk) {
          const unsigned s = gk % kStages;
          if (!(ok = waitBar(full[s], (gk / kStages) & 1u, abort))) break;
          const long want = (long)t * 1000 + kb;
          mmaUnit.push([&, s, b, t, kb, want] {
            if (stage[s].load() != want) bad = true;  // stage overwritten early
            if (kb == 0) {
              accTile[b] = t;
              accBlocks[b] = 1;
            } else {
              if (accTile[b].load() != t) bad = true;
              accBlocks[b].fetch_add(1);
            }
          });
          mmaUnit.push([&, s] { empty[s].arrive(); });  // tcgen05.commit
          jitter(g, 5);
        }
        if (!ok) break;
        mmaUnit.push([&, b] { accFull[b].arrive(); });
      }
      mmaUnit.push([&] { done.arrive(); });
      if (abort.load()) waitBar(done, 0, abort, true);
    });
    std::vector<std::thread> epi;
    for (int w = 0; w < kEpiWarps; ++w) {
      epi.emplace_back([&, w] {
        std::mt19937 g((unsigned)(seed * 13 + w));
        unsigned local = 0;
        for (int t = 0; t < tiles; ++t, ++local) {
          const unsigned b = local & 1u, use = local >> 1;
          if (!waitBar(accFull[b], use & 1u, abort)) break;
          // The four tcgen05.ld of this warp's rows and column half.
          for (int c = 0; c < 4; ++c) {
            if (accTile[b].load() != t || accBlocks[b].load() != kBlocks) bad = true;
            jitter(g, 3);
          }
          accEmpty[b].arrive();  // after the last read, before the stores
          jitter(g, 10);         // stores
          if (w == 0) storedCount[(size_t)t].fetch_add(1);
        }
      });
    }
    producer.join();
    mma.join();
    for (auto& th : epi) th.join();
    res.aborted = abort.load() != 0;
  }  // engines drain and stop
  for (auto& c : storedCount) {
    if (c.load() == 1) ++res.stored;
    if (c.load() > 1) res.ok = false;
  }
  res.ok = res.ok && !bad.load();
  return res;
}

// The CTA-pair kernel (gemmBiasActPairKernel) for one pair that owns `tiles`
// tiles. Barriers per CTA r; only CTA 0's full and accEmpty barriers are used.
Result runPair(int tiles, int kBlocks, int seed) {
  constexpr int kPairStages = 6;
  constexpr long kHalfBytes = 2 * 16 * 1024;  // one CTA's A and B halves per K block
  MBarrier full[2][kPairStages], empty[2][kPairStages], accFull[2][2], accEmpty[2][2], done;
  for (int r = 0; r < 2; ++r) {
    for (int s = 0; s < kPairStages; ++s) {
      full[r][s].init(1);
      empty[r][s].init(1);
    }
    for (int b = 0; b < 2; ++b) {
      accFull[r][b].init(1);
      accEmpty[r][b].init(2 * kEpiWarps);
    }
  }
  done.init(1);
  std::atomic<int> abort{0};
  std::atomic<long> stage[2][kPairStages];
  std::atomic<long> accTile[2][2], accBlocks[2][2];
  for (auto& cta : stage)
    for (auto& x : cta) x = -1;
  for (int r = 0; r < 2; ++r)
    for (int b = 0; b < 2; ++b) accTile[r][b] = accBlocks[r][b] = -1;
  std::atomic<bool> bad{false};
  std::vector<std::atomic<int>> storedCount((size_t)tiles * 2);
  for (auto& c : storedCount) c = 0;
  Result res;
  {
    Engine tma0(seed * 7 + 1, 30), tma1(seed * 7 + 3, 30), mmaUnit(seed * 7 + 2, 20);
    Engine* tmaOf[2] = {&tma0, &tma1};
    std::vector<std::thread> threads;
    for (int r = 0; r < 2; ++r) {
      threads.emplace_back([&, r] {  // producer of CTA r
        std::mt19937 g((unsigned)(seed + 17 * r));
        unsigned gk = 0;
        for (int t = 0; t < tiles && !abort.load(); ++t) {
          for (int kb = 0; kb < kBlocks; ++kb, ++gk) {
            const unsigned s = gk % kPairStages, round = gk / kPairStages;
            if (!waitBar(empty[r][s], (round & 1u) ^ 1u, abort)) break;
            if (r == 0) full[0][s].arriveExpectTx(2 * kHalfBytes);  // both CTAs' bytes
            const long tag = (long)t * 1000 + kb;
            // This CTA's loads land in its own stage and complete on CTA 0's barrier.
            tmaOf[r]->push([&, r, s, tag] {
              stage[r][s].store(tag);
              full[0][s].completeTx(kHalfBytes);
            });
            jitter(g, 5);
          }
        }
      });
    }
    threads.emplace_back([&] {  // MMA issuer, CTA 0
      std::mt19937 g((unsigned)seed + 1);
      unsigned gk = 0, local = 0;
      for (int t = 0; t < tiles && !abort.load(); ++t, ++local) {
        const unsigned b = local & 1u, use = local >> 1;
        if (!waitBar(accEmpty[0][b], (use & 1u) ^ 1u, abort)) break;
        bool ok = true;
        for (int kb = 0; kb < kBlocks; ++kb, ++gk) {
          const unsigned s = gk % kPairStages;
          if (!(ok = waitBar(full[0][s], (gk / kPairStages) & 1u, abort))) break;
          const long want = (long)t * 1000 + kb;
          mmaUnit.push([&, s, b, t, kb, want] {
            // The pair MMA reads both CTAs' stages and writes both TMEMs.
            if (stage[0][s].load() != want || stage[1][s].load() != want) bad = true;
            for (int r = 0; r < 2; ++r) {
              if (kb == 0) {
                accTile[r][b] = t;
                accBlocks[r][b] = 1;
              } else {
                if (accTile[r][b].load() != t) bad = true;
                accBlocks[r][b].fetch_add(1);
              }
            }
          });
          mmaUnit.push([&, s] {  // commit multicast to the pair
            empty[0][s].arrive();
            empty[1][s].arrive();
          });
          jitter(g, 5);
        }
        if (!ok) break;
        mmaUnit.push([&, b] {
          accFull[0][b].arrive();
          accFull[1][b].arrive();
        });
      }
      mmaUnit.push([&] { done.arrive(); });
      if (abort.load()) waitBar(done, 0, abort, true);
    });
    for (int r = 0; r < 2; ++r)
      for (int w = 0; w < kEpiWarps; ++w)
        threads.emplace_back([&, r, w] {  // epilogue warps of CTA r
          std::mt19937 g((unsigned)(seed * 13 + 100 * r + w));
          unsigned local = 0;
          for (int t = 0; t < tiles; ++t, ++local) {
            const unsigned b = local & 1u, use = local >> 1;
            if (!waitBar(accFull[r][b], use & 1u, abort)) break;
            for (int c = 0; c < 4; ++c) {
              if (accTile[r][b].load() != t || accBlocks[r][b].load() != kBlocks) bad = true;
              jitter(g, 3);
            }
            accEmpty[0][b].arrive();  // remote for CTA 1
            jitter(g, 10);
            if (w == 0) storedCount[(size_t)t * 2 + r].fetch_add(1);
          }
        });
    for (auto& th : threads) th.join();
    res.aborted = abort.load() != 0;
  }
  for (auto& c : storedCount) {
    if (c.load() == 1) ++res.stored;
    if (c.load() > 1) res.ok = false;
  }
  res.ok = res.ok && !bad.load();
  return res;
}

// The one-tile kernel (gemmBiasActKernel): one accumulator, one commit.
Result runSingle(int kBlocks, int seed) {
  MBarrier full[kStages], empty[kStages], accum;
  for (int s = 0; s < kStages; ++s) {
    full[s].init(1);
    empty[s].init(1);
  }
  accum.init(1);
  std::atomic<int> abort{0};
  std::atomic<long> stage[kStages];
  for (auto& x : stage) x = -1;
  std::atomic<long> blocks{0};
  std::atomic<bool> bad{false};
  std::atomic<int> storedWarps{0};
  constexpr long kBytes = 48 * 1024;
  Result res;
  {
    Engine tma(seed * 5 + 1, 30), mmaUnit(seed * 5 + 2, 20);
    std::thread producer([&] {
      for (int kb = 0; kb < kBlocks; ++kb) {
        const int s = kb % kStages;
        if (!waitBar(empty[s], ((unsigned)(kb / kStages) & 1u) ^ 1u, abort)) break;
        full[s].arriveExpectTx(kBytes);
        tma.push([&, s, kb] {
          stage[s].store(kb);
          full[s].completeTx(kBytes);
        });
      }
    });
    std::thread mma([&] {
      for (int kb = 0; kb < kBlocks; ++kb) {
        const int s = kb % kStages;
        if (!waitBar(full[s], (unsigned)(kb / kStages) & 1u, abort)) break;
        mmaUnit.push([&, s, kb] {
          if (stage[s].load() != kb) bad = true;
          blocks.fetch_add(1);
        });
        mmaUnit.push([&, s] { empty[s].arrive(); });
      }
      mmaUnit.push([&] { accum.arrive(); });
    });
    std::vector<std::thread> epi;
    for (int w = 0; w < kEpiWarps; ++w)
      epi.emplace_back([&] {
        if (!waitBar(accum, 0, abort)) return;
        if (blocks.load() != kBlocks) bad = true;
        storedWarps.fetch_add(1);
      });
    producer.join();
    mma.join();
    for (auto& th : epi) th.join();
    res.aborted = abort.load() != 0;
  }
  res.stored = storedWarps.load() == kEpiWarps ? 1 : 0;
  res.ok = !bad.load();
  return res;
}

}  // namespace

int main() {
  bool ok = true;
  for (int seed = 0; seed < 40 && ok; ++seed)
    for (int kBlocks : {1, 3, 4, 5, 12}) {
      Result r = runSingle(kBlocks, seed);
      ok = ok && r.ok && !r.aborted && r.stored == 1;
    }
  report("one-tile kernel: stages and accumulator hand-over", ok);

  ok = true;
  for (int seed = 0; seed < 25 && ok; ++seed)
    for (int tiles : {1, 2, 3, 7})
      for (int kBlocks : {1, 2, 5, 12}) {
        Result r = runPersistent(tiles, kBlocks, seed);
        if (!(r.ok && !r.aborted && r.stored == tiles)) {
          printf("  seed %d tiles %d kBlocks %d: ok %d aborted %d stored %d\n", seed, tiles,
                 kBlocks, r.ok, r.aborted, r.stored);
          ok = false;
        }
      }
  report("persistent kernel: stage ring across tiles, two accumulators", ok);

  ok = true;
  for (int seed = 0; seed < 15 && ok; ++seed)
    for (int tiles : {1, 2, 5})
      for (int kBlocks : {1, 4, 7, 12}) {
        Result r = runPair(tiles, kBlocks, seed);
        if (!(r.ok && !r.aborted && r.stored == 2 * tiles)) {
          printf("  pair seed %d tiles %d kBlocks %d: ok %d aborted %d stored %d\n", seed, tiles,
                 kBlocks, r.ok, r.aborted, r.stored);
          ok = false;
        }
      }
  report("CTA pair: shared full barrier, multicast commits, accEmpty x2", ok);

  ok = true;
  for (int seed = 0; seed < 10 && ok; ++seed) {
    const auto t0 = std::chrono::steady_clock::now();
    Result r = runPersistent(5, 4, seed, 9);  // stops inside the third tile
    const double s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    // Tiles that completed before the stop are intact; none after it.
    ok = r.ok && r.aborted && r.stored <= 2 && s < 4.0;
  }
  report("persistent kernel: a stopped producer ends every role", ok);

  printf("gemm_pipeline_model_test: %s\n", gFailed ? "FAIL" : "PASS");
  return gFailed ? 1 : 0;
}
