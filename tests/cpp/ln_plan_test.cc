// ln_plan_test.cc - CPU checks of the row-group LayerNorm backward's launch
// geometry (csrc/ops/ln_plan.h, the numbers the launcher uses) and of the
// kernel's schedule, restated on the host:
//   1. every plan fits the hardware and the shared-memory layout: threads per
//      CTA, shared memory, named-barrier ids, warp-sum slots, accumulator
//      reuse of the rings, partial rows against the scratch the callers size
//      (2 * tnops_ln_partial_rows() * C floats, 296 rows);
//   2. the per-thread cp.async destinations are disjoint, stay inside their
//      stage and are aligned to their copy size;
//   3. the row walk covers every row exactly once, and the stage ring with
//      cp.async.wait_group(kLnStages - 1) never reads a stage before its
//      copies have landed nor refills one that is still to be read;
//   4. the warp-sum slots double-buffered by row parity give every thread of
//      a group the sums of its current row, with real threads, a barrier per
//      row and random delays (the slots without parity are expected to fail
//      this check sooner or later, which the test does not require).
#include <stdio.h>
#include <stdlib.h>

#include <atomic>
#include <condition_variable>
#include <mutex>
#include <random>
#include <thread>
#include <vector>

#include "ln_plan.h"

using namespace tnops;

static int gFailures = 0;
#define CHECK(cond, ...)                                   \
  do {                                                     \
    if (!(cond)) {                                         \
      if (gFailures++ < 20) {                              \
        fprintf(stderr, "FAIL %s:%d: ", __FILE__, __LINE__); \
        fprintf(stderr, __VA_ARGS__);                      \
        fprintf(stderr, "\n");                             \
      }                                                    \
    }                                                      \
  } while (0)

constexpr int kSMs = 148;
constexpr int kPartialRows = 2 * kSMs;  // tnops_ln_partial_rows()
constexpr int kMaxSmemPerCta = 227 * 1024;

static void checkPlan(int rows, int C, int K) {
  const LnGroupPlan p = lnGroupPlan(rows, C, K, kSMs);
  const int threads = p.R * p.G;
  const int nwarps = p.G / 32;
  CHECK(p.G % 32 == 0 && p.G > 0, "C=%d K=%d: G=%d", C, K, p.G);
  CHECK(p.G * 4 * K >= C, "C=%d K=%d: G=%d does not cover the row", C, K, p.G);
  CHECK(nwarps <= kLnMaxWarpsPerGroup, "C=%d K=%d: %d warps per group", C, K, nwarps);
  CHECK(p.R >= 1 && p.R <= kLnMaxGroups, "C=%d K=%d: R=%d", C, K, p.R);
  CHECK(threads <= lnMaxThreads(K), "C=%d K=%d: %d threads", C, K, threads);
  CHECK(p.smemBytes <= kLnMaxSmemBytes && kLnMaxSmemBytes <= kMaxSmemPerCta,
        "C=%d K=%d: smem %d", C, K, p.smemBytes);
  // Accumulators [R][2C] floats reuse the rings.
  CHECK(p.R * 2 * C * 4 <= p.R * kLnStages * lnStageBytes(K, p.G),
        "C=%d K=%d: accumulators do not fit the rings", C, K);
  // Warp-sum slots: float2 index (grp * 2 + parity) * 8 + warp.
  CHECK(((p.R - 1) * 2 + 1) * kLnMaxWarpsPerGroup + (nwarps - 1) < kLnRedFloats / 2,
        "C=%d K=%d: warp-sum slot out of range", C, K);
  CHECK(p.blocks >= 1 && p.blocks <= kSMs && p.blocks <= kPartialRows,
        "rows=%d C=%d K=%d: %d blocks", rows, C, K, p.blocks);
  const int want = (rows + p.R - 1) / p.R;
  CHECK(p.blocks == (want < kSMs ? want : kSMs), "rows=%d: %d blocks", rows, p.blocks);
  // Ring bases: 16-byte aligned.
  for (int g = 0; g < p.R; ++g) {
    const long base = kLnRedFloats * 4L + (long)g * kLnStages * lnStageBytes(K, p.G);
    CHECK(base % 16 == 0, "ring base %ld", base);
  }
  // Per-thread copy destinations within one stage: disjoint, inside, aligned.
  const int sb = lnStageBytes(K, p.G);
  std::vector<unsigned char> owner(sb, 0);
  const int C4 = C / 4;
  for (int gt = 0; gt < p.G; ++gt) {
    if (!(gt < C4 / K)) continue;  // inactive threads copy nothing
    const int gyOff = 8 * K * gt, xOff = 8 * K * p.G + 16 * K * gt,
              rOff = 24 * K * p.G + 16 * K * gt;
    CHECK(gyOff % (8 * K) == 0 && xOff % 16 == 0 && rOff % 16 == 0, "alignment gt=%d", gt);
    const int spans[3][2] = {{gyOff, 8 * K}, {xOff, 16 * K}, {rOff, 16 * K}};
    for (auto& sp : spans) {
      CHECK(sp[0] + sp[1] <= sb, "C=%d K=%d gt=%d: copy past the stage", C, K, gt);
      for (int b = sp[0]; b < sp[0] + sp[1] && b < sb; ++b) {
        CHECK(owner[b] == 0, "C=%d K=%d: byte %d copied twice", C, K, b);
        owner[b] = 1;
      }
    }
    // The thread's columns lie inside the row.
    CHECK(4 * K * gt + 4 * K <= C, "C=%d K=%d gt=%d: columns past the row", C, K, gt);
  }
}

// Host restatement of the row walk and the stage ring of one group.
static void checkSchedule(int rows, int C, int K) {
  const LnGroupPlan p = lnGroupPlan(rows, C, K, kSMs);
  const int S = kLnStages;
  const int stride = p.blocks * p.R;
  std::vector<int> seen(rows, 0);
  for (int b = 0; b < p.blocks; ++b) {
    for (int g = 0; g < p.R; ++g) {
      const int first = b * p.R + g;
      std::vector<int> stageRow(S, -1);
      std::vector<bool> pendingRead(S, false);
      std::vector<std::vector<int>> groups;  // commit groups: rows copied
      auto issue = [&](int slot, int row) {
        CHECK(!pendingRead[slot], "refill of stage %d before it was read", slot);
        stageRow[slot] = row;
        pendingRead[slot] = true;
      };
      for (int j = 0; j < S - 1; ++j) {
        const int row = first + j * stride;
        std::vector<int> grp;
        if (row < rows) {
          issue(j, row);
          grp.push_back(row);
        }
        groups.push_back(grp);
      }
      int slot = 0;
      for (int row = first; row < rows; row += stride) {
        const int ahead = row + (S - 1) * stride;
        const int aslot = slot == 0 ? S - 1 : slot - 1;
        std::vector<int> grp;
        if (ahead < rows) {
          issue(aslot, ahead);
          grp.push_back(ahead);
        }
        groups.push_back(grp);
        // wait_group(S - 1): all but the newest S - 1 groups are complete.
        bool landed = false;
        for (size_t q = 0; q + (S - 1) < groups.size(); ++q)
          for (int r : groups[q]) landed |= r == row;
        CHECK(landed, "row %d read before its copies landed", row);
        CHECK(stageRow[slot] == row, "stage %d holds row %d, not %d", slot, stageRow[slot], row);
        pendingRead[slot] = false;
        ++seen[row];
        slot = slot + 1 == S ? 0 : slot + 1;
      }
    }
  }
  for (int r = 0; r < rows; ++r) CHECK(seen[r] == 1, "rows=%d: row %d seen %d times", rows, r, seen[r]);
}

// A reusable barrier for the threads of one group.
class Barrier {
 public:
  explicit Barrier(int n) : n_(n) {}
  void wait() {
    std::unique_lock<std::mutex> lk(m_);
    const long gen = gen_;
    if (++count_ == n_) {
      count_ = 0;
      ++gen_;
      cv_.notify_all();
    } else {
      cv_.wait(lk, [&] { return gen_ != gen; });
    }
  }

 private:
  std::mutex m_;
  std::condition_variable cv_;
  int n_, count_ = 0;
  long gen_ = 0;
};

// Threads stand for the warps of one group: each writes its warp sum for the
// current row into slot [parity][warp], waits at the group's barrier, then
// reads every warp's slot and checks that all are from the current row.
static void checkParitySlots(int nwarps, int nrows, unsigned seed) {
  std::vector<std::atomic<long>> slots(2 * kLnMaxWarpsPerGroup);
  for (auto& s : slots) s.store(-1);
  Barrier bar(nwarps);
  std::atomic<int> bad{0};
  std::vector<std::thread> th;
  for (int w = 0; w < nwarps; ++w) {
    th.emplace_back([&, w] {
      std::mt19937 rng(seed * 131u + (unsigned)w);
      int parity = 0;
      for (int row = 0; row < nrows; ++row) {
        if (rng() % 4 == 0) std::this_thread::yield();
        // The warp's value for this row (its lane-0 write).
        slots[parity * kLnMaxWarpsPerGroup + w].store((long)row * 64 + w);
        bar.wait();
        for (int k = 0; k < nwarps; ++k) {
          if (rng() % 8 == 0) std::this_thread::yield();
          const long v = slots[parity * kLnMaxWarpsPerGroup + k].load();
          if (v != (long)row * 64 + k) bad.fetch_add(1);
        }
        parity ^= 1;
      }
    });
  }
  for (auto& t : th) t.join();
  CHECK(bad.load() == 0, "nwarps=%d: %d stale warp sums", nwarps, bad.load());
}

int main() {
  const int rowCases[] = {1, 2, 3, 7, 8, 15, 16, 100, 333, 1183, 1184, 1185, 4096, 8192};
  int plans = 0;
  for (int C = 4; C <= 1024; C += 4) {
    for (int K = 1; K <= 2; ++K) {
      if (K == 2 && C % 8 != 0) continue;
      for (int rows : rowCases) {
        checkPlan(rows, C, K);
        ++plans;
      }
      checkPlan(65536, C, K);
    }
  }
  // The schedule for the shapes the trainers use and a spread of others.
  const int schedC[] = {36, 128, 640, 768, 772, 1024};
  for (int C : schedC)
    for (int K = 1; K <= 2; ++K) {
      if (K == 2 && C % 8 != 0) continue;
      for (int rows : rowCases) checkSchedule(rows, C, K);
    }
  for (int nw = 1; nw <= kLnMaxWarpsPerGroup; ++nw) checkParitySlots(nw, 2000, 7u + nw);
  if (gFailures != 0) {
    printf("ln_plan_test: FAIL (%d)\n", gFailures);
    return 1;
  }
  printf("ln_plan_test: %d plans, schedules and parity slots: PASS\n", plans);
  return 0;
}
