// rank_model_test.cc - threaded CPU model of the device protocols.
//
// One std::thread per rank runs the ring, one-shot, two-shot and NVLS
// algorithms of csrc/tnccl/allreduce.cu step for step on host memory (the
// warp-specialised teams of two-shot and NVLS as threads of their own, the
// NVLS multicast region as one copy per rank): the same protocol.h
// partition and mailbox layout, 64-bit sequence words written with release
// stores and polled with acquire loads, per-channel sequence counters that
// persist across collectives, and bounded waits. Channels of one rank run one
// after another on that rank's thread; channels never wait on each other, so
// this is one of the interleavings the GPU may produce.
//
// Checks:
//  * tiny-nccl's matrix (tests/ring_model_test.cc:163-171): nranks
//    {1,2,3,4,7} x count {0,1,2,5,8,31,113} x in/out of place, with a 7-element
//    chunk to force many tiles, for every algorithm, bit-exact against the
//    algorithm-aware oracle;
//  * BASELINE config 1: P = 4, ring FIFO 8 slots x 64 KiB, counts 1,048,576,
//    1,000,003 and 0, Uniform[-1,1) seeded per rank, fp32 and bf16;
//  * many collectives in a row on the same mailboxes (sequence continuity);
//  * the ticket replay of tiny-nccl (10,000 tickets over S slots);
//  * fault injection: a dropped publication makes every waiting rank give up
//    within the bound and report a timeout instead of hanging.
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <chrono>
#include <functional>
#include <memory>
#include <thread>
#include <vector>

#include "oracle.h"
#include "protocol.h"

using namespace tnccl;

namespace {

int gFailed = 0;
void report(const char* what, bool ok) {
  printf("%-52s %s\n", what, ok ? "ok" : "FAILED");
  fflush(stdout);
  if (!ok) ++gFailed;
}

enum Algo { kRing = 1, kOneShot = 2, kTwoShot = 3, kNvls = 4, kNvlsZc = 5 };

struct Config {
  int P = 4;
  int channels = 4;
  int osChannels = 2;
  int ringSlots = 4;
  uint64_t ringChunkElems = 16384;
  uint64_t tsChunkElems = 8192;
  int osSlots = 2;
  uint64_t osTileElems = 8192;
  int nvlsChannels = 2;
  uint64_t nvlsTileElems = 8192;
  uint64_t vec = 4;         // element granularity of chunk boundaries
  uint64_t minChunk = 4;
  int timeoutMs = 2000;
};

// Host model of one communicator: P mailboxes (elements stored as float, each
// value already rounded to the wire type), P sets of sequence counters.
struct World {
  Config cfg;
  MailboxLayout L;
  std::vector<std::vector<uint64_t>> mem;  // per rank, 8-byte aligned storage
  std::vector<std::vector<uint64_t>> counters;
  std::atomic<int> error{0};
  // Fault injection: rank `dropRank` skips its `dropAt`-th flag publication.
  int dropRank = -1;
  int dropAt = -1;
  std::vector<int> published;

  explicit World(const Config& c) : cfg(c) {
    LayoutConfig lc{};
    lc.nranks = c.P;
    lc.channels = c.channels;
    lc.osChannels = c.osChannels;
    lc.ringSlots = c.ringSlots;
    lc.ringChunkBytes = c.ringChunkElems * 4;
    lc.tsChunkBytes = c.tsChunkElems * 4;
    lc.osSlots = c.osSlots;
    lc.osTileBytes = c.osTileElems * 4;
    L = makeLayout(lc);
    mem.assign((size_t)c.P, std::vector<uint64_t>(L.totalBytes / 8, 0));
    counters.assign((size_t)c.P, std::vector<uint64_t>(kNumCounterFamilies * kMaxChannels, 0));
    published.assign((size_t)c.P, 0);
    mc.assign((size_t)c.P, std::vector<float>((size_t)c.nvlsChannels * kNvlsSlots * 2 *
                                                  c.nvlsTileElems, 0.f));
    const size_t ncount = (size_t)c.P * 2 * c.nvlsChannels * kNvlsSlots;
    mcCount.reset(new std::atomic<uint64_t>[ncount]);
    for (size_t i = 0; i < ncount; ++i) mcCount[i].store(0);
    for (int r = 0; r < c.P; ++r)
      for (int ch = 0; ch < c.channels; ++ch)
        for (int s = 0; s < c.ringSlots; ++s) *flag(r, ringCreditAt(L, ch, s)) = (uint64_t)s;
  }

  // NVLS: each rank's copy of the multicast region (input / output block per
  // channel and slot) and of the barrier counters; a multicast store or add
  // updates every rank's copy, a multicast reduce reads every rank's copy.
  std::vector<std::vector<float>> mc;
  std::unique_ptr<std::atomic<uint64_t>[]> mcCount;
  float* mcIn(int r, int c, int s) {
    return mc[(size_t)r].data() + ((size_t)c * kNvlsSlots + s) * 2 * cfg.nvlsTileElems;
  }
  float* mcOut(int r, int c, int s) { return mcIn(r, c, s) + cfg.nvlsTileElems; }
  std::atomic<uint64_t>& mcCounter(int r, int phase, int c, int s) {
    return mcCount[(((size_t)r * 2 + phase) * cfg.nvlsChannels + c) * kNvlsSlots + s];
  }
  // multimem.red.release: +1 on every rank's copy.
  void mcAdd(int self, int phase, int c, int s) {
    int n = __atomic_fetch_add(&published[(size_t)self], 1, __ATOMIC_RELAXED);
    if (self == dropRank && n == dropAt) return;  // injected loss
    for (int q = 0; q < cfg.P; ++q) mcCounter(q, phase, c, s).fetch_add(1, std::memory_order_release);
  }
  bool mcWait(int r, int phase, int c, int s, uint64_t want) {
    auto start = std::chrono::steady_clock::now();
    uint64_t spins = 0;
    while (mcCounter(r, phase, c, s).load(std::memory_order_acquire) < want) {
      if ((++spins & 1023) == 0) {
        if (error.load()) return false;
        if (std::chrono::steady_clock::now() - start > std::chrono::milliseconds(cfg.timeoutMs)) {
          error.store(5);
          return false;
        }
        std::this_thread::yield();
      }
    }
    return true;
  }

  // Zero-copy NVLS barrier counters ("entered", "stored") per rank and channel.
  std::unique_ptr<std::atomic<uint64_t>[]> zcCount{
      new std::atomic<uint64_t>[(size_t)kMaxRanks * 2 * kMaxChannels]()};
  std::atomic<uint64_t>& zcCounter(int r, int phase, int c) {
    return zcCount[((size_t)r * 2 + phase) * kMaxChannels + c];
  }
  void zcAdd(int self, int phase, int c) {
    int n = __atomic_fetch_add(&published[(size_t)self], 1, __ATOMIC_RELAXED);
    if (self == dropRank && n == dropAt) return;  // injected loss
    for (int q = 0; q < cfg.P; ++q) zcCounter(q, phase, c).fetch_add(1, std::memory_order_release);
  }
  bool zcWait(int r, int phase, int c, uint64_t want) {
    auto start = std::chrono::steady_clock::now();
    uint64_t spins = 0;
    while (zcCounter(r, phase, c).load(std::memory_order_acquire) < want) {
      if ((++spins & 1023) == 0) {
        if (error.load()) return false;
        if (std::chrono::steady_clock::now() - start > std::chrono::milliseconds(cfg.timeoutMs)) {
          error.store(5);
          return false;
        }
        std::this_thread::yield();
      }
    }
    return true;
  }

  char* base(int r) { return reinterpret_cast<char*>(mem[(size_t)r].data()); }
  uint64_t* flag(int r, uint64_t off) { return reinterpret_cast<uint64_t*>(base(r) + off); }
  float* data(int r, uint64_t off) { return reinterpret_cast<float*>(base(r) + off); }

  void publish(int self, int r, uint64_t off, uint64_t v) {
    int n = __atomic_fetch_add(&published[(size_t)self], 1, __ATOMIC_RELAXED);
    if (self == dropRank && n == dropAt) return;  // injected loss
    __atomic_store_n(flag(r, off), v, __ATOMIC_RELEASE);
  }

  // Bounded wait; false on timeout or when another rank already failed.
  bool wait(int r, uint64_t off, uint64_t want) {
    auto start = std::chrono::steady_clock::now();
    uint64_t spins = 0;
    while (__atomic_load_n(flag(r, off), __ATOMIC_ACQUIRE) < want) {
      if ((++spins & 1023) == 0) {
        if (error.load()) return false;
        if (std::chrono::steady_clock::now() - start >
            std::chrono::milliseconds(cfg.timeoutMs)) {
          error.store(5);
          return false;
        }
        std::this_thread::yield();
      }
    }
    return true;
  }
};

struct Job {
  int dtype;
  float alpha;
  const std::vector<std::vector<float>>* x;  // inputs (representable in dtype)
  std::vector<std::vector<float>>* y;        // outputs
  bool inPlace;
};

float rnd(int t, float f) { return oracle::roundTo(t, f); }

bool twoShot(World& w, int r, const Job& j, uint64_t count) {
  // Same structure as twoShotBody: per channel, a push, a reduce and a
  // gather role run concurrently (here: three threads), coupled only by the
  // peers' flags and by the local "gathered" counter that gates slot reuse.
  const Config& c = w.cfg;
  const int P = c.P;
  const MailboxLayout& L = w.L;
  ChunkPlan pl = makeChunkPlan(count, P, c.channels, c.tsChunkElems, c.minChunk, c.vec);
  const std::vector<float>& x = (*j.x)[(size_t)r];
  std::vector<float>& y = (*j.y)[(size_t)r];
  for (int ch = 0; ch < pl.channels; ++ch) {
    uint64_t& seq = w.counters[(size_t)r][kCounterTwoShot * kMaxChannels + ch];
    const uint64_t seq0 = seq;
    const uint64_t ntiles = channelTiles(pl.numTiles, pl.channels, ch);
    auto tileOf = [&](uint64_t t) { return (uint64_t)ch + t * (uint64_t)pl.channels; };
    auto slotOf = [&](uint64_t t) { return (int)((seq0 + t) % kTwoShotSlots); };
    std::atomic<uint64_t> gathered{0};
    std::atomic<int> fail{0};
    auto push = [&] {
      for (uint64_t t = 0; t < ntiles && !fail.load(); ++t) {
        if (t >= (uint64_t)kTwoShotSlots) {
          auto start = std::chrono::steady_clock::now();
          while (gathered.load(std::memory_order_acquire) < t - kTwoShotSlots + 1) {
            if (fail.load() || w.error.load() ||
                std::chrono::steady_clock::now() - start >
                    std::chrono::milliseconds(c.timeoutMs)) {
              fail.store(1);
              return;
            }
            std::this_thread::yield();
          }
        }
        for (int k = 1; k < P; ++k) {
          const int dst = (r + k) % P;
          Span sp = chunkSpan(pl, tileOf(t), dst, c.vec);
          float* out = w.data(dst, tsRsDataAt(L, ch, slotOf(t), r));
          for (uint64_t e = 0; e < sp.count; ++e) out[e] = x[sp.offset + e];
        }
        for (int p = 0; p < P; ++p)
          if (p != r) w.publish(r, p, tsRsFlagAt(L, ch, slotOf(t), r), seq0 + t + 1);
      }
    };
    auto reduce = [&] {
      for (uint64_t t = 0; t < ntiles; ++t) {
        const int slot = slotOf(t);
        const uint64_t want = seq0 + t + 1;
        for (int p = 0; p < P; ++p)
          if (p != r && !w.wait(r, tsRsFlagAt(L, ch, slot, p), want)) {
            fail.store(1);
            return;
          }
        Span own = chunkSpan(pl, tileOf(t), r, c.vec);
        for (uint64_t e = 0; e < own.count; ++e) {
          float acc = 0;
          for (int k = 0; k < P; ++k) {
            float v = k == r ? x[own.offset + e] : w.data(r, tsRsDataAt(L, ch, slot, k))[e];
            acc = k == 0 ? oracle::mul(j.alpha, v) : oracle::add(acc, oracle::mul(j.alpha, v));
          }
          acc = rnd(j.dtype, acc);
          y[own.offset + e] = acc;
          for (int p = 0; p < P; ++p)
            if (p != r) w.data(p, tsAgDataAt(L, ch, slot, r))[e] = acc;
        }
        for (int p = 0; p < P; ++p)
          if (p != r) w.publish(r, p, tsAgFlagAt(L, ch, slot, r), want);
      }
    };
    auto gather = [&] {
      for (uint64_t t = 0; t < ntiles; ++t) {
        const int slot = slotOf(t);
        for (int p = 0; p < P; ++p)
          if (p != r && !w.wait(r, tsAgFlagAt(L, ch, slot, p), seq0 + t + 1)) {
            fail.store(1);
            return;
          }
        for (int k = 1; k < P; ++k) {
          const int src = (r + P - k) % P;
          Span sp = chunkSpan(pl, tileOf(t), src, c.vec);
          const float* in = w.data(r, tsAgDataAt(L, ch, slot, src));
          for (uint64_t e = 0; e < sp.count; ++e) y[sp.offset + e] = in[e];
        }
        gathered.store(t + 1, std::memory_order_release);
      }
    };
    std::thread tp(push), tr(reduce);
    gather();
    tp.join();
    tr.join();
    if (fail.load()) return false;
    seq = seq0 + ntiles;
  }
  return true;
}

bool oneShot(World& w, int r, const Job& j, uint64_t count) {
  const Config& c = w.cfg;
  const int P = c.P;
  const MailboxLayout& L = w.L;
  BlockPlan pl = makeBlockPlan(count, c.osChannels, c.osTileElems, c.minChunk, c.vec);
  const std::vector<float>& x = (*j.x)[(size_t)r];
  std::vector<float>& y = (*j.y)[(size_t)r];
  const int S = c.osSlots;
  for (int ch = 0; ch < pl.channels; ++ch) {
    uint64_t& seq = w.counters[(size_t)r][kCounterOneShot * kMaxChannels + ch];
    for (uint64_t t = 0; t < channelTiles(pl.numTiles, pl.channels, ch); ++t) {
      const uint64_t tile = (uint64_t)ch + t * (uint64_t)pl.channels;
      Span sp = blockTileSpan(pl, tile);
      const int s = (int)(seq % (uint64_t)S);
      const uint64_t want = seq + 1;
      if (seq >= (uint64_t)S)
        for (int p = 0; p < P; ++p)
          if (p != r && !w.wait(r, osAckAt(L, ch, s, p), seq - (uint64_t)S + 1)) return false;
      for (int p = 0; p < P; ++p) {
        if (p == r) continue;
        float* out = w.data(p, osDataAt(L, ch, s, r));
        for (uint64_t e = 0; e < sp.count; ++e) out[e] = x[sp.offset + e];
      }
      for (int p = 0; p < P; ++p)
        if (p != r) w.publish(r, p, osFlagAt(L, ch, s, r), want);
      for (int p = 0; p < P; ++p)
        if (p != r && !w.wait(r, osFlagAt(L, ch, s, p), want)) return false;
      for (uint64_t e = 0; e < sp.count; ++e) {
        float acc = 0;
        for (int k = 0; k < P; ++k) {
          float v = k == r ? x[sp.offset + e] : w.data(r, osDataAt(L, ch, s, k))[e];
          acc = k == 0 ? oracle::mul(j.alpha, v) : oracle::add(acc, oracle::mul(j.alpha, v));
        }
        y[sp.offset + e] = rnd(j.dtype, acc);
      }
      for (int p = 0; p < P; ++p)
        if (p != r) w.publish(r, p, osAckAt(L, ch, s, r), want);
      ++seq;
    }
  }
  return true;
}

bool nvls(World& w, int r, const Job& j, uint64_t count) {
  // Same structure as nvlsKernel: per channel a copy-in, a switch and a
  // copy-out role (three threads) coupled by the per-slot multicast counters
  // (P x uses of the slot) and the local "copied out" counter. The switch
  // sums every rank's input copy in rank order (the real switch's order is
  // its own; the model checks the protocol, not the switch arithmetic).
  const Config& c = w.cfg;
  const int P = c.P;
  constexpr int S = kNvlsSlots;
  BlockPlan pl = makeBlockPlan(count, c.nvlsChannels, c.nvlsTileElems, c.minChunk, c.vec);
  const std::vector<float>& x = (*j.x)[(size_t)r];
  std::vector<float>& y = (*j.y)[(size_t)r];
  for (int ch = 0; ch < pl.channels; ++ch) {
    uint64_t& seq = w.counters[(size_t)r][kCounterNvls * kMaxChannels + ch];
    const uint64_t seq0 = seq;
    const uint64_t ntiles = channelTiles(pl.numTiles, pl.channels, ch);
    auto spanOf = [&](uint64_t t) { return blockTileSpan(pl, (uint64_t)ch + t * pl.channels); };
    auto slotOf = [&](uint64_t t) { return (int)((seq0 + t) % S); };
    auto usesOf = [&](uint64_t t) { return (seq0 + t) / S + 1; };
    std::atomic<uint64_t> copiedOut{0};
    std::atomic<int> fail{0};
    auto copyIn = [&] {
      for (uint64_t t = 0; t < ntiles && !fail.load(); ++t) {
        if (t >= (uint64_t)S) {
          auto start = std::chrono::steady_clock::now();
          while (copiedOut.load(std::memory_order_acquire) < t - S + 1) {
            if (fail.load() || w.error.load() ||
                std::chrono::steady_clock::now() - start > std::chrono::milliseconds(c.timeoutMs)) {
              fail.store(1);
              return;
            }
            std::this_thread::yield();
          }
        }
        const Span sp = spanOf(t);
        float* in = w.mcIn(r, ch, slotOf(t));
        for (uint64_t e = 0; e < sp.count; ++e) in[e] = x[sp.offset + e];
        w.mcAdd(r, 0, ch, slotOf(t));
      }
    };
    auto sw = [&] {
      for (uint64_t t = 0; t < ntiles; ++t) {
        const int s = slotOf(t);
        if (!w.mcWait(r, 0, ch, s, (uint64_t)P * usesOf(t))) {
          fail.store(1);
          return;
        }
        const Span sp = spanOf(t);
        const Span share = blockShare(divUp(sp.count, c.vec), P, r, 1);
        for (uint64_t e = share.offset * c.vec;
             e < (share.offset + share.count) * c.vec && e < sp.count; ++e) {
          float acc = w.mcIn(0, ch, s)[e];
          for (int q = 1; q < P; ++q) acc = oracle::add(acc, w.mcIn(q, ch, s)[e]);
          const float v = rnd(j.dtype, oracle::mul(j.alpha, acc));
          for (int q = 0; q < P; ++q) w.mcOut(q, ch, s)[e] = v;  // multicast store
        }
        w.mcAdd(r, 1, ch, s);
      }
    };
    auto copyOut = [&] {
      for (uint64_t t = 0; t < ntiles; ++t) {
        const int s = slotOf(t);
        if (!w.mcWait(r, 1, ch, s, (uint64_t)P * usesOf(t))) {
          fail.store(1);
          return;
        }
        const Span sp = spanOf(t);
        const float* out = w.mcOut(r, ch, s);
        for (uint64_t e = 0; e < sp.count; ++e) y[sp.offset + e] = out[e];
        copiedOut.store(t + 1, std::memory_order_release);
      }
    };
    std::thread ti(copyIn), ts(sw);
    copyOut();
    ti.join();
    ts.join();
    if (fail.load()) return false;
    seq = seq0 + ntiles;
  }
  return true;
}

bool nvlsZeroCopy(World& w, int r, const Job& j, uint64_t count) {
  // Same structure as nvlsZeroCopyKernel: one thread per channel; every
  // channel of every rank counts "entered" and "stored" on every rank, and
  // the switch reads every rank's buffer and writes every rank's output in
  // place. In place really is one buffer here (reads go to y, which starts
  // as a copy of x), so a read after another rank's store would show.
  // Messages that are not whole vectors take the staged kernel, as the host
  // does.
  const Config& c = w.cfg;
  if (count % c.vec != 0) return nvls(w, r, j, count);
  const int P = c.P;
  const uint64_t nv = count / c.vec;
  const int C = nvlsZcChannels(nv, P, c.nvlsChannels, 2);
  std::vector<std::vector<float>>& y = *j.y;
  const std::vector<std::vector<float>>& in = j.inPlace ? y : *j.x;
  std::atomic<int> fail{0};
  auto channel = [&](int ch) {
    uint64_t& seq = w.counters[(size_t)r][kCounterNvlsZc * kMaxChannels + ch];
    const uint64_t target = (uint64_t)P * (seq + 1);
    w.zcAdd(r, 0, ch);
    if (!w.zcWait(r, 0, ch, target)) {
      fail.store(1);
      return;
    }
    const Span sp = nvlsZcSpan(nv, P, r, C, ch);
    for (uint64_t e = sp.offset * c.vec; e < (sp.offset + sp.count) * c.vec; ++e) {
      float acc = in[0][e];
      for (int q = 1; q < P; ++q) acc = oracle::add(acc, in[(size_t)q][e]);
      const float v = rnd(j.dtype, oracle::mul(j.alpha, acc));
      for (int q = 0; q < P; ++q) y[(size_t)q][e] = v;  // multicast store
    }
    w.zcAdd(r, 1, ch);
    if (!w.zcWait(r, 1, ch, target)) {
      fail.store(1);
      return;
    }
    ++seq;
  };
  std::vector<std::thread> th;
  for (int ch = 1; ch < C; ++ch) th.emplace_back(channel, ch);
  channel(0);
  for (auto& t : th) t.join();
  return fail.load() == 0;
}

bool ring(World& w, int r, const Job& j, uint64_t count) {
  const Config& c = w.cfg;
  const int P = c.P;
  const MailboxLayout& L = w.L;
  const int S = c.ringSlots;
  ChunkPlan pl = makeChunkPlan(count, P, c.channels, c.ringChunkElems, c.minChunk, c.vec);
  const std::vector<float>& x = (*j.x)[(size_t)r];
  std::vector<float>& y = (*j.y)[(size_t)r];
  const int next = (r + 1) % P, prev = (r + P - 1) % P;
  for (int ch = 0; ch < pl.channels; ++ch) {
    uint64_t& ticket = w.counters[(size_t)r][kCounterRing * kMaxChannels + ch];
    uint64_t sendT = ticket, recvT = ticket;
    auto waitSend = [&]() { return w.wait(r, ringCreditAt(L, ch, (int)(sendT % S)), sendT); };
    auto waitRecv = [&]() { return w.wait(r, ringReadyAt(L, ch, (int)(recvT % S)), recvT + 1); };
    auto outSlot = [&]() { return w.data(next, ringDataAt(L, ch, (int)(sendT % S))); };
    auto inSlot = [&]() { return w.data(r, ringDataAt(L, ch, (int)(recvT % S))); };
    auto publish = [&]() {
      w.publish(r, next, ringReadyAt(L, ch, (int)(sendT % S)), sendT + 1);
      ++sendT;
    };
    auto release = [&]() {
      w.publish(r, prev, ringCreditAt(L, ch, (int)(recvT % S)), recvT + (uint64_t)S);
      ++recvT;
    };
    for (uint64_t t = 0; t < channelTiles(pl.numTiles, pl.channels, ch); ++t) {
      const uint64_t tile = (uint64_t)ch + t * (uint64_t)pl.channels;
      {
        Span sp = chunkSpan(pl, tile, ringChunkBehind(r, 1, P), c.vec);
        if (!waitSend()) return false;
        float* out = outSlot();
        for (uint64_t e = 0; e < sp.count; ++e)
          out[e] = rnd(j.dtype, oracle::mul(j.alpha, x[sp.offset + e]));
        publish();
      }
      for (int d = 2; d < P; ++d) {
        Span sp = chunkSpan(pl, tile, ringChunkBehind(r, d, P), c.vec);
        if (!waitRecv() || !waitSend()) return false;
        const float* in = inSlot();
        float* out = outSlot();
        for (uint64_t e = 0; e < sp.count; ++e)
          out[e] = rnd(j.dtype, oracle::add(in[e], oracle::mul(j.alpha, x[sp.offset + e])));
        release();
        publish();
      }
      {
        Span sp = chunkSpan(pl, tile, r, c.vec);
        if (!waitRecv() || !waitSend()) return false;
        const float* in = inSlot();
        float* out = outSlot();
        for (uint64_t e = 0; e < sp.count; ++e) {
          float v = rnd(j.dtype, oracle::add(in[e], oracle::mul(j.alpha, x[sp.offset + e])));
          y[sp.offset + e] = v;
          out[e] = v;
        }
        release();
        publish();
      }
      for (int d = 1; d < P - 1; ++d) {
        Span sp = chunkSpan(pl, tile, ringChunkBehind(r, d, P), c.vec);
        if (!waitRecv() || !waitSend()) return false;
        const float* in = inSlot();
        float* out = outSlot();
        for (uint64_t e = 0; e < sp.count; ++e) y[sp.offset + e] = out[e] = in[e];
        release();
        publish();
      }
      {
        Span sp = chunkSpan(pl, tile, ringChunkBehind(r, P - 1, P), c.vec);
        if (!waitRecv()) return false;
        const float* in = inSlot();
        for (uint64_t e = 0; e < sp.count; ++e) y[sp.offset + e] = in[e];
        release();
      }
    }
    ticket = sendT;
    if (sendT != recvT) return false;
  }
  return true;
}

// Runs one collective on every rank thread. Returns false if any rank failed.
bool collective(World& w, Algo a, const Job& j, uint64_t count) {
  const int P = w.cfg.P;
  std::vector<int> ok((size_t)P, 1);
  std::vector<std::thread> th;
  for (int r = 0; r < P; ++r) {
    th.emplace_back([&, r] {
      if (P == 1) {
        for (uint64_t e = 0; e < count; ++e)
          (*j.y)[0][e] = rnd(j.dtype, oracle::mul(j.alpha, (*j.x)[0][e]));
        return;
      }
      bool res = a == kRing      ? ring(w, r, j, count)
                 : a == kOneShot ? oneShot(w, r, j, count)
                 : a == kNvls    ? nvls(w, r, j, count)
                 : a == kNvlsZc  ? nvlsZeroCopy(w, r, j, count)
                                 : twoShot(w, r, j, count);
      ok[(size_t)r] = res ? 1 : 0;
    });
  }
  for (auto& t : th) t.join();
  for (int v : ok)
    if (!v) return false;
  return true;
}

// Builds inputs, runs `a`, compares every rank's output with the oracle.
bool checkOne(World& w, Algo a, int dtype, uint64_t count, bool inPlace, bool avg,
              uint64_t seed) {
  const int P = w.cfg.P;
  std::vector<std::vector<float>> x((size_t)P), y((size_t)P);
  std::vector<unsigned char> raw;
  for (int r = 0; r < P; ++r) {
    oracle::fillInput(dtype, seed, r, count, x[(size_t)r], raw);
    y[(size_t)r] = inPlace ? x[(size_t)r] : std::vector<float>(count, -7.0f);
  }
  const float alpha = avg ? 1.0f / (float)P : 1.0f;
  // In-place: the model reads x and writes y; on the device both are one
  // buffer. Reads of an element always precede its write there, which the
  // separate vectors model exactly.
  Job j{dtype, alpha, &x, &y, inPlace};
  if (!collective(w, a, j, count)) return false;
  std::vector<float> want;
  if (P == 1) {
    want.resize(count);
    for (uint64_t e = 0; e < count; ++e) want[e] = rnd(dtype, oracle::mul(alpha, x[0][e]));
  } else if (a == kRing) {
    ChunkPlan pl = makeChunkPlan(count, P, w.cfg.channels, w.cfg.ringChunkElems, w.cfg.minChunk,
                                 w.cfg.vec);
    oracle::ring(dtype, x, alpha, pl, w.cfg.vec, want);
  } else if (a == kNvls || a == kNvlsZc) {
    // The switch sums first and the pre-scale applies to the sum.
    want.resize(count);
    for (uint64_t e = 0; e < count; ++e) {
      float acc = x[0][e];
      for (int k = 1; k < P; ++k) acc = oracle::add(acc, x[(size_t)k][e]);
      want[e] = rnd(dtype, oracle::mul(alpha, acc));
    }
  } else {
    oracle::canonical(dtype, x, alpha, want);
  }
  for (int r = 0; r < P; ++r)
    for (uint64_t e = 0; e < count; ++e)
      if (memcmp(&y[(size_t)r][e], &want[e], 4) != 0) {
        printf("  rank %d elem %llu: got %.9g want %.9g\n", r, (unsigned long long)e,
               y[(size_t)r][e], want[e]);
        return false;
      }
  return true;
}

const char* algoName(Algo a) {
  return a == kRing      ? "ring"
         : a == kOneShot ? "oneshot"
         : a == kNvls    ? "nvls"
         : a == kNvlsZc  ? "nvls zero-copy"
                         : "twoshot";
}

void referenceMatrix() {
  for (Algo a : {kRing, kOneShot, kTwoShot, kNvls, kNvlsZc}) {
    bool ok = true;
    for (int P : {1, 2, 3, 4, 7}) {
      Config c;
      c.P = P;
      c.channels = 2;
      c.osChannels = 2;
      c.ringChunkElems = 7;  // tiny chunks force many tiles (as tiny-nccl's test)
      c.tsChunkElems = 7;
      c.osTileElems = 7;
      c.nvlsTileElems = 7;
      c.vec = 1;
      c.minChunk = 1;
      World w(c);
      uint64_t seed = 11;
      for (uint64_t n : {0ull, 1ull, 2ull, 5ull, 8ull, 31ull, 113ull})
        for (bool ip : {false, true}) ok = ok && checkOne(w, a, oracle::kF32, n, ip, false, seed++);
    }
    char name[96];
    snprintf(name, sizeof(name), "reference matrix (%s, 7-element chunks)", algoName(a));
    report(name, ok);
  }
}

void baselineConfig1() {
  Config c;
  c.P = 4;
  c.ringSlots = 8;
  c.ringChunkElems = 16384;  // 64 KiB of fp32 per slot
  c.channels = 4;
  for (Algo a : {kRing, kTwoShot, kOneShot, kNvls, kNvlsZc}) {
    for (int t : {oracle::kF32, oracle::kBF16}) {
      World w(c);
      bool ok = true;
      uint64_t seed = 2024;
      for (uint64_t n : {1048576ull, 1000003ull, 0ull, 1000003ull})
        ok = ok && checkOne(w, a, t, n, false, false, seed++);
      ok = ok && checkOne(w, a, t, 1000003, true, true, seed++);  // in place, pre-scale 1/P
      char name[96];
      snprintf(name, sizeof(name), "config1 P=4 8x64KiB %s %s", algoName(a),
               t == oracle::kF32 ? "fp32" : "bf16");
      report(name, ok);
    }
  }
}

void sequenceContinuity() {
  Config c;
  c.P = 3;
  c.channels = 3;
  c.ringChunkElems = 64;
  c.tsChunkElems = 64;
  c.osTileElems = 64;
  c.nvlsTileElems = 64;
  World w(c);
  bool ok = true;
  uint64_t seed = 5;
  // 200 collectives of varying size and algorithm on the same mailboxes.
  for (int i = 0; i < 200 && ok; ++i) {
    Algo a = (Algo)(1 + i % 5);
    uint64_t n = (uint64_t)((i * 37) % 900);
    ok = checkOne(w, a, i % 2 ? oracle::kBF16 : oracle::kF32, n, i % 5 == 0, i % 7 == 0, seed++);
  }
  report("200 mixed collectives on one mailbox set", ok);
}

// Randomised configurations: rank count, channel count, chunk / tile sizes
// small enough that every slot ring wraps many times, and random counts,
// algorithms, dtypes, in-place and pre-scale, three collectives per world.
void randomized() {
  uint64_t s = 0x9e3779b97f4a7c15ull;
  auto rnd = [&s](uint64_t n) {
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    return s % n;
  };
  bool ok = true;
  int worlds = 0;
  for (; worlds < 60 && ok; ++worlds) {
    Config c;
    c.P = 2 + (int)rnd(7);
    c.channels = 1 + (int)rnd(4);
    c.osChannels = 1 + (int)rnd(4);
    c.nvlsChannels = 1 + (int)rnd(3);
    c.ringSlots = 2 + (int)rnd(4);
    c.ringChunkElems = 4 * (1 + rnd(32));
    c.tsChunkElems = 4 * (1 + rnd(32));
    c.osSlots = 1 + (int)rnd(3);
    c.osTileElems = 4 * (1 + rnd(32));
    c.nvlsTileElems = 4 * (1 + rnd(32));
    World w(c);
    for (int k = 0; k < 3 && ok; ++k) {
      const Algo a = (Algo)(1 + rnd(5));
      const uint64_t n = rnd(5) == 0 ? rnd(8) : rnd(20000);
      ok = checkOne(w, a, rnd(2) ? oracle::kBF16 : oracle::kF32, n, rnd(2) == 0, rnd(3) == 0,
                    1000 + (uint64_t)worlds * 3 + (uint64_t)k);
      if (!ok) printf("  world %d: P=%d algo=%s count=%llu\n", worlds, c.P, algoName(a),
                      (unsigned long long)n);
    }
  }
  char name[96];
  snprintf(name, sizeof(name), "randomised configurations (%d worlds x 3)", worlds);
  report(name, ok);
}

// nvlsZcSpan over all (rank, channel) pairs covers [0, nv) exactly once, and
// nvlsZcChannels stays within 1 .. maxChannels.
void zeroCopyPartition() {
  bool ok = true;
  for (int P = 2; P <= kMaxRanks && ok; ++P)
    for (uint64_t nv : {0ull, 1ull, 2ull, 7ull, 15ull, 16ull, 17ull, 1000ull, 65537ull, 1ull << 26})
      for (int maxC : {1, 3, 32, kMaxChannels}) {
        const int C = nvlsZcChannels(nv, P, maxC, 1024);
        ok = ok && C >= 1 && C <= maxC;
        uint64_t next = 0;
        for (int r = 0; r < P && ok; ++r)
          for (int c = 0; c < C && ok; ++c) {
            const Span sp = nvlsZcSpan(nv, P, r, C, c);
            // Spans are contiguous in (rank, channel) order; empty ones may sit anywhere.
            if (sp.count == 0) continue;
            ok = sp.offset == next;
            next = sp.offset + sp.count;
          }
        ok = ok && next == nv;
        if (!ok) printf("  P=%d nv=%llu maxC=%d C=%d\n", P, (unsigned long long)nv, maxC, C);
      }
  report("zero-copy NVLS partition covers every vector once", ok);
}

void ticketReplay() {
  // tiny-nccl tests/ring_model_test.cc:149-159: credit == t before send,
  // ready = t + 1 on publish, credit = t + S on release.
  bool ok = true;
  for (int S : {2, 4, 8}) {
    std::vector<uint64_t> ready((size_t)S, 0), credit((size_t)S);
    for (int s = 0; s < S; ++s) credit[(size_t)s] = (uint64_t)s;
    for (uint64_t t = 0; t < 10000 && ok; ++t) {
      const size_t s = t % (uint64_t)S;
      ok = credit[s] == t && ready[s] == (t >= (uint64_t)S ? t - S + 1 : 0);
      ready[s] = t + 1;
      credit[s] = t + (uint64_t)S;
    }
  }
  report("ticket replay (10,000 tickets, S = 2/4/8)", ok);
}

void faultInjection() {
  for (Algo a : {kRing, kOneShot, kTwoShot, kNvls, kNvlsZc}) {
    Config c;
    c.P = 4;
    c.timeoutMs = 200;
    World w(c);
    w.dropRank = 2;
    w.dropAt = 3;  // the fourth flag rank 2 publishes never arrives
    auto t0 = std::chrono::steady_clock::now();
    std::vector<std::vector<float>> x(4), y(4);
    std::vector<unsigned char> raw;
    for (int r = 0; r < 4; ++r) {
      oracle::fillInput(oracle::kF32, 1, r, 100000, x[(size_t)r], raw);
      y[(size_t)r].assign(100000, 0.f);
    }
    Job j{oracle::kF32, 1.0f, &x, &y, false};
    bool completed = collective(w, a, j, 100000);
    double s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    char name[96];
    snprintf(name, sizeof(name), "dropped flag -> bounded timeout (%s)", algoName(a));
    report(name, !completed && w.error.load() == 5 && s < 5.0);
  }
}

}  // namespace

int main() {
  referenceMatrix();
  baselineConfig1();
  sequenceContinuity();
  randomized();
  zeroCopyPartition();
  ticketReplay();
  faultInjection();
  printf("rank_model_test: %s\n", gFailed ? "FAIL" : "PASS");
  return gFailed ? 1 : 0;
}
