// config_test.cc - host-side configuration and partition invariants, no GPU.
//
//  * loadConfig: defaults, environment overrides, clamping of out-of-range
//    values, the team-split parser and its fallback on malformed input;
//  * adaptConfig: the two-shot chunk per rank count (512 KiB tile, chunk
//    clamped to 32..256 KiB) and that an explicit TNCCL_TWOSHOT_CHUNK_BYTES
//    wins;
//  * configHash: equal for equal protocol fields, different when a field that
//    changes the mailbox layout differs, unchanged by rank-local knobs;
//  * TNCCL_TUNING_FILE: parsing, rejection of malformed lines, lookup, and
//    that the table is part of the configuration hash;
//  * makeLayout: areas and flag groups do not overlap, the canary lines sit
//    between them, alignment, and the total size;
//  * makeChunkPlan / chunkSpan and makeBlockPlan / blockTileSpan / blockShare:
//    every element is covered exactly once, chunk boundaries fall on vector
//    boundaries, for many counts, rank counts and channel counts.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <utility>
#include <vector>

#include "common.h"
#include "protocol.h"

using namespace tnccl;

namespace {

int gFailed = 0;
void check(bool ok, const char* what) {
  printf("%-60s %s\n", what, ok ? "ok" : "FAILED");
  if (!ok) ++gFailed;
}

void clearEnv() {
  for (const char* v :
       {"TNCCL_NCHANNELS", "TNCCL_ONESHOT_CHANNELS", "TNCCL_TWOSHOT_CHUNK_BYTES",
        "TNCCL_NTHREADS", "TNCCL_TWOSHOT_SPLIT", "TNCCL_NVLS_SPLIT", "TNCCL_TWOSHOT_STAGES",
        "TNCCL_TWOSHOT_PUSH_STAGE", "TNCCL_TWOSHOT_REDUCE_STAGE", "TNCCL_STAGE_MIN_BYTES",
        "TNCCL_ALGO", "TNCCL_TIMEOUT_MS", "TNCCL_ACQUIRE_LOAD", "TNCCL_NVLS_STAGE", "TNCCL_NET",
        "TNCCL_NET_CHANNELS", "TNCCL_NET_IF", "TNCCL_NET_SOCKBUF", "TNCCL_NET_SPIN_US"})
    unsetenv(v);
}

void defaultsAndOverrides() {
  clearEnv();
  setenv("TNCCL_DEBUG", "NONE", 1);  // the malformed-value cases below warn
  Config c = loadConfig();
  check(c.channels == 128 && c.osChannels == 64 && c.threads == 512, "defaults: channels, threads");
  check(c.tsSplit == (2 | (4 << 4)) && c.nvlsSplit == (1 | (4 << 4)), "defaults: team splits");
  check(c.stageMinBytes == (1 << 30) && c.acquireMode == 1, "defaults: staging off, ld.acquire");
  check(c.forcedAlgo == TNCCL_ALGO_AUTO && c.timeoutMs == 30000, "defaults: algorithm, timeout");

  setenv("TNCCL_NCHANNELS", "100000", 1);
  setenv("TNCCL_NTHREADS", "40", 1);
  setenv("TNCCL_TWOSHOT_SPLIT", "3,2", 1);
  setenv("TNCCL_ALGO", "twoshot", 1);
  setenv("TNCCL_TIMEOUT_MS", "0", 1);
  c = loadConfig();
  check(c.channels == kMaxChannels, "TNCCL_NCHANNELS clamped to kMaxChannels");
  check(c.threads == 128, "TNCCL_NTHREADS clamped to 128 (three teams need 4 warps)");
  check(c.tsSplit == (3 | (2 << 4)), "TNCCL_TWOSHOT_SPLIT=3,2 parsed");
  check(c.forcedAlgo == TNCCL_ALGO_TWOSHOT && c.timeoutMs == 1, "algorithm and timeout floor");

  setenv("TNCCL_TWOSHOT_SPLIT", "6,6", 1);  // 12 eighths: rejected
  setenv("TNCCL_NVLS_SPLIT", "garbage", 1);
  c = loadConfig();
  check(c.tsSplit == (2 | (4 << 4)) && c.nvlsSplit == (1 | (4 << 4)),
        "malformed splits fall back to the defaults");
  check(parseSplit("", 7) == 7 && parseSplit("1,1", 0) == (1 | (1 << 4)) &&
            parseSplit("0,3", 9) == 9 && parseSplit("4,4", 9) == 9 &&
            parseSplit("3,2x", 9) == 9,
        "parseSplit bounds");

  setenv("TNCCL_TWOSHOT_STAGES", "8", 1);
  setenv("TNCCL_TWOSHOT_PUSH_STAGE", "98304", 1);
  setenv("TNCCL_TWOSHOT_REDUCE_STAGE", "98304", 1);
  c = loadConfig();
  check((int64_t)c.tsStages * (c.tsPushStage + c.tsRedStage) <= 227 * 1024 - 256,
        "staging rings fit 227 KiB of shared memory");
  clearEnv();
}

void netKnobs() {
  clearEnv();
  Config c = loadConfig();
  check(c.netMode == 1 && c.netChannels == 2 && c.netIf.empty() && c.netSockBuf == 0 &&
            c.netSpinUs == 200,
        "socket-edge defaults: auto, 2 channels, derived address");
  check(parseNetMode("off") == 0 && parseNetMode("AUTO") == 1 && parseNetMode("force") == 2 &&
            parseNetMode("0") == 0 && parseNetMode("2") == 2 && parseNetMode("") == 1 &&
            parseNetMode("sometimes") == -1,
        "parseNetMode");
  setenv("TNCCL_NET", "force", 1);
  setenv("TNCCL_NET_CHANNELS", "64", 1);
  setenv("TNCCL_NET_IF", "10.0.0.7", 1);
  c = loadConfig();
  check(c.netMode == 2 && c.netChannels == 8 && c.netIf == "10.0.0.7",
        "TNCCL_NET=force, channels clamped to 8, TNCCL_NET_IF");
  setenv("TNCCL_NET", "sometimes", 1);
  c = loadConfig();
  check(c.netMode == 1, "malformed TNCCL_NET falls back to auto");
  Config a = loadConfig(), b = a;
  b.netMode = 2;
  check(configHash(a) != configHash(b), "configHash covers the socket-edge mode");
  b = a;
  b.netChannels = a.netChannels + 1;
  check(configHash(a) != configHash(b), "configHash covers the socket-edge channels");
  b = a;
  b.netIf = "192.168.0.1";
  b.netSpinUs = 5;
  b.netSockBuf = 4096;
  check(configHash(a) == configHash(b), "configHash ignores per-rank socket knobs");
  clearEnv();
}

void adaptChunks() {
  clearEnv();
  bool ok = true;
  for (int P = 1; P <= 16; ++P) {
    Config c = loadConfig();
    adaptConfig(c, P);
    int64_t want = (512 << 10) / P;
    want = std::min<int64_t>(std::max<int64_t>(want, 32 << 10), 256 << 10) / 16 * 16;
    ok = ok && c.tsChunkBytes == want;
  }
  check(ok, "two-shot chunk = 512 KiB / P clamped to 32..256 KiB");
  setenv("TNCCL_TWOSHOT_CHUNK_BYTES", "65536", 1);
  Config c = loadConfig();
  adaptConfig(c, 2);
  check(c.tsChunkBytes == 65536, "TNCCL_TWOSHOT_CHUNK_BYTES overrides the rank-count rule");
  clearEnv();
}

void hashes() {
  clearEnv();
  Config a = loadConfig(), b = loadConfig();
  check(configHash(a) == configHash(b), "configHash equal for equal configs");
  b.channels = a.channels - 1;
  check(configHash(a) != configHash(b), "configHash differs when the layout differs");
  b = a;
  b.threads = 256;
  b.tsSplit = 3 | (3 << 4);
  b.timeoutMs = 5;
  check(configHash(a) == configHash(b), "configHash ignores rank-local knobs");
  // Whether and with how many CTAs the zero-copy NVLS kernel runs must agree.
  b = a;
  b.nvlsZeroCopy = !a.nvlsZeroCopy;
  check(configHash(a) != configHash(b), "configHash covers TNCCL_NVLS_ZERO_COPY");
  b = a;
  b.nvlsZcChannels = a.nvlsZcChannels + 1;
  check(configHash(a) != configHash(b), "configHash covers TNCCL_NVLS_ZC_CHANNELS");
  check(a.nvlsZeroCopy == 1 && a.nvlsZcMinBytes == -1 && a.nvlsZcChannels == 32,
        "defaults: zero-copy NVLS on, minimum by rank count, 32 channels");
  Config r2 = a, r4 = a, r8 = a;
  adaptConfig(r2, 2);
  adaptConfig(r4, 4);
  adaptConfig(r8, 8);
  check(r2.nvlsZcMinBytes == INT64_MAX && r4.nvlsZcMinBytes == (64ll << 20) &&
            r8.nvlsZcMinBytes == (16ll << 20),
        "zero-copy AUTO minimum: never on 2 ranks, 64 MiB on 4, 16 MiB on 8");
}

// Random text never crashes the tuning-table parser; whatever it accepts is
// sorted and holds only valid rank counts and algorithms.
void fuzzedTuningTables() {
  uint64_t x = 0x2545F4914F6CDD1Dull;
  auto next = [&x] {
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    return x;
  };
  const char* pieces[] = {"8", "4", " ", "1048576", "oneshot", "twoshot", "ring", "nvls",
                          "\n", "#", "x", "-1", "99", "18446744073709551615", "\t", "auto"};
  bool ok = true;
  for (int it = 0; it < 5000; ++it) {
    std::string text;
    const int n = (int)(next() % 40);
    for (int k = 0; k < n; ++k) text += pieces[next() % (sizeof(pieces) / sizeof(pieces[0]))];
    TuningTable t;
    std::string err;
    if (parseTuningTable(text, &t, &err)) {
      for (size_t i = 0; i < t.entries.size(); ++i) {
        const TuningEntry& e = t.entries[i];
        ok = ok && e.nranks >= 1 && e.nranks <= kMaxRanks && e.algo > TNCCL_ALGO_AUTO &&
             e.algo < TNCCL_NUM_ALGOS;
        if (i) {
          const TuningEntry& p = t.entries[i - 1];
          ok = ok && (p.nranks < e.nranks || (p.nranks == e.nranks && p.maxBytes <= e.maxBytes));
        }
      }
    } else {
      ok = ok && !err.empty() && t.entries.empty();
    }
  }
  check(ok, "fuzzed tuning tables");
  TuningTable t;
  std::string err;
  check(!parseTuningTable("8 -1 ring\n", &t, &err) &&
            !parseTuningTable("8 99999999999999999999999 ring\n", &t, &err) &&
            !parseTuningTable("8 12abc ring\n", &t, &err) &&
            !parseTuningTable("8 4096 ring\n8 x ring\n", &t, &err) && t.entries.empty(),
        "tuning: negative / overflowing / malformed sizes rejected, table left empty");
}

void tuningTables() {
  TuningTable t;
  std::string err;
  const char* text =
      "# measured on 8 x B200\n"
      "8 1048576 oneshot\n"
      "8 268435456 twoshot   # mid sizes\n"
      "\n"
      "2 2097152 oneshot\n"
      "8 524288 oneshot\n";
  check(parseTuningTable(text, &t, &err) && t.entries.size() == 4, "tuning table parses");
  check(tunedAlgo(t, 8, 1) == TNCCL_ALGO_ONESHOT && tunedAlgo(t, 8, 1048577) == TNCCL_ALGO_TWOSHOT &&
            tunedAlgo(t, 8, 268435457) == -1 && tunedAlgo(t, 4, 100) == -1 &&
            tunedAlgo(t, 2, 2097152) == TNCCL_ALGO_ONESHOT,
        "tuning lookup: smallest max_bytes >= size, per rank count");
  check(!parseTuningTable("8 1024\n", &t, &err) && err.find("line 1") != std::string::npos,
        "tuning: missing field rejected with its line number");
  check(!parseTuningTable("4 1024 fastest\n", &t, &err) && !parseTuningTable("0 1 ring\n", &t, &err) &&
            !parseTuningTable("4 1024 auto\n", &t, &err) &&
            !parseTuningTable("4 1024 ring extra\n", &t, &err),
        "tuning: bad algorithm / rank count / trailing field rejected");

  clearEnv();
  Config a = loadConfig();
  const std::string path = "/tmp/tnccl_config_test_tuning.txt";
  FILE* f = fopen(path.c_str(), "w");
  fputs("2 4096 ring\n", f);
  fclose(f);
  setenv("TNCCL_TUNING_FILE", path.c_str(), 1);
  Config b = loadConfig();
  check(b.tuning.entries.size() == 1 && tunedAlgo(b.tuning, 2, 4096) == TNCCL_ALGO_RING,
        "TNCCL_TUNING_FILE loaded");
  check(configHash(a) != configHash(b), "configHash covers the tuning table");
  setenv("TNCCL_TUNING_FILE", "/nonexistent/tnccl.txt", 1);
  Config c = loadConfig();
  check(c.tuning.entries.empty(), "unreadable tuning file ignored");
  unsetenv("TNCCL_TUNING_FILE");
  remove(path.c_str());
}

void teamSplits() {
  bool ok = true;
  for (int nw = 3; nw <= 32; ++nw)
    for (int a = 0; a < 16; ++a)
      for (int b = 0; b < 16; ++b) {
        const TeamWarps t = teamWarps(nw, a | (b << 4));
        ok = ok && t.first >= 1 && t.second >= 1 && t.third >= 1 &&
             t.first + t.second + t.third == nw;
      }
  const TeamWarps d = teamWarps(16, 2 | (4 << 4));
  check(ok && d.first == 4 && d.second == 8 && d.third == 4,
        "team split: every team >= 1 warp for any split, 16 warps 2,4 -> 4/8/4");
}

void layouts() {
  bool ok = true;
  for (int P : {2, 3, 4, 8, 16}) {
    LayoutConfig lc{};
    lc.nranks = P;
    lc.channels = 96;
    lc.osChannels = 64;
    lc.ringSlots = 4;
    lc.ringChunkBytes = 256 << 10;
    lc.tsChunkBytes = (512 << 10) / P;
    lc.osSlots = 2;
    lc.osTileBytes = 32 << 10;
    const MailboxLayout L = makeLayout(lc);
    const uint64_t C = 96;
    std::vector<std::pair<uint64_t, uint64_t>> areas = {
        {L.ringDataOff, C * 4 * lc.ringChunkBytes},
        {L.tsRsDataOff, C * kTwoShotSlots * P * lc.tsChunkBytes},
        {L.tsAgDataOff, C * kTwoShotSlots * P * lc.tsChunkBytes},
        {L.osDataOff, 64ull * 2 * P * lc.osTileBytes},
        {L.ringReadyOff, C * 4 * 8},
        {L.ringCreditOff, C * 4 * 8},
        {L.tsRsFlagOff, C * kTwoShotSlots * P * 8},
        {L.tsAgFlagOff, C * kTwoShotSlots * P * 8},
        {L.osFlagOff, 64ull * 2 * P * 8},
        {L.osAckOff, 64ull * 2 * P * 8},
    };
    for (int k = 0; k < kNumCanaries; ++k) areas.push_back({L.canaryOff[k], kCanaryBytes});
    std::sort(areas.begin(), areas.end());
    for (size_t i = 0; i + 1 < areas.size(); ++i)
      ok = ok && areas[i].first + areas[i].second <= areas[i + 1].first;
    ok = ok && areas.back().first + areas.back().second <= L.totalBytes;
    ok = ok && L.totalBytes % 4096 == 0 && L.tsRsDataOff % 4096 == 0 && L.osDataOff % 4096 == 0;
    // The canary after an area starts exactly where the area ends.
    ok = ok && L.canaryOff[0] == L.ringDataOff + C * 4 * lc.ringChunkBytes;
    ok = ok && L.canaryOff[1] == L.tsRsDataOff + C * kTwoShotSlots * P * lc.tsChunkBytes;
    ok = ok && L.canaryOff[2] == L.tsAgDataOff + C * kTwoShotSlots * P * lc.tsChunkBytes;
  }
  check(ok, "mailbox areas, flags and canaries do not overlap");
  const uint64_t tb = 512 << 10;
  check(nvlsCounterAt(tb, 64, 1, 127, kNvlsSlots - 1) + 8 <= nvlsRegionBytes(tb, 64) &&
            nvlsCounterAt(tb, 64, 0, 0, 0) == nvlsDataBytes(tb, 64),
        "NVLS counters follow the data blocks inside the region");
  check(nvlsZcCounterAt(tb, 64, 0, 0) == nvlsCounterAt(tb, 64, 1, kMaxChannels - 1, kNvlsSlots - 1) + 8 &&
            nvlsZcCounterAt(tb, 64, 1, kMaxChannels - 1) + 8 <= nvlsRegionBytes(tb, 64),
        "zero-copy NVLS counters follow the staged kernel's inside the region");
}

void plans() {
  bool ok = true;
  uint64_t seed = 12345;
  auto rnd = [&seed]() {
    seed = seed * 6364136223846793005ull + 1442695040888963407ull;
    return seed >> 33;
  };
  for (int it = 0; it < 400 && ok; ++it) {
    const uint64_t V = (it % 2) ? 4 : 8;
    const uint64_t count = (it < 20) ? (uint64_t)it : rnd() % 3000000;
    const int P = 2 + (int)(rnd() % 15);
    const int channels = 1 + (int)(rnd() % 128);
    const uint64_t maxChunk = 16 * (1 + rnd() % 4096);
    ChunkPlan cp = makeChunkPlan(count, P, channels, maxChunk, 16, V);
    std::vector<unsigned char> seen(count, 0);
    for (uint64_t t = 0; t < cp.numTiles; ++t)
      for (int j = 0; j < P; ++j) {
        const Span s = chunkSpan(cp, t, j, V);
        ok = ok && (s.count == 0 || s.offset % V == 0) && s.offset + s.count <= count;
        for (uint64_t e = s.offset; e < s.offset + s.count && ok; ++e) ok = ++seen[e] == 1;
      }
    for (uint64_t e = 0; e < count && ok; ++e) ok = seen[e] == 1;
    ok = ok && cp.channels >= 1 && cp.channels <= channels;

    BlockPlan bp = makeBlockPlan(count, channels, maxChunk, 16, V);
    std::fill(seen.begin(), seen.end(), 0);
    for (uint64_t t = 0; t < bp.numTiles; ++t) {
      const Span s = blockTileSpan(bp, t);
      for (uint64_t e = s.offset; e < s.offset + s.count && ok; ++e) ok = ++seen[e] == 1;
      // NVLS shares: every vector of the tile belongs to exactly one rank.
      const uint64_t nv = divUp(s.count, V);
      uint64_t covered = 0;
      for (int r = 0; r < P; ++r) {
        const Span sh = blockShare(nv, P, r, 1);
        ok = ok && sh.offset == covered;
        covered += sh.count;
      }
      ok = ok && covered == nv;
    }
    for (uint64_t e = 0; e < count && ok; ++e) ok = seen[e] == 1;
  }
  check(ok, "chunk / block / share plans cover every element once");
}

}  // namespace

int main() {
  defaultsAndOverrides();
  netKnobs();
  adaptChunks();
  hashes();
  tuningTables();
  fuzzedTuningTables();
  teamSplits();
  layouts();
  plans();
  printf("config_test: %s\n", gFailed ? "FAIL" : "PASS");
  return gFailed ? 1 : 0;
}
