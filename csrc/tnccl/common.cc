#include "common.h"

#include "protocol.h"

#include <errno.h>
#include <stdio.h>
#include <string.h>
#include <strings.h>
#include <unistd.h>

#include <algorithm>
#include <mutex>

namespace tnccl {

int logLevel() {
  static int level = [] {
    const char* v = getenv("TNCCL_DEBUG");
    if (v == nullptr) return (int)kLogWarn;
    if (strcasecmp(v, "NONE") == 0) return (int)kLogNone;
    if (strcasecmp(v, "INFO") == 0) return (int)kLogInfo;
    if (strcasecmp(v, "TRACE") == 0) return (int)kLogTrace;
    return (int)kLogWarn;
  }();
  return level;
}

void logf(int level, const char* fmt, ...) {
  if (level > logLevel()) return;
  static std::mutex mu;
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  const char* tag = level == kLogWarn ? "WARN" : level == kLogInfo ? "INFO" : "TRACE";
  std::lock_guard<std::mutex> lock(mu);
  fprintf(stderr, "[tnccl pid %d] %s %s\n", (int)getpid(), tag, buf);
}

int64_t envInt(const char* name, int64_t dflt) {
  const char* v = getenv(name);
  if (v == nullptr || *v == '\0') return dflt;
  char* end = nullptr;
  long long x = strtoll(v, &end, 0);
  if (end == v || (end && *end != '\0')) {
    TN_WARN("ignoring malformed %s=%s", name, v);
    return dflt;
  }
  return (int64_t)x;
}

std::string envStr(const char* name, const char* dflt) {
  const char* v = getenv(name);
  return (v == nullptr || *v == '\0') ? std::string(dflt) : std::string(v);
}

int parseAlgo(const std::string& s) {
  if (s.empty() || strcasecmp(s.c_str(), "auto") == 0) return TNCCL_ALGO_AUTO;
  if (strcasecmp(s.c_str(), "ring") == 0) return TNCCL_ALGO_RING;
  if (strcasecmp(s.c_str(), "oneshot") == 0) return TNCCL_ALGO_ONESHOT;
  if (strcasecmp(s.c_str(), "twoshot") == 0) return TNCCL_ALGO_TWOSHOT;
  if (strcasecmp(s.c_str(), "nvls") == 0) return TNCCL_ALGO_NVLS;
  return -1;
}

int parseNetMode(const std::string& s) {
  if (s.empty() || strcasecmp(s.c_str(), "auto") == 0 || s == "1") return 1;
  if (strcasecmp(s.c_str(), "off") == 0 || s == "0") return 0;
  if (strcasecmp(s.c_str(), "force") == 0 || s == "2") return 2;
  return -1;
}

static int clampInt(int64_t v, int lo, int hi) {
  return (int)(v < lo ? lo : v > hi ? hi : v);
}

static int64_t roundTo16(int64_t v) { return v < 16 ? 16 : (v + 15) / 16 * 16; }

Config loadConfig() {
  Config c{};
  c.channels = clampInt(envInt("TNCCL_NCHANNELS", 128), 1, kMaxChannels);
  c.osChannels = clampInt(envInt("TNCCL_ONESHOT_CHANNELS", 64), 1, kMaxChannels);
  c.ringSlots = clampInt(envInt("TNCCL_SLOTS", 4), 2, 16);
  c.ringChunkBytes = roundTo16(envInt("TNCCL_CHUNK_BYTES", 256 << 10));
  c.tsChunkBytes = roundTo16(envInt("TNCCL_TWOSHOT_CHUNK_BYTES", 0));  // 0: by nranks
  c.osSlots = clampInt(envInt("TNCCL_ONESHOT_SLOTS", 2), 1, 8);
  c.osTileBytes = roundTo16(envInt("TNCCL_ONESHOT_TILE_BYTES", 32 << 10));
  c.nvlsChannels = clampInt(envInt("TNCCL_NVLS_CHANNELS", 64), 1, kMaxChannels);
  c.nvlsTileBytes = roundTo16(envInt("TNCCL_NVLS_TILE_BYTES", 512 << 10));
  c.nvlsEnable = (int)envInt("TNCCL_NVLS_ENABLE", 1);
  // Off until it has been measured against the staged kernel.
  c.nvlsZeroCopy = envInt("TNCCL_NVLS_ZERO_COPY", 1) ? 1 : 0;
  c.nvlsZcMinBytes = envInt("TNCCL_NVLS_ZC_MIN_BYTES", -1);  // -1: by rank count
  c.nvlsZcChannels = clampInt(envInt("TNCCL_NVLS_ZC_CHANNELS", 32), 1, kMaxChannels);
  int algo = parseAlgo(envStr("TNCCL_ALGO", "auto"));
  if (algo < 0) {
    TN_WARN("unknown TNCCL_ALGO; using auto");
    algo = TNCCL_ALGO_AUTO;
  }
  c.forcedAlgo = algo;
  c.timeoutMs = envInt("TNCCL_TIMEOUT_MS", 30000);
  if (c.timeoutMs < 1) c.timeoutMs = 1;
  c.bootstrapTimeoutMs = envInt("TNCCL_BOOTSTRAP_TIMEOUT_MS", 30000);
  if (c.bootstrapTimeoutMs < 1) c.bootstrapTimeoutMs = 1;
  c.threads = clampInt(envInt("TNCCL_NTHREADS", 512), 128, 512) / 32 * 32;
  c.useCuMem = (int)envInt("TNCCL_CUMEM_ENABLE", 1);
  c.oneShotMaxBytes = envInt("TNCCL_ONESHOT_MAX_BYTES", 0);
  c.nvlsMinBytes = envInt("TNCCL_NVLS_MIN_BYTES", 0);
  c.traceEvents = envInt("TNCCL_TRACE", 0) ? clampInt(envInt("TNCCL_TRACE_EVENTS", 4096), 16, 1 << 20)
                                            : 0;
  c.tsSplit = parseSplit(envStr("TNCCL_TWOSHOT_SPLIT", ""), 2 | (4 << 4));
  c.nvlsSplit = parseSplit(envStr("TNCCL_NVLS_SPLIT", ""), 1 | (4 << 4));
  c.acquireMode = envInt("TNCCL_ACQUIRE_LOAD", 1) ? 1 : 0;
  // Staging sizes: a stage is split among up to 16 sources and every buffer
  // stays 16-byte aligned; 256 bytes of mbarriers plus all rings fit the
  // 227 KiB of shared memory a CTA can have (fewer stages otherwise).
  const int64_t kSmem = 227 * 1024 - 256;
  c.tsStages = clampInt(envInt("TNCCL_TWOSHOT_STAGES", 2), 1, 8);
  c.tsPushStage = clampInt(envInt("TNCCL_TWOSHOT_PUSH_STAGE", 32 << 10), 4 << 10, 96 << 10) / 256 * 256;
  c.tsRedStage = clampInt(envInt("TNCCL_TWOSHOT_REDUCE_STAGE", 64 << 10), 4 << 10, 128 << 10) / 256 * 256;
  auto tsBytes = [&c]() { return (int64_t)c.tsStages * (c.tsPushStage + c.tsRedStage); };
  while (c.tsStages > 1 && tsBytes() > kSmem) --c.tsStages;
  if (tsBytes() > kSmem) c.tsPushStage = c.tsRedStage = 32 << 10;
  c.nvlsStages = clampInt(envInt("TNCCL_NVLS_STAGES", 2), 1, 8);
  c.nvlsStage = clampInt(envInt("TNCCL_NVLS_STAGE", 48 << 10), 4 << 10, 96 << 10) / 256 * 256;
  while (c.nvlsStages > 1 && (int64_t)c.nvlsStages * c.nvlsStage > kSmem) --c.nvlsStages;
  // TMA staging of the two-shot push / reduce and NVLS copy-in loads is
  // opt-in (TNCCL_STAGE_MIN_BYTES): the register path was as fast or faster
  // at every size measured, on 4 x B200 (648 vs 631 GB/s at 256 MiB) and on
  // 8 (618 vs 367 at 256 MiB, 654 vs 484 at 1 GiB): a bulk-copy stage has a
  // fixed cost that short per-peer pieces do not amortise.
  c.stageMinBytes = clampInt(envInt("TNCCL_STAGE_MIN_BYTES", 1 << 30), 0, 1 << 30);
  c.tuning = loadTuningTable();
  c.netMode = parseNetMode(envStr("TNCCL_NET", "auto"));
  if (c.netMode < 0) {
    TN_WARN("unknown TNCCL_NET (want off, auto or force); using auto");
    c.netMode = 1;
  }
  c.netChannels = clampInt(envInt("TNCCL_NET_CHANNELS", 2), 1, 8);
  c.netIf = envStr("TNCCL_NET_IF", "");
  c.netSockBuf = clampInt(envInt("TNCCL_NET_SOCKBUF", 0), 0, 1 << 30);
  c.netSpinUs = clampInt(envInt("TNCCL_NET_SPIN_US", 200), 0, 1000000);
  return c;
}

int parseSplit(const std::string& s, int dflt) {
  int a = 0, b = 0;
  char extra = 0;
  if (s.empty()) return dflt;
  if (sscanf(s.c_str(), "%d,%d%c", &a, &b, &extra) != 2 || a < 1 || b < 1 || a + b > 7) {
    TN_WARN("malformed team split '%s' (want a,b in eighths, a + b <= 7); using default",
            s.c_str());
    return dflt;
  }
  return a | (b << 4);
}

uint64_t configHash(const Config& c) {
  // FNV-1a over the fields that change the device protocol or the mailbox
  // layout. Timeouts and thread counts may differ across ranks.
  uint64_t h = 1469598103934665603ull;
  auto mix = [&h](int64_t v) {
    for (int i = 0; i < 8; ++i) {
      h ^= (uint64_t)((v >> (8 * i)) & 0xff);
      h *= 1099511628211ull;
    }
  };
  mix(c.channels);
  mix(c.osChannels);
  mix(c.ringSlots);
  mix(c.ringChunkBytes);
  mix(c.tsChunkBytes);
  mix(c.osSlots);
  mix(c.osTileBytes);
  mix(c.nvlsChannels);
  mix(c.nvlsTileBytes);
  mix(c.nvlsEnable);
  mix(c.nvlsZeroCopy);
  mix(c.nvlsZcMinBytes);
  mix(c.nvlsZcChannels);
  mix(c.forcedAlgo);
  mix(c.useCuMem);
  mix(c.oneShotMaxBytes);
  mix(c.nvlsMinBytes);
  // Which ring edges are socket edges, and the ring channels they carry.
  mix(c.netMode);
  mix(c.netChannels);
  // Every rank must pick the same algorithm for a message.
  for (const TuningEntry& e : c.tuning.entries) {
    mix(e.nranks);
    mix((int64_t)e.maxBytes);
    mix(e.algo);
  }
  return h;
}

}  // namespace tnccl

namespace tnccl {

void adaptConfig(Config& c, int nranks) {
  if (nranks < 1) nranks = 1;
  // Two-shot: a 512 KiB tile per channel split into one chunk per rank, so
  // the mailbox (channels x slots x tile x 2) does not grow with nranks.
  // Measured on 2 x B200: 256 KiB chunks reach 590-625 GB/s bus bandwidth
  // at 256 MiB with 64-128 channels; 64 KiB chunks lose a third.
  if (c.tsChunkBytes <= 16 && envInt("TNCCL_TWOSHOT_CHUNK_BYTES", 0) == 0) {
    int64_t chunk = (int64_t)(512 << 10) / nranks;
    chunk = chunk < (32 << 10) ? (32 << 10) : chunk > (256 << 10) ? (256 << 10) : chunk;
    c.tsChunkBytes = chunk / 16 * 16;
  }
  // Smallest registered message AUTO sends through the zero-copy NVLS
  // kernel. Measured on 8 x B200: it beats two-shot from 32 MiB and NCCL
  // from 32 MiB to 4 GiB (fp32 and bf16), is level with two-shot at 16 MiB
  // and behind below; on 2 x B200 two-shot wins at every size (the switch
  // step moves 1.5 x the message per direction there, two-shot 1 x), so
  // 2 ranks never take it. 3 to 7 ranks: not measured; 64 MiB.
  if (c.nvlsZcMinBytes < 0)
    c.nvlsZcMinBytes = nranks >= 8 ? (16ll << 20) : nranks >= 3 ? (64ll << 20) : INT64_MAX;
}

bool parseTuningTable(const std::string& text, TuningTable* out, std::string* error) {
  out->entries.clear();
  size_t pos = 0;
  int lineNo = 0;
  while (pos <= text.size()) {
    size_t end = text.find('\n', pos);
    if (end == std::string::npos) end = text.size();
    std::string line = text.substr(pos, end - pos);
    pos = end + 1;
    ++lineNo;
    const size_t hash = line.find('#');
    if (hash != std::string::npos) line.resize(hash);
    if (line.find_first_not_of(" \t\r") == std::string::npos) continue;
    int nranks = 0;
    unsigned long long maxBytes = 0;
    char sizeText[32] = {0};
    char algoName[32] = {0};
    char extra[2] = {0};
    // The size is read as text first: %llu alone would take "-1" as 2^64 - 1.
    char* sizeEnd = nullptr;
    errno = 0;
    if (sscanf(line.c_str(), "%d %31s %31s %1s", &nranks, sizeText, algoName, extra) != 3 ||
        nranks < 1 || nranks > kMaxRanks || sizeText[0] < '0' || sizeText[0] > '9' ||
        (maxBytes = strtoull(sizeText, &sizeEnd, 10), *sizeEnd != '\0' || errno == ERANGE)) {
      if (error) *error = "line " + std::to_string(lineNo) + ": want <nranks> <max_bytes> <algo>";
      out->entries.clear();
      return false;
    }
    const int algo = parseAlgo(algoName);
    if (algo <= TNCCL_ALGO_AUTO) {
      if (error) *error = "line " + std::to_string(lineNo) + ": unknown algorithm " + algoName;
      out->entries.clear();
      return false;
    }
    out->entries.push_back(TuningEntry{nranks, (uint64_t)maxBytes, algo});
  }
  std::sort(out->entries.begin(), out->entries.end(),
            [](const TuningEntry& a, const TuningEntry& b) {
              return a.nranks != b.nranks ? a.nranks < b.nranks : a.maxBytes < b.maxBytes;
            });
  return true;
}

TuningTable loadTuningTable() {
  TuningTable t;
  const std::string path = envStr("TNCCL_TUNING_FILE", "");
  if (path.empty()) return t;
  FILE* f = fopen(path.c_str(), "r");
  if (f == nullptr) {
    TN_WARN("TNCCL_TUNING_FILE %s cannot be read; using the built-in thresholds", path.c_str());
    return t;
  }
  std::string text;
  char buf[4096];
  size_t n;
  while ((n = fread(buf, 1, sizeof(buf), f)) > 0) text.append(buf, n);
  fclose(f);
  std::string err;
  if (!parseTuningTable(text, &t, &err)) {
    TN_WARN("TNCCL_TUNING_FILE %s: %s; using the built-in thresholds", path.c_str(), err.c_str());
    t.entries.clear();
  }
  return t;
}

int tunedAlgo(const TuningTable& t, int nranks, uint64_t bytes) {
  for (const TuningEntry& e : t.entries)
    if (e.nranks == nranks && bytes <= e.maxBytes) return e.algo;
  return -1;
}

}  // namespace tnccl
