// common.h - logging, environment configuration and small helpers for the
// host side of the library.
#pragma once

#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include <string>
#include <vector>

#include "tnccl.h"

namespace tnccl {

// TNCCL_DEBUG=WARN|INFO|TRACE selects host log verbosity (default: WARN).
enum LogLevel { kLogNone = 0, kLogWarn = 1, kLogInfo = 2, kLogTrace = 3 };
int logLevel();
void logf(int level, const char* fmt, ...) __attribute__((format(printf, 2, 3)));

#define TN_WARN(...) ::tnccl::logf(::tnccl::kLogWarn, __VA_ARGS__)
#define TN_INFO(...) ::tnccl::logf(::tnccl::kLogInfo, __VA_ARGS__)
#define TN_TRACE(...) ::tnccl::logf(::tnccl::kLogTrace, __VA_ARGS__)

// Integer environment variable with a default; malformed values fall back to
// the default with a warning.
int64_t envInt(const char* name, int64_t dflt);
std::string envStr(const char* name, const char* dflt);

// AUTO tuning table (TNCCL_TUNING_FILE): text lines "<nranks> <max_bytes>
// <algo>", '#' starts a comment. For a communicator of nranks ranks, a
// message of b bytes uses the algorithm of the line with the smallest
// max_bytes >= b among that rank count's lines; sizes above every line keep
// the built-in rule. benchmarks/make_tuning_table.py writes such a file from
// a measured sweep.
struct TuningEntry {
  int nranks;
  uint64_t maxBytes;
  int algo;
};
struct TuningTable {
  std::vector<TuningEntry> entries;  // sorted by (nranks, maxBytes)
};
// Parses `text`; false (*error set, the table left empty) on a malformed
// line.
bool parseTuningTable(const std::string& text, TuningTable* out, std::string* error);
// The table's algorithm for (nranks, bytes), or -1 when no line applies.
int tunedAlgo(const TuningTable& t, int nranks, uint64_t bytes);

// Tunables read once per communicator. They must be equal on every rank; the
// bootstrap hello carries their hash and rank 0 rejects a mismatch.
struct Config {
  int channels;          // TNCCL_NCHANNELS (ring / two-shot CTAs)
  int osChannels;        // TNCCL_ONESHOT_CHANNELS
  int ringSlots;         // TNCCL_SLOTS
  int64_t ringChunkBytes;  // TNCCL_CHUNK_BYTES
  int64_t tsChunkBytes;    // TNCCL_TWOSHOT_CHUNK_BYTES
  int osSlots;
  int64_t osTileBytes;     // TNCCL_ONESHOT_TILE_BYTES
  int nvlsChannels;        // TNCCL_NVLS_CHANNELS
  int64_t nvlsTileBytes;   // TNCCL_NVLS_TILE_BYTES
  int nvlsEnable;          // TNCCL_NVLS_ENABLE (0 off, 1 on if supported)
  // Zero-copy NVLS over registered buffers (register.cc).
  int nvlsZeroCopy;        // TNCCL_NVLS_ZERO_COPY (1 on, the default; 0 off)
  int64_t nvlsZcMinBytes;  // TNCCL_NVLS_ZC_MIN_BYTES: AUTO uses it from here up
                           // (-1: by rank count, resolved by adaptConfig)
  int nvlsZcChannels;      // TNCCL_NVLS_ZC_CHANNELS (CTAs per launch)
  int forcedAlgo;          // TNCCL_ALGO (tncclAlgo_t)
  int64_t timeoutMs;       // TNCCL_TIMEOUT_MS: device wait bound
  int64_t bootstrapTimeoutMs;  // TNCCL_BOOTSTRAP_TIMEOUT_MS
  int threads;             // TNCCL_NTHREADS (threads per CTA)
  int useCuMem;            // TNCCL_CUMEM_ENABLE (0: legacy cudaIpc)
  // AUTO thresholds in bytes (0 = derive from nranks).
  int64_t oneShotMaxBytes;   // TNCCL_ONESHOT_MAX_BYTES
  int64_t nvlsMinBytes;      // TNCCL_NVLS_MIN_BYTES
  int traceEvents;           // TNCCL_TRACE=1: records per channel (TNCCL_TRACE_EVENTS)
  // Warp split of the warp-specialised kernels, in eighths of a CTA's warps
  // for the first two teams (packed a | b << 4; the third team gets the
  // rest). Local to a rank: it does not change the protocol.
  int tsSplit;               // TNCCL_TWOSHOT_SPLIT "push,reduce" (default 2,4)
  int nvlsSplit;             // TNCCL_NVLS_SPLIT "copy-in,switch" (default 1,4)
  int acquireMode;           // TNCCL_ACQUIRE_LOAD (1: ld.acquire.sys, 0: fence)
  int tsStages;              // TNCCL_TWOSHOT_STAGES (1..8, default 2)
  int tsPushStage;           // TNCCL_TWOSHOT_PUSH_STAGE bytes (default 32 KiB)
  int tsRedStage;            // TNCCL_TWOSHOT_REDUCE_STAGE bytes (default 64 KiB)
  int nvlsStages;            // TNCCL_NVLS_STAGES (1..8, default 2)
  int nvlsStage;             // TNCCL_NVLS_STAGE bytes (default 48 KiB)
  int stageMinBytes;         // TNCCL_STAGE_MIN_BYTES (default 1 GiB: staging off)
  TuningTable tuning;        // TNCCL_TUNING_FILE (empty: built-in AUTO rule)
  // Socket ring edges (net.h). TNCCL_NET: "off", "auto" (edges between
  // ranks on different hosts) or "force" (every ring edge, also on one host).
  int netMode;               // 0 off, 1 auto, 2 force
  int netChannels;           // TNCCL_NET_CHANNELS: ring channels of a socket edge (1..8)
  std::string netIf;         // TNCCL_NET_IF: IPv4 address to listen on ("": derived)
  int netSockBuf;            // TNCCL_NET_SOCKBUF: SO_SNDBUF / SO_RCVBUF (0: system)
  int netSpinUs;             // TNCCL_NET_SPIN_US: proxy busy-poll window
};

// Loads TNCCL_TUNING_FILE when set (a missing or malformed file warns and
// yields an empty table).
TuningTable loadTuningTable();

// Parses "a,b" (eighths, each 1..6, a + b <= 7) into a | b << 4.
int parseSplit(const std::string& s, int dflt);

Config loadConfig();
// Fills in the defaults that depend on the rank count (called before the
// configuration hash is exchanged, so every rank derives the same values).
void adaptConfig(Config& c, int nranks);
uint64_t configHash(const Config& c);

int parseAlgo(const std::string& s);
// "off" / "auto" / "force" (or 0 / 1 / 2); -1 when malformed.
int parseNetMode(const std::string& s);

}  // namespace tnccl
