// protocol.h - partition, tile geometry and mailbox layout shared by host
// code, device kernels and the CPU rank model.
//
// Everything here is pure integer arithmetic on __host__ __device__ inline
// functions, so the kernels, the launcher and tests/cpp/rank_model_test.cc use
// one copy of the index math (tiny-nccl keeps its index math in
// src/device.cuh:16-75 and re-implements it in tests/ring_model_test.cc:16-30;
// sharing one header removes that duplication).
//
// Work decomposition (all algorithms):
//   * A message of N elements is cut into tiles. For the ring and the
//     two-shot algorithm a tile holds P chunks (one per rank); for one-shot and
//     NVLS a tile is one contiguous block that every rank contributes in full.
//   * Tile k is handled by channel (CTA) k % C, so one channel walks tiles
//     c, c + C, c + 2C, ... in order. Every rank derives the same tile list
//     from (N, P, C, chunk), so per-channel FIFO sequence numbers advance
//     identically on all ranks without any host-side ticket.
//   * Chunk boundaries are multiples of the 16-byte vector width V, so only
//     the very end of the message can need scalar accesses.
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define TN_HD __host__ __device__ __forceinline__
#else
#define TN_HD inline
#endif

namespace tnccl {

constexpr int kMaxRanks = 16;
constexpr int kMaxChannels = 128;
constexpr int kVectorBytes = 16;
// Smallest chunk (bytes) the planners use, so that small messages occupy few
// channels instead of many nearly empty ones.
constexpr uint64_t kRingMinChunkBytes = 4096;
constexpr uint64_t kTwoShotMinChunkBytes = 2048;
constexpr uint64_t kOneShotMinTileBytes = 4096;
constexpr uint64_t kNvlsMinTileBytes = 16384;
// Two-shot keeps up to kTwoShotSlots tiles in flight per channel.
constexpr int kTwoShotSlots = 4;
// NVLS keeps up to kNvlsSlots tiles in flight per channel.
constexpr int kNvlsSlots = 4;

// Counter families kept in device memory, one array of kMaxChannels each.
enum CounterFamily : int {
  kCounterRing = 0,
  kCounterOneShot = 1,
  kCounterTwoShot = 2,
  kCounterNvls = 3,
  kCounterNvlsZc = 4,  // zero-copy NVLS over registered buffers
  kNumCounterFamilies = 5
};

TN_HD uint64_t divUp(uint64_t a, uint64_t b) { return (a + b - 1) / b; }
TN_HD uint64_t roundUp(uint64_t a, uint64_t b) { return divUp(a, b) * b; }
TN_HD uint64_t minU64(uint64_t a, uint64_t b) { return a < b ? a : b; }
TN_HD uint64_t maxU64(uint64_t a, uint64_t b) { return a > b ? a : b; }

struct Span {
  uint64_t offset;  // element offset into the message
  uint64_t count;   // elements
};

// ---------------------------------------------------------------------------
// Chunked tiles (ring, two-shot): tile = P chunks.
// ---------------------------------------------------------------------------
struct ChunkPlan {
  uint64_t count;       // N
  uint64_t chunkElems;  // elements per chunk in a full tile (multiple of V)
  uint64_t tileElems;   // P * chunkElems
  uint64_t numTiles;    // ceil(N / tileElems)
  int nranks;
  int channels;         // channels actually used (<= requested, >= 1)
};

// Picks the chunk so that the message spreads over all channels, but never
// exceeds the mailbox chunk capacity and never drops below minChunkElems.
TN_HD ChunkPlan makeChunkPlan(uint64_t count, int nranks, int channels,
                              uint64_t maxChunkElems, uint64_t minChunkElems,
                              uint64_t vecElems) {
  ChunkPlan p{};
  p.count = count;
  p.nranks = nranks;
  uint64_t want = roundUp(divUp(count, (uint64_t)nranks * (uint64_t)channels),
                          vecElems);
  want = maxU64(want, minChunkElems);
  want = minU64(want, maxChunkElems);
  if (want == 0) want = vecElems;
  p.chunkElems = want;
  p.tileElems = want * (uint64_t)nranks;
  p.numTiles = count == 0 ? 0 : divUp(count, p.tileElems);
  uint64_t used = minU64((uint64_t)channels, p.numTiles);
  p.channels = used == 0 ? 1 : (int)used;
  return p;
}

// Element range of tile k.
TN_HD Span tileSpan(const ChunkPlan& p, uint64_t tile) {
  uint64_t base = tile * p.tileElems;
  uint64_t len = p.count > base ? minU64(p.tileElems, p.count - base) : 0;
  return Span{base, len};
}

// Element range of chunk j inside tile k. A full tile uses chunkElems per
// chunk; the final partial tile spreads its remainder evenly over the ranks
// (rounded to the vector width), so some trailing chunks may be empty.
TN_HD Span chunkSpan(const ChunkPlan& p, uint64_t tile, int chunk,
                     uint64_t vecElems) {
  Span t = tileSpan(p, tile);
  uint64_t cl = t.count == p.tileElems
                    ? p.chunkElems
                    : roundUp(divUp(t.count, (uint64_t)p.nranks), vecElems);
  uint64_t off = minU64((uint64_t)chunk * cl, t.count);
  uint64_t n = minU64(cl, t.count - off);
  return Span{t.offset + off, n};
}

// Number of tiles channel c processes.
TN_HD uint64_t channelTiles(uint64_t numTiles, int channels, int c) {
  return numTiles > (uint64_t)c ? divUp(numTiles - (uint64_t)c, (uint64_t)channels)
                                : 0;
}

// ---------------------------------------------------------------------------
// Block tiles (one-shot, NVLS): tile = one block every rank contributes.
// ---------------------------------------------------------------------------
struct BlockPlan {
  uint64_t count;
  uint64_t tileElems;
  uint64_t numTiles;
  int channels;
};

TN_HD BlockPlan makeBlockPlan(uint64_t count, int channels,
                              uint64_t maxTileElems, uint64_t minTileElems,
                              uint64_t vecElems) {
  BlockPlan p{};
  p.count = count;
  uint64_t want = roundUp(divUp(count, (uint64_t)channels), vecElems);
  want = maxU64(want, minTileElems);
  want = minU64(want, maxTileElems);
  if (want == 0) want = vecElems;
  p.tileElems = want;
  p.numTiles = count == 0 ? 0 : divUp(count, want);
  uint64_t used = minU64((uint64_t)channels, p.numTiles);
  p.channels = used == 0 ? 1 : (int)used;
  return p;
}

TN_HD Span blockTileSpan(const BlockPlan& p, uint64_t tile) {
  uint64_t base = tile * p.tileElems;
  uint64_t len = p.count > base ? minU64(p.tileElems, p.count - base) : 0;
  return Span{base, len};
}

// Rank r's share of a block tile for NVLS reduce (split evenly over P ranks
// in vector units).
TN_HD Span blockShare(uint64_t tileCount, int nranks, int rank,
                      uint64_t vecElems) {
  uint64_t cl = roundUp(divUp(tileCount, (uint64_t)nranks), vecElems);
  uint64_t off = minU64((uint64_t)rank * cl, tileCount);
  return Span{off, minU64(cl, tileCount - off)};
}

// ---------------------------------------------------------------------------
// Ring: chunk schedule of the reduce-scatter / all-gather rotation.
// ---------------------------------------------------------------------------
TN_HD int ringChunkBehind(int rank, int distance, int nranks) {
  int s = (rank - distance) % nranks;
  return s < 0 ? s + nranks : s;
}

// Messages per tile on every ring edge: P-1 reduce-scatter + P-1 all-gather.
TN_HD uint64_t ringMessagesPerTile(int nranks) {
  return 2ull * (uint64_t)(nranks - 1);
}

// ---------------------------------------------------------------------------
// Mailbox layout. One unicast allocation per rank, mapped by every peer.
// Flags are 64-bit sequence words; each word has exactly one writer.
// ---------------------------------------------------------------------------
struct MailboxLayout {
  int nranks;
  int channels;       // channels provisioned for ring/two-shot
  int osChannels;     // channels provisioned for one-shot

  // ring FIFO: data + ready live in the consumer, credit in the producer.
  int ringSlots;
  uint64_t ringChunkBytes;
  uint64_t ringDataOff, ringReadyOff, ringCreditOff;

  // two-shot: per channel and slot, P reduce-scatter chunks + P all-gather
  // chunks (two slots so that one tile's all-gather overlaps the next
  // tile's reduce-scatter).
  uint64_t tsChunkBytes;
  uint64_t tsRsDataOff, tsAgDataOff, tsRsFlagOff, tsAgFlagOff;

  // one-shot: per channel and slot, P blocks; flag per source, ack per consumer.
  int osSlots;
  uint64_t osTileBytes;
  uint64_t osDataOff, osFlagOff, osAckOff;

  // Canary lines after every data area and after the flag block: filled
  // with kCanaryByte at init and checked by tncclCommValidate / destroy, so
  // a write past the end of an area shows up (kNumCanaries regions of
  // kCanaryBytes).
  uint64_t canaryOff[5];

  uint64_t totalBytes;
};

constexpr int kNumCanaries = 5;
constexpr uint64_t kCanaryBytes = 128;
constexpr unsigned char kCanaryByte = 0xA5;

struct LayoutConfig {
  int nranks;
  int channels;
  int osChannels;
  int ringSlots;
  uint64_t ringChunkBytes;
  uint64_t tsChunkBytes;
  int osSlots;
  uint64_t osTileBytes;
};

TN_HD uint64_t alignUp(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

// Warp counts of the three teams of a warp-specialised CTA of nw >= 3 warps:
// split = a | b << 4 asks for a/8 and b/8 of the warps for the first two
// teams; every team gets at least one warp and the third the rest.
struct TeamWarps {
  int first, second, third;
};
TN_HD TeamWarps teamWarps(int nw, int split) {
  int a = nw * (split & 15) / 8, b = nw * ((split >> 4) & 15) / 8;
  a = a < 1 ? 1 : a > nw - 2 ? nw - 2 : a;
  b = b < 1 ? 1 : b > nw - 1 - a ? nw - 1 - a : b;
  return TeamWarps{a, b, nw - a - b};
}

inline MailboxLayout makeLayout(const LayoutConfig& c) {
  MailboxLayout L{};
  const uint64_t P = (uint64_t)c.nranks;
  const uint64_t C = (uint64_t)c.channels;
  L.nranks = c.nranks;
  L.channels = c.channels;
  L.osChannels = c.osChannels;
  L.ringSlots = c.ringSlots;
  L.ringChunkBytes = c.ringChunkBytes;
  L.tsChunkBytes = c.tsChunkBytes;
  L.osSlots = c.osSlots;
  L.osTileBytes = c.osTileBytes;

  uint64_t off = 0;
  L.ringDataOff = off;
  off += C * (uint64_t)c.ringSlots * c.ringChunkBytes;
  L.canaryOff[0] = off;
  off = alignUp(off + kCanaryBytes, 4096);
  L.tsRsDataOff = off;
  off += C * kTwoShotSlots * P * c.tsChunkBytes;
  L.canaryOff[1] = off;
  off = alignUp(off + kCanaryBytes, 128);
  L.tsAgDataOff = off;
  off += C * kTwoShotSlots * P * c.tsChunkBytes;
  L.canaryOff[2] = off;
  off = alignUp(off + kCanaryBytes, 4096);
  L.osDataOff = off;
  off += (uint64_t)c.osChannels * (uint64_t)c.osSlots * P * c.osTileBytes;
  L.canaryOff[3] = off;
  off = alignUp(off + kCanaryBytes, 4096);
  // Flag words. Each group starts on its own 128-byte line.
  L.ringReadyOff = off;
  off = alignUp(off + C * (uint64_t)c.ringSlots * 8, 128);
  L.ringCreditOff = off;
  off = alignUp(off + C * (uint64_t)c.ringSlots * 8, 128);
  L.tsRsFlagOff = off;
  off = alignUp(off + C * kTwoShotSlots * P * 8, 128);
  L.tsAgFlagOff = off;
  off = alignUp(off + C * kTwoShotSlots * P * 8, 128);
  L.osFlagOff = off;
  off = alignUp(off + (uint64_t)c.osChannels * (uint64_t)c.osSlots * P * 8, 128);
  L.osAckOff = off;
  off = alignUp(off + (uint64_t)c.osChannels * (uint64_t)c.osSlots * P * 8, 128);
  L.canaryOff[4] = off;
  off += kCanaryBytes;
  L.totalBytes = alignUp(off, 4096);
  return L;
}

// Address helpers (byte offsets from a rank's mailbox base).
TN_HD uint64_t ringDataAt(const MailboxLayout& L, int c, int s) {
  return L.ringDataOff + ((uint64_t)c * L.ringSlots + s) * L.ringChunkBytes;
}
TN_HD uint64_t ringReadyAt(const MailboxLayout& L, int c, int s) {
  return L.ringReadyOff + ((uint64_t)c * L.ringSlots + s) * 8;
}
TN_HD uint64_t ringCreditAt(const MailboxLayout& L, int c, int s) {
  return L.ringCreditOff + ((uint64_t)c * L.ringSlots + s) * 8;
}
TN_HD uint64_t tsSlotIndex(const MailboxLayout& L, int c, int slot, int src) {
  return ((uint64_t)c * kTwoShotSlots + (uint64_t)slot) * L.nranks + src;
}
TN_HD uint64_t tsRsDataAt(const MailboxLayout& L, int c, int slot, int src) {
  return L.tsRsDataOff + tsSlotIndex(L, c, slot, src) * L.tsChunkBytes;
}
TN_HD uint64_t tsAgDataAt(const MailboxLayout& L, int c, int slot, int src) {
  return L.tsAgDataOff + tsSlotIndex(L, c, slot, src) * L.tsChunkBytes;
}
TN_HD uint64_t tsRsFlagAt(const MailboxLayout& L, int c, int slot, int src) {
  return L.tsRsFlagOff + tsSlotIndex(L, c, slot, src) * 8;
}
TN_HD uint64_t tsAgFlagAt(const MailboxLayout& L, int c, int slot, int src) {
  return L.tsAgFlagOff + tsSlotIndex(L, c, slot, src) * 8;
}
TN_HD uint64_t osDataAt(const MailboxLayout& L, int c, int s, int src) {
  return L.osDataOff +
         (((uint64_t)c * L.osSlots + s) * L.nranks + src) * L.osTileBytes;
}
TN_HD uint64_t osFlagAt(const MailboxLayout& L, int c, int s, int src) {
  return L.osFlagOff + (((uint64_t)c * L.osSlots + s) * L.nranks + src) * 8;
}
TN_HD uint64_t osAckAt(const MailboxLayout& L, int c, int s, int consumer) {
  return L.osAckOff +
         (((uint64_t)c * L.osSlots + s) * L.nranks + consumer) * 8;
}
// NVLS multicast region: per channel kNvlsSlots pairs of an input block and
// an output block, then the barrier counters: one 64-bit word per phase
// ("copied in", "stored"), channel and slot that every rank increments with
// a multicast add (multimem.red) once per use of the slot, so each rank's
// copy counts all ranks. A rank cannot count use k + 1 of a slot before
// every rank counted use k (the slot is reused only after all ranks stored
// it), so a count of P * k means every rank finished use k.
TN_HD uint64_t nvlsInAt(uint64_t tileBytes, int c, int slot) {
  return ((uint64_t)c * kNvlsSlots + (uint64_t)slot) * 2 * tileBytes;
}
TN_HD uint64_t nvlsOutAt(uint64_t tileBytes, int c, int slot) {
  return nvlsInAt(tileBytes, c, slot) + tileBytes;
}
TN_HD uint64_t nvlsDataBytes(uint64_t tileBytes, int channels) {
  return (uint64_t)channels * kNvlsSlots * 2 * tileBytes;
}
TN_HD uint64_t nvlsCounterAt(uint64_t tileBytes, int channels, int phase, int c, int slot) {
  return nvlsDataBytes(tileBytes, channels) +
         (((uint64_t)phase * kMaxChannels + c) * kNvlsSlots + slot) * 8;
}
// After those, the zero-copy kernel's barrier counters: one 64-bit word per
// phase ("entered", "stored") and channel, counted once per launch by every
// rank, so P x launches means every rank finished that phase of a launch.
TN_HD uint64_t nvlsZcCounterAt(uint64_t tileBytes, int channels, int phase, int c) {
  return nvlsDataBytes(tileBytes, channels) + 2ull * kMaxChannels * kNvlsSlots * 8 +
         ((uint64_t)phase * kMaxChannels + c) * 8;
}
TN_HD uint64_t nvlsRegionBytes(uint64_t tileBytes, int channels) {
  return nvlsDataBytes(tileBytes, channels) +
         alignUp(2ull * kMaxChannels * kNvlsSlots * 8 + 2ull * kMaxChannels * 8, 4096);
}

// ---------------------------------------------------------------------------
// Zero-copy NVLS (buffers registered with tncclCommRegister): the message is
// nv 16-byte vectors; rank r reduces its share blockShare(nv, P, r, 1), and
// channel c of C takes an even contiguous part of that share. C depends on
// the message size only, so it is the same on every rank, and every channel
// runs (possibly with nothing to reduce) so that the barrier counts agree.
// ---------------------------------------------------------------------------
TN_HD int nvlsZcChannels(uint64_t nv, int nranks, int maxChannels, uint64_t minVecsPerChannel) {
  const uint64_t perRank = divUp(nv, (uint64_t)nranks);
  const uint64_t want = divUp(perRank, minVecsPerChannel == 0 ? 1 : minVecsPerChannel);
  const uint64_t cap = maxChannels < 1 ? 1 : (uint64_t)maxChannels;
  return (int)(want < 1 ? 1 : minU64(want, cap));
}
TN_HD Span nvlsZcSpan(uint64_t nv, int nranks, int rank, int channels, int c) {
  const Span share = blockShare(nv, nranks, rank, 1);
  const uint64_t per = divUp(share.count, (uint64_t)channels);
  const uint64_t off = minU64((uint64_t)c * per, share.count);
  return Span{share.offset + off, minU64(per, share.count - off)};
}

// ---------------------------------------------------------------------------
// One ring edge's FIFO as the ring kernel and the socket proxy see it: per
// channel c and slot s (index c * slots + s) a payload of chunkBytes, a ready
// word (ticket + 1 once the payload of that ticket is written) and a credit
// word (the first ticket that may use the slot; slot s starts at s). For an
// NVLink edge the payload and ready words live in the consumer's mailbox and
// the credits in the producer's, so both ends poll local memory. For a socket
// edge all of them live in one host-mapped buffer per direction (layout:
// makeNetFifoLayout) that the rank's kernel shares with its proxy thread,
// plus a payload-size word per slot, since a frame carries exactly the bytes
// the kernel wrote.
// ---------------------------------------------------------------------------
struct RingFifo {
  char* data;
  uint64_t* ready;
  uint64_t* credit;
  uint64_t* bytes;  // payload bytes per slot (socket edges; null for NVLink)
  uint64_t chunkBytes;
  int slots;
};

TN_HD uint64_t ringFifoIndex(const RingFifo& f, int c, uint64_t ticket) {
  return (uint64_t)c * (uint64_t)f.slots + ticket % (uint64_t)f.slots;
}
TN_HD char* ringFifoData(const RingFifo& f, int c, uint64_t ticket) {
  return f.data + ringFifoIndex(f, c, ticket) * f.chunkBytes;
}

// The FIFO of the NVLink edge producer -> consumer, from the two mailboxes.
TN_HD RingFifo nvlinkRingFifo(char* consumer, char* producer, const MailboxLayout& L) {
  return RingFifo{consumer + L.ringDataOff,
                  reinterpret_cast<uint64_t*>(consumer + L.ringReadyOff),
                  reinterpret_cast<uint64_t*>(producer + L.ringCreditOff), nullptr,
                  L.ringChunkBytes, L.ringSlots};
}

struct NetFifoLayout {
  int channels;
  int slots;
  uint64_t chunkBytes;
  uint64_t readyOff, creditOff, bytesOff;
  uint64_t totalBytes;
};

TN_HD NetFifoLayout makeNetFifoLayout(int channels, int slots, uint64_t chunkBytes) {
  NetFifoLayout L{};
  const uint64_t n = (uint64_t)channels * (uint64_t)slots;
  L.channels = channels;
  L.slots = slots;
  L.chunkBytes = chunkBytes;
  L.readyOff = alignUp(n * chunkBytes, 128);
  L.creditOff = alignUp(L.readyOff + n * 8, 128);
  L.bytesOff = alignUp(L.creditOff + n * 8, 128);
  L.totalBytes = alignUp(L.bytesOff + n * 8, 4096);
  return L;
}

TN_HD RingFifo netRingFifo(char* base, const NetFifoLayout& L) {
  return RingFifo{base, reinterpret_cast<uint64_t*>(base + L.readyOff),
                  reinterpret_cast<uint64_t*>(base + L.creditOff),
                  reinterpret_cast<uint64_t*>(base + L.bytesOff), L.chunkBytes, L.slots};
}

// Socket frame: ticket (8 bytes) and payload bytes (4 bytes), big-endian,
// then the payload. The close frame (ticket kNetCloseTicket, no payload) ends
// a connection cleanly; a connection that ends without it is a failure.
constexpr uint32_t kNetFrameHeaderBytes = 12;
constexpr uint64_t kNetCloseTicket = ~0ull;

}  // namespace tnccl
