// oracle.h - host reference for the all-reduce tests: seeded inputs, element
// type rounding, and order-aware sums that reproduce each algorithm's
// summation order bit for bit.
//
//   canonical (one-shot, two-shot): y = fl(...fl(fl(a*x0) + fl(a*x1)) ... )
//                                  in fp32, rounded once to T.
//   ring: chunk s is folded from rank s+1 around to rank s and every hop's
//         partial sum is rounded to T (it travels on the wire as T).
#pragma once

#include <stdint.h>
#include <string.h>

#include <vector>

#include "protocol.h"

namespace oracle {

enum Type { kF32 = 0, kBF16 = 1, kF16 = 2 };

inline size_t typeSize(int t) { return t == kF32 ? 4 : 2; }

inline uint64_t splitmix(uint64_t& s) {
  uint64_t z = (s += 0x9e3779b97f4a7c15ull);
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

// Uniform[-1, 1) with 24 random bits.
inline float uniform(uint64_t& s) {
  return (float)((splitmix(s) >> 40) * (1.0 / 16777216.0)) * 2.0f - 1.0f;
}

inline uint16_t f2bf(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
inline float bf2f(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
inline uint16_t f2h(float f) {
  _Float16 h = (_Float16)f;
  uint16_t u;
  memcpy(&u, &h, 2);
  return u;
}
inline float h2f(uint16_t u) {
  _Float16 h;
  memcpy(&h, &u, 2);
  return (float)h;
}

// Rounds an fp32 value to T and back.
inline float roundTo(int t, float f) {
  if (t == kBF16) return bf2f(f2bf(f));
  if (t == kF16) return h2f(f2h(f));
  return f;
}

// Fills raw bytes of T with rank r's seeded input (values representable in T).
inline void fillInput(int t, uint64_t seed, int rank, size_t n, std::vector<float>& vals,
                      std::vector<unsigned char>& raw) {
  uint64_t s = seed * 1000003ull + (uint64_t)rank;
  vals.resize(n);
  raw.resize(n * typeSize(t));
  for (size_t i = 0; i < n; ++i) {
    float v = roundTo(t, uniform(s));
    vals[i] = v;
    if (t == kF32) {
      memcpy(&raw[i * 4], &v, 4);
    } else {
      uint16_t u = t == kBF16 ? f2bf(v) : f2h(v);
      memcpy(&raw[i * 2], &u, 2);
    }
  }
}

inline float rawToFloat(int t, const unsigned char* p) {
  if (t == kF32) {
    float f;
    memcpy(&f, p, 4);
    return f;
  }
  uint16_t u;
  memcpy(&u, p, 2);
  return t == kBF16 ? bf2f(u) : h2f(u);
}

// Volatile-free fp32 arithmetic with one rounding per operation.
inline float mul(float a, float b) {
  volatile float r = a * b;
  return r;
}
inline float add(float a, float b) {
  volatile float r = a + b;
  return r;
}

inline void canonical(int t, const std::vector<std::vector<float>>& x, float alpha,
                      std::vector<float>& y) {
  const size_t n = x[0].size();
  y.resize(n);
  for (size_t i = 0; i < n; ++i) {
    float acc = mul(alpha, x[0][i]);
    for (size_t r = 1; r < x.size(); ++r) acc = add(acc, mul(alpha, x[r][i]));
    y[i] = roundTo(t, acc);
  }
}

// Chunk index of element e under a ring chunk plan.
inline int chunkOf(const tnccl::ChunkPlan& p, uint64_t e, uint64_t vecElems) {
  const uint64_t tile = e / p.tileElems;
  for (int j = 0; j < p.nranks; ++j) {
    tnccl::Span s = tnccl::chunkSpan(p, tile, j, vecElems);
    if (e >= s.offset && e < s.offset + s.count) return j;
  }
  return -1;
}

inline void ring(int t, const std::vector<std::vector<float>>& x, float alpha,
                 const tnccl::ChunkPlan& p, uint64_t vecElems, std::vector<float>& y) {
  const int P = (int)x.size();
  const size_t n = x[0].size();
  y.resize(n);
  for (size_t i = 0; i < n; ++i) {
    const int s = chunkOf(p, i, vecElems);
    int r = (s + 1) % P;
    float acc = roundTo(t, mul(alpha, x[(size_t)r][i]));
    for (int k = 2; k <= P; ++k) {
      r = (s + k) % P;
      acc = roundTo(t, add(acc, mul(alpha, x[(size_t)r][i])));
    }
    y[i] = acc;
  }
}

}  // namespace oracle
