// ln_plan.h - launch geometry and shared-memory layout of the row-group
// LayerNorm backward (lnBwdGroupKernel, layernorm.cu). Plain C++ so that the
// CPU test (tests/cpp/ln_plan_test.cc) checks the very numbers the launcher
// uses.
//
// A group of G threads owns one row at a time; each thread owns K
// consecutive float4 column groups (4K columns). A CTA holds R groups and the
// grid has at most one CTA per SM. Dynamic shared memory:
//   [0, kLnRedFloats floats)   warp sums: [group][row parity][warp][2]
//   then R rings of kLnStages stages, one ring per group; a stage holds a
//   row's gy (8K bytes per thread), x_out and residual gradient (16K each):
//     gy [8K G] | x_out [16K G] | g_res [16K G]
// After the row loop the rings are reused for the per-group [dW | dB]
// accumulators (R * 2C floats).
#pragma once

#if defined(__CUDACC__)
#define TNOPS_HD __host__ __device__
#else
#define TNOPS_HD
#endif

namespace tnops {

constexpr int kLnMaxGroups = 15;            // R limit: named barriers 1..15
constexpr int kLnStages = 3;                // ring stages per group (2 rows ahead)
constexpr int kLnMaxWarpsPerGroup = 8;      // warp-sum slots per group and parity
constexpr int kLnRedFloats = 16 * 2 * kLnMaxWarpsPerGroup * 2;
constexpr int kLnRingBudget = 200 * 1024;   // stage-ring bytes per CTA

TNOPS_HD constexpr int lnStageBytes(int K, int G) { return 40 * K * G; }
TNOPS_HD constexpr int lnMaxThreads(int K) { return K == 1 ? 1024 : 768; }
// Largest dynamic shared memory any plan asks for (set once per device).
constexpr int kLnMaxSmemBytes = kLnRedFloats * 4 + kLnRingBudget;

struct LnGroupPlan {
  int K;           // float4 column groups per thread
  int G;           // threads per row group (a multiple of 32)
  int R;           // row groups per CTA
  int blocks;      // CTAs (= partial rows written)
  int smemBytes;   // dynamic shared memory per CTA
};

// K = 2 needs C % 8 == 0 (and 16-byte aligned bf16 rows, checked by the
// caller); C % 4 == 0, 0 < C <= 1024, rows > 0.
inline LnGroupPlan lnGroupPlan(int rows, int C, int K, int sms) {
  LnGroupPlan p{};
  p.K = K;
  p.G = 32 * ((C / (4 * K) + 31) / 32);
  p.R = lnMaxThreads(K) / p.G;
  if (p.R > kLnMaxGroups) p.R = kLnMaxGroups;
  const int ringR = kLnRingBudget / (kLnStages * lnStageBytes(K, p.G));
  if (p.R > ringR) p.R = ringR;
  p.blocks = (rows + p.R - 1) / p.R;
  if (p.blocks > sms) p.blocks = sms;
  p.smemBytes = kLnRedFloats * 4 + p.R * kLnStages * lnStageBytes(K, p.G);
  return p;
}

}  // namespace tnops
