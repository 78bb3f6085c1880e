// gemm_tcgen05.cu - bf16 GEMM with a fused bias (+ tanh-GELU) epilogue on the
// 5th-generation tensor cores: tcgen05.mma with the fp32 accumulator in TMEM,
// operands staged by TMA (cp.async.bulk.tensor, 128-byte swizzle) through a
// 4-stage shared-memory ring.
//
//   pre = bf16(x w^T + bias)         x [M, K], w [N, K] (nn.Linear layout)
//   act = bf16(gelu_tanh(pre))       (GELU variant; gelu of the rounded pre,
//                                     as when pre is materialised first)
//
// One CTA computes one 128 x 256 output tile with three warp roles:
//   warp 0     one thread issues the TMA loads of each 64-wide K block (A:
//              128 x 64, B: 256 x 64) into the next free stage;
//   warp 1     allocates 256 TMEM columns, and one thread issues four
//              tcgen05.mma 128x256x16 per K block, then tcgen05.commit to the
//              stage's "empty" barrier (the stage is free once those MMAs have
//              read it) and, after the last block, to the accumulator barrier;
//   warps 2-9  wait for the accumulator, read it with tcgen05.ld (warp w owns
//              TMEM lanes 32 (w % 4) .. +31, i.e. those output rows; warps
//              2-5 take columns 0-127 of the tile, warps 6-9 columns
//              128-255), add the bias, apply GELU, round to bf16 and store.
//              Eight epilogue warps, two per SM sub-partition, keep the
//              epilogue of a tile shorter than the main loop of the next.
// Operands are K-major in shared memory, rows of 128 bytes in 8-row swizzle
// atoms of 1024 bytes: the UMMA descriptor holds the start address, a
// leading offset of 16 bytes and an 8-row stride of 1024 bytes, layout
// SWIZZLE_128B, version 1; successive K = 16 slices start 32 bytes further.
//
// Every mbarrier wait is bounded (globaltimer). On expiry the CTA records a
// code in gTcgen05Status, the other roles stop at their next wait, the
// producer waits (bounded) for the TMA loads it issued, the MMA thread
// commits and waits (bounded) for the MMAs it issued, and the TMEM columns
// are freed before the CTA returns. No load uses cluster multicast; the
// kernel reads this GPU's memory only.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "common.cuh"
#include "tnccl_ops.h"

namespace tnops {
namespace {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;  // bf16: 128 bytes, one swizzle row
constexpr int kStages = 4;
constexpr int kEpiWarps = 8;  // two per TMEM lane quarter
constexpr int kThreads = 64 + kEpiWarps * 32;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kStageA = kBM * kBK * 2;  // 16 KiB
constexpr uint32_t kStageB = kBN * kBK * 2;  // 32 KiB
// Epilogue staging: per epilogue warp a 32 x 32 bf16 block of pre and one of
// act (2 KiB each, 64-byte swizzle), written out by TMA tensor stores.
constexpr uint32_t kEpiBuf = 4096;
constexpr uint32_t kEpiBytes = kEpiWarps * kEpiBuf;
constexpr uint32_t kSmemBytes =
    kStages * (kStageA + kStageB) + kEpiBytes + 1024;  // + alignment slack
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s per wait

__device__ unsigned int gTcgen05Status;  // first failure code (0: none)

__device__ __forceinline__ uint32_t smemAddr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ uint64_t globalTimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbarInit(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smemAddr(bar)), "r"(count));
}
__device__ __forceinline__ void mbarExpectTx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smemAddr(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbarTryWait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smemAddr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits until the phase of `parity` completed. Gives up when *abort is set
// (unless ignoreAbort) or after kWaitNs; on a timeout records `code`.
__device__ __forceinline__ bool mbarWait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                         unsigned code, bool ignoreAbort = false) {
  if (mbarTryWait(bar, parity)) return true;
  const uint64_t t0 = globalTimer();
  for (uint32_t it = 1;; ++it) {
    if (mbarTryWait(bar, parity)) return true;
    if ((it & 63) == 0) {
      if (!ignoreAbort && *abort) return false;
      if (globalTimer() - t0 > kWaitNs) {
        atomicCAS(&gTcgen05Status, 0u, code);
        *abort = 1;
        return false;
      }
    }
  }
}
__device__ __forceinline__ void tmaLoad2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smemAddr(bar))
      : "memory");
}
__device__ __forceinline__ void fenceBeforeSync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fenceAfterSync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// K-major operand tile in shared memory, 128-byte swizzle (see the header).
__device__ __forceinline__ uint64_t smemDesc(uint32_t addr) {
  uint64_t d = (uint64_t)((addr & 0x3FFFFu) >> 4);  // start address, bits [0,14)
  d |= (uint64_t)1 << 16;                           // leading byte offset 16 B, bits [16,30)
  d |= (uint64_t)(1024 >> 4) << 32;                 // 8-row stride 1024 B, bits [32,46)
  d |= (uint64_t)1 << 46;                           // descriptor version 1, bits [46,48)
  d |= (uint64_t)2 << 61;                           // SWIZZLE_128B, bits [61,64)
  return d;
}
// Instruction descriptor of kind::f16: bf16 x bf16 -> f32, both K-major,
// M = 128, N = 256, dense.
__host__ __device__ constexpr uint32_t instrDesc() {
  return (1u << 4)                       // D format f32, bits [4,6)
         | (1u << 7)                     // A format bf16, bits [7,10)
         | (1u << 10)                    // B format bf16, bits [10,13)
         | ((uint32_t)(kBN >> 3) << 17)  // N >> 3, bits [17,23)
         | ((uint32_t)(kBM >> 4) << 24); // M >> 4, bits [24,29)
}
__device__ __forceinline__ void mma(uint32_t tmemD, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmemD),
      "l"(a), "l"(b), "r"(instrDesc()), "r"(accumulate)
      : "memory");
}
// Arrives on `bar` once every tcgen05.mma this thread issued before has completed.
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smemAddr(bar))
      : "memory");
}
__device__ __forceinline__ void tmemLoad32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// tanh-GELU, 0.5 x (1 + tanh(u)) with u = k0 (x + k1 x^3), evaluated in the
// equivalent form x / (1 + e^(-2u)) (1 + tanh(u) = 2 / (1 + e^(-2u))): no
// cancellation where tanh(u) is near -1, so the relative error stays near
// that of the hardware ex2 and the fast division (~1e-6), far below the bf16
// rounding of the result. Saturates correctly: x for large u, -0 for very
// negative u.
__device__ __forceinline__ float ex2Approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float geluTanh(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2 / pi)
  const float k0k1 = 0.7978845608028654f * 0.044715f;
  const float m2log2e = -2.0f * 1.4426950408889634f;
  // |u| <= 40 keeps e^(-2u) finite; gelu is x or -0 to float precision there.
  const float u = fminf(fmaxf(x * fmaf(k0k1, x * x, k0), -40.0f), 40.0f);
  return __fdividef(x, 1.0f + ex2Approx(u * m2log2e));
}
__device__ __forceinline__ uint32_t packBf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void tmaStore2d(const CUtensorMap* map, int x, int y, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(src)
               : "memory");
}
__device__ __forceinline__ void stShared16(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                           uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

// Epilogue of one warp's 32 x 32 block (lane = row row0 + lane, columns
// col0 .. +31, the fp32 accumulator values in v): bias (the same 32 values
// for every lane, four broadcast 16-byte loads), rounding to bf16, GELU of
// the rounded value; the bf16 rows go to this warp's staging buffers in the
// 64-byte swizzle (16-byte piece j of row r at piece j ^ ((r >> 1) & 3),
// which keeps the eight lanes of each store phase on distinct banks), and
// one lane writes each block with a TMA tensor store. The tensor maps clip
// rows and columns past M and N; a block that starts past them is skipped. A buffer is rewritten only after the
// previous store from it has been read.
template <bool GELU>
__device__ __forceinline__ void epilogueChunk(const float (&v)[32], int lane, int row0, int col0,
                                              int M, int N, const uint16_t* __restrict__ bias,
                                              const CUtensorMap* mapPre,
                                              const CUtensorMap* mapAct, uint32_t bufPre,
                                              uint32_t bufAct, bool hasPre) {
  uint4 bb[4] = {};
  if (bias) {
#pragma unroll
    for (int g = 0; g < 4; ++g)
      if (col0 + g * 8 < N) bb[g] = __ldg(reinterpret_cast<const uint4*>(bias + col0) + g);
  }
  uint32_t pw[16], aw[16];
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const uint32_t bw[4] = {bb[g].x, bb[g].y, bb[g].z, bb[g].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float x0 = v[g * 8 + 2 * i] + __uint_as_float(bw[i] << 16);
      const float x1 = v[g * 8 + 2 * i + 1] + __uint_as_float(bw[i] & 0xffff0000u);
      const uint32_t p = packBf16(x0, x1);
      pw[g * 4 + i] = p;
      if (GELU)
        aw[g * 4 + i] = packBf16(geluTanh(__uint_as_float(p << 16)),
                                 geluTanh(__uint_as_float(p & 0xffff0000u)));
    }
  }
  if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
  __syncwarp();
  const uint32_t rowOff = (uint32_t)lane * 64u, sw = ((uint32_t)lane >> 1) & 3u;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const uint32_t at = rowOff + 16u * ((uint32_t)g ^ sw);
    if (hasPre) stShared16(bufPre + at, pw[4 * g], pw[4 * g + 1], pw[4 * g + 2], pw[4 * g + 3]);
    if (GELU) stShared16(bufAct + at, aw[4 * g], aw[4 * g + 1], aw[4 * g + 2], aw[4 * g + 3]);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp();
  if (lane == 0 && row0 < M && col0 < N) {  // blocks wholly past the edge are not stored
    if (hasPre) tmaStore2d(mapPre, col0, row0, bufPre);
    if (GELU) tmaStore2d(mapAct, col0, row0, bufAct);
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  }
}
// Before a warp's staging buffers go away: its stores have completed.
__device__ __forceinline__ void epilogueDrain(int lane) {
  if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  __syncwarp();
}

template <bool GELU>
__global__ void __launch_bounds__(kThreads, 1)
    gemmBiasActKernel(const __grid_constant__ CUtensorMap mapA,
                      const __grid_constant__ CUtensorMap mapB,
                      const __grid_constant__ CUtensorMap mapPre,
                      const __grid_constant__ CUtensorMap mapAct,
                      const uint16_t* __restrict__ bias, int hasPre, int M, int N, int K) {
  __shared__ __align__(8) uint64_t sFull[kStages];
  __shared__ __align__(8) uint64_t sEmpty[kStages];
  __shared__ __align__(8) uint64_t sAccum;
  __shared__ uint32_t sTmem;
  __shared__ int sAbort;
  extern __shared__ uint8_t dsmem[];
  // Stage buffers start on a 1024-byte boundary (swizzle atoms).
  const uint32_t base = (smemAddr(dsmem) + 1023u) & ~1023u;
  const uint32_t stageA0 = base, stageB0 = base + kStages * kStageA;
  const uint32_t epi0 = base + kStages * (kStageA + kStageB);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kBN, m0 = blockIdx.y * kBM;
  const int kBlocks = (K + kBK - 1) / kBK;
  volatile int* abort = &sAbort;

  if (threadIdx.x == 0) {
    sAbort = 0;
    for (int s = 0; s < kStages; ++s) {
      mbarInit(&sFull[s], 1);
      mbarInit(&sEmpty[s], 1);
    }
    mbarInit(&sAccum, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smemAddr(&sTmem)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fenceBeforeSync();
  __syncthreads();
  fenceAfterSync();
  const uint32_t tmem = sTmem;

  if (warp == 0 && lane == 0) {
    // Producer.
    int issued = 0;
    for (int kb = 0; kb < kBlocks; ++kb) {
      const int s = kb % kStages;
      const uint32_t round = (uint32_t)(kb / kStages);
      // A fresh barrier counts as having completed the phase before its first.
      if (!mbarWait(&sEmpty[s], (round & 1u) ^ 1u, abort, 1)) break;
      mbarExpectTx(&sFull[s], kStageA + kStageB);
      tmaLoad2d(stageA0 + s * kStageA, &mapA, kb * kBK, m0, &sFull[s]);
      tmaLoad2d(stageB0 + s * kStageB, &mapB, kb * kBK, n0, &sFull[s]);
      issued = kb + 1;
    }
    if (*abort) {
      // No TMA write may land after the CTA is gone.
      for (int kb = issued > kStages ? issued - kStages : 0; kb < issued; ++kb)
        mbarWait(&sFull[kb % kStages], (uint32_t)(kb / kStages) & 1u, abort, 4, true);
    }
  } else if (warp == 1 && lane == 0) {
    // MMA issuer.
    for (int kb = 0; kb < kBlocks; ++kb) {
      const int s = kb % kStages;
      if (!mbarWait(&sFull[s], (uint32_t)(kb / kStages) & 1u, abort, 2)) break;
      fenceAfterSync();
      const uint32_t a = stageA0 + s * kStageA, b = stageB0 + s * kStageB;
#pragma unroll
      for (int k = 0; k < kBK / 16; ++k)
        mma(tmem, smemDesc(a + k * 32), smemDesc(b + k * 32), (kb | k) != 0 ? 1u : 0u);
      commit(&sEmpty[s]);
    }
    commit(&sAccum);  // also after an abort: the MMAs issued so far
    if (*abort) mbarWait(&sAccum, 0, abort, 5, true);
  } else if (warp >= 2) {
    // Epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 = tile rows, in
    // the column half (warp - 2) / 4.
    const int quarter = warp & 3;
    const int c0 = ((warp - 2) >> 2) * (kBN / 2);
    const uint32_t bufPre = epi0 + (uint32_t)(warp - 2) * kEpiBuf, bufAct = bufPre + kEpiBuf / 2;
    // tcgen05.ld is warp-collective: the whole warp proceeds only if every
    // lane saw the accumulator complete.
    const bool ready = mbarWait(&sAccum, 0, abort, 3);
    if (__all_sync(0xffffffffu, ready)) {
      fenceAfterSync();
#pragma unroll 1
      for (int c = c0; c < c0 + kBN / 2; c += 32) {
        float v[32];
        tmemLoad32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c, v);
        epilogueChunk<GELU>(v, lane, m0 + quarter * 32, n0 + c, M, N, bias, &mapPre, &mapAct,
                            bufPre, bufAct, hasPre != 0);
      }
    }
    epilogueDrain(lane);
  }
  fenceBeforeSync();
  __syncthreads();
  if (warp == 1) {
    fenceAfterSync();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

__device__ __forceinline__ void mbarArrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smemAddr(bar)) : "memory");
}

// Persistent variant: one CTA per SM walks the tiles t = blockIdx.x,
// blockIdx.x + gridDim.x, ... (row-tile major, so neighbouring CTAs share A).
// The producer's stage ring runs across tile boundaries, and the 512 TMEM
// columns hold two accumulators: the MMA issuer fills accumulator t % 2 while
// the epilogue drains the other. accFull[b] (MMA commit) and accEmpty[b] (one
// arrival per epilogue warp after its last tcgen05.ld of that buffer) hand
// the buffers back and forth; use u of buffer b waits for phase u of
// accFull[b] and, on the MMA side, for phase u - 1 of accEmpty[b].
template <bool GELU>
__global__ void __launch_bounds__(kThreads, 1)
    gemmBiasActPersistentKernel(const __grid_constant__ CUtensorMap mapA,
                                const __grid_constant__ CUtensorMap mapB,
                                const __grid_constant__ CUtensorMap mapPre,
                                const __grid_constant__ CUtensorMap mapAct,
                                const uint16_t* __restrict__ bias, int hasPre, int M, int N,
                                int K) {
  __shared__ __align__(8) uint64_t sFull[kStages];
  __shared__ __align__(8) uint64_t sEmpty[kStages];
  __shared__ __align__(8) uint64_t sAccFull[2];
  __shared__ __align__(8) uint64_t sAccEmpty[2];
  __shared__ __align__(8) uint64_t sDone;
  __shared__ uint32_t sTmem;
  __shared__ int sAbort;
  extern __shared__ uint8_t dsmem[];
  const uint32_t base = (smemAddr(dsmem) + 1023u) & ~1023u;
  const uint32_t stageA0 = base, stageB0 = base + kStages * kStageA;
  const uint32_t epi0 = base + kStages * (kStageA + kStageB);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tilesN = (N + kBN - 1) / kBN;
  const int tiles = tilesN * ((M + kBM - 1) / kBM);
  const int kBlocks = (K + kBK - 1) / kBK;
  volatile int* abort = &sAbort;

  if (threadIdx.x == 0) {
    sAbort = 0;
    for (int s = 0; s < kStages; ++s) {
      mbarInit(&sFull[s], 1);
      mbarInit(&sEmpty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbarInit(&sAccFull[b], 1);
      mbarInit(&sAccEmpty[b], kEpiWarps);  // one arrival per epilogue warp
    }
    mbarInit(&sDone, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smemAddr(&sTmem)),
                 "r"(2 * kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fenceBeforeSync();
  __syncthreads();
  fenceAfterSync();
  const uint32_t tmem = sTmem;

  if (warp == 0 && lane == 0) {
    // Producer: one stage sequence over all of this CTA's tiles.
    uint32_t g = 0;  // K blocks issued
    for (int t = blockIdx.x; t < tiles && !*abort; t += gridDim.x) {
      const int m0 = (t / tilesN) * kBM, n0 = (t % tilesN) * kBN;
      for (int kb = 0; kb < kBlocks; ++kb, ++g) {
        const uint32_t s = g % kStages, round = g / kStages;
        if (!mbarWait(&sEmpty[s], (round & 1u) ^ 1u, abort, 1)) break;
        mbarExpectTx(&sFull[s], kStageA + kStageB);
        tmaLoad2d(stageA0 + s * kStageA, &mapA, kb * kBK, m0, &sFull[s]);
        tmaLoad2d(stageB0 + s * kStageB, &mapB, kb * kBK, n0, &sFull[s]);
      }
    }
    if (*abort)
      for (uint32_t q = g > (uint32_t)kStages ? g - kStages : 0; q < g; ++q)
        mbarWait(&sFull[q % kStages], (q / kStages) & 1u, abort, 4, true);
  } else if (warp == 1 && lane == 0) {
    // MMA issuer.
    uint32_t g = 0, local = 0;
    for (int t = blockIdx.x; t < tiles && !*abort; t += gridDim.x, ++local) {
      const uint32_t b = local & 1u, use = local >> 1;
      if (!mbarWait(&sAccEmpty[b], (use & 1u) ^ 1u, abort, 2)) break;
      fenceAfterSync();
      const uint32_t acc = tmem + b * kTmemCols;
      bool ok = true;
      for (int kb = 0; kb < kBlocks; ++kb, ++g) {
        const uint32_t s = g % kStages;
        if (!(ok = mbarWait(&sFull[s], (g / kStages) & 1u, abort, 2))) break;
        fenceAfterSync();
        const uint32_t a = stageA0 + s * kStageA, bb = stageB0 + s * kStageB;
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k)
          mma(acc, smemDesc(a + k * 32), smemDesc(bb + k * 32), (kb | k) != 0 ? 1u : 0u);
        commit(&sEmpty[s]);
      }
      if (!ok) break;
      commit(&sAccFull[b]);
    }
    commit(&sDone);  // every MMA issued so far
    if (*abort) mbarWait(&sDone, 0, abort, 5, true);
  } else if (warp >= 2) {
    // Epilogue: TMEM lane quarter warp % 4, column half (warp - 2) / 4.
    const int quarter = warp & 3;
    const int c0 = ((warp - 2) >> 2) * (kBN / 2);
    const uint32_t bufPre = epi0 + (uint32_t)(warp - 2) * kEpiBuf, bufAct = bufPre + kEpiBuf / 2;
    uint32_t local = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++local) {
      const uint32_t b = local & 1u, use = local >> 1;
      const bool ready = mbarWait(&sAccFull[b], use & 1u, abort, 3);
      if (!__all_sync(0xffffffffu, ready)) break;
      fenceAfterSync();
      const int m0 = (t / tilesN) * kBM, n0 = (t % tilesN) * kBN;
      const uint32_t acc = tmem + b * kTmemCols + ((uint32_t)(quarter * 32) << 16);
#pragma unroll 1
      for (int c = c0; c < c0 + kBN / 2; c += 32) {
        float v[32];
        tmemLoad32(acc + (uint32_t)c, v);
        if (c + 32 == c0 + kBN / 2) {
          // Last read of this buffer: hand it back before the stores.
          fenceBeforeSync();
          __syncwarp();
          if (lane == 0) mbarArrive(&sAccEmpty[b]);
        }
        epilogueChunk<GELU>(v, lane, m0 + quarter * 32, n0 + c, M, N, bias, &mapPre, &mapAct,
                            bufPre, bufAct, hasPre != 0);
      }
    }
    epilogueDrain(lane);
  }
  fenceBeforeSync();
  __syncthreads();
  if (warp == 1) {
    fenceAfterSync();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(2 * kTmemCols)
                 : "memory");
  }
}

// ---------------------------------------------------------------------------
// CTA-pair variant (tcgen05 cta_group::2): a cluster of two CTAs on the two
// SMs of a TPC computes one 256 x 256 tile per step, persistent over the
// tiles. CTA r of the pair stages rows 128 r .. +127 of the tile's A block
// and of its B block (16 KiB each per 64-wide K block) in its own shared
// memory; the even CTA issues tcgen05.mma.cta_group::2 (M 256, N 256), which
// reads A and B from both CTAs at the same shared-memory offsets and writes
// the fp32 accumulator rows 128 r .. +127 into CTA r's TMEM. Per K block each
// SM loads 32 KiB from L2 for 128 x 256 x 64 of MMA, two thirds of the
// one-CTA tile's 48 KiB, and six stages fit in shared memory.
//
// Hand-offs (the even CTA's barriers unless noted):
//   full[s]      the even producer arms it for both CTAs' bytes (64 KiB);
//                both producers' TMA loads (cta_group::2 form, no multicast)
//                complete on it;
//   empty[s]     in each CTA, count 1: the MMA commit multicast to the pair;
//   accFull[b]   in each CTA: the commit after a tile's last K block;
//   accEmpty[b]  count 2 x 8: every epilogue warp of both CTAs arrives
//                (the odd CTA's remotely) after its last read of buffer b.
// Both CTAs meet at cluster barriers after set-up and before teardown, so
// neither leaves while the other can still reach its shared memory or TMEM.
// Every wait is bounded as in the other variants; on expiry the even CTA
// drains its loads and MMAs and the odd CTA, whose loads complete on the
// even CTA's barriers, gives its loads a bounded grace period before the
// final cluster barrier.
// ---------------------------------------------------------------------------
constexpr int kPairBM = 256;
constexpr int kPairStages = 6;
constexpr uint32_t kHalf = 128 * kBK * 2;  // 16 KiB: 128 rows x 64 K of bf16
constexpr uint32_t kPairSmemBytes = kPairStages * 2 * kHalf + kEpiBytes + 1024;

__device__ __forceinline__ uint32_t clusterRank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared variable in CTA 0 of the cluster.
__device__ __forceinline__ uint32_t inLeader(const void* p) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(d) : "r"(smemAddr(p)));
  return d;
}
__device__ __forceinline__ void clusterSync() {
  asm volatile("barrier.cluster.arrive.release;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ void tmaLoadPair(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t leaderBar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(leaderBar)
      : "memory");
}
__host__ __device__ constexpr uint32_t instrDescPair() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(256 >> 3) << 17) |
         ((uint32_t)(kPairBM >> 4) << 24);
}
__device__ __forceinline__ void mmaPair(uint32_t tmemD, uint64_t a, uint64_t b,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, "
      "{%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}" ::"r"(tmemD),
      "l"(a), "l"(b), "r"(instrDescPair()), "r"(accumulate), "r"(0u)
      : "memory");
}
// Arrives on `bar` in both CTAs of the pair once the pair MMAs issued so far
// have completed.
__device__ __forceinline__ void commitPair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;" ::"r"(smemAddr(bar)),
      "h"((uint16_t)3)
      : "memory");
}
__device__ __forceinline__ void commitPairLocal(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smemAddr(bar))
               : "memory");
}
__device__ __forceinline__ void mbarArriveRemote(uint32_t clusterAddr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(clusterAddr)
               : "memory");
}

template <bool GELU>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemmBiasActPairKernel(const __grid_constant__ CUtensorMap mapA,
                          const __grid_constant__ CUtensorMap mapB,
                          const __grid_constant__ CUtensorMap mapPre,
                          const __grid_constant__ CUtensorMap mapAct,
                          const uint16_t* __restrict__ bias, int hasPre, int M, int N, int K) {
  __shared__ __align__(8) uint64_t sFull[kPairStages];
  __shared__ __align__(8) uint64_t sEmpty[kPairStages];
  __shared__ __align__(8) uint64_t sAccFull[2];
  __shared__ __align__(8) uint64_t sAccEmpty[2];
  __shared__ __align__(8) uint64_t sDone;
  __shared__ uint32_t sTmem;
  __shared__ int sAbort;
  extern __shared__ uint8_t dsmem[];
  const uint32_t base = (smemAddr(dsmem) + 1023u) & ~1023u;
  const uint32_t stageA0 = base, stageB0 = base + kPairStages * kHalf;
  const uint32_t epi0 = base + kPairStages * 2 * kHalf;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = clusterRank();
  const int pair = (int)(blockIdx.x >> 1), pairs = (int)(gridDim.x >> 1);
  const int tilesN = (N + 255) / 256;
  const int tiles = tilesN * ((M + kPairBM - 1) / kPairBM);
  const int kBlocks = (K + kBK - 1) / kBK;
  volatile int* abort = &sAbort;

  if (threadIdx.x == 0) {
    sAbort = 0;
    for (int s = 0; s < kPairStages; ++s) {
      mbarInit(&sFull[s], 1);
      mbarInit(&sEmpty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbarInit(&sAccFull[b], 1);
      mbarInit(&sAccEmpty[b], 2 * kEpiWarps);
    }
    mbarInit(&sDone, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    // Both CTAs' warp 1, the same shared-memory destination in each.
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smemAddr(&sTmem)),
                 "r"(2 * kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  fenceBeforeSync();
  __syncthreads();
  clusterSync();  // barriers initialised and TMEM allocated in both CTAs
  fenceAfterSync();
  const uint32_t tmem = sTmem;

  if (warp == 0 && lane == 0) {
    // Producer (both CTAs): this CTA's halves of A and B.
    uint32_t g = 0;
    for (int t = pair; t < tiles && !*abort; t += pairs) {
      const int m0 = (t / tilesN) * kPairBM + (int)rank * 128;
      const int n0 = (t % tilesN) * 256 + (int)rank * 128;
      for (int kb = 0; kb < kBlocks; ++kb, ++g) {
        const uint32_t s = g % kPairStages, round = g / kPairStages;
        if (!mbarWait(&sEmpty[s], (round & 1u) ^ 1u, abort, 1)) break;
        if (rank == 0) mbarExpectTx(&sFull[s], 4 * kHalf);  // both CTAs' A and B halves
        const uint32_t bar = inLeader(&sFull[s]);
        tmaLoadPair(stageA0 + s * kHalf, &mapA, kb * kBK, m0, bar);
        tmaLoadPair(stageB0 + s * kHalf, &mapB, kb * kBK, n0, bar);
      }
    }
    if (*abort) {
      if (rank == 0) {
        for (uint32_t q = g > (uint32_t)kPairStages ? g - kPairStages : 0; q < g; ++q)
          mbarWait(&sFull[q % kPairStages], (q / kPairStages) & 1u, abort, 4, true);
      } else {
        // This CTA's loads complete on the even CTA's barriers: let them land.
        const uint64_t t0 = globalTimer();
        while (globalTimer() - t0 < 200000ull) {
        }
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // MMA issuer (even CTA only).
    uint32_t g = 0, local = 0;
    for (int t = pair; t < tiles && !*abort; t += pairs, ++local) {
      const uint32_t b = local & 1u, use = local >> 1;
      if (!mbarWait(&sAccEmpty[b], (use & 1u) ^ 1u, abort, 2)) break;
      fenceAfterSync();
      const uint32_t acc = tmem + b * kTmemCols;
      bool ok = true;
      for (int kb = 0; kb < kBlocks; ++kb, ++g) {
        const uint32_t s = g % kPairStages;
        if (!(ok = mbarWait(&sFull[s], (g / kPairStages) & 1u, abort, 2))) break;
        fenceAfterSync();
        const uint32_t a = stageA0 + s * kHalf, bb = stageB0 + s * kHalf;
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k)
          mmaPair(acc, smemDesc(a + k * 32), smemDesc(bb + k * 32), (kb | k) != 0 ? 1u : 0u);
        commitPair(&sEmpty[s]);
      }
      if (!ok) break;
      commitPair(&sAccFull[b]);
    }
    commitPairLocal(&sDone);
    if (*abort) mbarWait(&sDone, 0, abort, 5, true);
  } else if (warp >= 2) {
    // Epilogue (both CTAs): this CTA's 128 rows of the tile; TMEM lane
    // quarter warp % 4, column half (warp - 2) / 4.
    const int quarter = warp & 3;
    const int c0 = ((warp - 2) >> 2) * 128;
    const uint32_t bufPre = epi0 + (uint32_t)(warp - 2) * kEpiBuf, bufAct = bufPre + kEpiBuf / 2;
    uint32_t local = 0;
    for (int t = pair; t < tiles; t += pairs, ++local) {
      const uint32_t b = local & 1u, use = local >> 1;
      const bool ready = mbarWait(&sAccFull[b], use & 1u, abort, 3);
      if (!__all_sync(0xffffffffu, ready)) break;
      fenceAfterSync();
      const int m0 = (t / tilesN) * kPairBM + (int)rank * 128, n0 = (t % tilesN) * 256;
      const uint32_t acc = tmem + b * kTmemCols + ((uint32_t)(quarter * 32) << 16);
#pragma unroll 1
      for (int c = c0; c < c0 + 128; c += 32) {
        float v[32];
        tmemLoad32(acc + (uint32_t)c, v);
        if (c + 32 == c0 + 128) {
          fenceBeforeSync();
          __syncwarp();
          if (lane == 0) mbarArriveRemote(inLeader(&sAccEmpty[b]));
        }
        epilogueChunk<GELU>(v, lane, m0 + quarter * 32, n0 + c, M, N, bias, &mapPre, &mapAct,
                            bufPre, bufAct, hasPre != 0);
      }
    }
    epilogueDrain(lane);
  }
  fenceBeforeSync();
  __syncthreads();
  clusterSync();  // neither CTA leaves while the pair's MMAs or arrivals can reach it
  if (warp == 1) {
    fenceAfterSync();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(2 * kTmemCols)
                 : "memory");
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encodeTiled() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// [rows, K] row-major bf16, box {64, boxRows}, 128-byte swizzle, zero fill.
bool makeMap(CUtensorMap* map, const void* base, int rows, int K, int boxRows) {
  EncodeTiledFn fn = encodeTiled();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)boxRows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [rows, cols] row-major bf16 output, box {32, 32} (one epilogue warp's
// block), 64-byte swizzle, as the epilogue stages it.
bool makeOutMap(CUtensorMap* map, const void* base, int rows, int cols) {
  EncodeTiledFn fn = encodeTiled();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {32, 32};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Output maps of pre and act; a missing output gets a copy of the other
// map (never stored through: hasPre / GELU select the stores).
bool makeOutMaps(CUtensorMap* mapPre, CUtensorMap* mapAct, const void* pre, const void* act,
                 int M, int N) {
  if (pre && !makeOutMap(mapPre, pre, M, N)) return false;
  if (act && !makeOutMap(mapAct, act, M, N)) return false;
  if (!pre) *mapPre = *mapAct;
  if (!act) *mapAct = *mapPre;
  return true;
}

template <bool GELU, bool PERSISTENT>
int launchGemm(const void* x, const void* w, const void* bias, void* pre, void* act, int M, int N,
               int K, cudaStream_t stream) {
  auto kernel = PERSISTENT ? gemmBiasActPersistentKernel<GELU> : gemmBiasActKernel<GELU>;
  // Opt in to the shared memory once per device (bit d of `done`); the SM
  // count of that device sizes the persistent grid.
  static std::atomic<uint64_t> done{0};
  static int sms[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 3;
  const uint64_t bit = dev < 64 ? (1ull << dev) : 0;
  if (!(done.load(std::memory_order_acquire) & bit)) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSmemBytes) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms[dev & 63], cudaDevAttrMultiProcessorCount, dev) !=
            cudaSuccess)
      return 3;
    done.fetch_or(bit, std::memory_order_acq_rel);
  }
  CUtensorMap mapA, mapB, mapPre, mapAct;
  if (!makeMap(&mapA, x, M, K, kBM) || !makeMap(&mapB, w, N, K, kBN) ||
      !makeOutMaps(&mapPre, &mapAct, pre, act, M, N))
    return 4;
  const int tilesN = (N + kBN - 1) / kBN, tilesM = (M + kBM - 1) / kBM;
  dim3 grid((unsigned)tilesN, (unsigned)tilesM);
  if (PERSISTENT) {
    const int tiles = tilesN * tilesM, n = sms[dev & 63] > 0 ? sms[dev & 63] : 148;
    grid = dim3((unsigned)(tiles < n ? tiles : n));
  }
  kernel<<<grid, kThreads, kSmemBytes, stream>>>(mapA, mapB, mapPre, mapAct,
                                                 static_cast<const uint16_t*>(bias),
                                                 pre != nullptr ? 1 : 0, M, N, K);
  gLaunches.fetch_add(1, std::memory_order_relaxed);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

template <bool GELU>
int launchGemmPair(const void* x, const void* w, const void* bias, void* pre, void* act, int M,
                   int N, int K, cudaStream_t stream) {
  auto kernel = gemmBiasActPairKernel<GELU>;
  static std::atomic<uint64_t> done{0};
  static int sms[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 3;
  const uint64_t bit = dev < 64 ? (1ull << dev) : 0;
  if (!(done.load(std::memory_order_acquire) & bit)) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kPairSmemBytes) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms[dev & 63], cudaDevAttrMultiProcessorCount, dev) !=
            cudaSuccess)
      return 3;
    done.fetch_or(bit, std::memory_order_acq_rel);
  }
  // Each CTA of a pair loads 128 rows of A and 128 rows of B per K block.
  CUtensorMap mapA, mapB, mapPre, mapAct;
  if (!makeMap(&mapA, x, M, K, 128) || !makeMap(&mapB, w, N, K, 128) ||
      !makeOutMaps(&mapPre, &mapAct, pre, act, M, N))
    return 4;
  const int tiles = ((N + 255) / 256) * ((M + kPairBM - 1) / kPairBM);
  const int pairs = (sms[dev & 63] > 0 ? sms[dev & 63] : 148) / 2;
  const unsigned grid = 2u * (unsigned)(tiles < pairs ? tiles : pairs);
  kernel<<<grid, kThreads, kPairSmemBytes, stream>>>(mapA, mapB, mapPre, mapAct,
                                                     static_cast<const uint16_t*>(bias),
                                                     pre != nullptr ? 1 : 0, M, N, K);
  gLaunches.fetch_add(1, std::memory_order_relaxed);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace tnops

using namespace tnops;

// pre = bf16(x w^T + bias) and, with gelu, act = bf16(gelu_tanh(pre)); bias
// and pre may be null (not both outputs). `persistent` selects the kernel:
// 0 one 128 x 256 tile per CTA, 1 one CTA per SM walking the tiles with two
// TMEM accumulators, 2 CTA pairs (cta_group::2) walking 256 x 256 tiles. Requirements: K % 8 == 0
// (TMA row pitch), N % 8 == 0, 16-byte aligned x, w, pre, act. Returns 0 on
// launch.
extern "C" int tnops_gemm_bias_act(const void* x, const void* w, const void* bias, void* pre,
                                   void* act, int M, int N, int K, int gelu, int persistent,
                                   cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0 || K % 8 != 0 || N % 8 != 0 || !aligned16(x) ||
      !aligned16(w) || (pre && !aligned16(pre)) || (act && !aligned16(act)) ||
      (gelu && act == nullptr) || (!gelu && pre == nullptr))
    return 1;
  if (persistent == 2)
    return gelu ? launchGemmPair<true>(x, w, bias, pre, act, M, N, K, stream)
                : launchGemmPair<false>(x, w, bias, pre, act, M, N, K, stream);
  if (persistent)
    return gelu ? launchGemm<true, true>(x, w, bias, pre, act, M, N, K, stream)
                : launchGemm<false, true>(x, w, bias, pre, act, M, N, K, stream);
  return gelu ? launchGemm<true, false>(x, w, bias, pre, act, M, N, K, stream)
              : launchGemm<false, false>(x, w, bias, pre, act, M, N, K, stream);
}

// First failure code a tcgen05 GEMM recorded (1-3: a wait of the producer,
// MMA issuer or epilogue timed out; 4-5: a drain after that timed out), 0 if
// none; `reset` clears it. Synchronises the device.
extern "C" unsigned tnops_tcgen05_status(int reset) {
  unsigned v = 0;
  cudaMemcpyFromSymbol(&v, gTcgen05Status, sizeof(v));
  if (reset) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(gTcgen05Status, &z, sizeof(z));
  }
  return v;
}
