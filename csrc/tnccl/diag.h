// diag.h - diagnostic entry point (not part of the stable API).
#pragma once

#include <stddef.h>

#include "tnccl.h"

#ifdef __cplusplus
extern "C" {
#endif

// Times `iters` launches of one NVLink/HBM primitive (see diag.cu) on this
// rank and returns the mean milliseconds per launch. Every rank must call it
// with the same arguments at the same time. It overwrites the ring data area
// of the mailboxes, which holds no state between collectives.
tncclResult tncclDiagBench(tncclComm_t comm, int mode, size_t bytes, int ctas, int threads,
                           int unroll, size_t chunk, int iters, cudaStream_t stream,
                           float* msPerIter);

#ifdef __cplusplus
}
#endif
