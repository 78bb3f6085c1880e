// diag.h - diagnostic entry point (not part of the stable API).
#pragma once

#include <stddef.h>

#include "tnccl.h"

#ifdef __cplusplus
extern "C" {
#endif

// Launches one kernel that waits, bounded by timeoutMs, on a device word that
// is never written. After the stream completes, tncclCommGetAsyncError
// reports TNCCL_TIMEOUT and the communicator refuses further collectives.
tncclResult tncclDiagWaitTimeout(tncclComm_t comm, int timeoutMs, cudaStream_t stream);

// 1 if this build of the library has the kernels' debug protocol checks
// compiled in (TNCCL_DEVICE_CHECKS=1), 0 otherwise.
int tncclDiagDeviceChecks(void);

// Overwrites guard line `which` (0 .. 4) of this rank's mailbox from the host
// (cudaMemset), so a test can check that tncclCommValidate notices.
tncclResult tncclDiagCorruptCanary(tncclComm_t comm, int which);

#ifdef __cplusplus
}
#endif

#ifdef __cplusplus
extern "C" {
#endif

// Copies the phase-trace records (TNCCL_TRACE=1) of channel `channel` into
// out (pairs of {globaltimer ns, tag}, oldest first, at most maxRecords) and
// stores their number in *n. Synchronizes the device first.
tncclResult tncclCommTraceRead(tncclComm_t comm, int channel, unsigned long long* out,
                               size_t maxRecords, size_t* n);

#ifdef __cplusplus
}
#endif

#ifdef __cplusplus
extern "C" {
#endif

// Single-GPU emulation of an nranks communicator (emulate.cc): all ranks'
// mailboxes in the current device's memory, all ranks' channels in one
// cooperative launch. For tests and profiles of ring / one-shot / two-shot.
typedef struct tncclEmu* tncclEmu_t;
tncclResult tncclEmuCreate(tncclEmu_t* emu, int nranks);
tncclResult tncclEmuAllReduce(tncclEmu_t emu, const void* const* send, void* const* recv,
                              size_t count, tncclDataType_t dtype, tncclRedOp_t op,
                              float preScale, tncclAlgo_t algo, cudaStream_t stream);
tncclResult tncclEmuGetAsyncError(tncclEmu_t emu, tncclResult* asyncError);
tncclResult tncclEmuDestroy(tncclEmu_t emu);

#ifdef __cplusplus
}
#endif
