// api.cc - small public entry points: unique id, error strings, version,
// communicator queries, asynchronous error and abort. tncclGetErrorString
// returns the same strings for codes 0-4 as tiny-nccl src/api.cc:98-113;
// everything else here is new.
#include "comm.h"

using namespace tnccl;

extern "C" tncclResult tncclGetUniqueId(tncclUniqueId* id) { return bootstrapNewId(id); }

extern "C" tncclResult tncclGetUniqueIdTcp(tncclUniqueId* id, const char* ipv4, int port) {
  return bootstrapNewTcpId(id, ipv4, port);
}

extern "C" const char* tncclGetErrorString(tncclResult result) {
  switch (result) {
    case TNCCL_SUCCESS:
      return "success";
    case TNCCL_INVALID_ARGUMENT:
      return "invalid argument";
    case TNCCL_UNSUPPORTED:
      return "unsupported configuration";
    case TNCCL_SYSTEM_ERROR:
      return "system error";
    case TNCCL_CUDA_ERROR:
      return "CUDA error";
    case TNCCL_TIMEOUT:
      return "timed out waiting for a peer";
    case TNCCL_ABORTED:
      return "communicator aborted";
    default:
      return "unknown tnccl error";
  }
}

extern "C" const char* tncclAlgoName(tncclAlgo_t algo) {
  switch (algo) {
    case TNCCL_ALGO_AUTO:
      return "auto";
    case TNCCL_ALGO_RING:
      return "ring";
    case TNCCL_ALGO_ONESHOT:
      return "oneshot";
    case TNCCL_ALGO_TWOSHOT:
      return "twoshot";
    case TNCCL_ALGO_NVLS:
      return "nvls";
    default:
      return "unknown";
  }
}

extern "C" tncclResult tncclGetVersion(int* version) {
  if (version == nullptr) return TNCCL_INVALID_ARGUMENT;
  *version = TNCCL_VERSION_CODE;
  return TNCCL_SUCCESS;
}

extern "C" unsigned long long tncclGetLaunchCount(void) {
  return gLaunchCount.load(std::memory_order_relaxed);
}

extern "C" tncclResult tncclCommCount(tncclComm_t comm, int* nranks) {
  if (comm == nullptr || nranks == nullptr) return TNCCL_INVALID_ARGUMENT;
  *nranks = comm->nranks;
  return TNCCL_SUCCESS;
}

extern "C" tncclResult tncclCommUserRank(tncclComm_t comm, int* rank) {
  if (comm == nullptr || rank == nullptr) return TNCCL_INVALID_ARGUMENT;
  *rank = comm->rank;
  return TNCCL_SUCCESS;
}

extern "C" tncclResult tncclCommCuDevice(tncclComm_t comm, int* device) {
  if (comm == nullptr || device == nullptr) return TNCCL_INVALID_ARGUMENT;
  *device = comm->device;
  return TNCCL_SUCCESS;
}

extern "C" tncclResult tncclCommGetInfo(tncclComm_t comm, tncclCommInfo* info) {
  if (comm == nullptr || info == nullptr) return TNCCL_INVALID_ARGUMENT;
  *info = tncclCommInfo{};
  info->rank = comm->rank;
  info->nranks = comm->nranks;
  info->device = comm->device;
  info->channels = comm->cfg.channels;
  info->nvlsEnabled = comm->nvls.enabled ? 1 : 0;
  info->ipcMode = comm->ipcMode;
  info->mailboxBytes = comm->local.bytes;
  info->nvlsBytes = comm->nvls.enabled ? comm->nvls.bytes : 0;
  info->sizeThresholds[0] = comm->oneShotMaxBytes;
  info->sizeThresholds[1] = comm->nvlsMinBytes;
  info->ringChunkBytes = (size_t)comm->cfg.ringChunkBytes;
  info->ringMinChunkBytes = kRingMinChunkBytes;
  info->oneShotChannels = comm->cfg.osChannels;
  info->nvlsChannels = comm->nvls.enabled ? comm->nvls.channels : 0;
  info->netSendSocket = comm->net.send ? 1 : 0;
  info->netRecvSocket = comm->net.recv ? 1 : 0;
  info->netChannels = comm->net.any ? comm->net.layout.channels : 0;
  for (const Registration& g : comm->regs) info->registrations += g.used ? 1 : 0;
  info->zeroCopyLaunches = comm->zeroCopyLaunches;
  return TNCCL_SUCCESS;
}

extern "C" tncclResult tncclCommGetNetStats(tncclComm_t comm, tncclNetStats* stats) {
  if (comm == nullptr || stats == nullptr) return TNCCL_INVALID_ARGUMENT;
  *stats = tncclNetStats{};
  const NetProxy* p = comm->net.proxy;
  if (p == nullptr) return TNCCL_SUCCESS;
  stats->framesSent = p->framesSent.load();
  stats->framesReceived = p->framesReceived.load();
  stats->bytesSent = p->bytesSent.load();
  stats->bytesReceived = p->bytesReceived.load();
  stats->partialWrites = p->partialWrites.load();
  stats->partialReads = p->partialReads.load();
  stats->creditStalls = p->creditStalls.load();
  stats->failed = p->error.load();
  return TNCCL_SUCCESS;
}

extern "C" tncclResult tncclCommValidate(tncclComm_t comm, int* corrupted) {
  if (comm == nullptr || corrupted == nullptr) return TNCCL_INVALID_ARGUMENT;
  if (comm->streamBound && cudaStreamSynchronize(comm->boundStream) != cudaSuccess)
    return TNCCL_CUDA_ERROR;
  return countBadCanaries(comm, corrupted);
}

extern "C" tncclResult tncclCommSetMaxChannels(tncclComm_t comm, int maxChannels) {
  if (comm == nullptr || maxChannels < 0) return TNCCL_INVALID_ARGUMENT;
  comm->maxChannels = maxChannels;
  return TNCCL_SUCCESS;
}

extern "C" tncclResult tncclCommGetAsyncError(tncclComm_t comm, tncclResult* asyncError) {
  if (comm == nullptr || asyncError == nullptr) return TNCCL_INVALID_ARGUMENT;
  const int e = comm->hostStatus ? comm->hostStatus->error : 0;
  if (e == 0) {
    *asyncError = comm->aborted ? TNCCL_ABORTED : TNCCL_SUCCESS;
  } else {
    *asyncError = e > 0 && e < TNCCL_NUM_RESULTS ? (tncclResult)e : TNCCL_SYSTEM_ERROR;
  }
  return TNCCL_SUCCESS;
}

extern "C" tncclResult tncclCommAbort(tncclComm_t comm) {
  if (comm == nullptr) return TNCCL_INVALID_ARGUMENT;
  comm->aborted = true;
  if (comm->hostStatus) {
    comm->hostStatus->abort = 1;
    __sync_synchronize();
  }
  return TNCCL_SUCCESS;
}
