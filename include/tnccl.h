/*
 * tnccl.h - public C API of tnccl-b200, a collective library for NVIDIA B200
 * (sm_100a) GPUs: NVLink 5 / NVSwitch within a node, TCP socket ring edges
 * between nodes.
 *
 * The first five entry points and the first five result codes keep the names,
 * values and semantics of tiny-nccl's include/tnccl.h:11-51. Everything after
 * them is appended (new result codes take new values; existing values never
 * change).
 *
 * Contract (same as tiny-nccl unless stated):
 *  - One process per GPU, one rank per process. Ranks on several hosts
 *    (TNCCL_BOOTSTRAP_ADDR for the rendezvous) are linked by socket ring edges
 *    (TNCCL_NET); such a communicator runs the ring algorithm only.
 *  - tncclCommInitRank and tncclCommDestroy are blocking collectives when
 *    nranks > 1: every rank calls them, in the same order.
 *  - The communicator captures the CUDA device that is current at init and is
 *    used from one host thread at a time.
 *  - The first collective binds the communicator to its stream; a collective
 *    on another stream returns TNCCL_UNSUPPORTED.
 *  - A collective returns once its work is enqueued; completion is observed
 *    through the stream.
 *  - All ranks issue the same collectives with the same count and datatype in
 *    the same order.
 *  - send/recv must be either the same pointer (in place) or fully disjoint.
 *  - Communication memory is a fixed set of mailbox slots sized at init; it
 *    does not grow with the tensor size. The bootstrap socket only carries
 *    control metadata, never tensor data.
 *
 * Differences from tiny-nccl:
 *  - Every device-side wait is bounded (TNCCL_TIMEOUT_MS, default 30000 ms).
 *    When a wait expires the kernel records TNCCL_TIMEOUT in host-mapped
 *    memory and returns instead of hanging; tncclCommGetAsyncError reports it
 *    and later collectives on that communicator fail fast.
 *  - tncclCommAbort makes in-flight device waits return promptly.
 *  - Collectives may be captured into CUDA graphs: FIFO sequence numbers live
 *    in device memory, so a replayed launch continues the sequence.
 */
#ifndef TNCCL_H_
#define TNCCL_H_

#include <stddef.h>

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TNCCL_VERSION_MAJOR 1
#define TNCCL_VERSION_MINOR 0
#define TNCCL_VERSION_PATCH 0
#define TNCCL_VERSION_CODE \
  (TNCCL_VERSION_MAJOR * 10000 + TNCCL_VERSION_MINOR * 100 + TNCCL_VERSION_PATCH)

typedef struct tncclComm* tncclComm_t;

typedef struct {
  unsigned char bytes[128];
} tncclUniqueId;

typedef enum {
  TNCCL_SUCCESS = 0,
  TNCCL_INVALID_ARGUMENT = 1,
  TNCCL_UNSUPPORTED = 2,
  TNCCL_SYSTEM_ERROR = 3,
  TNCCL_CUDA_ERROR = 4,
  /* appended */
  TNCCL_TIMEOUT = 5,  /* a bounded device wait expired (peer missing, count
                         mismatch, or another contract violation) */
  TNCCL_ABORTED = 6,  /* the communicator was aborted */
  TNCCL_NUM_RESULTS = 7
} tncclResult;

typedef enum {
  tncclFloat32 = 0,
  tncclBfloat16 = 1,
  tncclFloat16 = 2,
  tncclNumTypes = 3
} tncclDataType_t;

typedef enum {
  tncclSum = 0,
  tncclAvg = 1, /* sum with every input pre-scaled by 1/nranks */
  tncclNumOps = 2
} tncclRedOp_t;

typedef enum {
  TNCCL_ALGO_AUTO = 0,    /* pick by message size from the tuning table */
  TNCCL_ALGO_RING = 1,    /* multi-channel ring reduce-scatter + all-gather */
  TNCCL_ALGO_ONESHOT = 2, /* every rank pushes its data to every peer */
  TNCCL_ALGO_TWOSHOT = 3, /* all-peer reduce-scatter + all-gather */
  TNCCL_ALGO_NVLS = 4,    /* NVSwitch multimem reduce + multicast store */
  TNCCL_NUM_ALGOS = 5
} tncclAlgo_t;

/* ---- tiny-nccl surface ------------------------------------------------- */

tncclResult tncclGetUniqueId(tncclUniqueId* id);

/* Blocking collective initialization for nranks > 1. Every rank calls it
 * once with the same id and nranks, a unique rank, and its own CUDA device
 * current. Returns TNCCL_UNSUPPORTED if two ranks share a device or a peer
 * pair lacks P2P access or native peer atomics. */
tncclResult tncclCommInitRank(tncclComm_t* comm, int nranks, tncclUniqueId id,
                              int rank);

/* FP32 SUM all-reduce; same as tncclAllReduce(..., tncclFloat32, tncclSum). */
tncclResult tncclAllReduceSumF32(const float* send, float* recv, size_t count,
                                 tncclComm_t comm, cudaStream_t stream);

/* Blocking collective for nranks > 1. Synchronizes the bound stream, then
 * tears the IPC/NVLS mappings down in two barrier phases so that every
 * importer closes before any exporter frees. Always consumes comm, including
 * on error. If a safe teardown cannot be proven, device memory is retained
 * until the process exits. */
tncclResult tncclCommDestroy(tncclComm_t comm);

const char* tncclGetErrorString(tncclResult result);

/* ---- appended surface ---------------------------------------------------- */

/* General all-reduce. recv[i] = sum over ranks r of (scale * send_r[i]),
 * accumulated in fp32 and stored as dtype. scale is 1 for tncclSum and
 * 1/nranks for tncclAvg. */
tncclResult tncclAllReduce(const void* send, void* recv, size_t count,
                           tncclDataType_t dtype, tncclRedOp_t op,
                           tncclComm_t comm, cudaStream_t stream);

/* All-reduce with an explicit pre-scale (applied to every input before the
 * sum, fused into the kernel) and an explicit algorithm. algo must be the
 * same on every rank. op == tncclAvg multiplies preScale by 1/nranks. */
tncclResult tncclAllReduceEx(const void* send, void* recv, size_t count,
                             tncclDataType_t dtype, tncclRedOp_t op,
                             float preScale, tncclAlgo_t algo,
                             tncclComm_t comm, cudaStream_t stream);

typedef struct {
  int rank;
  int nranks;
  int device;
  int channels;             /* CTAs (channels) per all-peer/ring launch */
  int nvlsEnabled;          /* 1 if the NVLS path is mapped and usable */
  int ipcMode;              /* 0: single rank, 1: cuMem POSIX fd, 2: cudaIpc */
  size_t mailboxBytes;      /* unicast mailbox bytes per rank (constant) */
  size_t nvlsBytes;         /* multicast-bound bytes per rank (constant) */
  unsigned long long sizeThresholds[4]; /* AUTO switch points in bytes:
                                           [0] one-shot max, [1] NVLS min */
  size_t ringChunkBytes;    /* ring chunk capacity per FIFO slot */
  size_t ringMinChunkBytes; /* smallest ring chunk the planner uses */
  int oneShotChannels;
  int nvlsChannels;
  int netSendSocket;        /* 1: this rank's ring edge to rank + 1 is a socket edge */
  int netRecvSocket;        /* 1: its ring edge from rank - 1 is a socket edge */
  int netChannels;          /* ring channels when the communicator has socket edges */
  int registrations;        /* live tncclCommRegister registrations */
  unsigned long long zeroCopyLaunches; /* all-reduces that ran the zero-copy NVLS kernel */
} tncclCommInfo;

tncclResult tncclCommGetInfo(tncclComm_t comm, tncclCommInfo* info);

/* Traffic of this rank's socket ring edges (all zero without them). */
typedef struct {
  unsigned long long framesSent, framesReceived;
  unsigned long long bytesSent, bytesReceived;
  unsigned long long partialWrites, partialReads; /* frames that took several calls */
  unsigned long long creditStalls; /* received frames that waited for the kernel */
  int failed;                      /* tncclResult of the proxy's failure, 0 if none */
} tncclNetStats;
tncclResult tncclCommGetNetStats(tncclComm_t comm, tncclNetStats* stats);
tncclResult tncclCommCount(tncclComm_t comm, int* nranks);
tncclResult tncclCommUserRank(tncclComm_t comm, int* rank);
tncclResult tncclCommCuDevice(tncclComm_t comm, int* device);

/* Caps the CTAs (channels) of every later ring / two-shot / one-shot / NVLS
 * launch on this communicator at maxChannels (clamped to 1 .. the configured
 * count; 0 restores the configured count). A collective that overlaps with
 * compute (the DDP hook) leaves the other SMs to the compute kernels. Local
 * to the rank and stream-ordered like any launch parameter; ranks must use
 * the same cap for collectives on registered buffers (the zero-copy NVLS
 * kernel's grid follows it, and its barriers count every CTA of every rank). */
tncclResult tncclCommSetMaxChannels(tncclComm_t comm, int maxChannels);

/* Waits for the bound stream, then checks the guard lines placed after every
 * mailbox area of this rank (filled with a pattern at init). *corrupted is
 * the number of guard lines that were overwritten (0 = intact). Local. */
tncclResult tncclCommValidate(tncclComm_t comm, int* corrupted);

/* The algorithm TNCCL_ALGO_AUTO would use for this message. */
tncclResult tncclCommSelectAlgo(tncclComm_t comm, size_t count,
                                tncclDataType_t dtype, tncclAlgo_t* algo);

/* Reads the error recorded by device code (TNCCL_SUCCESS if none). Does not
 * synchronize; call after the stream has completed to see a final state. */
tncclResult tncclCommGetAsyncError(tncclComm_t comm, tncclResult* asyncError);

/* Sets the abort word that every device wait polls. In-flight waits return,
 * the communicator stops accepting collectives, and only tncclCommDestroy is
 * valid afterwards. Local only: it does not notify peers. */
tncclResult tncclCommAbort(tncclComm_t comm);

/* A unique id for a TCP rendezvous: rank 0 listens on ipv4:port (dotted
 * quad; the address must be rank 0's), the other ranks connect there. Needed
 * when ranks run on several hosts; tncclGetUniqueId does the same when
 * TNCCL_BOOTSTRAP_ADDR=<ipv4>:<port> is set. */
tncclResult tncclGetUniqueIdTcp(tncclUniqueId* id, const char* ipv4, int port);

/* ---- registered buffers (zero-copy NVLS) ---------------------------------
 * tncclMemAlloc returns device memory on the current device (a cuMem
 * allocation, rounded up to the multicast granularity) that can be bound to
 * an NVSwitch multicast object; cudaMalloc memory cannot. tncclMemFree
 * synchronizes the device first, like cudaFree, and refuses memory that is
 * still registered. */
tncclResult tncclMemAlloc(void** ptr, size_t size);
tncclResult tncclMemFree(void* ptr);

/* Collective: every rank calls it in the same order with a buffer of the
 * same size inside a tncclMemAlloc allocation (at its start, or at an offset
 * that is a multiple of the multicast granularity). It binds the buffer to a
 * multicast object of its own on every rank. An NVLS all-reduce whose send
 * and recv both lie in registered buffers, at the same offsets on every
 * rank, 16-byte aligned and a multiple of 16 bytes long, then reduces
 * straight from the senders' buffers and stores into every receiver's, with
 * no copy through the communicator's own region (TNCCL_NVLS_ZERO_COPY=0
 * turns that off; AUTO takes it from TNCCL_NVLS_ZC_MIN_BYTES, 16 MiB on 8
 * ranks). TNCCL_UNSUPPORTED when the communicator has no NVLS. */
tncclResult tncclCommRegister(tncclComm_t comm, void* buff, size_t size, void** handle);
/* Collective: waits for the bound stream, then unbinds on every rank
 * (two barriers, as tncclCommDestroy). tncclCommDestroy deregisters what is
 * left. */
tncclResult tncclCommDeregister(tncclComm_t comm, void* handle);

const char* tncclAlgoName(tncclAlgo_t algo);
tncclResult tncclGetVersion(int* version);

/* Number of kernels this library has launched in this process. */
unsigned long long tncclGetLaunchCount(void);

#ifdef __cplusplus
}
#endif

#endif /* TNCCL_H_ */
