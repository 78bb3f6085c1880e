// tnccl_ext.cpp - PyTorch binding of the collective library.
//
// Exposes a Communicator class over the C API of include/tnccl.h. Tensors are
// validated here (device, dtype, contiguity, shape); the collective is
// enqueued on the caller's current CUDA stream (the first call binds the
// communicator to that stream, as the C API requires).
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include <string>
#include <vector>

#include "diag.h"
#include "tnccl.h"

namespace py = pybind11;

namespace {

void check(tncclResult r, const char* what) {
  if (r != TNCCL_SUCCESS)
    throw std::runtime_error(std::string(what) + ": " + tncclGetErrorString(r) + " (" +
                             std::to_string((int)r) + ")");
}

tncclDataType_t toDtype(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat:
      return tncclFloat32;
    case at::kBFloat16:
      return tncclBfloat16;
    case at::kHalf:
      return tncclFloat16;
    default:
      throw std::invalid_argument("tnccl: dtype must be float32, bfloat16 or float16");
  }
}

tncclAlgo_t parseAlgo(const std::string& a) {
  if (a == "auto") return TNCCL_ALGO_AUTO;
  if (a == "ring") return TNCCL_ALGO_RING;
  if (a == "oneshot") return TNCCL_ALGO_ONESHOT;
  if (a == "twoshot") return TNCCL_ALGO_TWOSHOT;
  if (a == "nvls") return TNCCL_ALGO_NVLS;
  throw std::invalid_argument("tnccl: unknown algorithm '" + a + "'");
}

tncclRedOp_t parseOp(const std::string& op) {
  if (op == "sum") return tncclSum;
  if (op == "avg") return tncclAvg;
  throw std::invalid_argument("tnccl: op must be 'sum' or 'avg'");
}

class Communicator {
 public:
  Communicator(const py::bytes& id, int nranks, int rank) {
    std::string s = id;
    if (s.size() != sizeof(tncclUniqueId))
      throw std::invalid_argument("tnccl: unique id must be 128 bytes");
    tncclUniqueId uid;
    memcpy(uid.bytes, s.data(), sizeof(uid.bytes));
    tncclResult r;
    {
      py::gil_scoped_release nogil;  // blocking collective
      r = tncclCommInitRank(&comm_, nranks, uid, rank);
    }
    check(r, "tncclCommInitRank");
    check(tncclCommGetInfo(comm_, &info_), "tncclCommGetInfo");
  }

  at::Tensor allReduce(at::Tensor input, c10::optional<at::Tensor> output, const std::string& op,
                       double scale, const std::string& algo) {
    live();
    TORCH_CHECK(input.is_cuda(), "tnccl: input must be a CUDA tensor");
    TORCH_CHECK(input.get_device() == info_.device, "tnccl: input is on device ",
                input.get_device(), " but the communicator uses device ", info_.device);
    TORCH_CHECK(input.is_contiguous(), "tnccl: input must be contiguous");
    at::Tensor out = output.has_value() ? *output : input;
    TORCH_CHECK(out.is_cuda() && out.get_device() == info_.device && out.is_contiguous(),
                "tnccl: output must be a contiguous tensor on the communicator's device");
    TORCH_CHECK(out.scalar_type() == input.scalar_type() && out.numel() == input.numel(),
                "tnccl: output must match the input's dtype and size");
    c10::cuda::CUDAGuard guard(info_.device);
    cudaStream_t stream = c10::cuda::getCurrentCUDAStream(info_.device).stream();
    check(tncclAllReduceEx(input.data_ptr(), out.data_ptr(), (size_t)input.numel(),
                           toDtype(input), parseOp(op), (float)scale, parseAlgo(algo), comm_,
                           stream),
          "tncclAllReduceEx");
    return out;
  }

  // Raw-pointer variant for callers that manage their own buffers (bench
  // harness, CUDA-graph capture of preallocated buffers).
  void allReducePtr(uint64_t send, uint64_t recv, uint64_t count, int dtype, const std::string& op,
                    double scale, const std::string& algo, uint64_t stream) {
    live();
    c10::cuda::CUDAGuard guard(info_.device);
    check(tncclAllReduceEx(reinterpret_cast<const void*>(send), reinterpret_cast<void*>(recv),
                           (size_t)count, (tncclDataType_t)dtype, parseOp(op), (float)scale,
                           parseAlgo(algo), comm_, reinterpret_cast<cudaStream_t>(stream)),
          "tncclAllReduceEx");
  }

  std::string selectAlgo(int64_t numel, at::ScalarType st) {
    live();
    at::Tensor probe = at::empty({0}, at::TensorOptions().dtype(st));
    tncclAlgo_t a;
    check(tncclCommSelectAlgo(comm_, (size_t)numel, toDtype(probe), &a), "tncclCommSelectAlgo");
    return tncclAlgoName(a);
  }

  int validate() {
    live();
    int bad = 0;
    check(tncclCommValidate(comm_, &bad), "tncclCommValidate");
    return bad;
  }

  void diagCorruptCanary(int which) {
    live();
    check(tncclDiagCorruptCanary(comm_, which), "tncclDiagCorruptCanary");
  }

  void setMaxChannels(int n) {
    live();
    check(tncclCommSetMaxChannels(comm_, n), "tncclCommSetMaxChannels");
  }

  int asyncError() {
    live();
    tncclResult r;
    check(tncclCommGetAsyncError(comm_, &r), "tncclCommGetAsyncError");
    return (int)r;
  }

  void abort() {
    live();
    check(tncclCommAbort(comm_), "tncclCommAbort");
  }

  void destroy() {
    if (comm_ == nullptr) return;
    tncclComm_t c = comm_;
    comm_ = nullptr;
    tncclResult r;
    {
      py::gil_scoped_release nogil;
      r = tncclCommDestroy(c);
    }
    check(r, "tncclCommDestroy");
  }

  py::dict info() {
    if (comm_ != nullptr) check(tncclCommGetInfo(comm_, &info_), "tncclCommGetInfo");
    py::dict d;
    d["rank"] = info_.rank;
    d["nranks"] = info_.nranks;
    d["device"] = info_.device;
    d["channels"] = info_.channels;
    d["nvls"] = (bool)info_.nvlsEnabled;
    d["ipc"] = info_.ipcMode == 1 ? "cumem" : info_.ipcMode == 2 ? "cudaipc" : "none";
    d["mailbox_bytes"] = (uint64_t)info_.mailboxBytes;
    d["nvls_bytes"] = (uint64_t)info_.nvlsBytes;
    d["oneshot_max_bytes"] = (uint64_t)info_.sizeThresholds[0];
    d["nvls_min_bytes"] = (uint64_t)info_.sizeThresholds[1];
    d["socket_send_edge"] = (bool)info_.netSendSocket;
    d["socket_recv_edge"] = (bool)info_.netRecvSocket;
    d["socket_channels"] = info_.netChannels;
    d["registrations"] = info_.registrations;
    d["zero_copy_launches"] = (uint64_t)info_.zeroCopyLaunches;
    return d;
  }

  py::dict netStats() const {
    live();
    tncclNetStats st{};
    check(tncclCommGetNetStats(comm_, &st), "tncclCommGetNetStats");
    py::dict d;
    d["frames_sent"] = st.framesSent;
    d["frames_received"] = st.framesReceived;
    d["bytes_sent"] = st.bytesSent;
    d["bytes_received"] = st.bytesReceived;
    d["partial_writes"] = st.partialWrites;
    d["partial_reads"] = st.partialReads;
    d["credit_stalls"] = st.creditStalls;
    d["failed"] = st.failed;
    return d;
  }

  // Self test of the bounded device waits (see tncclDiagWaitTimeout).
  void diagWaitTimeout(int timeoutMs) {
    live();
    c10::cuda::CUDAGuard guard(info_.device);
    check(tncclDiagWaitTimeout(comm_, timeoutMs,
                               c10::cuda::getCurrentCUDAStream(info_.device).stream()),
          "tncclDiagWaitTimeout");
  }

  // Phase-trace records of one channel as a flat list [t0, tag0, t1, tag1, ...].
  std::vector<uint64_t> traceRead(int channel, int64_t maxRecords) {
    live();
    std::vector<unsigned long long> buf((size_t)maxRecords * 2);
    size_t n = 0;
    check(tncclCommTraceRead(comm_, channel, buf.data(), (size_t)maxRecords, &n),
          "tncclCommTraceRead");
    return std::vector<uint64_t>(buf.begin(), buf.begin() + 2 * n);
  }

  // Collective: binds a tensor that lies in tncclMemAlloc memory (memEmpty)
  // for the zero-copy NVLS all-reduce; returns the registration handle.
  uint64_t registerTensor(const at::Tensor& t) {
    live();
    TORCH_CHECK(t.is_cuda() && t.get_device() == info_.device && t.is_contiguous(),
                "tnccl: register needs a contiguous tensor on the communicator's device");
    c10::cuda::CUDAGuard guard(info_.device);
    void* h = nullptr;
    tncclResult r;
    {
      py::gil_scoped_release nogil;  // blocking collective
      r = tncclCommRegister(comm_, t.data_ptr(), (size_t)t.nbytes(), &h);
    }
    check(r, "tncclCommRegister");
    return reinterpret_cast<uint64_t>(h);
  }

  void deregister(uint64_t handle) {
    live();
    c10::cuda::CUDAGuard guard(info_.device);
    tncclResult r;
    {
      py::gil_scoped_release nogil;  // blocking collective
      r = tncclCommDeregister(comm_, reinterpret_cast<void*>(handle));
    }
    check(r, "tncclCommDeregister");
  }

  int rank() const { return info_.rank; }
  int size() const { return info_.nranks; }
  int device() const { return info_.device; }
  bool alive() const { return comm_ != nullptr; }

 private:
  void live() const {
    if (comm_ == nullptr) throw std::runtime_error("tnccl: communicator was destroyed");
  }
  tncclComm_t comm_ = nullptr;
  tncclCommInfo info_{};
};

// Single-GPU emulation of an n-rank communicator (tests and kernel profiles).
class Emulator {
 public:
  explicit Emulator(int nranks) { check(tncclEmuCreate(&emu_, nranks), "tncclEmuCreate"); }
  ~Emulator() {
    if (emu_) tncclEmuDestroy(emu_);
  }
  void allReduce(const std::vector<at::Tensor>& ins, const std::vector<at::Tensor>& outs,
                 const std::string& op, double scale, const std::string& algo) {
    TORCH_CHECK(emu_ != nullptr, "tnccl: emulator was destroyed");
    TORCH_CHECK(!ins.empty() && ins.size() == outs.size(), "tnccl: one input and output per rank");
    std::vector<const void*> s;
    std::vector<void*> r;
    for (size_t k = 0; k < ins.size(); ++k) {
      TORCH_CHECK(ins[k].is_cuda() && ins[k].is_contiguous() && outs[k].is_contiguous() &&
                      ins[k].numel() == ins[0].numel() && outs[k].numel() == ins[0].numel() &&
                      ins[k].scalar_type() == ins[0].scalar_type() &&
                      outs[k].scalar_type() == ins[0].scalar_type(),
                  "tnccl: emulated ranks need matching contiguous CUDA tensors");
      s.push_back(ins[k].data_ptr());
      r.push_back(outs[k].data_ptr());
    }
    cudaStream_t stream = c10::cuda::getCurrentCUDAStream(ins[0].get_device()).stream();
    check(tncclEmuAllReduce(emu_, s.data(), r.data(), (size_t)ins[0].numel(), toDtype(ins[0]),
                            parseOp(op), (float)scale, parseAlgo(algo), stream),
          "tncclEmuAllReduce");
  }
  int asyncError() {
    tncclResult e = TNCCL_SUCCESS;
    check(tncclEmuGetAsyncError(emu_, &e), "tncclEmuGetAsyncError");
    return (int)e;
  }
  void destroy() {
    if (emu_) check(tncclEmuDestroy(emu_), "tncclEmuDestroy");
    emu_ = nullptr;
  }

 private:
  tncclEmu_t emu_ = nullptr;
};

// nbytes of tncclMemAlloc memory on `device` as a uint8 tensor; the memory
// goes back through tncclMemFree when the last view of the tensor dies.
at::Tensor memEmpty(int64_t nbytes, int device) {
  TORCH_CHECK(nbytes > 0, "tnccl: mem_empty needs a positive size");
  c10::cuda::CUDAGuard guard(device);
  void* p = nullptr;
  check(tncclMemAlloc(&p, (size_t)nbytes), "tncclMemAlloc");
  return torch::from_blob(
      p, {nbytes}, [](void* q) { tncclMemFree(q); },
      at::TensorOptions().dtype(at::kByte).device(at::kCUDA, device));
}

py::bytes getUniqueId() {
  tncclUniqueId id;
  check(tncclGetUniqueId(&id), "tncclGetUniqueId");
  return py::bytes(reinterpret_cast<const char*>(id.bytes), sizeof(id.bytes));
}

py::bytes getUniqueIdTcp(const std::string& ipv4, int port) {
  tncclUniqueId id;
  check(tncclGetUniqueIdTcp(&id, ipv4.c_str(), port), "tncclGetUniqueIdTcp");
  return py::bytes(reinterpret_cast<const char*>(id.bytes), sizeof(id.bytes));
}

}  // namespace

void registerOps(py::module_& m);  // ops_ext.cpp

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "tnccl-b200 native binding";
  py::class_<Communicator>(m, "Communicator")
      .def(py::init<const py::bytes&, int, int>(), py::arg("unique_id"), py::arg("nranks"),
           py::arg("rank"))
      .def("all_reduce", &Communicator::allReduce, py::arg("input"),
           py::arg("output") = py::none(), py::arg("op") = "sum", py::arg("scale") = 1.0,
           py::arg("algo") = "auto")
      .def("all_reduce_ptr", &Communicator::allReducePtr, py::arg("send"), py::arg("recv"),
           py::arg("count"), py::arg("dtype"), py::arg("op") = "sum", py::arg("scale") = 1.0,
           py::arg("algo") = "auto", py::arg("stream") = 0)
      .def("select_algo", &Communicator::selectAlgo)
      .def("set_max_channels", &Communicator::setMaxChannels, py::arg("max_channels"))
      .def("validate", &Communicator::validate)
      .def("diag_corrupt_canary", &Communicator::diagCorruptCanary, py::arg("which"))
      .def("async_error", &Communicator::asyncError)
      .def("abort", &Communicator::abort)
      .def("destroy", &Communicator::destroy)
      .def("info", &Communicator::info)
      .def("net_stats", &Communicator::netStats)
      .def("diag_wait_timeout", &Communicator::diagWaitTimeout)
      .def("trace_read", &Communicator::traceRead)
      .def("register", &Communicator::registerTensor, py::arg("tensor"))
      .def("deregister", &Communicator::deregister, py::arg("handle"))
      .def_property_readonly("rank", &Communicator::rank)
      .def_property_readonly("size", &Communicator::size)
      .def_property_readonly("device", &Communicator::device)
      .def_property_readonly("alive", &Communicator::alive);
  py::class_<Emulator>(m, "Emulator")
      .def(py::init<int>(), py::arg("nranks"))
      .def("all_reduce", &Emulator::allReduce, py::arg("inputs"), py::arg("outputs"),
           py::arg("op") = "sum", py::arg("scale") = 1.0, py::arg("algo") = "twoshot")
      .def("async_error", &Emulator::asyncError)
      .def("destroy", &Emulator::destroy);
  m.def("get_unique_id", &getUniqueId);
  m.def("mem_empty", &memEmpty, py::arg("nbytes"), py::arg("device"));
  m.def("get_unique_id_tcp", &getUniqueIdTcp);
  m.def("launch_count", []() { return tncclGetLaunchCount(); });
  // 1 when the loaded collective library is the build with the device
  // protocol checks (lib/checked/libtnccl.so).
  m.def("device_checks", []() { return tncclDiagDeviceChecks(); });
  m.def("error_string", [](int r) { return std::string(tncclGetErrorString((tncclResult)r)); });
  m.def("version", []() {
    int v = 0;
    tncclGetVersion(&v);
    return v;
  });
  registerOps(m);
}
