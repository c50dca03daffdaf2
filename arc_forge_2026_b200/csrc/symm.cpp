// Symmetric device heap for the in-kernel collectives: every rank allocates one buffer of the same size, the
// ranks swap CUDA IPC handles (the host plumbing passes them through torch.distributed), and each rank maps every
// peer's buffer. Regions are carved at the same byte offsets on all ranks, so a kernel reaches "region R of rank p"
// as peer_base[p] + offset(R) and can load from or store to it directly over NVLink.
//
// This replaces the reference's pinned-host POSIX-shm region (hostcomm.py:200-320, hostcomm.cu:1-11): on an
// NVSwitch system the peers' HBM is one load/store away, so nothing is staged through host memory.
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

class SymmHeap {
 public:
  SymmHeap(int64_t bytes, int64_t rank, int64_t world, int64_t device)
      : bytes_(bytes), rank_((int)rank), world_((int)world), device_((int)device), peers_(world, 0) {
    if (bytes <= 0 || world < 1 || rank < 0 || rank >= world) throw std::invalid_argument("SymmHeap: bad sizes");
    check(cudaSetDevice(device_), "cudaSetDevice");
    check(cudaMalloc(&base_, (size_t)bytes_), "cudaMalloc(symmetric heap)");
    check(cudaMemset(base_, 0, (size_t)bytes_), "cudaMemset(symmetric heap)");
    check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    peers_[rank_] = (int64_t)(uintptr_t)base_;
  }

  ~SymmHeap() { close(); }

  // the IPC handle of this rank's buffer (opaque bytes; empty when there is only one rank)
  pybind11::bytes handle() const {
    if (world_ == 1) return pybind11::bytes("");
    cudaIpcMemHandle_t h;
    check(cudaSetDevice(device_), "cudaSetDevice");
    check(cudaIpcGetMemHandle(&h, base_), "cudaIpcGetMemHandle");
    return pybind11::bytes(reinterpret_cast<const char*>(&h), sizeof(h));
  }

  // map every peer's buffer from the handles of all ranks (in rank order)
  void open(const std::vector<std::string>& handles) {
    if ((int)handles.size() != world_) throw std::invalid_argument("SymmHeap.open: need one handle per rank");
    check(cudaSetDevice(device_), "cudaSetDevice");
    for (int p = 0; p < world_; ++p) {
      if (p == rank_ || peers_[p]) continue;
      if (handles[p].size() != sizeof(cudaIpcMemHandle_t)) throw std::invalid_argument("SymmHeap.open: bad handle");
      cudaIpcMemHandle_t h;
      std::memcpy(&h, handles[p].data(), sizeof(h));
      void* ptr = nullptr;
      check(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
      peers_[p] = (int64_t)(uintptr_t)ptr;
    }
  }

  void close() {
    if (!base_) return;
    cudaSetDevice(device_);
    cudaDeviceSynchronize();
    for (int p = 0; p < world_; ++p)
      if (p != rank_ && peers_[p]) cudaIpcCloseMemHandle(reinterpret_cast<void*>((uintptr_t)peers_[p]));
    cudaFree(base_);
    base_ = nullptr;
    std::fill(peers_.begin(), peers_.end(), 0);
  }

  int64_t base() const { return (int64_t)(uintptr_t)base_; }
  // this rank's buffer as a uint8 tensor (a view: the heap object must outlive it)
  at::Tensor tensor() const {
    if (!base_) throw std::runtime_error("SymmHeap: closed");
    return torch::from_blob(base_, {bytes_}, [](void*) {},
                            torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device_));
  }
  std::vector<int64_t> peers() const { return peers_; }
  int64_t bytes() const { return bytes_; }
  int64_t rank() const { return rank_; }
  int64_t world() const { return world_; }

 private:
  int64_t bytes_;
  int rank_, world_, device_;
  void* base_ = nullptr;
  std::vector<int64_t> peers_;
};

// Pinned, device-mapped host memory of an exact size (the torch pinned allocator rounds large blocks up to a power
// of two, which for a ~100 GB KV pool would double the host memory). Kernels read and write it through
// device_ptr(); the host sees it as a uint8 tensor.
class HostPool {
 public:
  explicit HostPool(int64_t bytes) : bytes_(bytes) {
    if (bytes <= 0) throw std::invalid_argument("HostPool: size must be positive");
    check(cudaHostAlloc(&host_, (size_t)bytes, cudaHostAllocMapped | cudaHostAllocPortable), "cudaHostAlloc");
    check(cudaHostGetDevicePointer(&dev_, host_, 0), "cudaHostGetDevicePointer");
  }
  ~HostPool() { close(); }
  void close() {
    if (host_) cudaFreeHost(host_);
    host_ = nullptr;
    dev_ = nullptr;
  }
  int64_t device_ptr() const { return (int64_t)(uintptr_t)dev_; }
  int64_t bytes() const { return bytes_; }
  at::Tensor tensor() const {
    if (!host_) throw std::runtime_error("HostPool: closed");
    return torch::from_blob(host_, {bytes_}, [](void*) {}, torch::TensorOptions().dtype(torch::kUInt8));
  }

 private:
  int64_t bytes_;
  void* host_ = nullptr;
  void* dev_ = nullptr;
};

}  // namespace

void register_symm(pybind11::module& m) {
  pybind11::class_<HostPool>(m, "HostPool")
      .def(pybind11::init<int64_t>(), pybind11::arg("bytes"))
      .def("device_ptr", &HostPool::device_ptr)
      .def("tensor", &HostPool::tensor)
      .def("close", &HostPool::close)
      .def_property_readonly("bytes", &HostPool::bytes);
  pybind11::class_<SymmHeap>(m, "SymmHeap")
      .def(pybind11::init<int64_t, int64_t, int64_t, int64_t>(), pybind11::arg("bytes"), pybind11::arg("rank"),
           pybind11::arg("world"), pybind11::arg("device"))
      .def("handle", &SymmHeap::handle)
      .def("open", &SymmHeap::open)
      .def("close", &SymmHeap::close)
      .def("base", &SymmHeap::base)
      .def("tensor", &SymmHeap::tensor)
      .def("peers", &SymmHeap::peers)
      .def_property_readonly("bytes", &SymmHeap::bytes)
      .def_property_readonly("rank", &SymmHeap::rank)
      .def_property_readonly("world", &SymmHeap::world);
}
