// Python bindings of the native runtime (module weightbridge_b200._C).
// Device tables and buffers are passed as integer addresses (tensor.data_ptr()), streams as
// cudaStream_t handles (torch.cuda.Stream.cuda_stream).
#include <torch/extension.h>

#include <cuda_runtime.h>

#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "wb_board.h"
#include "wb_common.h"
#include "wb_cpu.h"
#include "wb_ipc.h"
#include "wb_splitq.h"
#include "wb_synth.h"
#include "wb_transfer.h"

namespace py = pybind11;

namespace {

template <typename T>
T* P(uint64_t a) {
  return reinterpret_cast<T*>(a);
}

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

void transfer(uint64_t items, uint32_t n_items, uint64_t bulk, uint32_t n_bulk, uint64_t qdescs, uint64_t qwork,
              uint32_t n_qwork, uint32_t piece_bytes, uint32_t spin_limit, uint64_t counter, uint64_t flags,
              uint32_t n_flags, uint64_t epoch, uint64_t status, int mode, int grid, uint64_t stream,
              uint64_t qmaps = 0, uint64_t qtma = 0) {
  if (mode == 0 && n_bulk) throw std::invalid_argument("bulk items need a TMA mode (1-3)");
  if ((qmaps != 0) != (qtma != 0)) throw std::invalid_argument("quant tensor maps need their validity bytes");
  if (qmaps % 64) throw std::invalid_argument("quant tensor maps must be 64-byte aligned");
  if (piece_bytes % 16) throw std::invalid_argument("piece_bytes must be a multiple of 16");
  wb::TransferArgs a{};
  a.items = P<const wb::Item>(items);
  a.n_items = n_items;
  a.bulk_items = P<const wb::Item>(bulk);
  a.n_bulk = n_bulk;
  a.qdescs = P<const wb::QuantDesc>(qdescs);
  a.qwork = P<const wb::QuantWork>(qwork);
  a.n_qwork = n_qwork;
  a.piece_bytes = piece_bytes;
  a.mbar_spin_limit = spin_limit;
  a.sig.counter = P<uint32_t>(counter);
  a.sig.flag_addrs = P<const uint64_t>(flags);
  a.sig.n_flags = n_flags;
  a.sig.epoch = P<const uint64_t>(epoch);
  a.sig.status = P<uint32_t>(status);
  a.qmaps = mode != 0 ? P<const uint8_t>(qmaps) : nullptr;      // the vector mode has no quant stages
  a.qtma = mode != 0 ? P<const uint8_t>(qtma) : nullptr;
  if (a.sig.counter && !a.sig.epoch) throw std::invalid_argument("a completion signal needs an epoch word");
  check(wb::launch_transfer(a, mode, grid, reinterpret_cast<cudaStream_t>(stream)), "transfer launch");
}

// One call per launch for the per-sync path: with `epoch` >= 0 write it into the pinned host word
// and copy it to the device epoch word on `stream`, then launch the kernel with the completion
// signal; with `epoch` < 0 launch without a signal.  `a` holds the program's fixed arguments:
// (items, n_items, bulk, n_bulk, qdescs, qwork, n_qwork, piece_bytes, spin_limit, counter,
//  flags, n_flags, epoch_dev, status, mode, grid, epoch_host, qmaps, qtma).
void transfer_launch(const py::tuple& a, int64_t epoch, uint64_t stream) {
  if (a.size() != 19) throw std::invalid_argument("transfer_launch: 19 fixed arguments expected");
  auto u = [&](size_t i) { return a[i].cast<uint64_t>(); };
  const bool sig = epoch >= 0;
  const auto st = reinterpret_cast<cudaStream_t>(stream);
  if (sig) {
    int64_t* host = reinterpret_cast<int64_t*>(u(16));
    *host = epoch;
    check(cudaMemcpyAsync(reinterpret_cast<void*>(u(12)), host, 8, cudaMemcpyHostToDevice, st), "epoch copy");
  }
  transfer(u(0), (uint32_t)u(1), u(2), (uint32_t)u(3), u(4), u(5), (uint32_t)u(6), (uint32_t)u(7), (uint32_t)u(8),
           sig ? u(9) : 0, u(10), sig ? (uint32_t)u(11) : 0, u(12), u(13), a[14].cast<int>(), a[15].cast<int>(), stream,
           u(17), u(18));
}

// Tensor maps of the quant descriptors (host arrays): returns how many qualified for the TMA path.
uint32_t encode_quant_maps(uint64_t descs, uint32_t n, uint64_t maps, uint64_t valid) {
  return wb::encode_quant_maps(P<const wb::QuantDesc>(descs), n, P<uint8_t>(maps), P<uint8_t>(valid));
}

// Synchronous read of `n` 8-byte words of device memory through a pinned host buffer.
py::list read_words(uint64_t dev, uint64_t host, int64_t n) {
  check(cudaMemcpy(reinterpret_cast<void*>(host), reinterpret_cast<const void*>(dev), 8 * (size_t)n,
                   cudaMemcpyDeviceToHost), "read_words");
  py::list out;
  const int64_t* h = reinterpret_cast<const int64_t*>(host);
  for (int64_t i = 0; i < n; ++i) out.append(h[i]);
  return out;
}

void wait_flags(uint64_t flags, uint32_t n, uint64_t epoch, uint64_t timeout_ns, uint64_t status, uint64_t where,
                uint64_t stream) {
  check(wb::launch_wait_flags(P<const uint64_t>(flags), n, P<const uint64_t>(epoch), timeout_ns, P<uint32_t>(status),
                              P<uint32_t>(where), reinterpret_cast<cudaStream_t>(stream)),
        "wait_flags launch");
}

void cpu_execute(uint64_t items, size_t n_items, uint64_t qdescs, uint64_t qwork, size_t n_qwork) {
  py::gil_scoped_release nogil;
  wb::cpu_execute(P<const wb::Item>(items), n_items, P<const wb::QuantDesc>(qdescs), P<const wb::QuantWork>(qwork),
                  n_qwork);
}

void split_amax(uint64_t pieces, uint32_t n, uint64_t partial, uint64_t stream) {
  check(wb::launch_split_amax(P<const wb::SplitPiece>(pieces), n, P<float>(partial),
                              reinterpret_cast<cudaStream_t>(stream)),
        "split_amax launch");
}

void split_quant(uint64_t pieces, uint32_t n, uint64_t amax, uint64_t stream) {
  check(wb::launch_split_quant(P<const wb::SplitPiece>(pieces), n, P<const float>(amax),
                               reinterpret_cast<cudaStream_t>(stream)),
        "split_quant launch");
}

void cpu_split_amax(uint64_t pieces, size_t n, uint64_t partial) {
  py::gil_scoped_release nogil;
  wb::cpu_split_amax(P<const wb::SplitPiece>(pieces), n, P<float>(partial));
}

void cpu_split_quant(uint64_t pieces, size_t n, uint64_t amax) {
  py::gil_scoped_release nogil;
  wb::cpu_split_quant(P<const wb::SplitPiece>(pieces), n, P<const float>(amax));
}

// Data pointers of a list of tensors (lists / tuples of tensors flattened in order) as one
// bytes object, 8 bytes each and 0 for anything else: the sender's cheap exact check that a
// state_dict still holds the tensors its plan was compiled for.
void append_ptrs(const py::handle& h, std::string& out, int depth) {
  uint64_t p = 0;
  if (THPVariable_Check(h.ptr())) {
    p = reinterpret_cast<uint64_t>(THPVariable_Unpack(h.ptr()).data_ptr());
  } else if (depth == 0 && (py::isinstance<py::list>(h) || py::isinstance<py::tuple>(h))) {
    for (const auto& e : py::reinterpret_borrow<py::sequence>(h)) append_ptrs(e, out, 1);
    p = ~uint64_t(0);  // end of a list
  }
  out.append(reinterpret_cast<const char*>(&p), 8);
}

// Fingerprint of a state_dict for the sender's per-sync check that it still holds the tensors
// its program was compiled for: the entry count, then per entry (in dict order) the name's
// hash and the data pointer(s) of its tensor or list of tensors.  One pass over the dict with
// PyDict_Next; str hashes are cached by Python, and the tensor type check is skipped while the
// type repeats.
py::bytes state_key(const py::dict& d) {
  std::string out;
  out.reserve(16 * static_cast<size_t>(PyDict_Size(d.ptr())) + 8);
  const uint64_t n = static_cast<uint64_t>(PyDict_Size(d.ptr()));
  out.append(reinterpret_cast<const char*>(&n), 8);
  PyObject *key = nullptr, *val = nullptr;
  Py_ssize_t pos = 0;
  PyTypeObject* tensor_type = nullptr;       // last type seen to be a tensor type
  auto ptr_of = [&](PyObject* o) -> uint64_t {
    if (Py_TYPE(o) != tensor_type) {
      if (!THPVariable_Check(o)) return 0;
      tensor_type = Py_TYPE(o);
    }
    return reinterpret_cast<uint64_t>(THPVariable_Unpack(o).data_ptr());
  };
  while (PyDict_Next(d.ptr(), &pos, &key, &val)) {
    const Py_hash_t kh = PyObject_Hash(key);
    if (kh == -1) throw py::error_already_set();
    out.append(reinterpret_cast<const char*>(&kh), 8);
    uint64_t p = 0;
    if (PyList_Check(val) || PyTuple_Check(val)) {
      const Py_ssize_t m = PySequence_Fast_GET_SIZE(val);
      PyObject** items = PySequence_Fast_ITEMS(val);
      for (Py_ssize_t i = 0; i < m; ++i) {
        const uint64_t q = ptr_of(items[i]);
        out.append(reinterpret_cast<const char*>(&q), 8);
      }
      p = ~uint64_t(0);  // end of a list
    } else {
      p = ptr_of(val);
    }
    out.append(reinterpret_cast<const char*>(&p), 8);
  }
  return py::bytes(out);
}

py::bytes data_ptrs(const py::list& tensors) {
  std::string out;
  out.reserve(tensors.size() * 8);
  for (const auto& h : tensors) append_ptrs(h, out, 0);
  return py::bytes(out);
}

void synth_fill(uint64_t dst, uint32_t dtype, uint64_t key, double std, const std::vector<int64_t>& ext,
                const std::vector<int64_t>& vstride, const std::vector<int64_t>& lo,
                const std::vector<int64_t>& lstride, uint64_t stream) {
  const size_t n = ext.size();
  if (n < 1 || n > (size_t)wb::kSynthMaxDims || vstride.size() != n || lo.size() != n || lstride.size() != n)
    throw std::invalid_argument("synth_fill: 1-8 dimensions with one extent, stride, start and logical stride each");
  if (!wb::synth_dtype_supported(dtype)) throw std::invalid_argument("synth_fill: dtype code not supported");
  wb::SynthDesc d{};
  d.dst = dst;
  d.ndim = (int32_t)n;
  d.dtype = dtype;
  d.key = key;
  d.std = std;
  for (size_t k = 0; k < n; ++k) {
    d.ext[k] = ext[k];
    d.vstride[k] = vstride[k];
    d.lo[k] = lo[k];
    d.lstride[k] = lstride[k];
  }
  check(wb::launch_synth_fill(d, reinterpret_cast<cudaStream_t>(stream)), "synth_fill launch");
}

int num_sms(int device) {
  int v = 0;
  check(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device), "cudaDeviceGetAttribute");
  return v;
}

py::tuple vmm_tuple(const wb::VmmAlloc& a) { return py::make_tuple(a.ptr, a.size, a.handle); }

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "weightbridge_b200 native runtime: sm_100a transfer kernel, CPU executor, IPC/VMM/multicast";
  m.def("transfer", &transfer, "launch the persistent transfer kernel", py::arg("items"), py::arg("n_items"),
        py::arg("bulk"), py::arg("n_bulk"), py::arg("qdescs"), py::arg("qwork"), py::arg("n_qwork"),
        py::arg("piece_bytes"), py::arg("spin_limit"), py::arg("counter"), py::arg("flags"), py::arg("n_flags"),
        py::arg("epoch"), py::arg("status"), py::arg("mode"), py::arg("grid"), py::arg("stream"),
        py::arg("qmaps") = 0, py::arg("qtma") = 0);
  m.def("encode_quant_maps", &encode_quant_maps, "tensor maps of the quant descriptors the TMA path can load");
  m.def("transfer_launch", &transfer_launch, "epoch copy and transfer launch of one program, in one call");
  m.def("read_words", &read_words, "synchronous read of device words through a pinned buffer");
  m.def("wait_flags", &wait_flags, "launch a bounded wait on flag words");
  m.def("bulk_stages", &wb::bulk_stages);
  m.def("cpu_execute", &cpu_execute, "run work tables on the host");
  m.def("split_amax", &split_amax, "launch the per-piece amax kernel of split fp8 blocks");
  m.def("split_quant", &split_quant, "launch the quantisation kernel of split fp8 blocks");
  m.def("cpu_split_amax", &cpu_split_amax, "per-piece amax of split fp8 blocks on the host");
  m.def("cpu_split_quant", &cpu_split_quant, "quantise split fp8 block pieces on the host");
  m.def("board_publish", &wb::board_publish, "store a handshake slot's fields, then its epoch (release)");
  m.def("board_wait", [](uint64_t base, const std::vector<int64_t>& offs, int64_t target, int64_t max_ns) {
          py::gil_scoped_release nogil;
          return wb::board_wait(base, offs, target, max_ns);
        }, "wait until every slot's epoch reaches target (bounded; the GIL is released)");
  m.def("board_read", &wb::board_read, "a handshake slot's epoch and fields");
  m.def("num_sms", &num_sms);
  m.def("synth_fill", &synth_fill, "fill a strided view with the synthetic weights");
  m.def("synth_dtype_supported", &wb::synth_dtype_supported);
  m.def("data_ptrs", &data_ptrs, "data pointers of a list of tensors, 8 bytes each");
  m.def("state_key", &state_key, "fingerprint of a state_dict: entry names' hashes and tensor data pointers");
  m.def("addr_range", [](uint64_t p) {
    auto r = wb::addr_range(p);
    return py::make_tuple(r.base, r.size);
  });
  m.def("ipc_handle", [](uint64_t base) { return py::bytes(wb::ipc_handle(base)); });
  m.def("ipc_open", [](py::bytes h) { return wb::ipc_open(std::string(h)); });
  m.def("ipc_close", &wb::ipc_close);
  m.def("device_uuid", [](int d) { return py::bytes(wb::device_uuid(d)); });
  m.def("can_access_peer", &wb::can_access_peer);
  m.def("enable_peer_access", &wb::enable_peer_access);
  m.def("vmm_granularity", &wb::vmm_granularity);
  m.def("vmm_alloc", [](size_t size, int dev) { return vmm_tuple(wb::vmm_alloc(size, dev)); });
  m.def("vmm_export_fd", &wb::vmm_export_fd);
  m.def("vmm_import_fd", [](int fd, size_t size, int dev) { return vmm_tuple(wb::vmm_import_fd(fd, size, dev)); });
  m.def("vmm_free", [](uint64_t ptr, uint64_t size, uint64_t handle) { wb::vmm_free(wb::VmmAlloc{ptr, size, handle}); });
  m.def("multicast_supported", &wb::multicast_supported);
  m.def("mc_create", &wb::mc_create);
  m.def("mc_import_fd", &wb::mc_import_fd);
  m.def("mc_add_device", &wb::mc_add_device);
  m.def("mc_bind_mem", &wb::mc_bind_mem);
  m.def("mc_unbind", &wb::mc_unbind);
  m.def("mc_map", [](uint64_t mc, size_t size, int dev) { return vmm_tuple(wb::mc_map(mc, size, dev)); });
  m.def("mem_release", &wb::mem_release);
  m.def("va_unmap", &wb::va_unmap);
  m.attr("ITEM_SIZE") = (int)sizeof(wb::Item);
  m.attr("QDESC_SIZE") = (int)sizeof(wb::QuantDesc);
  m.attr("QWORK_SIZE") = (int)sizeof(wb::QuantWork);
  m.attr("SPIECE_SIZE") = (int)sizeof(wb::SplitPiece);
  m.attr("ST_MBAR_TIMEOUT") = (int)wb::ST_MBAR_TIMEOUT;
  m.attr("ST_FLAG_TIMEOUT") = (int)wb::ST_FLAG_TIMEOUT;
  m.attr("ST_FLAG_STALE") = (int)wb::ST_FLAG_STALE;
  m.attr("ST_BAD_ITEM") = (int)wb::ST_BAD_ITEM;
  m.attr("ST_BAD_QUANT") = (int)wb::ST_BAD_QUANT;
}
