// ferrum_gpu._native — the Python boundary, mirroring the reference's PyO3
// module (crates/ferrum-gpu-py/src/lib.rs:389-604) on top of the C ABI in
// include/ferrum_fft.h:
//   version()
//   cuda.Device(ordinal=0) with .sync()
//   fft.fft_1d_c2c_pow2(arr, log_n, direction="forward", normalize=False, device=None)
//   fft.fft_2d_c2c_pow2(arr, log_n, direction="forward", normalize=False, device=None)
// Validation order and ValueError messages follow lib.rs:455-477 and
// :537-558; the accepted ranges are wider (1D log_n up to 26, 2D log_n 2..14
// and batched (B, N, N) images). The GIL is released for all GPU work, as in
// lib.rs:490-497, and the call returns when the result is in host memory.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>

#include <complex>
#include <mutex>
#include <sstream>
#include <string>

#include "../../include/ferrum_fft.h"

namespace py = pybind11;

namespace {

class Device {
 public:
  explicit Device(int ordinal) : ordinal_(ordinal) {
    ferrum_status s = ferrum_device_create(ordinal, &handle_);
    if (s != FERRUM_OK) {
      std::ostringstream os;
      os << "CudaContext::new(" << ordinal << "): " << ferrum_last_error();
      throw py::value_error(os.str());
    }
  }
  ~Device() {
    if (handle_) ferrum_device_destroy(handle_);
  }
  Device(const Device&) = delete;
  Device& operator=(const Device&) = delete;

  void sync() {
    ferrum_status s;
    {
      py::gil_scoped_release release;
      s = ferrum_device_sync(handle_);
    }
    if (s != FERRUM_OK) throw py::value_error(std::string("sync: ") + ferrum_last_error());
  }
  ferrum_device* handle() const { return handle_; }
  int ordinal() const { return ordinal_; }
  // Address of the C handle, for callers that bind the C ABI directly.
  uintptr_t handle_address() const { return reinterpret_cast<uintptr_t>(handle_); }

 private:
  int ordinal_ = 0;
  ferrum_device* handle_ = nullptr;
};

// device=None: the reference builds a transient context and module per call
// (lib.rs:252-264, about 200 ms). Here one handle per process is created on
// first use and reused; results are identical. The handle is never
// destroyed: a static destructor would run after the CUDA runtime has shut
// down at process exit, and the driver reclaims the device memory anyway.
Device& default_device() {
  static std::once_flag once;
  static Device* dev = nullptr;
  static std::string* error = new std::string();
  std::call_once(once, [] {
    try {
      dev = new Device(0);
    } catch (const std::exception& e) {
      *error = e.what();
    }
  });
  if (!dev) throw py::value_error(*error);
  return *dev;
}

int parse_direction(const std::string& direction) {
  if (direction == "forward") return FERRUM_FORWARD;
  if (direction == "inverse") return FERRUM_INVERSE;
  // Rust's {:?} formatting of the offending &str (lib.rs:473-475).
  throw py::value_error("direction must be 'forward' or 'inverse', got \"" + direction + "\"");
}

void require_complex64(const py::array& arr) {
  if (!arr.dtype().is(py::dtype::of<std::complex<float>>()))
    throw py::type_error("argument 'arr': expected a numpy.ndarray of dtype complex64, got " +
                         std::string(py::str(arr.dtype())));
}

using CArr = py::array_t<std::complex<float>, py::array::c_style>;

py::array fft_1d(py::array arr, unsigned log_n, const std::string& direction, bool normalize,
                 py::object device) {
  if (log_n < FERRUM_MIN_LOG_N || log_n > FERRUM_MAX_LOG_N_1D)
    throw py::value_error("log_n must be in [2, 26], got " + std::to_string(log_n));
  require_complex64(arr);
  if (arr.ndim() != 1)
    throw py::type_error("argument 'arr': expected a 1-D array, got " +
                         std::to_string(arr.ndim()) + " dimensions");
  const size_t n = size_t(1) << log_n;
  CArr in = CArr::ensure(arr);
  const size_t total = (size_t)in.size();
  if (total == 0 || total % n != 0) {
    std::ostringstream os;
    os << "arr len " << total << " must be a positive multiple of N = " << n;
    throw py::value_error(os.str());
  }
  const size_t batch = total / n;
  const int dir = parse_direction(direction);
  Device& dev = device.is_none() ? default_device() : device.cast<Device&>();
  CArr out((py::ssize_t)total);
  const void* ip = in.data();
  void* op = out.mutable_data();
  ferrum_status s;
  {
    py::gil_scoped_release release;
    s = ferrum_fft_1d_c2c_pow2_host(dev.handle(), ip, op, (int)log_n, batch, dir, normalize ? 1 : 0);
  }
  if (s != FERRUM_OK) throw py::value_error(std::string("ferrum-gpu fft error: ") + ferrum_last_error());
  return out;
}

py::array fft_2d(py::array arr, unsigned log_n, const std::string& direction, bool normalize,
                 py::object device) {
  if (log_n < FERRUM_MIN_LOG_N || log_n > FERRUM_MAX_LOG_N_2D)
    throw py::value_error("2D requires log_n in [2, 14]; got " + std::to_string(log_n));
  require_complex64(arr);
  const py::ssize_t n = py::ssize_t(1) << log_n;
  const bool shape_ok = (arr.ndim() == 2 && arr.shape(0) == n && arr.shape(1) == n) ||
                        (arr.ndim() == 3 && arr.shape(0) > 0 && arr.shape(1) == n && arr.shape(2) == n);
  if (!shape_ok) {
    // Rust Debug formatting of the shape slice (lib.rs:544-548).
    std::ostringstream os;
    os << "arr shape [";
    for (py::ssize_t i = 0; i < arr.ndim(); ++i) os << (i ? ", " : "") << arr.shape(i);
    os << "] != (" << n << ", " << n << ")";
    throw py::value_error(os.str());
  }
  const int dir = parse_direction(direction);
  Device& dev = device.is_none() ? default_device() : device.cast<Device&>();
  CArr in = CArr::ensure(arr);
  const size_t batch = arr.ndim() == 3 ? (size_t)arr.shape(0) : 1;
  std::vector<py::ssize_t> shape(arr.shape(), arr.shape() + arr.ndim());
  CArr out(shape);
  const void* ip = in.data();
  void* op = out.mutable_data();
  ferrum_status s;
  {
    py::gil_scoped_release release;
    s = ferrum_fft_2d_c2c_pow2_host(dev.handle(), ip, op, (int)log_n, batch, dir, normalize ? 1 : 0);
  }
  if (s != FERRUM_OK)
    throw py::value_error(std::string("ferrum-gpu fft 2d error: ") + ferrum_last_error());
  return out;
}

}  // namespace

PYBIND11_MODULE(_native, m) {
  m.doc() = "ferrum-gpu B200 FFT path (sm_100a kernels behind the C ABI in ferrum_fft.h)";
  m.def("version", [] { return std::string(ferrum_version()); }, "Returns the library version.");

  py::module_ cuda = m.def_submodule("cuda", "CUDA device handles");
  py::class_<Device>(cuda, "Device", py::module_local(false))
      .def(py::init<int>(), py::arg("ordinal") = 0,
           "Open a CUDA device and upload the twiddle tables once.")
      .def("sync", &Device::sync, "Wait for all work on the device.")
      .def_property_readonly("ordinal", &Device::ordinal)
      .def_property_readonly("handle_address", &Device::handle_address,
                             "Address of the ferrum_device* C handle.");

  py::module_ fft = m.def_submodule("fft", "Power-of-two complex-to-complex FFTs");
  fft.def("fft_1d_c2c_pow2", &fft_1d, py::arg("arr"), py::arg("log_n"),
          py::arg("direction") = "forward", py::arg("normalize") = false,
          py::arg("device") = py::none(),
          "Batched 1D C2C FFT of a complex64 array of length batch * 2**log_n.");
  fft.def("fft_2d_c2c_pow2", &fft_2d, py::arg("arr"), py::arg("log_n"),
          py::arg("direction") = "forward", py::arg("normalize") = false,
          py::arg("device") = py::none(),
          "2D C2C FFT of a complex64 (N, N) or (B, N, N) array, N = 2**log_n.");
}
