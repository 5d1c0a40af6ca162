// Generic kernel-module substrate behind the C ABI: zeroed device buffers,
// synchronous copies, loading a compiled module (PTX text or a cubin /
// fatbin image), kernel lookup by name and launch on a stream. The
// reference's backend contract offers the same operations
// (crates/ferrum-gpu-core/src/backend.rs:12-77: alloc_zeros, copy_h2d,
// copy_d2h, load_module, get_kernel, launch, default_stream, sync_stream);
// its vector-add examples run on them. Built on the CUDA runtime's library
// API (cudaLibraryLoadData / cudaLibraryGetKernel), so no driver-API link is
// needed.
#include <cuda_runtime.h>

#include <string>

#include "runtime.h"

struct ferrum_module {
  ferrum_device* dev = nullptr;
  cudaLibrary_t lib = nullptr;
};

using namespace ferrum;

namespace {

ferrum_status require_device(const ferrum_device* dev, const char* what) {
  if (dev == nullptr || dev->tables == nullptr)
    return set_error(FERRUM_ERR_INVALID_ARG, std::string(what) + ": device handle is NULL or destroyed");
  return FERRUM_OK;
}

}  // namespace

extern "C" {

ferrum_status ferrum_buffer_alloc_zeros(ferrum_device* dev, size_t bytes, void** out) {
  clear_error();
  if (ferrum_status s = require_device(dev, "buffer_alloc_zeros")) return s;
  if (out == nullptr || bytes == 0)
    return set_error(FERRUM_ERR_INVALID_ARG, "buffer_alloc_zeros: out is NULL or bytes is 0");
  *out = nullptr;
  DeviceGuard guard(dev->ordinal);
  if (guard.status() != cudaSuccess) return cuda_error(guard.status(), "cudaSetDevice");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return cuda_error(e, "buffer_alloc_zeros: cudaMalloc");
  }
  e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_error(e, "buffer_alloc_zeros: cudaMemset");
  }
  *out = p;
  return FERRUM_OK;
}

ferrum_status ferrum_buffer_free(ferrum_device* dev, void* buf) {
  clear_error();
  if (ferrum_status s = require_device(dev, "buffer_free")) return s;
  if (buf == nullptr) return FERRUM_OK;
  DeviceGuard guard(dev->ordinal);
  cudaError_t e = cudaFree(buf);
  return e == cudaSuccess ? FERRUM_OK : cuda_error(e, "buffer_free");
}

ferrum_status ferrum_copy_h2d(ferrum_device* dev, void* dst_dev, const void* src_host, size_t bytes) {
  clear_error();
  if (ferrum_status s = require_device(dev, "copy_h2d")) return s;
  if ((dst_dev == nullptr || src_host == nullptr) && bytes > 0)
    return set_error(FERRUM_ERR_INVALID_ARG, "copy_h2d: NULL pointer");
  DeviceGuard guard(dev->ordinal);
  cudaError_t e = cudaMemcpy(dst_dev, src_host, bytes, cudaMemcpyHostToDevice);
  return e == cudaSuccess ? FERRUM_OK : cuda_error(e, "copy_h2d");
}

ferrum_status ferrum_copy_d2h(ferrum_device* dev, void* dst_host, const void* src_dev, size_t bytes) {
  clear_error();
  if (ferrum_status s = require_device(dev, "copy_d2h")) return s;
  if ((dst_host == nullptr || src_dev == nullptr) && bytes > 0)
    return set_error(FERRUM_ERR_INVALID_ARG, "copy_d2h: NULL pointer");
  DeviceGuard guard(dev->ordinal);
  cudaError_t e = cudaMemcpy(dst_host, src_dev, bytes, cudaMemcpyDeviceToHost);
  return e == cudaSuccess ? FERRUM_OK : cuda_error(e, "copy_d2h");
}

ferrum_status ferrum_module_load(ferrum_device* dev, const void* image, ferrum_module** out) {
  clear_error();
  if (ferrum_status s = require_device(dev, "module_load")) return s;
  if (image == nullptr || out == nullptr)
    return set_error(FERRUM_ERR_INVALID_ARG, "module_load: image or out is NULL");
  *out = nullptr;
  DeviceGuard guard(dev->ordinal);
  if (guard.status() != cudaSuccess) return cuda_error(guard.status(), "cudaSetDevice");
  cudaLibrary_t lib = nullptr;
  cudaError_t e = cudaLibraryLoadData(&lib, image, nullptr, nullptr, 0, nullptr, nullptr, 0);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();  // reported here; not left for a later call to find
    return cuda_error(e, "module_load: cudaLibraryLoadData");
  }
  auto* m = new ferrum_module();
  m->dev = dev;
  m->lib = lib;
  *out = m;
  return FERRUM_OK;
}

ferrum_status ferrum_module_unload(ferrum_module* module) {
  clear_error();
  if (module == nullptr) return FERRUM_OK;
  DeviceGuard guard(module->dev->ordinal);
  cudaError_t e = cudaLibraryUnload(module->lib);
  delete module;
  return e == cudaSuccess ? FERRUM_OK : cuda_error(e, "module_unload");
}

ferrum_status ferrum_module_kernel(ferrum_module* module, const char* name, void** kernel_out) {
  clear_error();
  if (module == nullptr || name == nullptr || kernel_out == nullptr)
    return set_error(FERRUM_ERR_INVALID_ARG, "module_kernel: NULL argument");
  *kernel_out = nullptr;
  DeviceGuard guard(module->dev->ordinal);
  cudaKernel_t k = nullptr;
  cudaError_t e = cudaLibraryGetKernel(&k, module->lib, name);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();  // reported here; not left for a later call to find
    return cuda_error(e, (std::string("module_kernel: no kernel named ") + name).c_str());
  }
  *kernel_out = reinterpret_cast<void*>(k);
  return FERRUM_OK;
}

ferrum_status ferrum_launch(ferrum_device* dev, void* kernel, const unsigned grid[3],
                            const unsigned block[3], unsigned shared_bytes, void** args,
                            void* stream) {
  clear_error();
  if (ferrum_status s = require_device(dev, "launch")) return s;
  if (kernel == nullptr || grid == nullptr || block == nullptr)
    return set_error(FERRUM_ERR_INVALID_ARG, "launch: NULL kernel, grid or block");
  for (int i = 0; i < 3; ++i)
    if (grid[i] == 0 || block[i] == 0)
      return set_error(FERRUM_ERR_INVALID_ARG, "launch: grid and block dimensions must be >= 1");
  DeviceGuard guard(dev->ordinal);
  if (guard.status() != cudaSuccess) return cuda_error(guard.status(), "cudaSetDevice");
  (void)cudaGetLastError();  // an earlier unrelated error is not this launch's
  cudaError_t e = cudaLaunchKernel(reinterpret_cast<const void*>(kernel),
                                   dim3(grid[0], grid[1], grid[2]),
                                   dim3(block[0], block[1], block[2]), args, shared_bytes,
                                   (cudaStream_t)stream);
  return e == cudaSuccess ? FERRUM_OK : cuda_error(e, "launch");
}

ferrum_status ferrum_stream_sync(ferrum_device* dev, void* stream) {
  clear_error();
  if (ferrum_status s = require_device(dev, "stream_sync")) return s;
  DeviceGuard guard(dev->ordinal);
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  return e == cudaSuccess ? FERRUM_OK : cuda_error(e, "stream_sync");
}

}  // extern "C"
