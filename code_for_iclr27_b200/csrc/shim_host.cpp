// lazy_recall._host, backed by liblrk: page-locking of the recall transport's
// shared-memory DMA slots (csrc/host.cpp:5-18 of the reference).
#include <pybind11/pybind11.h>

#include <cstdint>
#include <stdexcept>
#include <string>

#include "lrk.h"

namespace {

void register_host(uint64_t address, uint64_t bytes) {
  if (lrk_register_host(reinterpret_cast<void *>(address), static_cast<size_t>(bytes)) != LRK_OK)
    throw std::runtime_error(lrk_last_error());
}

void unregister_host(uint64_t address) {
  if (lrk_unregister_host(reinterpret_cast<void *>(address)) != LRK_OK) throw std::runtime_error(lrk_last_error());
}

// Device address of registered host memory (for reading it from kernels).
uint64_t device_pointer(uint64_t address) {
  void *device = nullptr;
  if (lrk_host_device_pointer(reinterpret_cast<void *>(address), &device) != LRK_OK)
    throw std::runtime_error(lrk_last_error());
  return reinterpret_cast<uint64_t>(device);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, module) {
  module.def("register_host", &register_host);
  module.def("unregister_host", &unregister_host);
  module.def("device_pointer", &device_pointer);
}
