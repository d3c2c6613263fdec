// Owning device allocation (cudaMalloc / cudaFree), movable, not copyable.
#pragma once

#include <stddef.h>

namespace nemotron_cuda {

class DeviceBuffer {
 public:
  DeviceBuffer() = default;
  explicit DeviceBuffer(size_t bytes);
  ~DeviceBuffer();
  DeviceBuffer(DeviceBuffer&& o) noexcept;
  DeviceBuffer& operator=(DeviceBuffer&& o) noexcept;
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
  void* get() const { return p_; }
  template <class T>
  T* as() const {
    return static_cast<T*>(p_);
  }
  size_t bytes() const { return n_; }

 private:
  void* p_ = nullptr;
  size_t n_ = 0;
};

}  // namespace nemotron_cuda
