// Exception-to-status translation shared by the extern "C" entry points:
// every entry runs its body through guarded(), which maps C++ exceptions to a
// cq_status and a thread-local message, the way catcher-ffi wraps its Rust
// calls (crates/catcher-ffi/src/lib.rs:703-722, :779-786).
#pragma once

#include <memory>
#include <new>
#include <string>
#include <vector>

#include "artifact.hpp"
#include "cqartifact.h"
#include "cqlinear.h"
#include "qlinear.hpp"

namespace nemotron_cuda {

inline std::string& last_error_slot() {
  thread_local std::string message;
  return message;
}

template <class F>
cq_status guarded(F&& f) {
  try {
    f();
    last_error_slot().clear();
    return CQ_OK;
  } catch (const Error& e) {
    last_error_slot() = e.what();
    return e.status();
  } catch (const std::bad_alloc&) {
    last_error_slot() = "host allocation failed";
    return CQ_RUNTIME_ERROR;
  } catch (const std::exception& e) {
    last_error_slot() = e.what();
    return CQ_RUNTIME_ERROR;
  } catch (...) {
    last_error_slot() = "unknown error";
    return CQ_RUNTIME_ERROR;
  }
}

inline void need_handle(const void* h, const char* what) {
  if (h == nullptr) throw_invalid(std::string(what) + " must not be null");
}

}  // namespace nemotron_cuda

// A layer handle: owns its layer, or borrows one that an encoder owns.
struct cq_linear {
  std::unique_ptr<nemotron_cuda::QuantizedLinear> owned;
  nemotron_cuda::QuantizedLinear* impl = nullptr;
  bool borrowed = false;
};

// An opened artifact and its manifest names (cq_artifact_tensor_name order).
struct cq_artifact {
  std::unique_ptr<nemotron_cuda::Artifact> impl;
  std::vector<std::string> names;
};
