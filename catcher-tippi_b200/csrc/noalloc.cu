// Device scratch for callers that cannot allocate device memory.
//
// Who cannot allocate: a streaming transcriber that feeds the encoder from a
// real-time audio path (catcher_push_audio is called per captured block), and
// hosts that run under a fixed GPU memory budget fixed at start-up.  For them
// cudaMalloc in the middle of a stream is not acceptable: it can block for
// milliseconds, it synchronises with work already queued on the device, and it
// can fail under memory pressure long after the session has started.
//
// The one piece of scratch the quantized linear needs is the f16 copy of bf16
// activations (plus one scale per row) that the batched tensor-core path
// stages before its GEMM.  cq_linear_forward_noalloc takes that scratch from
// the file-scope array below instead of the layer's own workspace.  The array
// is part of the library's device image: every GPU that loads the library
// holds it until the process exits.
#include <cuda_runtime.h>

#include <mutex>
#include <vector>

#include "qlinear.hpp"

namespace {

// Maximum scratch: rows * input_dims * 2 bytes (f16 activations, rounded up to
// 256 bytes) + rows * 4 bytes (row scales) must fit, e.g. 896 rows at
// input_dims 4096 (64 streams x 14 frames through an FFN down projection).
constexpr size_t kNoAllocScratchBytes = 8u << 20;  // 8 MiB

// In host code this name is only a stand-in for the device symbol: its device
// address comes from cudaGetSymbolAddress below, per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
std::vector<void*> g_addr;  // device address of the array, per device

}  // namespace

namespace nemotron_cuda {

size_t noalloc_scratch_capacity() { return kNoAllocScratchBytes; }

// Device address of the scratch array on `device`.  Looked up once per device,
// with that device current, on the first no-allocation call there, which
// therefore must come before any stream capture: a first call on a capturing
// stream is rejected with a message that says so.  The cached address lives as
// long as the process's device context; like every handle of this library it
// does not survive a cudaDeviceReset.
void* noalloc_scratch_address(int device, cudaStream_t stream) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (device < 0) throw_invalid("invalid device " + std::to_string(device));
  if (g_addr.size() <= static_cast<size_t>(device)) g_addr.resize(device + 1, nullptr);
  if (g_addr[device] == nullptr) {
    DeviceGuard guard(device);
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    const cudaError_t qs = cudaStreamIsCapturing(stream, &capture);
    if (qs != cudaSuccess || capture != cudaStreamCaptureStatusNone) {
      if (qs != cudaSuccess) (void)cudaGetLastError();
      throw_invalid("the first no-allocation call on device " + std::to_string(device) +
                    " looks up its scratch address and must not run during stream capture;"
                    " make one call before capturing");
    }
    void* p = nullptr;
    check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch),
               "cudaGetSymbolAddress(no-allocation scratch)");
    g_addr[device] = p;
  }
  return g_addr[device];
}

}  // namespace nemotron_cuda
