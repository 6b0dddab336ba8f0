// Relay cell pass without any allocation: the variant of mb_cell_pass for
// callers that cannot allocate device memory themselves or through us.
//
// Who needs it: hosts that embed the evaluator inside a runtime owning every
// device allocation (a Rust or C++ engine that hands the library only the
// buffers it manages, a process running under a fixed device-memory budget,
// code that must not call into the CUDA allocator at all). mb_cell_pass asks
// the caller for an (n_cov x h) fp32 scratch buffer; this entry point uses a
// fixed array compiled into the library instead, so the caller passes only
// its inputs and outputs.
//
// The scratch is one file-scope __device__ array of kScratchFloats floats
// (16 MiB). Every GPU that loads the library holds it until the process
// exits. Its device address is looked up with cudaGetSymbolAddress on the
// device the call runs on (that device current): the first call on a device
// does it, and so does every later call whose stream is not being captured,
// so the address stays right after a device reset reloads the module. A call
// inside a stream capture reuses the last address looked up on that device;
// make the first call on each device before any stream capture.
//
// All calls share the one array and it keeps the previous call's contents.
// Nothing here needs it cleared: the cell kernel writes every row
// [0, n_cov) before the window reduction reads it. Calls that overlap on the
// GPU (different streams, or different host threads on one device) race on
// the array; serialise them.
#include <mutex>

#include "common.cuh"

namespace mb {
namespace noalloc {

constexpr int64_t kScratchFloats = int64_t(4) * 1024 * 1024;  // 16 MiB
__device__ __align__(256) float g_relay_scratch[kScratchFloats];

constexpr int kMaxDevices = 64;
float* g_scratch_of_device[kMaxDevices] = {};
std::mutex g_scratch_mutex;

// The device address of the scratch array on the current device (looked up
// again unless `stream` is being captured).
int scratch_address(float** out, cudaStream_t stream) {
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return fail(MB_LAUNCH_FAILED, "cell_pass_noalloc: cudaGetDevice: %s", cudaGetErrorString(err));
  if (dev < 0 || dev >= kMaxDevices) return fail(MB_UNSUPPORTED, "cell_pass_noalloc: device %d out of range", dev);
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &capture) != cudaSuccess) capture = cudaStreamCaptureStatusActive;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_of_device[dev] == nullptr || capture == cudaStreamCaptureStatusNone) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_relay_scratch);
    if (err != cudaSuccess || p == nullptr) {
      if (g_scratch_of_device[dev] == nullptr)
        return fail(MB_LAUNCH_FAILED, "cell_pass_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(err));
      p = g_scratch_of_device[dev];
    }
    g_scratch_of_device[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_of_device[dev];
  return MB_OK;
}

}  // namespace noalloc
}  // namespace mb

extern "C" int mb_cell_pass_noalloc(const void* x, int x_dtype, int64_t n_windows, const float* emb, int64_t n_cls,
                                    const int64_t* cell_ptr, int64_t n_cov, const int64_t* edge_window,
                                    const int64_t* edge_class, const int64_t* win_ptr, const int64_t* edge_wcell,
                                    int64_t h, void* out, int out_dtype, void* stream) {
  MB_REQUIRE(n_cov >= 0 && h > 0, "cell_pass_noalloc: bad sizes");
  MB_REQUIRE(n_cov <= mb::noalloc::kScratchFloats / h,
             "cell_pass_noalloc: %lld covered cells x width %lld need %lld floats of scratch; the fixed buffer "
             "holds %lld (use mb_cell_pass with a caller buffer)",
             (long long)n_cov, (long long)h, (long long)(n_cov * h), (long long)mb::noalloc::kScratchFloats);
  float* scratch = nullptr;
  const int st = mb::noalloc::scratch_address(&scratch, as_stream(stream));
  if (st != MB_OK) return st;
  return mb_cell_pass(x, x_dtype, n_windows, emb, n_cls, cell_ptr, n_cov, edge_window, edge_class, win_ptr,
                      edge_wcell, h, scratch, out, out_dtype, stream);
}
