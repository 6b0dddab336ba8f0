// Library identity, error reporting, and the device error word.
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

namespace mb {

static thread_local char t_message[1024] = "";

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_message, sizeof(t_message), fmt, ap);
  va_end(ap);
  return status;
}

int launch_status(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return fail(MB_LAUNCH_FAILED, "%s: %s", what, cudaGetErrorString(err));
  return MB_OK;
}

}  // namespace mb

extern "C" {

int mb_version(void) { return 1; }

const char* mb_last_error(void) { return mb::t_message; }

int mb_device_error(void* stream, uint32_t* code, int clear) {
  MB_REQUIRE(code != nullptr, "mb_device_error: code is NULL");
  cudaStream_t s = mb::as_stream(stream);
  cudaError_t err = cudaMemcpyFromSymbolAsync(code, mb::g_device_error, sizeof(uint32_t), 0,
                                              cudaMemcpyDeviceToHost, s);
  if (err == cudaSuccess) err = cudaStreamSynchronize(s);
  if (err == cudaSuccess && clear && *code != 0) {
    const uint32_t zero = 0;
    err = cudaMemcpyToSymbolAsync(mb::g_device_error, &zero, sizeof(uint32_t), 0, cudaMemcpyHostToDevice, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
  }
  if (err != cudaSuccess) return mb::fail(MB_LAUNCH_FAILED, "mb_device_error: %s", cudaGetErrorString(err));
  return MB_OK;
}

}  // extern "C"
