// Integer table derivations: CSR pointers over sorted keys, stable argsort,
// index gathers. Bit-exact with the torch compositions the reference runs per
// forward (cell_latents.py:96-165, cell_nodes.py:23-94,
// message_passing.py:495-517, window_latents.py:38-56).
#include <cub/device/device_radix_sort.cuh>

#include "common.cuh"

namespace mb {

// ptr[d] = lower_bound(keys, d) for d in [0, n_dest]. Thread i owns the gap
// between keys[i-1] and keys[i]; every d in (keys[i-1], keys[i]] maps to i.
__global__ void csr_from_sorted_kernel(const int64_t* __restrict__ keys, int64_t n, int64_t n_dest,
                                       int64_t* __restrict__ ptr) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i <= n; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t lo = (i == 0) ? -1 : keys[i - 1];
    int64_t hi = (i == n) ? n_dest : keys[i];
    if (i < n && (hi < 0 || hi >= n_dest)) { report(ERR_INDEX); continue; }
    if (hi < lo) { report(ERR_UNSORTED); continue; }
    if (lo < -1) lo = -1;
    for (int64_t d = lo + 1; d <= hi; ++d) ptr[d] = i;
  }
}

__global__ void iota_kernel(int64_t* out, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = i;
}

__global__ void gather_i64_kernel(const int64_t* __restrict__ src, int64_t n_src, const int64_t* __restrict__ idx,
                                  int64_t n, int64_t* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t j = idx[i];
    if (j < 0 || j >= n_src) { report(ERR_INDEX); out[i] = 0; continue; }
    out[i] = src[j];
  }
}

__global__ void radius_class_kernel(const int64_t* __restrict__ orbit, const int64_t* __restrict__ own,
                                    const int64_t* __restrict__ on_axis, const int64_t* __restrict__ order,
                                    int64_t n, int64_t* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t j = order ? order[i] : i;
    if (j < 0 || j >= n) { report(ERR_INDEX); out[i] = 0; continue; }
    out[i] = orbit[j] + 48 * (own[j] + 2 * on_axis[j]);
  }
}

__global__ void div_kernel(const int64_t* __restrict__ x, int64_t n, int64_t divisor, int64_t* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = x[i] / divisor;
}

static inline int grid_for(int64_t n, int threads = 256) {
  int64_t g = cdiv(n, threads);
  if (g < 1) g = 1;
  if (g > 148 * 32) g = 148 * 32;
  return (int)g;
}

// One buffer for CUB's temp storage plus the iota payload. The size query
// reads the current device's properties, so it needs a visible GPU.
static cudaError_t cub_bytes(int64_t n, int key_bits, size_t* temp) {
  *temp = 0;
  return cub::DeviceRadixSort::SortPairs<int64_t, int64_t>(nullptr, *temp, (const int64_t*)nullptr,
                                                           (int64_t*)nullptr, (const int64_t*)nullptr,
                                                           (int64_t*)nullptr, (int)n, 0, key_bits);
}

}  // namespace mb

extern "C" {

int mb_csr_from_sorted(const int64_t* keys, int64_t n, int64_t n_dest, int64_t* ptr, void* stream) {
  MB_REQUIRE(n >= 0 && n_dest >= 0, "csr_from_sorted: negative size");
  MB_REQUIRE(ptr != nullptr && (n == 0 || keys != nullptr), "csr_from_sorted: null pointer");
  mb::csr_from_sorted_kernel<<<mb::grid_for(n + 1), 256, 0, mb::as_stream(stream)>>>(keys, n, n_dest, ptr);
  return mb::launch_status("csr_from_sorted");
}

int mb_argsort_workspace(int64_t n, int key_bits, int64_t* bytes) {
  MB_REQUIRE(bytes != nullptr, "argsort_workspace: bytes is NULL");
  MB_REQUIRE(n >= 0 && n < (int64_t)INT32_MAX, "argsort_workspace: n=%lld out of range", (long long)n);
  MB_REQUIRE(key_bits >= 1 && key_bits <= 63, "argsort_workspace: key_bits=%d", key_bits);
  size_t temp = 0;
  cudaError_t err = mb::cub_bytes(n, key_bits, &temp);
  if (err != cudaSuccess) {
    cudaGetLastError();
    return mb::fail(MB_UNSUPPORTED, "argsort_workspace: %s", cudaGetErrorString(err));
  }
  *bytes = (int64_t)(((temp + 255) / 256) * 256 + (size_t)n * sizeof(int64_t));
  return MB_OK;
}

int mb_argsort(const int64_t* keys, int64_t n, int key_bits, int64_t* sorted_keys, int64_t* order, void* workspace,
               int64_t workspace_bytes, void* stream) {
  MB_REQUIRE(n >= 0 && n < (int64_t)INT32_MAX, "argsort: n=%lld out of range", (long long)n);
  MB_REQUIRE(key_bits >= 1 && key_bits <= 63, "argsort: key_bits=%d", key_bits);
  if (n == 0) return MB_OK;
  MB_REQUIRE(keys && sorted_keys && order && workspace, "argsort: null pointer");
  int64_t need = 0;
  int st = mb_argsort_workspace(n, key_bits, &need);
  if (st != MB_OK) return st;
  MB_REQUIRE(workspace_bytes >= need, "argsort: workspace %lld < %lld bytes", (long long)workspace_bytes,
             (long long)need);
  cudaStream_t s = mb::as_stream(stream);
  size_t temp = 0;
  mb::cub_bytes(n, key_bits, &temp);
  size_t temp_aligned = ((temp + 255) / 256) * 256;
  int64_t* iota = reinterpret_cast<int64_t*>(static_cast<char*>(workspace) + temp_aligned);
  mb::iota_kernel<<<mb::grid_for(n), 256, 0, s>>>(iota, n);
  cudaError_t err = cub::DeviceRadixSort::SortPairs<int64_t, int64_t>(workspace, temp, keys, sorted_keys, iota, order,
                                                                      (int)n, 0, key_bits, s);
  if (err != cudaSuccess) return mb::fail(MB_LAUNCH_FAILED, "argsort: %s", cudaGetErrorString(err));
  return mb::launch_status("argsort");
}

int mb_gather_i64(const int64_t* src, int64_t n_src, const int64_t* idx, int64_t n, int64_t* out, void* stream) {
  MB_REQUIRE(n >= 0, "gather_i64: negative size");
  if (n == 0) return MB_OK;
  MB_REQUIRE(src && idx && out, "gather_i64: null pointer");
  mb::gather_i64_kernel<<<mb::grid_for(n), 256, 0, mb::as_stream(stream)>>>(src, n_src, idx, n, out);
  return mb::launch_status("gather_i64");
}

int mb_radius_class(const int64_t* orbit, const int64_t* own, const int64_t* on_axis, const int64_t* order, int64_t n,
                    int64_t* out, void* stream) {
  MB_REQUIRE(n >= 0, "radius_class: negative size");
  if (n == 0) return MB_OK;
  MB_REQUIRE(orbit && own && on_axis && out, "radius_class: null pointer");
  mb::radius_class_kernel<<<mb::grid_for(n), 256, 0, mb::as_stream(stream)>>>(orbit, own, on_axis, order, n, out);
  return mb::launch_status("radius_class");
}

int mb_div_i64(const int64_t* x, int64_t n, int64_t divisor, int64_t* out, void* stream) {
  MB_REQUIRE(n >= 0 && divisor > 0, "div_i64: bad arguments");
  if (n == 0) return MB_OK;
  MB_REQUIRE(x && out, "div_i64: null pointer");
  mb::div_kernel<<<mb::grid_for(n), 256, 0, mb::as_stream(stream)>>>(x, n, divisor, out);
  return mb::launch_status("div_i64");
}

}  // extern "C"
