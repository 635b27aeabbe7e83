// Shared internals of libpowersparse_b200: status handling and small device helpers.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <cstdint>
#include <stdexcept>
#include <string>

namespace psb {

// Errors travel as C++ exceptions inside the library and become status codes
// at the extern "C" boundary (ps_capi.cu).  The two kinds mirror the reference's
// convention: std::invalid_argument for caller errors, std::runtime_error for
// CUDA failures (utils/cuda_utils.h:7-14 of the reference).
struct CudaError : std::runtime_error {
  cudaError_t code;
  CudaError(cudaError_t c, const std::string& what) : std::runtime_error(what), code(c) {}
};

inline void check_cuda(cudaError_t status, const char* expr, const char* file, int line) {
  if (status != cudaSuccess)
    throw CudaError(status, std::string(file) + ":" + std::to_string(line) + ": " + expr + ": " +
                                cudaGetErrorString(status));
}

#define PSB_CUDA(call) ::psb::check_cuda((call), #call, __FILE__, __LINE__)
#define PSB_LAUNCH_CHECK() ::psb::check_cuda(cudaGetLastError(), "kernel launch", __FILE__, __LINE__)

constexpr int kWarp = 32;

// Multiprocessor count of the current device (cached per device): grid-stride
// kernels launch a fixed number of CTAs per SM.
inline int device_sms() {
  static std::atomic<int> cache[64] = {};
  int dev = 0;
  PSB_CUDA(cudaGetDevice(&dev));
  const bool cached = dev >= 0 && dev < 64;
  if (cached) {
    const int v = cache[dev].load(std::memory_order_relaxed);
    if (v > 0) return v;
  }
  int v = 0;
  PSB_CUDA(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev));
  if (cached) cache[dev].store(v, std::memory_order_relaxed);
  return v;
}

__host__ __device__ inline int ceil_div(int a, int b) { return (a + b - 1) / b; }
__host__ __device__ inline long long ceil_div_ll(long long a, long long b) { return (a + b - 1) / b; }

inline int bits_for(unsigned long long max_value) {
  int b = 0;
  while (b < 64 && (max_value >> b) != 0) ++b;
  return b;
}

// A device buffer owned by the library (freed on scope exit, also on throw).
template <typename T>
struct DeviceArray {
  T* ptr = nullptr;
  size_t count = 0;
  DeviceArray() = default;
  explicit DeviceArray(size_t n) { reset(n); }
  DeviceArray(const DeviceArray&) = delete;
  DeviceArray& operator=(const DeviceArray&) = delete;
  DeviceArray(DeviceArray&& o) noexcept : ptr(o.ptr), count(o.count) { o.ptr = nullptr; o.count = 0; }
  DeviceArray& operator=(DeviceArray&& o) noexcept {
    if (this != &o) { release(); ptr = o.ptr; count = o.count; o.ptr = nullptr; o.count = 0; }
    return *this;
  }
  ~DeviceArray() { release(); }
  void reset(size_t n) {
    release();
    count = n;
    if (n) PSB_CUDA(cudaMalloc(reinterpret_cast<void**>(&ptr), n * sizeof(T)));
  }
  void release() noexcept {
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    count = 0;
  }
  T* release_ownership() { T* p = ptr; ptr = nullptr; count = 0; return p; }
  T* get() const { return ptr; }
};

// The library's stream-ordered memory pool on `device`, for the scratch of the
// preprocessing.  Its release threshold is unlimited, so memory given back stays
// mapped for the next allocation (the row sort's buffers become the column sort's)
// instead of being returned at every synchronization; trim_scratch_pool hands it
// back to the device when a build ends.
inline cudaMemPool_t scratch_pool(int device) {
  static std::mutex mu;
  static cudaMemPool_t pools[64] = {};
  if (device < 0 || device >= 64) throw std::invalid_argument("device ordinal out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (!pools[device]) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = device;
    cudaMemPool_t pool = nullptr;
    PSB_CUDA(cudaMemPoolCreate(&pool, &props));
    unsigned long long keep = ~0ULL;
    PSB_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep));
    pools[device] = pool;
  }
  return pools[device];
}

// Returns the unused memory of the current device's scratch pool after waiting for
// the device (memory freed in stream order is unused only once the free has run).
inline void trim_scratch_pool() noexcept {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return;
  cudaDeviceSynchronize();
  try {
    cudaMemPoolTrimTo(scratch_pool(device), 0);
  } catch (...) {
  }
}

// A device buffer in stream order: taken from the scratch pool on `stream` and given
// back with cudaFreeAsync on the same stream at scope exit, so work already queued
// on that stream may still use it and neither step waits for the device.
template <typename T>
struct StreamArray {
  T* ptr = nullptr;
  cudaStream_t stream = nullptr;
  StreamArray(size_t n, cudaStream_t s) : stream(s) {
    if (!n) return;
    int device = 0;
    PSB_CUDA(cudaGetDevice(&device));
    PSB_CUDA(cudaMallocFromPoolAsync(reinterpret_cast<void**>(&ptr), n * sizeof(T), scratch_pool(device), s));
  }
  StreamArray(const StreamArray&) = delete;
  StreamArray& operator=(const StreamArray&) = delete;
  ~StreamArray() { release(); }
  // Gives the buffer back now (in stream order).
  void release() noexcept {
    if (ptr) cudaFreeAsync(ptr, stream);
    ptr = nullptr;
  }
  T* get() const { return ptr; }
};

}  // namespace psb
