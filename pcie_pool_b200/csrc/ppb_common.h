// Shared host-side helpers for the pcie_pool_b200 native core.
//
// The core links the CUDA runtime statically and reaches the few driver entry
// points it needs (stream memory operations) through
// cudaGetDriverEntryPointByVersion, so the module has no link-time dependency
// on libcuda and can be built on a machine without a GPU driver.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>

namespace ppb {

class CudaError : public std::runtime_error {
 public:
  CudaError(const std::string& what, cudaError_t code)
      : std::runtime_error(what), code_(code) {}
  cudaError_t code() const { return code_; }

 private:
  cudaError_t code_;
};

inline void check_cuda(cudaError_t rc, const char* what) {
  if (rc != cudaSuccess) {
    throw CudaError(std::string(what) + ": " + cudaGetErrorName(rc) + " (" +
                        cudaGetErrorString(rc) + ")",
                    rc);
  }
}

#define PPB_CUDA(expr) ::ppb::check_cuda((expr), #expr)

// RAII guard that restores the current device on scope exit.
class DeviceGuard {
 public:
  explicit DeviceGuard(int device) {
    check_cuda(cudaGetDevice(&prev_), "cudaGetDevice");
    if (device != prev_) check_cuda(cudaSetDevice(device), "cudaSetDevice");
  }
  ~DeviceGuard() { cudaSetDevice(prev_); }
  DeviceGuard(const DeviceGuard&) = delete;
  DeviceGuard& operator=(const DeviceGuard&) = delete;

 private:
  int prev_ = 0;
};

// Stream memory operations from the driver API.  Values follow cuda.h:
// CU_STREAM_WAIT_VALUE_GEQ compares (int32_t)(*addr - value) >= 0, which is
// wrap-around safe for the monotonically increasing lane counters used here.
enum : unsigned int {
  kWaitGeq = 0x0,
  kWaitFlush = 1u << 30,
  kWriteDefault = 0x0,
};

struct DriverApi {
  using WaitValue32Fn = int (*)(cudaStream_t, unsigned long long, uint32_t,
                                unsigned int);
  using WriteValue32Fn = int (*)(cudaStream_t, unsigned long long, uint32_t,
                                 unsigned int);
  WaitValue32Fn wait_value32 = nullptr;
  WriteValue32Fn write_value32 = nullptr;

  static const DriverApi& get();
};

// Stream-ordered 32-bit wait / write on a device-visible address.
void stream_wait_geq(cudaStream_t stream, const void* addr, uint32_t value,
                     bool flush);
void stream_write(cudaStream_t stream, void* addr, uint32_t value);

}  // namespace ppb
