#include "ppb_common.h"

#include <mutex>

namespace ppb {

const DriverApi& DriverApi::get() {
  static DriverApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q1 = cudaDriverEntryPointSymbolNotFound;
    cudaDriverEntryPointQueryResult q2 = cudaDriverEntryPointSymbolNotFound;
    void* fn = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuStreamWaitValue32", &fn, 12000, cudaEnableDefault,
                                         &q1) == cudaSuccess &&
        q1 == cudaDriverEntryPointSuccess) {
      api.wait_value32 = reinterpret_cast<DriverApi::WaitValue32Fn>(fn);
    }
    fn = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuStreamWriteValue32", &fn, 12000, cudaEnableDefault,
                                         &q2) == cudaSuccess &&
        q2 == cudaDriverEntryPointSuccess) {
      api.write_value32 = reinterpret_cast<DriverApi::WriteValue32Fn>(fn);
    }
  });
  if (api.wait_value32 == nullptr || api.write_value32 == nullptr) {
    throw std::runtime_error(
        "CUDA driver does not provide cuStreamWaitValue32/cuStreamWriteValue32");
  }
  return api;
}

void stream_wait_geq(cudaStream_t stream, const void* addr, uint32_t value, bool flush) {
  const int rc = DriverApi::get().wait_value32(
      stream, reinterpret_cast<unsigned long long>(addr), value,
      kWaitGeq | (flush ? kWaitFlush : 0u));
  if (rc != 0) {
    throw std::runtime_error("cuStreamWaitValue32 failed with CUresult " + std::to_string(rc));
  }
}

void stream_write(cudaStream_t stream, void* addr, uint32_t value) {
  const int rc = DriverApi::get().write_value32(
      stream, reinterpret_cast<unsigned long long>(addr), value, kWriteDefault);
  if (rc != 0) {
    throw std::runtime_error("cuStreamWriteValue32 failed with CUresult " + std::to_string(rc));
  }
}

}  // namespace ppb
