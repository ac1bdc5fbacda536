// Device-local sm_100a kernels that complement the lane kernels:
//   * fp8 e4m3 128x128 block quantisation of a bf16 matrix already in HBM,
//   * fixed-size unit gather / scatter (paged-KV blocks <-> contiguous),
//   * variable-range pack / unpack,
//   * fused AdamW step over fp32 master/m/v + bf16 grads emitting bf16 params,
//   * an SM/HBM interference generator (the reference's dummy compute,
//     cpp/src/dummy_compute_cuda.cu:23-35, generalised to a tunable CTA count),
//   * the chunk checksum on device and on the host.
// All take raw addresses and a stream so they serve both the engine and the
// torch-facing Python wrappers.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <utility>

namespace ppb {

struct AdamParams {
  double lr = 1e-3;
  double beta1 = 0.9;
  double beta2 = 0.999;
  double eps = 1e-8;
  double weight_decay = 0.0;
  double grad_scale = 1.0;  // multiplies the incoming gradient
  int step = 1;
};

cudaError_t fp8_block_quant(const void* src_bf16, uint64_t rows, uint64_t cols, void* q_e4m3,
                            float* scales, cudaStream_t stream);
cudaError_t fp8_block_dequant(const void* q_e4m3, const float* scales, uint64_t rows,
                              uint64_t cols, void* out_bf16, cudaStream_t stream);
cudaError_t gather_units(const uint64_t* unit_addr_dev, uint64_t units, uint32_t unit_bytes,
                         void* dst, cudaStream_t stream);
cudaError_t scatter_units(const void* src, const uint64_t* unit_addr_dev, uint64_t units,
                          uint32_t unit_bytes, cudaStream_t stream);
cudaError_t pack_ranges(const uint64_t* addr_dev, const uint64_t* bytes_dev, const uint64_t* pos_dev,
                        uint64_t n, void* dst, cudaStream_t stream);
cudaError_t unpack_ranges(const void* src, const uint64_t* addr_dev, const uint64_t* bytes_dev,
                          const uint64_t* pos_dev, uint64_t n, cudaStream_t stream);
cudaError_t fused_adamw(float* master, float* m, float* v, const void* grad_bf16, void* param_bf16,
                        uint64_t n, const AdamParams& p, cudaStream_t stream);
cudaError_t interference(float* buf, uint64_t n, int iters, int ctas, cudaStream_t stream);
// Device checksum of [ptr, ptr+bytes) into out_dev[2] (zeroed by the call).
cudaError_t checksum_device(const void* ptr, uint64_t bytes, unsigned long long* out_dev,
                            cudaStream_t stream);
std::pair<uint64_t, uint64_t> checksum_host(const void* ptr, uint64_t bytes);

}  // namespace ppb
