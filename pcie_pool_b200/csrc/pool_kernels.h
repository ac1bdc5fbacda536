// Descriptors and launchers for the fused lane kernels.
//
//   land  (H2D, runs on the destination GPU): waits for a lane's "ready"
//         counter, pulls the staged chunk out of the (peer) staging slot with
//         TMA bulk loads over NVLink, applies the landing op (copy, paged-KV
//         scatter, fp8 block quantisation), accumulates the chunk checksum and
//         releases the slot by advancing the lane's "free" counter with a
//         system-scope release store.
//   push  (D2H, runs on the source GPU): waits for the lane's "free" counter,
//         gathers/copies the chunk into the (peer) staging slot, checksums it
//         and publishes it by advancing the lane's "ready" counter.
//
// Reference behaviour these replace: the relay leg in the reference is a
// cudaMemcpyPeerAsync per chunk followed by a full-slot cudaMemsetAsync
// (cpp/src/executor_cuda.cu:223-238, :274-287).  Here the leg is one
// persistent kernel per transfer with no per-chunk API call on the device side.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "adamw.cuh"

namespace ppb {

enum LaneOp : uint32_t {
  kOpCopy = 0,          // contiguous chunk -> dst + dst_off (or src + src_off -> slot)
  kOpScatterUnits = 1,  // H2D: fixed-size units -> unit_addr[unit] (paged-KV reload)
  kOpGatherUnits = 2,   // D2H: unit_addr[unit] -> contiguous (paged-KV offload)
  kOpFp8Quant = 3,      // H2D: bf16 rows -> fp8 e4m3 + fp32 per-128x128 scales
  kOpScatterRanges = 4, // H2D: variable ranges -> range_addr (unpack)
  kOpGatherRanges = 5,  // D2H: variable ranges -> contiguous (pack)
  kOpAdamW = 6,         // H2D round trip: fp32 optimizer-state tiles are updated in
                        // their staging slot with the local bf16 grads (bf16 params
                        // out), then copied back to the host (streamed optimizer step)
};

// Streamed-optimizer state layout, host and slot: tiles of kAdamTileParams
// parameters, each [master | exp_avg | exp_avg_sq] as fp32 (24 KiB, one
// shared-memory stage).  Parameter i lives in tile i / kAdamTileParams.
constexpr uint32_t kAdamTileParams = 2048;
constexpr uint32_t kAdamTileBytes = 3u * 4u * kAdamTileParams;

enum StatusCode : int {
  kStatusOk = 0,
  kStatusReadyTimeout = 1,
  kStatusCopyTimeout = 2,
  kStatusBadArgument = 3,
  kStatusFreeTimeout = 4,
};

// One lane of a transfer as seen by the lane kernel.
struct LaneDesc {
  uint8_t* ring;          // staging ring base (peer pointer for relay lanes)
  uint32_t* ready;        // producer -> consumer counter
  uint32_t* freec;        // consumer -> producer counter
  uint64_t slot_bytes;
  uint32_t chunk_begin;   // first chunk of this lane in the chunk table
  uint32_t chunk_count;
  uint32_t cta_begin;     // CTA group of this lane
  uint32_t cta_count;
  uint32_t in_place;      // 1: no staging, the data sits at its final place
  uint32_t slots;
  // Round trip (kOpAdamW): the kernel publishes a processed chunk here for the
  // copy-out stream, which frees the slot itself (freec is then unused).
  uint32_t* donec;
};

struct ChunkDesc {
  uint64_t dev_off;   // H2D: destination offset; D2H: source offset (Copy)
  uint64_t host_off;  // offset on the host side (for stats / in-place D2H)
  uint32_t bytes;
  uint32_t seq;       // lane counter value that publishes this chunk
  uint32_t slot;      // staging slot index
  uint32_t unit0;     // first unit / first range / first row (op dependent)
  uint32_t tensor;    // fp8: tensor table index
  uint32_t count;     // ranges: number of ranges in this chunk
};

// Fp8 landing target: a row-major [rows, cols] bf16 matrix that lands as
// e4m3 [rows, cols] plus fp32 scales [ceil(rows/128), cols/128].
struct QuantTensor {
  uint8_t* q;
  float* scales;
  uint32_t rows;
  uint32_t cols;
};

struct LaneKernelParams {
  const LaneDesc* lanes;
  const ChunkDesc* chunks;
  uint32_t num_lanes;
  uint32_t op;
  uint8_t* dev;                 // device buffer base (dst for H2D, src for D2H)
  const uint64_t* unit_addr;    // per-unit device addresses (scatter/gather)
  const uint64_t* range_addr;   // per-range device addresses (pack/unpack)
  const uint32_t* range_bytes;  // per-range sizes
  const uint64_t* range_pos;    // per-range start within the chunk stream
  uint32_t unit_bytes;
  uint32_t checksum;
  const QuantTensor* tensors;
  uint32_t* done;               // per-chunk arrival counters (zeroed per transfer)
  unsigned long long* csum;     // per-chunk {sum, weighted} (zeroed per transfer)
  int* status;                  // {code, lane, chunk, detail} (first error wins)
  uint64_t timeout_ns;
  // Optional per-chunk device trace (nullptr: off), kTraceWords words per
  // kernel chunk of %globaltimer nanoseconds: {wait begin, ready (land: chunk
  // published / push: slot free), chunk done (last CTA of the lane group),
  // CTAs that finished the chunk}.
  unsigned long long* trace;
  // kOpAdamW: local bf16 gradients in, bf16 parameters out (nparams each)
  const uint16_t* grads;
  uint16_t* params_out;
  uint64_t nparams;
  AdamCoeffs adam;
};

constexpr int kTraceWords = 4;

constexpr int kLaneThreads = 256;
constexpr uint32_t kTileBytes = 32768;
constexpr int kStages = 4;
constexpr size_t kLaneSmemBytes = size_t(kStages) * kTileBytes + 128;

// Launch the landing kernel (H2D) / push kernel (D2H) with `grid` CTAs.
cudaError_t launch_land(const LaneKernelParams& p, int grid, cudaStream_t stream);
cudaError_t launch_push(const LaneKernelParams& p, int grid, cudaStream_t stream);

// Max co-resident lane CTAs on one device (the grid must fit so that no CTA of
// a lane group waits for SM space while its siblings wait for it).
int lane_kernel_max_ctas(int device);

}  // namespace ppb
