// PoolEngine: the persistent data plane of pcie_pool_b200.
//
// One engine lives in the data-plane process and holds contexts on every GPU
// it may use.  Per device and per direction (H2D, D2H) it owns
//   * a main/join stream, a lane-kernel stream and a copy-engine stream, so
//     one GPU's H2D and D2H transfers run at the same time on the full-duplex
//     PCIe link (same-direction transfers on one target run in submit order),
//   * a relay staging ring (`slots` x `slot_bytes`) used while the device
//     lends its PCIe link to another GPU, plus a landing ring used for staged
//     ops on its own direct lane,
//   * 32-bit lane counters (ready / free for each ring) in one mailbox,
// all allocated once and reused by every transfer (the reference re-creates
// its runtime, staging slots and peer mappings per transfer:
// turbobus/worker/cuda_executor.py:67-75).  A transfer that overlaps (host or
// device bytes) a pending transfer of the other direction on the same target
// is ordered after it.
//
// A transfer is a set of lanes (the target's direct PCIe lane plus relay
// lanes), each with an ordered chunk list.  For H2D each relay lane runs
//     wait(free >= seq - slots) ; memcpy host->slot ; write(ready = seq)
// on the relay's copy-in stream, and one landing kernel on the target pulls
// every lane's slots over NVLink (pool_kernels.cu).  D2H mirrors it with the
// push kernel on the source GPU and memcpy slot->host on the relay.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <chrono>
#include <cstdint>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "pool_kernels.h"

namespace ppb {

struct EngineOptions {
  uint64_t slot_bytes = 16ull << 20;
  int slots = 3;
  int ctas_per_lane = 4;
  uint64_t coalesce_bytes = 64ull << 20;  // max merged plain direct-lane copy
  double timeout_s = 10.0;  // device-side bound on every wait of a lane kernel
  bool enable_peer_access = true;
};

struct ChunkSpec {
  uint64_t src_off = 0;  // H2D: host offset; D2H: device offset
  uint64_t dst_off = 0;  // H2D: device offset; D2H: host offset
  uint64_t bytes = 0;
  uint32_t unit0 = 0;    // scatter/gather units; fp8 first row; ranges first index
  uint32_t tensor = 0;   // fp8 tensor index
  uint32_t count = 0;    // ranges in this chunk
};

struct LaneSpec {
  int device = -1;       // GPU whose PCIe link carries the lane (== target: direct)
  std::vector<ChunkSpec> chunks;
};

struct QuantTensorSpec {
  uint64_t q = 0;        // device address of the e4m3 output
  uint64_t scales = 0;   // device address of the fp32 scales
  uint32_t rows = 0;
  uint32_t cols = 0;
};

// Streamed optimizer step (op kOpAdamW): device tensors and hyper-parameters.
struct AdamStepSpec {
  uint64_t grads = 0;    // bf16 gradients on the target, nparams elements
  uint64_t params = 0;   // bf16 parameters written on the target, nparams elements
  uint64_t nparams = 0;
  double lr = 1e-3;      // scalars in double: the kernel's factors are formed from them
  double beta1 = 0.9;
  double beta2 = 0.999;
  double eps = 1e-8;
  double weight_decay = 0.0;
  double grad_scale = 1.0;
  int step = 1;          // 1-based step count (bias correction)
};

struct TransferSpec {
  int direction = 0;     // 0 = H2D, 1 = D2H
  int target = 0;
  uint64_t host_ptr = 0;
  uint64_t host_bytes = 0;
  uint64_t dev_ptr = 0;
  uint64_t dev_bytes = 0;
  std::vector<LaneSpec> lanes;
  int op = kOpCopy;
  bool checksum = false;
  bool stage_direct = false;  // route a plain-copy direct lane through the landing ring
  // Serialised mode: H2D issues and finishes every copy-engine copy before the
  // landing kernel starts; D2H starts the copy-out after the push kernel ends.
  // No kernel then waits on a copy running beside it, so the transfer also
  // completes when a profiler serialises all GPU work.  Each staged lane may
  // hold at most `slots` chunks (nothing frees a slot mid-transfer).
  bool serialize = false;
  int debug_drop_publish = -1;  // tests: lane whose "ready" publications are skipped
  bool trace = false;        // record per-chunk %globaltimer stamps (TransferResult::trace)
  int ctas_per_lane = 0;     // 0: engine default
  double timeout_s = 0.0;    // 0: engine default
  uint32_t unit_bytes = 0;
  std::vector<uint64_t> unit_addrs;   // per-unit device addresses
  std::vector<uint64_t> range_addrs;  // per-range device addresses
  std::vector<uint32_t> range_bytes;
  std::vector<uint64_t> range_pos;    // start of each range inside its chunk stream
  std::vector<QuantTensorSpec> tensors;
  AdamStepSpec adam;                  // kOpAdamW: host_ptr is the fp32 state image
};

struct LaneStats {
  int device = -1;
  bool direct = false;
  uint64_t bytes = 0;
  uint64_t chunks = 0;
  double cuda_ms = 0.0;
};

struct TransferResult {
  uint64_t id = 0;
  bool ok = false;
  int status_code = 0;
  int error_lane = -1;
  int error_chunk = -1;
  int error_detail = 0;
  std::string error;
  uint64_t bytes = 0;
  double cuda_ms = 0.0;
  double submit_to_complete_ms = 0.0;
  double gib_per_s = 0.0;
  std::vector<LaneStats> lanes;
  std::vector<uint64_t> checksums;  // 2 per chunk, lanes in spec order
  // 4 per chunk when TransferSpec::trace: {wait begin, ready, done, CTAs} in
  // device nanoseconds (%globaltimer), zeros for chunks no kernel touched
  std::vector<uint64_t> trace;
};

class PoolEngine {
 public:
  PoolEngine(const std::vector<int>& devices, const EngineOptions& options);
  ~PoolEngine();
  PoolEngine(const PoolEngine&) = delete;
  PoolEngine& operator=(const PoolEngine&) = delete;

  uint64_t submit(const TransferSpec& spec);
  // Waits up to `host_timeout_s` (<=0: derived from the device timeout).
  TransferResult wait(uint64_t id, double host_timeout_s);
  bool query(uint64_t id);

  const std::vector<int>& devices() const { return devices_; }
  const EngineOptions& options() const { return options_; }
  // Raw pointers for tests / probes.
  uint64_t relay_ring(int device);
  uint64_t mailbox(int device);
  // Counter values as the host believes them: H2D relay ring, H2D landing
  // ring, D2H relay ring, D2H landing ring.
  std::vector<uint64_t> issued(int device);
  int max_lane_ctas(int device);

 private:
  struct Ring {
    uint8_t* base = nullptr;
    uint32_t* ready = nullptr;
    uint32_t* freec = nullptr;
    uint32_t* donec = nullptr;  // round trips: kernel -> copy-out
    uint64_t issued = 0;       // chunks ever published through this ring
    int last_dir = -1;
    int last_target = -1;
    cudaEvent_t last_done = nullptr;  // end of the last transfer that used it
    bool poisoned = false;
  };
  struct Dev {
    int device = -1;
    // indexed by direction (0 = H2D, 1 = D2H); copy[0] carries host->device
    // copies, copy[1] device->host copies, whichever GPU is the target
    cudaStream_t main[2] = {nullptr, nullptr};
    cudaStream_t kern[2] = {nullptr, nullptr};
    cudaStream_t copy[2] = {nullptr, nullptr};
    uint32_t* mbox = nullptr;  // 12 counters, each on its own 128-byte line
    Ring relay[2], land[2];
    std::vector<cudaEvent_t> free_events;
    // Lane-kernel scratch (descriptor tables, checksums, status, arrival
    // counters): device buffers made once and reused, one per transfer in
    // flight; a buffer returns here when its transfer is waited on.
    std::vector<std::pair<uint8_t*, size_t>> free_scratch;
    std::vector<uint8_t*> quarantine;  // scratch of transfers abandoned by the watchdog
    int max_ctas = 0;
    bool can_flush_remote_writes = false;
  };
  struct Pending;

  Dev& dev(int device);
  void ensure_ring(Dev& d, Ring& r, bool relay);
  cudaEvent_t take_event(Dev& d);
  void give_event(Dev& d, cudaEvent_t e);
  std::pair<uint8_t*, size_t> take_scratch(Dev& d, size_t bytes);
  void give_scratch(Dev& d, std::pair<uint8_t*, size_t> b);
  void* take_pinned(size_t bytes);
  void give_pinned(void* p);
  void reset_rings(Pending& p);

  std::vector<int> devices_;
  EngineOptions options_;
  std::map<int, std::unique_ptr<Dev>> devs_;
  std::mutex mu_;
  std::atomic<uint64_t> next_id_{1};
  std::map<uint64_t, std::unique_ptr<Pending>> pending_;
  std::vector<std::pair<void*, size_t>> pinned_free_;
  std::map<void*, size_t> pinned_used_;
};

// Pinned host memory helpers (cudaHostRegister with portable + mapped flags so
// every GPU context of the process can DMA from/to it).
void host_register(uint64_t ptr, uint64_t bytes);
void host_unregister(uint64_t ptr);

}  // namespace ppb
