#include "engine.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <thread>

#include <nvtx3/nvToolsExt.h>

#include "ppb_common.h"

namespace ppb {

namespace {

// Mailbox layout: per direction six 32-bit counters (relay ready, relay
// free, landing ready, landing free, relay done, landing done), each on its
// own 128-byte line.  "done" is only used by round trips (kOpAdamW): the
// kernel publishes a processed chunk and the copy-out stream frees the slot.
constexpr int kCounterStride = 128 / 4;
constexpr int kRelayReady = 0;
constexpr int kRelayFree = 1;
constexpr int kLandReady = 2;
constexpr int kLandFree = 3;
constexpr int kRelayDone = 4;
constexpr int kLandDone = 5;
constexpr int kCountersPerDir = 6;
constexpr size_t kMailboxBytes = 128 * 2 * kCountersPerDir;
uint32_t* counter(uint32_t* mbox, int dir, int which) {
  return mbox + (dir * kCountersPerDir + which) * kCounterStride;
}

// Of the lane-kernel CTAs that can be resident on one GPU, landing kernels
// (H2D; fp8 quantisation wants many CTAs) get two thirds and push kernels
// (D2H) one third, so one transfer of each direction always fits side by side
// and no CTA of either waits for the other to leave the GPU.
int direction_cta_budget(int max_ctas, bool h2d) {
  const int d2h = std::max(1, max_ctas / 3);
  return h2d ? std::max(1, max_ctas - d2h) : d2h;
}
constexpr uint32_t kRescueStride = 0x40000000u;

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

double event_ms(cudaEvent_t a, cudaEvent_t b) {
  float ms = 0.f;
  if (cudaEventElapsedTime(&ms, a, b) != cudaSuccess) {
    cudaGetLastError();
    return 0.0;
  }
  return static_cast<double>(ms);
}

bool is_pinned_host(const void* p) {
  cudaPointerAttributes attr{};
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return attr.type == cudaMemoryTypeHost;
}

bool can_flush_remote_writes(int device) {
  int v = 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrCanFlushRemoteWrites, device) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return v != 0;
}

}  // namespace

// NVTX annotations (header-only NVTX3: free when no tool is attached).  One
// range per transfer from submit to the end of wait() (started and ended on
// possibly different host threads), a nested push/pop range around each
// lane's copy-engine enqueue and around each lane-kernel launch, all in the
// "pcie_pool_b200" domain.
nvtxDomainHandle_t nvtx_domain() {
  static nvtxDomainHandle_t d = nvtxDomainCreateA("pcie_pool_b200");
  return d;
}

nvtxRangeId_t nvtx_start(const std::string& msg, uint32_t color) {
  nvtxEventAttributes_t a{};
  a.version = NVTX_VERSION;
  a.size = NVTX_EVENT_ATTRIB_STRUCT_SIZE;
  a.colorType = NVTX_COLOR_ARGB;
  a.color = color;
  a.messageType = NVTX_MESSAGE_TYPE_ASCII;
  a.message.ascii = msg.c_str();
  return nvtxDomainRangeStartEx(nvtx_domain(), &a);
}

struct NvtxScope {
  explicit NvtxScope(const std::string& msg, uint32_t color) {
    nvtxEventAttributes_t a{};
    a.version = NVTX_VERSION;
    a.size = NVTX_EVENT_ATTRIB_STRUCT_SIZE;
    a.colorType = NVTX_COLOR_ARGB;
    a.color = color;
    a.messageType = NVTX_MESSAGE_TYPE_ASCII;
    a.message.ascii = msg.c_str();
    nvtxDomainRangePushEx(nvtx_domain(), &a);
  }
  ~NvtxScope() { nvtxDomainRangePop(nvtx_domain()); }
};

struct PoolEngine::Pending {
  struct LaneRec {
    int device = -1;
    bool direct = false;
    bool kernel = false;     // processed by the lane kernel
    bool staged = false;     // goes through a staging ring
    bool in_place = false;   // kernel reads/writes data at its final place
    bool roundtrip = false;  // kOpAdamW: chunks return to the host after the kernel
    Ring* ring = nullptr;
    cudaStream_t stream = nullptr;
    cudaStream_t out = nullptr;  // round trip: the copy-out (device->host) stream
    Dev* d = nullptr;
    cudaEvent_t t0 = nullptr, t1 = nullptr;
    cudaEvent_t t_in = nullptr;   // round trip: end of the copy-in leg
    cudaEvent_t t_out = nullptr;  // round trip: end of the copy-out leg
    uint64_t seq0 = 0;       // ring->issued before this lane's first chunk
    uint64_t bytes = 0;
    uint64_t chunks = 0;
    int first_chunk = -1;    // index into the kernel chunk table
  };
  uint64_t id = 0;
  int target = 0;
  int direction = 0;
  nvtxRangeId_t nvtx = 0;   // transfer range (submit -> wait)
  size_t total_chunks = 0;  // chunks in spec order (for the checksum vector)
  std::vector<int> spec_chunk_to_kernel;  // spec-order chunk -> kernel chunk (-1: none)
  std::vector<int> kernel_lane_to_spec;   // kernel lane index -> spec lane index
  bool trace = false;
  std::vector<LaneRec> lanes;
  std::vector<Ring*> rings;
  std::vector<int> ring_devices;
  cudaEvent_t start = nullptr, stop = nullptr, kern_done = nullptr;
  std::pair<uint8_t*, size_t> scratch{nullptr, 0};  // device scratch (reused buffer)
  void* desc_host = nullptr;
  void* result_host = nullptr;
  size_t kernel_chunks = 0;
  bool has_kernel = false;
  uint64_t bytes = 0;
  double timeout_s = 0.0;
  std::chrono::steady_clock::time_point t_submit;
  // bytes the transfer touches, for ordering against the other direction
  uint64_t host_lo = 0, host_hi = 0, dev_lo = 0, dev_hi = 0;
  bool dev_known = false;  // false: scattered device addresses (treated as overlapping)
};

PoolEngine::PoolEngine(const std::vector<int>& devices, const EngineOptions& options)
    : devices_(devices), options_(options) {
  if (devices_.empty()) throw std::invalid_argument("PoolEngine needs at least one device");
  if (options_.slot_bytes == 0 || options_.slot_bytes % 256 != 0)
    throw std::invalid_argument("slot_bytes must be a positive multiple of 256");
  if (options_.slot_bytes > (1ull << 31))
    throw std::invalid_argument("slot_bytes must be at most 2 GiB");
  if (options_.slots < 1) throw std::invalid_argument("slots must be >= 1");
  if (options_.ctas_per_lane < 1) throw std::invalid_argument("ctas_per_lane must be >= 1");
  int count = 0;
  PPB_CUDA(cudaGetDeviceCount(&count));
  for (int d : devices_) {
    if (d < 0 || d >= count) throw std::invalid_argument("device index out of range");
  }
  int prev = 0;
  PPB_CUDA(cudaGetDevice(&prev));
  for (int d : devices_) {
    auto D = std::make_unique<Dev>();
    D->device = d;
    PPB_CUDA(cudaSetDevice(d));
    int lo = 0, hi = 0;
    PPB_CUDA(cudaDeviceGetStreamPriorityRange(&lo, &hi));
    for (int dir = 0; dir < 2; ++dir) {
      PPB_CUDA(cudaStreamCreateWithFlags(&D->main[dir], cudaStreamNonBlocking));
      PPB_CUDA(cudaStreamCreateWithPriority(&D->kern[dir], cudaStreamNonBlocking, hi));
      PPB_CUDA(cudaStreamCreateWithFlags(&D->copy[dir], cudaStreamNonBlocking));
    }
    void* mb = nullptr;
    PPB_CUDA(cudaMalloc(&mb, kMailboxBytes));
    PPB_CUDA(cudaMemset(mb, 0, kMailboxBytes));
    D->mbox = static_cast<uint32_t*>(mb);
    for (int dir = 0; dir < 2; ++dir) {
      D->relay[dir].ready = counter(D->mbox, dir, kRelayReady);
      D->relay[dir].freec = counter(D->mbox, dir, kRelayFree);
      D->land[dir].ready = counter(D->mbox, dir, kLandReady);
      D->land[dir].freec = counter(D->mbox, dir, kLandFree);
      D->relay[dir].donec = counter(D->mbox, dir, kRelayDone);
      D->land[dir].donec = counter(D->mbox, dir, kLandDone);
    }
    // Keep freed stream-ordered allocations cached in the pool.
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, d) == cudaSuccess) {
      uint64_t thr = ~0ull;
      cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
    }
    cudaGetLastError();
    D->max_ctas = lane_kernel_max_ctas(d);
    D->can_flush_remote_writes = can_flush_remote_writes(d);
    devs_[d] = std::move(D);
  }
  if (options_.enable_peer_access) {
    for (int a : devices_) {
      PPB_CUDA(cudaSetDevice(a));
      for (int b : devices_) {
        if (a == b) continue;
        int can = 0;
        PPB_CUDA(cudaDeviceCanAccessPeer(&can, a, b));
        if (!can) continue;
        const cudaError_t rc = cudaDeviceEnablePeerAccess(b, 0);
        if (rc == cudaErrorPeerAccessAlreadyEnabled) {
          cudaGetLastError();
        } else {
          check_cuda(rc, "cudaDeviceEnablePeerAccess");
        }
      }
    }
  }
  PPB_CUDA(cudaSetDevice(prev));
}

PoolEngine::~PoolEngine() {
  // Best effort: bounded wait for everything in flight, then release.
  for (auto& kv : pending_) {
    auto& P = *kv.second;
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(30);
    while (cudaEventQuery(P.stop) == cudaErrorNotReady &&
           std::chrono::steady_clock::now() < deadline) {
      std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
  }
  cudaGetLastError();
  for (auto& kv : devs_) {
    Dev& D = *kv.second;
    cudaSetDevice(D.device);
    for (int dir = 0; dir < 2; ++dir) {
      cudaStreamSynchronize(D.main[dir]);
      cudaStreamSynchronize(D.kern[dir]);
      cudaStreamSynchronize(D.copy[dir]);
    }
    for (Ring* r : {&D.relay[0], &D.land[0], &D.relay[1], &D.land[1]}) {
      if (r->base) {
        cudaMemset(r->base, 0, options_.slot_bytes * options_.slots);
        cudaFree(r->base);
      }
    }
    if (D.mbox) cudaFree(D.mbox);
    for (auto& b : D.free_scratch) cudaFree(b.first);
    for (auto* b : D.quarantine) cudaFree(b);
    for (auto e : D.free_events) cudaEventDestroy(e);
    for (int dir = 0; dir < 2; ++dir) {
      cudaStreamDestroy(D.main[dir]);
      cudaStreamDestroy(D.kern[dir]);
      cudaStreamDestroy(D.copy[dir]);
    }
  }
  for (auto& kv : pending_) {
    if (kv.second->scratch.first) {
      cudaSetDevice(kv.second->target);
      cudaFree(kv.second->scratch.first);
    }
    if (kv.second->desc_host) cudaFreeHost(kv.second->desc_host);
    if (kv.second->result_host) cudaFreeHost(kv.second->result_host);
  }
  for (auto& p : pinned_free_) cudaFreeHost(p.first);
  for (auto& p : pinned_used_) cudaFreeHost(p.first);
  cudaGetLastError();
}

PoolEngine::Dev& PoolEngine::dev(int device) {
  auto it = devs_.find(device);
  if (it == devs_.end()) throw std::invalid_argument("device is not managed by this engine");
  return *it->second;
}

void PoolEngine::ensure_ring(Dev& d, Ring& r, bool) {
  if (r.base) return;
  DeviceGuard g(d.device);
  void* p = nullptr;
  PPB_CUDA(cudaMalloc(&p, options_.slot_bytes * options_.slots));
  PPB_CUDA(cudaMemset(p, 0, options_.slot_bytes * options_.slots));
  r.base = static_cast<uint8_t*>(p);
}

cudaEvent_t PoolEngine::take_event(Dev& d) {
  if (!d.free_events.empty()) {
    cudaEvent_t e = d.free_events.back();
    d.free_events.pop_back();
    return e;
  }
  DeviceGuard g(d.device);
  cudaEvent_t e;
  PPB_CUDA(cudaEventCreate(&e));
  return e;
}

void PoolEngine::give_event(Dev& d, cudaEvent_t e) {
  if (e) d.free_events.push_back(e);
}

std::pair<uint8_t*, size_t> PoolEngine::take_scratch(Dev& d, size_t bytes) {
  // Smallest free buffer that fits; else a new one (rounded up to 1 MiB so a
  // few sizes cover every transfer; made once, then reused).
  size_t best = d.free_scratch.size();
  for (size_t i = 0; i < d.free_scratch.size(); ++i) {
    if (d.free_scratch[i].second >= bytes &&
        (best == d.free_scratch.size() || d.free_scratch[i].second < d.free_scratch[best].second))
      best = i;
  }
  if (best != d.free_scratch.size()) {
    auto b = d.free_scratch[best];
    d.free_scratch.erase(d.free_scratch.begin() + static_cast<long>(best));
    return b;
  }
  const size_t cap = align_up(std::max<size_t>(bytes, 1), size_t(1) << 20);
  DeviceGuard g(d.device);
  void* p = nullptr;
  PPB_CUDA(cudaMalloc(&p, cap));
  return {static_cast<uint8_t*>(p), cap};
}

void PoolEngine::give_scratch(Dev& d, std::pair<uint8_t*, size_t> b) {
  if (b.first) d.free_scratch.push_back(b);
}

void* PoolEngine::take_pinned(size_t bytes) {
  bytes = std::max<size_t>(align_up(bytes, 4096), 65536);
  for (size_t i = 0; i < pinned_free_.size(); ++i) {
    if (pinned_free_[i].second >= bytes) {
      auto e = pinned_free_[i];
      pinned_free_.erase(pinned_free_.begin() + static_cast<long>(i));
      pinned_used_[e.first] = e.second;
      return e.first;
    }
  }
  void* p = nullptr;
  PPB_CUDA(cudaMallocHost(&p, bytes));
  pinned_used_[p] = bytes;
  return p;
}

void PoolEngine::give_pinned(void* p) {
  if (!p) return;
  auto it = pinned_used_.find(p);
  if (it == pinned_used_.end()) return;
  pinned_free_.emplace_back(it->first, it->second);
  pinned_used_.erase(it);
}

uint64_t PoolEngine::relay_ring(int device) {
  std::lock_guard<std::mutex> g(mu_);
  Dev& d = dev(device);
  ensure_ring(d, d.relay[0], true);
  return reinterpret_cast<uint64_t>(d.relay[0].base);
}

uint64_t PoolEngine::mailbox(int device) {
  std::lock_guard<std::mutex> g(mu_);
  return reinterpret_cast<uint64_t>(dev(device).mbox);
}

std::vector<uint64_t> PoolEngine::issued(int device) {
  std::lock_guard<std::mutex> g(mu_);
  Dev& d = dev(device);
  return {d.relay[0].issued, d.land[0].issued, d.relay[1].issued, d.land[1].issued};
}

int PoolEngine::max_lane_ctas(int device) {
  std::lock_guard<std::mutex> g(mu_);
  return dev(device).max_ctas;
}

// Reset the counters of rings that saw an error once nothing uses them.
void PoolEngine::reset_rings(Pending& P) {
  for (size_t i = 0; i < P.rings.size(); ++i) {
    Ring* r = P.rings[i];
    if (!r->poisoned) continue;
    DeviceGuard g(P.ring_devices[i]);
    cudaMemset(r->ready, 0, 4);
    cudaMemset(r->freec, 0, 4);
    cudaMemset(r->donec, 0, 4);
    cudaDeviceSynchronize();
    r->issued = 0;
    r->poisoned = false;
    r->last_dir = -1;
    r->last_target = -1;
  }
  cudaGetLastError();
}

namespace {

void validate_spec(const TransferSpec& s, uint64_t slot_bytes, size_t slots) {
  if (s.direction != 0 && s.direction != 1) throw std::invalid_argument("direction must be 0 or 1");
  if (s.host_ptr == 0 || s.dev_ptr == 0) throw std::invalid_argument("null buffer pointer");
  if (s.lanes.empty()) throw std::invalid_argument("transfer has no lanes");
  const bool h2d = s.direction == 0;
  switch (s.op) {
    case kOpCopy:
      break;
    case kOpScatterUnits:
    case kOpFp8Quant:
    case kOpScatterRanges:
      if (!h2d) throw std::invalid_argument("scatter/fp8 ops land data: H2D only");
      break;
    case kOpGatherUnits:
    case kOpGatherRanges:
      if (h2d) throw std::invalid_argument("gather ops push data: D2H only");
      break;
    case kOpAdamW:
      if (!h2d) throw std::invalid_argument("the streamed optimizer step is an H2D round trip");
      if (s.adam.nparams == 0 || s.adam.grads == 0 || s.adam.params == 0 || s.adam.grads % 16 != 0 ||
          s.adam.params % 16 != 0)
        throw std::invalid_argument("adamw needs 16-byte aligned grads and params and nparams > 0");
      if (s.adam.step < 1) throw std::invalid_argument("adamw step must be >= 1");
      if (s.host_ptr % 16 != 0) throw std::invalid_argument("adamw state image must be 16-byte aligned");
      break;
    default:
      throw std::invalid_argument("unknown lane op");
  }
  if (s.op == kOpScatterUnits || s.op == kOpGatherUnits) {
    if (s.unit_bytes == 0 || s.unit_bytes % 16 != 0)
      throw std::invalid_argument("unit_bytes must be a positive multiple of 16");
    for (uint64_t a : s.unit_addrs)
      if (a == 0 || a % 16 != 0) throw std::invalid_argument("unit address must be 16-byte aligned");
  }
  if (s.op == kOpScatterRanges || s.op == kOpGatherRanges) {
    if (s.range_addrs.size() != s.range_bytes.size() || s.range_pos.size() != s.range_bytes.size())
      throw std::invalid_argument("range tables must have equal lengths");
    for (size_t i = 0; i < s.range_bytes.size(); ++i) {
      if (s.range_bytes[i] == 0 || s.range_bytes[i] > kTileBytes || s.range_bytes[i] % 16 != 0 ||
          s.range_addrs[i] % 16 != 0 || s.range_pos[i] % 16 != 0)
        throw std::invalid_argument(
            "ranges must be 16-byte aligned, non-empty and at most one tile (32 KiB)");
    }
  }
  for (const auto& L : s.lanes) {
    for (const auto& c : L.chunks) {
      if (c.bytes == 0) throw std::invalid_argument("empty chunk");
      if (c.bytes > 0xffffffffull) throw std::invalid_argument("chunk larger than 4 GiB");
      const uint64_t host_off = h2d ? c.src_off : c.dst_off;
      const uint64_t dev_off = h2d ? c.dst_off : c.src_off;
      if (host_off + c.bytes > s.host_bytes) throw std::invalid_argument("chunk exceeds host buffer");
      if (s.op == kOpCopy && dev_off + c.bytes > s.dev_bytes)
        throw std::invalid_argument("chunk exceeds device buffer");
      const bool staged = L.device != s.target || s.op != kOpCopy || s.stage_direct;
      if (staged && c.bytes > slot_bytes)
        throw std::invalid_argument("chunk larger than the staging slot");
      if (staged && s.serialize && L.chunks.size() > slots)
        throw std::invalid_argument("serialized transfer: a staged lane holds more chunks than slots");
      if (s.op == kOpScatterUnits || s.op == kOpGatherUnits) {
        if (c.bytes % s.unit_bytes != 0) throw std::invalid_argument("chunk not a whole number of units");
        if (uint64_t(c.unit0) + c.bytes / s.unit_bytes > s.unit_addrs.size())
          throw std::invalid_argument("chunk units exceed the unit table");
      }
      if (s.op == kOpScatterRanges || s.op == kOpGatherRanges) {
        if (c.count == 0 || uint64_t(c.unit0) + c.count > s.range_bytes.size())
          throw std::invalid_argument("chunk ranges exceed the range table");
        uint64_t sum = 0;
        for (uint32_t k = 0; k < c.count; ++k) {
          if (s.range_pos[c.unit0 + k] != sum) throw std::invalid_argument("range positions must be packed");
          sum += s.range_bytes[c.unit0 + k];
        }
        if (sum != c.bytes) throw std::invalid_argument("chunk bytes must equal its ranges");
      }
      if (s.op == kOpAdamW) {
        const uint64_t tiles = (s.adam.nparams + kAdamTileParams - 1) / kAdamTileParams;
        if (c.bytes % kAdamTileBytes != 0 || c.src_off % 16 != 0)
          throw std::invalid_argument("adamw chunks must be whole 16-byte aligned state tiles");
        if (uint64_t(c.unit0) + c.bytes / kAdamTileBytes > tiles)
          throw std::invalid_argument("adamw chunk tiles exceed the parameter count");
        if (c.src_off != uint64_t(c.unit0) * kAdamTileBytes)
          throw std::invalid_argument("adamw chunk offset must match its first tile");
      }
      if (s.op == kOpFp8Quant) {
        if (c.tensor >= s.tensors.size()) throw std::invalid_argument("fp8 tensor index out of range");
        const auto& T = s.tensors[c.tensor];
        if (T.cols == 0 || T.cols % 128 != 0) throw std::invalid_argument("fp8 landing needs cols % 128 == 0");
        const uint64_t rb = uint64_t(T.cols) * 2;
        if (c.bytes % rb != 0) throw std::invalid_argument("fp8 chunk must hold whole rows");
        if (c.unit0 % 128 != 0) throw std::invalid_argument("fp8 chunk must start on a 128-row tile");
        if (uint64_t(c.unit0) + c.bytes / rb > T.rows) throw std::invalid_argument("fp8 chunk rows exceed tensor");
        if (T.q == 0 || T.scales == 0 || T.q % 16 != 0 || T.scales % 4 != 0)
          throw std::invalid_argument("fp8 outputs must be aligned device buffers");
      }
    }
  }
}

}  // namespace

uint64_t PoolEngine::submit(const TransferSpec& s) {
  std::lock_guard<std::mutex> guard(mu_);
  validate_spec(s, options_.slot_bytes, static_cast<size_t>(options_.slots));
  const bool h2d = s.direction == 0;
  Dev& T = dev(s.target);
  for (const auto& L : s.lanes) dev(L.device);  // every lane device is managed
  if (!is_pinned_host(reinterpret_cast<void*>(s.host_ptr)))
    throw std::invalid_argument("host buffer is not page-locked (register it first)");

  auto Pp = std::make_unique<Pending>();
  Pending& P = *Pp;
  P.id = next_id_.fetch_add(1);
  P.target = s.target;
  P.direction = s.direction;
  P.timeout_s = s.timeout_s > 0 ? s.timeout_s : options_.timeout_s;
  P.t_submit = std::chrono::steady_clock::now();
  P.nvtx = nvtx_start("transfer " + std::to_string(P.id) + (s.direction == 0 ? " h2d" : " d2h") + " target " +
                          std::to_string(s.target) + " lanes " + std::to_string(s.lanes.size()) + " op " +
                          std::to_string(s.op),
                      0xFF2E86C1u);

  // ---- classify lanes --------------------------------------------------------
  for (const auto& L : s.lanes) {
    Pending::LaneRec R;
    R.device = L.device;
    R.direct = L.device == s.target;
    R.d = &dev(L.device);
    R.staged = !R.direct || s.op != kOpCopy || s.stage_direct;
    R.in_place = R.direct && !R.staged && s.checksum;
    R.kernel = R.staged || R.in_place;
    if (R.staged) {
      R.ring = R.direct ? &T.land[s.direction] : &R.d->relay[s.direction];
      ensure_ring(*R.d, *R.ring, !R.direct);
    } else if (R.in_place && h2d) {
      R.ring = &T.land[0];  // counters only: CE publishes, the kernel verifies in place
    }
    R.stream = R.d->copy[s.direction];
    R.roundtrip = s.op == kOpAdamW;
    if (R.roundtrip) R.out = R.d->copy[1];
    for (const auto& c : L.chunks) R.bytes += c.bytes;
    R.chunks = L.chunks.size();
    P.bytes += R.bytes;
    P.lanes.push_back(R);
  }

  // ---- footprint, for ordering against the other direction ---------------------
  P.host_lo = s.host_ptr;
  P.host_hi = s.host_ptr + s.host_bytes;
  P.dev_known = s.op == kOpCopy;
  P.dev_lo = s.dev_ptr;
  P.dev_hi = s.dev_ptr + s.dev_bytes;

  // ---- ring hand-over: a ring whose target changes must be idle -----------------
  for (auto& R : P.lanes) {
    if (!R.ring) continue;
    if (std::find(P.rings.begin(), P.rings.end(), R.ring) != P.rings.end()) {
      throw std::invalid_argument("two lanes of one transfer use the same device");
    }
    P.rings.push_back(R.ring);
    P.ring_devices.push_back(R.d->device);
  }
  for (size_t i = 0; i < P.rings.size(); ++i) {
    Ring* r = P.rings[i];
    const bool switching = r->last_dir != -1 && (r->last_dir != s.direction || r->last_target != s.target);
    if (switching || r->poisoned) {
      // Drain the pending transfers that use this ring (bounded) so no other
      // producer/consumer still advances its counters.
      for (auto& kv : pending_) {
        const auto& kr = kv.second->rings;
        if (std::find(kr.begin(), kr.end(), r) == kr.end()) continue;
        const auto deadline = std::chrono::steady_clock::now() +
                              std::chrono::duration<double>(kv.second->timeout_s * 2 + 5);
        while (cudaEventQuery(kv.second->stop) == cudaErrorNotReady) {
          if (std::chrono::steady_clock::now() > deadline)
            throw std::runtime_error("ring hand-over: previous transfer did not finish");
          std::this_thread::sleep_for(std::chrono::microseconds(100));
        }
      }
      cudaGetLastError();
      if (r->poisoned) {
        Pending tmp;
        tmp.rings = {r};
        tmp.ring_devices = {P.ring_devices[i]};
        reset_rings(tmp);
      }
    }
  }

  // ---- kernel tables ---------------------------------------------------------
  std::vector<LaneDesc> lanes_d;
  std::vector<ChunkDesc> chunks_d;
  int kernel_lanes = 0;
  for (const auto& R : P.lanes) kernel_lanes += R.kernel ? 1 : 0;
  int cpl = s.ctas_per_lane > 0 ? s.ctas_per_lane : options_.ctas_per_lane;
  if (kernel_lanes > 0) {
    if (T.max_ctas <= 0) throw std::runtime_error("lane kernel cannot be resident on target");
    const int budget = direction_cta_budget(T.max_ctas, h2d);
    if (kernel_lanes > budget) throw std::invalid_argument("more kernel lanes than resident CTAs");
    cpl = std::max(1, std::min(cpl, budget / kernel_lanes));
  }
  uint32_t cta = 0;
  for (size_t li = 0; li < s.lanes.size(); ++li) {
    auto& R = P.lanes[li];
    const auto& L = s.lanes[li];
    if (R.ring) R.seq0 = R.ring->issued;
    if (R.kernel) {
      P.kernel_lane_to_spec.push_back(static_cast<int>(li));
      LaneDesc d{};
      d.ring = R.staged ? R.ring->base : nullptr;
      d.ready = R.ring ? R.ring->ready : nullptr;
      // a round trip's slots are freed by its copy-out stream, not the kernel
      d.freec = R.ring && !R.roundtrip ? R.ring->freec : nullptr;
      d.donec = R.roundtrip ? R.ring->donec : nullptr;
      d.slot_bytes = options_.slot_bytes;
      d.slots = static_cast<uint32_t>(options_.slots);
      d.chunk_begin = static_cast<uint32_t>(chunks_d.size());
      d.chunk_count = static_cast<uint32_t>(L.chunks.size());
      d.cta_begin = cta;
      d.cta_count = static_cast<uint32_t>(cpl);
      d.in_place = R.in_place ? 1u : 0u;
      cta += static_cast<uint32_t>(cpl);
      R.first_chunk = static_cast<int>(chunks_d.size());
      for (size_t k = 0; k < L.chunks.size(); ++k) {
        const auto& c = L.chunks[k];
        ChunkDesc cd{};
        cd.dev_off = h2d ? c.dst_off : c.src_off;
        cd.host_off = h2d ? c.src_off : c.dst_off;
        cd.bytes = static_cast<uint32_t>(c.bytes);
        cd.seq = R.ring ? static_cast<uint32_t>(R.seq0 + k + 1) : 0u;
        cd.slot = R.ring ? static_cast<uint32_t>((R.seq0 + k) % options_.slots) : 0u;
        cd.unit0 = c.unit0;
        cd.tensor = c.tensor;
        cd.count = c.count;
        chunks_d.push_back(cd);
      }
      lanes_d.push_back(d);
    }
    if (R.ring) R.ring->issued += L.chunks.size();
  }
  // spec-order chunk -> kernel chunk
  for (size_t li = 0; li < s.lanes.size(); ++li) {
    for (size_t k = 0; k < s.lanes[li].chunks.size(); ++k) {
      P.spec_chunk_to_kernel.push_back(P.lanes[li].kernel ? P.lanes[li].first_chunk + int(k) : -1);
    }
  }
  P.total_chunks = P.spec_chunk_to_kernel.size();
  P.kernel_chunks = chunks_d.size();
  P.has_kernel = kernel_lanes > 0;

  // ---- device scratch layout ----------------------------------------------------
  const size_t nk = std::max<size_t>(chunks_d.size(), 1);
  size_t off = 0;
  const size_t o_lanes = off; off = align_up(off + lanes_d.size() * sizeof(LaneDesc), 256);
  const size_t o_chunks = off; off = align_up(off + chunks_d.size() * sizeof(ChunkDesc), 256);
  const size_t o_units = off; off = align_up(off + s.unit_addrs.size() * 8, 256);
  const size_t o_raddr = off; off = align_up(off + s.range_addrs.size() * 8, 256);
  const size_t o_rbytes = off; off = align_up(off + s.range_bytes.size() * 4, 256);
  const size_t o_rpos = off; off = align_up(off + s.range_pos.size() * 8, 256);
  const size_t o_tensors = off; off = align_up(off + s.tensors.size() * sizeof(QuantTensor), 256);
  const size_t upload_bytes = off;
  const size_t o_csum = off; off = align_up(off + nk * 16, 256);
  const size_t o_status = off; off = align_up(off + 16, 256);
  const size_t o_trace = off; off = align_up(off + (s.trace ? nk * kTraceWords * 8 : 0), 256);
  const size_t o_done = off; off = align_up(off + nk * 4, 256);
  const size_t scratch_bytes = off;
  const size_t result_bytes = o_done - o_csum;  // csum + status (+ trace)
  P.trace = s.trace;

  DeviceGuard tg(s.target);
  P.start = take_event(T);
  P.stop = take_event(T);
  P.kern_done = take_event(T);
  for (auto& R : P.lanes) {
    R.t0 = take_event(*R.d);
    R.t1 = take_event(*R.d);
    if (R.roundtrip) {
      R.t_in = take_event(*R.d);
      R.t_out = take_event(*R.d);
    }
  }

  cudaStream_t tmain = T.main[s.direction];
  cudaStream_t tkern = T.kern[s.direction];
  // Order after pending transfers of the other direction on this target that
  // touch the same host or device bytes (save-then-restore of one region).
  for (auto& kv : pending_) {
    const Pending& Q = *kv.second;
    if (Q.target != s.target || Q.direction == s.direction) continue;
    const bool host_overlap = Q.host_lo < P.host_hi && P.host_lo < Q.host_hi;
    const bool dev_overlap = !Q.dev_known || !P.dev_known || (Q.dev_lo < P.dev_hi && P.dev_lo < Q.dev_hi);
    if (host_overlap || dev_overlap) PPB_CUDA(cudaStreamWaitEvent(tmain, Q.stop, 0));
  }
  PPB_CUDA(cudaEventRecord(P.start, tmain));
  for (auto& R : P.lanes) {
    DeviceGuard lg(R.device);
    PPB_CUDA(cudaStreamWaitEvent(R.stream, P.start, 0));
    PPB_CUDA(cudaEventRecord(R.t0, R.stream));
    if (R.roundtrip) PPB_CUDA(cudaStreamWaitEvent(R.out, P.start, 0));
  }

  // Pipelined (default): the kernel is queued before any copy-engine work so a
  // failed launch leaves no relay stream waiting on it.  Serialised: H2D
  // launches after the copies (below); D2H copies start after the kernel.
  const bool kernel_after_copies = s.serialize && h2d;
  auto launch_kernel = [&]() {
    if (!P.has_kernel) return;
    P.desc_host = take_pinned(upload_bytes + 256);
    P.result_host = take_pinned(result_bytes + 256);
    uint8_t* h = static_cast<uint8_t*>(P.desc_host);
    std::memset(h, 0, upload_bytes);
    auto put = [&](size_t o, const void* src, size_t n) { if (n) std::memcpy(h + o, src, n); };
    put(o_lanes, lanes_d.data(), lanes_d.size() * sizeof(LaneDesc));
    put(o_chunks, chunks_d.data(), chunks_d.size() * sizeof(ChunkDesc));
    put(o_units, s.unit_addrs.data(), s.unit_addrs.size() * 8);
    put(o_raddr, s.range_addrs.data(), s.range_addrs.size() * 8);
    put(o_rbytes, s.range_bytes.data(), s.range_bytes.size() * 4);
    put(o_rpos, s.range_pos.data(), s.range_pos.size() * 8);
    std::vector<QuantTensor> qt;
    for (const auto& t : s.tensors)
      qt.push_back(QuantTensor{reinterpret_cast<uint8_t*>(t.q), reinterpret_cast<float*>(t.scales), t.rows, t.cols});
    put(o_tensors, qt.data(), qt.size() * sizeof(QuantTensor));

    P.scratch = take_scratch(T, scratch_bytes);
    PPB_CUDA(cudaStreamWaitEvent(tkern, P.start, 0));
    uint8_t* dsc = P.scratch.first;
    PPB_CUDA(cudaMemcpyAsync(dsc, h, upload_bytes, cudaMemcpyHostToDevice, tkern));
    PPB_CUDA(cudaMemsetAsync(dsc + o_csum, 0, scratch_bytes - o_csum, tkern));

    LaneKernelParams kp{};
    kp.lanes = reinterpret_cast<const LaneDesc*>(dsc + o_lanes);
    kp.chunks = reinterpret_cast<const ChunkDesc*>(dsc + o_chunks);
    kp.num_lanes = static_cast<uint32_t>(lanes_d.size());
    kp.op = static_cast<uint32_t>(s.op);
    kp.dev = reinterpret_cast<uint8_t*>(s.dev_ptr);
    kp.unit_addr = reinterpret_cast<const uint64_t*>(dsc + o_units);
    kp.range_addr = reinterpret_cast<const uint64_t*>(dsc + o_raddr);
    kp.range_bytes = reinterpret_cast<const uint32_t*>(dsc + o_rbytes);
    kp.range_pos = reinterpret_cast<const uint64_t*>(dsc + o_rpos);
    kp.unit_bytes = s.unit_bytes;
    kp.checksum = s.checksum ? 1u : 0u;
    kp.tensors = reinterpret_cast<const QuantTensor*>(dsc + o_tensors);
    kp.done = reinterpret_cast<uint32_t*>(dsc + o_done);
    kp.csum = reinterpret_cast<unsigned long long*>(dsc + o_csum);
    kp.status = reinterpret_cast<int*>(dsc + o_status);
    kp.timeout_ns = static_cast<uint64_t>(P.timeout_s * 1e9);
    kp.trace = s.trace ? reinterpret_cast<unsigned long long*>(dsc + o_trace) : nullptr;
    if (s.op == kOpAdamW) {
      const auto& a = s.adam;
      kp.grads = reinterpret_cast<const uint16_t*>(a.grads);
      kp.params_out = reinterpret_cast<uint16_t*>(a.params);
      kp.nparams = a.nparams;
      kp.adam = AdamCoeffs::make(a.lr, a.beta1, a.beta2, a.eps, a.weight_decay, a.grad_scale, a.step);
    }
    // Launch before any copy-engine work is queued: if the launch fails no
    // relay stream is left waiting for a kernel that never runs.
    cudaError_t lrc;
    {
      NvtxScope k(std::string(h2d ? "land_kernel" : "push_kernel") + " launch: " + std::to_string(cta) + " CTAs, " +
                      std::to_string(chunks_d.size()) + " chunks",
                  0xFF28B463u);
      lrc = h2d ? launch_land(kp, static_cast<int>(cta), tkern) : launch_push(kp, static_cast<int>(cta), tkern);
    }
    if (lrc != cudaSuccess) {
      cudaStreamSynchronize(tkern);  // the scratch upload is done before reuse
      give_scratch(T, P.scratch);
      P.scratch = {nullptr, 0};
      for (auto& R : P.lanes) {
        if (!R.ring) continue;
        R.ring->issued = R.seq0;
        // serialised H2D: the copies already published their chunks
        if (kernel_after_copies) R.ring->poisoned = true;
      }
      give_pinned(P.desc_host);
      give_pinned(P.result_host);
      check_cuda(lrc, "lane kernel launch");
    }
    PPB_CUDA(cudaMemcpyAsync(P.result_host, dsc + o_csum, result_bytes, cudaMemcpyDeviceToHost, tkern));
    PPB_CUDA(cudaEventRecord(P.kern_done, tkern));
  };

  // ---- copy-engine side, chunks interleaved round-robin across lanes ------------
  const uint8_t* host = reinterpret_cast<const uint8_t*>(s.host_ptr);
  uint8_t* devp = reinterpret_cast<uint8_t*>(s.dev_ptr);
  std::vector<size_t> next(s.lanes.size(), 0);
  std::vector<uint64_t> left(s.lanes.size(), 0);
  for (size_t li = 0; li < s.lanes.size(); ++li)
    for (const auto& c : s.lanes[li].chunks) left[li] += c.bytes;
  // Lanes whose copies depend on nothing (a direct lane copying straight to
  // or from its final place) are queued first, so their copy engine starts
  // while the kernel's descriptors are still being prepared; a failed kernel
  // launch leaves them nothing to wait for.
  const bool direct_first = !s.serialize;
  auto enqueue = [&](bool unstaged_only) {
  bool any = true;
  while (any) {
    any = false;
    for (size_t li = 0; li < s.lanes.size(); ++li) {
      const auto& L = s.lanes[li];
      auto& R = P.lanes[li];
      if (unstaged_only && R.staged) continue;
      const size_t k = next[li];
      if (k >= L.chunks.size()) continue;
      any = true;
      next[li] = k + 1;
      const auto& c = L.chunks[k];
      DeviceGuard lg(R.device);
      if (!R.staged) {
        // Plain direct lane: merge chunks that are contiguous on both sides
        // into one copy-engine transfer and publish the last chunk's
        // sequence number once for the group.  A group takes at most half of
        // the lane's remaining bytes (and at most coalesce_bytes), so the
        // groups shrink towards the end: the kernel's in-place checksum of a
        // group overlaps the copy of the next, and what is left after the
        // last copy is one chunk's checksum.
        const uint64_t cap = std::min<uint64_t>(options_.coalesce_bytes, std::max<uint64_t>(c.bytes, left[li] / 2));
        size_t end = k + 1;
        uint64_t run = c.bytes;
        while (end < L.chunks.size()) {
          const auto& nx = L.chunks[end];
          const auto& pv = L.chunks[end - 1];
          if (nx.src_off != pv.src_off + pv.bytes || nx.dst_off != pv.dst_off + pv.bytes ||
              run + nx.bytes > cap)
            break;
          run += nx.bytes;
          ++end;
        }
        next[li] = end;
        left[li] -= run;
        const uint32_t last_seq = R.ring ? static_cast<uint32_t>(R.seq0 + end) : 0u;
        const bool pub = static_cast<int>(li) != s.debug_drop_publish;
        if (h2d) {
          PPB_CUDA(cudaMemcpyAsync(devp + c.dst_off, host + c.src_off, run, cudaMemcpyHostToDevice, R.stream));
          if (R.in_place && pub) stream_write(R.stream, R.ring->ready, last_seq);
        } else {
          PPB_CUDA(cudaMemcpyAsync(const_cast<uint8_t*>(host) + c.dst_off, devp + c.src_off, run,
                                   cudaMemcpyDeviceToHost, R.stream));
        }
        continue;
      }
      const uint32_t seq = R.ring ? static_cast<uint32_t>(R.seq0 + k + 1) : 0u;
      uint8_t* slot = R.staged ? R.ring->base + ((R.seq0 + k) % options_.slots) * options_.slot_bytes : nullptr;
      const bool publish = static_cast<int>(li) != s.debug_drop_publish;
      if (h2d) {
        if (R.staged) {
          stream_wait_geq(R.stream, R.ring->freec, seq - static_cast<uint32_t>(options_.slots), false);
          PPB_CUDA(cudaMemcpyAsync(slot, host + c.src_off, c.bytes, cudaMemcpyHostToDevice, R.stream));
          if (publish) stream_write(R.stream, R.ring->ready, seq);
          if (R.roundtrip) {
            // copy-out leg: once the kernel has updated the chunk in the slot
            stream_wait_geq(R.out, R.ring->donec, seq, R.d->can_flush_remote_writes);
            PPB_CUDA(cudaMemcpyAsync(const_cast<uint8_t*>(host) + c.src_off, slot, c.bytes,
                                     cudaMemcpyDeviceToHost, R.out));
            stream_write(R.out, R.ring->freec, seq);
          }
        } else {
          PPB_CUDA(cudaMemcpyAsync(devp + c.dst_off, host + c.src_off, c.bytes, cudaMemcpyHostToDevice, R.stream));
          if (R.in_place && publish) stream_write(R.stream, R.ring->ready, seq);
        }
      } else {
        uint8_t* hdst = const_cast<uint8_t*>(host) + c.dst_off;
        if (R.staged) {
          stream_wait_geq(R.stream, R.ring->ready, seq, R.d->can_flush_remote_writes);
          PPB_CUDA(cudaMemcpyAsync(hdst, slot, c.bytes, cudaMemcpyDeviceToHost, R.stream));
          stream_write(R.stream, R.ring->freec, seq);
        } else {
          PPB_CUDA(cudaMemcpyAsync(hdst, devp + c.src_off, c.bytes, cudaMemcpyDeviceToHost, R.stream));
        }
      }
    }
  }

  };
  {
    NvtxScope enqueue_scope("copy-engine enqueue: " + std::to_string(s.lanes.size()) + " lanes", 0xFFF39C12u);
    if (direct_first) enqueue(true);
  }
  if (!kernel_after_copies) launch_kernel();
  if (s.serialize && !h2d && P.has_kernel) {
    for (auto& R : P.lanes) {
      DeviceGuard lg(R.device);
      PPB_CUDA(cudaStreamWaitEvent(R.stream, P.kern_done, 0));
    }
  }
  {
    NvtxScope enqueue_scope("copy-engine enqueue: " + std::to_string(s.lanes.size()) + " lanes", 0xFFF39C12u);
    enqueue(false);
  }

  for (auto& R : P.lanes) {
    DeviceGuard lg(R.device);
    if (R.roundtrip) {
      // the lane ends when its copy-out leg ends
      PPB_CUDA(cudaEventRecord(R.t_in, R.stream));
      PPB_CUDA(cudaEventRecord(R.t_out, R.out));
      PPB_CUDA(cudaStreamWaitEvent(R.stream, R.t_out, 0));
    }
    PPB_CUDA(cudaEventRecord(R.t1, R.stream));
  }
  if (kernel_after_copies && P.has_kernel) {
    DeviceGuard kg(s.target);
    for (auto& R : P.lanes) PPB_CUDA(cudaStreamWaitEvent(tkern, R.roundtrip ? R.t_in : R.t1, 0));
    launch_kernel();
  }
  PPB_CUDA(cudaSetDevice(s.target));
  for (auto& R : P.lanes) PPB_CUDA(cudaStreamWaitEvent(tmain, R.t1, 0));
  if (P.has_kernel) PPB_CUDA(cudaStreamWaitEvent(tmain, P.kern_done, 0));
  PPB_CUDA(cudaEventRecord(P.stop, tmain));

  for (size_t i = 0; i < P.rings.size(); ++i) {
    P.rings[i]->last_dir = s.direction;
    P.rings[i]->last_target = s.target;
  }
  const uint64_t id = P.id;
  pending_[id] = std::move(Pp);
  return id;
}

bool PoolEngine::query(uint64_t id) {
  std::lock_guard<std::mutex> g(mu_);
  auto it = pending_.find(id);
  if (it == pending_.end()) throw std::invalid_argument("unknown transfer id");
  const cudaError_t rc = cudaEventQuery(it->second->stop);
  if (rc == cudaErrorNotReady) return false;
  check_cuda(rc, "cudaEventQuery");
  return true;
}

TransferResult PoolEngine::wait(uint64_t id, double host_timeout_s) {
  std::unique_ptr<Pending> Pp;
  cudaEvent_t stop = nullptr;
  double tmo = 0.0;
  {
    std::lock_guard<std::mutex> g(mu_);
    auto it = pending_.find(id);
    if (it == pending_.end()) throw std::invalid_argument("unknown transfer id");
    stop = it->second->stop;
    tmo = host_timeout_s > 0 ? host_timeout_s : it->second->timeout_s * 2 + 10.0;
  }
  // Poll without holding the lock so other threads can keep submitting.
  const auto t_wait = std::chrono::steady_clock::now();
  const auto deadline = t_wait + std::chrono::duration<double>(tmo);
  bool done = false;
  bool rescued = false;
  while (true) {
    const cudaError_t rc = cudaEventQuery(stop);
    if (rc == cudaSuccess) { done = true; break; }
    if (rc != cudaErrorNotReady) { check_cuda(rc, "cudaEventQuery(transfer stop)"); }
    const auto now = std::chrono::steady_clock::now();
    if (now > deadline) break;
    // Small transfers finish within tens of microseconds: poll without
    // sleeping for the first 200 us, then back off to 20 us sleeps.
    if (now - t_wait < std::chrono::microseconds(200)) {
      std::this_thread::yield();
    } else {
      std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
  }
  const auto t_done = std::chrono::steady_clock::now();
  std::lock_guard<std::mutex> g(mu_);
  auto it = pending_.find(id);
  Pp = std::move(it->second);
  pending_.erase(it);
  Pending& P = *Pp;
  if (P.nvtx) nvtxDomainRangeEnd(nvtx_domain(), P.nvtx);
  if (!done) {
    // Watchdog: something never advanced (kernel not scheduled, peer stuck).
    // Push every counter of this transfer far ahead from the host so no copy
    // engine stays parked in a stream wait, then give it a bounded drain.
    rescued = true;
    for (size_t i = 0; i < P.rings.size(); ++i) {
      Ring* r = P.rings[i];
      DeviceGuard dg(P.ring_devices[i]);
      const uint32_t v = static_cast<uint32_t>(r->issued) + kRescueStride;
      cudaStream_t rs;
      if (cudaStreamCreateWithFlags(&rs, cudaStreamNonBlocking) == cudaSuccess) {
        cudaMemcpyAsync(r->ready, &v, 4, cudaMemcpyHostToDevice, rs);
        cudaMemcpyAsync(r->freec, &v, 4, cudaMemcpyHostToDevice, rs);
        cudaMemcpyAsync(r->donec, &v, 4, cudaMemcpyHostToDevice, rs);
        cudaStreamSynchronize(rs);
        cudaStreamDestroy(rs);
      }
      r->poisoned = true;
    }
    const auto d2 = std::chrono::steady_clock::now() + std::chrono::duration<double>(P.timeout_s + 5);
    while (cudaEventQuery(stop) == cudaErrorNotReady && std::chrono::steady_clock::now() < d2)
      std::this_thread::sleep_for(std::chrono::microseconds(200));
    cudaGetLastError();
  }

  TransferResult res;
  res.id = P.id;
  res.bytes = P.bytes;
  res.submit_to_complete_ms =
      std::chrono::duration<double, std::milli>(t_done - P.t_submit).count();
  if (done) {
    res.cuda_ms = event_ms(P.start, P.stop);
    if (res.cuda_ms > 0) res.gib_per_s = (double(P.bytes) / double(1ull << 30)) / (res.cuda_ms / 1e3);
  }
  for (auto& R : P.lanes) {
    LaneStats ls;
    ls.device = R.device;
    ls.direct = R.direct;
    ls.bytes = R.bytes;
    ls.chunks = R.chunks;
    if (done) ls.cuda_ms = event_ms(R.t0, R.t1);
    res.lanes.push_back(ls);
  }
  res.checksums.assign(P.total_chunks * 2, 0);
  int code = 0;
  if (P.has_kernel && done) {
    const uint8_t* rh = static_cast<const uint8_t*>(P.result_host);
    const size_t nk = std::max<size_t>(P.kernel_chunks, 1);
    const uint64_t* cs = reinterpret_cast<const uint64_t*>(rh);
    const int* st = reinterpret_cast<const int*>(rh + align_up(nk * 16, 256));
    for (size_t i = 0; i < P.spec_chunk_to_kernel.size(); ++i) {
      const int kc = P.spec_chunk_to_kernel[i];
      if (kc >= 0) {
        res.checksums[2 * i] = cs[2 * kc];
        res.checksums[2 * i + 1] = cs[2 * kc + 1];
      }
    }
    if (P.trace) {
      const uint64_t* tr = reinterpret_cast<const uint64_t*>(rh + align_up(nk * 16, 256) + 256);
      res.trace.assign(P.total_chunks * kTraceWords, 0);
      for (size_t i = 0; i < P.spec_chunk_to_kernel.size(); ++i) {
        const int kc = P.spec_chunk_to_kernel[i];
        if (kc >= 0)
          for (int w = 0; w < kTraceWords; ++w) res.trace[kTraceWords * i + w] = tr[kTraceWords * kc + w];
      }
    }
    code = st[0];
    // the kernel reports its own lane / chunk indices: map them to spec order
    res.error_lane = st[1];
    if (st[1] >= 0 && static_cast<size_t>(st[1]) < P.kernel_lane_to_spec.size())
      res.error_lane = P.kernel_lane_to_spec[st[1]];
    res.error_chunk = st[2];
    for (size_t i = 0; st[2] >= 0 && i < P.spec_chunk_to_kernel.size(); ++i) {
      if (P.spec_chunk_to_kernel[i] == st[2]) {
        res.error_chunk = static_cast<int>(i);
        break;
      }
    }
    res.error_detail = st[3];
  }
  if (!done) {
    res.status_code = -1;
    res.error = "transfer did not complete within the host timeout (watchdog released its lanes)";
  } else if (code != 0) {
    res.status_code = code;
    static const char* names[] = {"ok", "timeout waiting for a staged chunk", "timeout in a bulk copy",
                                  "bad argument", "timeout waiting for a free staging slot"};
    res.error = std::string("lane kernel error: ") + (code >= 0 && code <= 4 ? names[code] : "unknown");
    for (Ring* r : P.rings) r->poisoned = true;
  }
  res.ok = done && code == 0;
  // Return resources.
  Dev& T = dev(P.target);
  give_event(T, P.start);
  give_event(T, P.stop);
  give_event(T, P.kern_done);
  for (auto& R : P.lanes) {
    give_event(*R.d, R.t0);
    give_event(*R.d, R.t1);
    give_event(*R.d, R.t_in);
    give_event(*R.d, R.t_out);
  }
  if (done || cudaEventQuery(stop) == cudaSuccess) {
    give_scratch(T, P.scratch);
  } else if (P.scratch.first) {
    // The kernel may still run (its own waits are bounded): keep the buffer
    // out of reuse until the engine is destroyed.
    T.quarantine.push_back(P.scratch.first);
  }
  cudaGetLastError();
  P.scratch = {nullptr, 0};
  give_pinned(P.desc_host);
  give_pinned(P.result_host);
  if (!res.ok) {
    // Poisoned rings are reset once every transfer touching them is done.
    bool others = false;
    for (auto& kv : pending_) {
      for (Ring* r : kv.second->rings)
        if (std::find(P.rings.begin(), P.rings.end(), r) != P.rings.end()) others = true;
    }
    if (!others && done) reset_rings(P);
  }
  (void)rescued;
  return res;
}

void host_register(uint64_t ptr, uint64_t bytes) {
  if (ptr == 0 || bytes == 0) throw std::invalid_argument("host_register: empty range");
  PPB_CUDA(cudaHostRegister(reinterpret_cast<void*>(ptr), bytes,
                            cudaHostRegisterPortable | cudaHostRegisterMapped));
}

void host_unregister(uint64_t ptr) {
  if (ptr == 0) throw std::invalid_argument("host_unregister: null pointer");
  PPB_CUDA(cudaHostUnregister(reinterpret_cast<void*>(ptr)));
}

}  // namespace ppb
