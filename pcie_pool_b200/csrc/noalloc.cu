// Allocation-free entry point: land_kernel with its scratch in a static
// device array (contract in noalloc.h).
#include "noalloc.h"

#include <atomic>
#include <cstddef>
#include <mutex>

#include <cuda_runtime.h>

#include "pool_kernels.h"

namespace {

using ppb::ChunkDesc;
using ppb::LaneDesc;
using ppb::LaneKernelParams;

// Scratch layout (byte offsets, every region 256-byte aligned).
constexpr size_t kOffLane = 0;
constexpr size_t kOffReady = 256;
constexpr size_t kOffStatus = 512;
constexpr size_t kOffBadUnit = 640;  // first bad unit index + 1 (0: table is good)
constexpr size_t kOffDone = 768;
constexpr size_t kOffCsum = kOffDone + size_t(PPB_NOALLOC_MAX_CHUNKS) * sizeof(uint32_t);
constexpr size_t kOffChunks = kOffCsum + size_t(PPB_NOALLOC_MAX_CHUNKS) * 2 * sizeof(unsigned long long);
constexpr size_t kScratchUsed = kOffChunks + size_t(PPB_NOALLOC_MAX_CHUNKS) * sizeof(ChunkDesc);
static_assert(sizeof(LaneDesc) <= kOffReady - kOffLane, "lane descriptor region");
static_assert(kOffBadUnit + 8 <= kOffDone && kOffStatus + 16 <= kOffBadUnit, "status regions");
static_assert(kOffCsum % 256 == 0 && kOffChunks % 256 == 0, "scratch regions stay 256-byte aligned");
static_assert(kScratchUsed <= PPB_NOALLOC_SCRATCH_BYTES, "scratch array too small for the layout");

constexpr int kMaxDevices = 64;

}  // namespace

static __device__ __align__(256) unsigned char g_noalloc_scratch[PPB_NOALLOC_SCRATCH_BYTES];

namespace {

std::mutex g_setup_mu;
std::atomic<unsigned char*> g_scratch[kMaxDevices];
std::atomic<int> g_max_ctas[kMaxDevices];

// Writes the lane and chunk tables and clears counters, checksums and status.
__global__ void noalloc_prepare(unsigned char* s, const uint8_t* src, uint64_t src_bytes,
                                uint64_t chunk_bytes, uint32_t nchunks, uint32_t unit_bytes,
                                uint32_t ctas, uint32_t scatter) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i == 0) {
    LaneDesc L;
    L.ring = const_cast<uint8_t*>(src);
    L.ready = reinterpret_cast<uint32_t*>(s + kOffReady);
    L.freec = nullptr;
    L.slot_bytes = chunk_bytes;
    L.chunk_begin = 0;
    L.chunk_count = nchunks;
    L.cta_begin = 0;
    L.cta_count = ctas;
    L.in_place = 0;
    L.slots = nchunks;
    L.donec = nullptr;  // not a round trip
    *reinterpret_cast<LaneDesc*>(s + kOffLane) = L;
    *reinterpret_cast<uint32_t*>(s + kOffReady) = 1u;  // every chunk is published (seq 1)
    int* st = reinterpret_cast<int*>(s + kOffStatus);
    st[0] = st[1] = st[2] = st[3] = 0;
    *reinterpret_cast<unsigned long long*>(s + kOffBadUnit) = ~0ull;
  }
  if (i < nchunks) {
    const uint64_t off = uint64_t(i) * chunk_bytes;
    const uint64_t left = src_bytes - off;
    ChunkDesc c;
    c.dev_off = off;
    c.host_off = off;
    c.bytes = static_cast<uint32_t>(left < chunk_bytes ? left : chunk_bytes);
    c.seq = 1u;
    c.slot = i;
    c.unit0 = scatter ? static_cast<uint32_t>(off / unit_bytes) : 0u;
    c.tensor = 0u;
    c.count = 0u;
    reinterpret_cast<ChunkDesc*>(s + kOffChunks)[i] = c;
    reinterpret_cast<uint32_t*>(s + kOffDone)[i] = 0u;
    unsigned long long* cs = reinterpret_cast<unsigned long long*>(s + kOffCsum);
    cs[2 * i] = 0ull;
    cs[2 * i + 1] = 0ull;
  }
}

// Checks every unit address of a scatter (non-null, 16-byte aligned) and
// records the first bad unit.  Grid-stride over all units.
__global__ void noalloc_check_units(unsigned char* s, const uint64_t* unit_addrs, uint64_t units) {
  unsigned long long* bad = reinterpret_cast<unsigned long long*>(s + kOffBadUnit);
  for (uint64_t u = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; u < units;
       u += uint64_t(gridDim.x) * blockDim.x) {
    const uint64_t a = unit_addrs[u];
    if (a == 0 || (a & 15u) != 0) atomicMin(bad, static_cast<unsigned long long>(u + 1));
  }
}

// After the check: a bad table empties the lane (the landing kernel then
// issues no copy at all) and reports kStatusBadArgument with the unit index.
__global__ void noalloc_gate(unsigned char* s) {
  const unsigned long long bad = *reinterpret_cast<unsigned long long*>(s + kOffBadUnit);
  if (bad == ~0ull) return;
  reinterpret_cast<LaneDesc*>(s + kOffLane)->chunk_count = 0;
  int* st = reinterpret_cast<int*>(s + kOffStatus);
  st[0] = ppb::kStatusBadArgument;
  st[1] = 0;
  st[2] = -1;
  st[3] = static_cast<int>(bad - 1);
}

struct CurrentDevice {
  int prev = -1;
  cudaError_t rc = cudaSuccess;
  explicit CurrentDevice(int dev) {
    rc = cudaGetDevice(&prev);
    if (rc == cudaSuccess && prev != dev) rc = cudaSetDevice(dev);
  }
  ~CurrentDevice() {
    int now = -1;
    if (prev >= 0 && cudaGetDevice(&now) == cudaSuccess && now != prev) cudaSetDevice(prev);
  }
};

int setup_locked(int device) {
  if (g_scratch[device].load(std::memory_order_acquire) != nullptr) return 0;
  CurrentDevice cur(device);
  if (cur.rc != cudaSuccess) return static_cast<int>(cur.rc);
  void* p = nullptr;
  const cudaError_t rc = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (rc != cudaSuccess) return static_cast<int>(rc);
  if (p == nullptr) return PPB_NOALLOC_E_SETUP;
  // Also sets the land kernel's shared-memory attribute on this device.
  const int max_ctas = ppb::lane_kernel_max_ctas(device);
  if (max_ctas <= 0) return PPB_NOALLOC_E_SETUP;
  g_max_ctas[device].store(max_ctas, std::memory_order_relaxed);
  g_scratch[device].store(static_cast<unsigned char*>(p), std::memory_order_release);
  return 0;
}

int ensure_setup(int device, unsigned char** out) {
  unsigned char* s = g_scratch[device].load(std::memory_order_acquire);
  if (s == nullptr) {
    std::lock_guard<std::mutex> g(g_setup_mu);
    const int rc = setup_locked(device);
    if (rc != 0) return rc;
    s = g_scratch[device].load(std::memory_order_acquire);
  }
  *out = s;
  return 0;
}

}  // namespace

extern "C" {

__attribute__((visibility("default"))) int ppb_noalloc_setup(int device) {
  if (device < 0 || device >= kMaxDevices) return PPB_NOALLOC_E_ARGUMENT;
  unsigned char* s = nullptr;
  return ensure_setup(device, &s);
}

__attribute__((visibility("default"))) int ppb_noalloc_land(
    int device, int op, const void* src, uint64_t src_bytes, void* dst, uint64_t dst_bytes,
    const uint64_t* unit_addrs, uint32_t unit_bytes, uint64_t chunk_bytes, uint32_t ctas,
    int checksum, uint64_t timeout_ns, void* stream) {
  // ---- argument checks: no CUDA call before these pass ----
  if (device < 0 || device >= kMaxDevices) return PPB_NOALLOC_E_ARGUMENT;
  if (op != PPB_NOALLOC_OP_COPY && op != PPB_NOALLOC_OP_SCATTER_UNITS) return PPB_NOALLOC_E_ARGUMENT;
  if (src == nullptr || src_bytes == 0 || chunk_bytes == 0 || ctas == 0) return PPB_NOALLOC_E_ARGUMENT;
  if (chunk_bytes > 0xFFFFFFFFull) return PPB_NOALLOC_E_TOO_LARGE;
  const uint64_t nchunks = (src_bytes + chunk_bytes - 1) / chunk_bytes;
  if (nchunks > PPB_NOALLOC_MAX_CHUNKS) return PPB_NOALLOC_E_TOO_LARGE;
  if (op == PPB_NOALLOC_OP_COPY) {
    if (dst == nullptr || dst_bytes < src_bytes) return PPB_NOALLOC_E_ARGUMENT;
  } else {
    // The scatter moves whole units with 16-byte bulk copies: the source, the
    // unit size and (checked on the device) every unit address must be
    // 16-byte aligned.
    if (unit_addrs == nullptr || unit_bytes == 0 || unit_bytes % 16 != 0) return PPB_NOALLOC_E_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(src) & 15u) != 0) return PPB_NOALLOC_E_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(unit_addrs) & 7u) != 0) return PPB_NOALLOC_E_ARGUMENT;
    if (src_bytes % unit_bytes != 0 || chunk_bytes % unit_bytes != 0) return PPB_NOALLOC_E_ARGUMENT;
    if (src_bytes / unit_bytes > 0xFFFFFFFFull) return PPB_NOALLOC_E_TOO_LARGE;
  }

  unsigned char* s = nullptr;
  int rc = ensure_setup(device, &s);
  if (rc != 0) return rc;
  CurrentDevice cur(device);
  if (cur.rc != cudaSuccess) return static_cast<int>(cur.rc);
  const uint32_t max_ctas = static_cast<uint32_t>(g_max_ctas[device].load(std::memory_order_relaxed));
  const uint32_t grid = ctas < max_ctas ? ctas : max_ctas;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  const uint32_t n = static_cast<uint32_t>(nchunks);
  noalloc_prepare<<<(n + 255) / 256, 256, 0, st>>>(s, static_cast<const uint8_t*>(src), src_bytes,
                                                   chunk_bytes, n, unit_bytes, grid,
                                                   op == PPB_NOALLOC_OP_SCATTER_UNITS ? 1u : 0u);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return static_cast<int>(e);
  if (op == PPB_NOALLOC_OP_SCATTER_UNITS) {
    const uint64_t units = src_bytes / unit_bytes;
    const uint64_t want = (units + 255) / 256;
    const unsigned int blocks = static_cast<unsigned int>(want < 1184 ? want : 1184);
    noalloc_check_units<<<blocks, 256, 0, st>>>(s, unit_addrs, units);
    noalloc_gate<<<1, 1, 0, st>>>(s);
    e = cudaGetLastError();
    if (e != cudaSuccess) return static_cast<int>(e);
  }

  LaneKernelParams p{};
  p.lanes = reinterpret_cast<const LaneDesc*>(s + kOffLane);
  p.chunks = reinterpret_cast<const ChunkDesc*>(s + kOffChunks);
  p.num_lanes = 1;
  p.op = op == PPB_NOALLOC_OP_COPY ? ppb::kOpCopy : ppb::kOpScatterUnits;
  p.dev = static_cast<uint8_t*>(dst);
  p.unit_addr = unit_addrs;
  p.unit_bytes = unit_bytes;
  p.checksum = checksum ? 1u : 0u;
  p.done = reinterpret_cast<uint32_t*>(s + kOffDone);
  p.csum = reinterpret_cast<unsigned long long*>(s + kOffCsum);
  p.status = reinterpret_cast<int*>(s + kOffStatus);
  p.timeout_ns = timeout_ns ? timeout_ns : 10ull * 1000000000ull;
  e = ppb::launch_land(p, static_cast<int>(grid), st);
  return static_cast<int>(e);
}

__attribute__((visibility("default"))) int ppb_noalloc_result(int device, int* status4,
                                                              unsigned long long* csum,
                                                              uint32_t chunks, void* stream) {
  if (device < 0 || device >= kMaxDevices || status4 == nullptr) return PPB_NOALLOC_E_ARGUMENT;
  if (chunks > PPB_NOALLOC_MAX_CHUNKS) return PPB_NOALLOC_E_TOO_LARGE;
  unsigned char* s = g_scratch[device].load(std::memory_order_acquire);
  if (s == nullptr) return PPB_NOALLOC_E_SETUP;
  CurrentDevice cur(device);
  if (cur.rc != cudaSuccess) return static_cast<int>(cur.rc);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(status4, s + kOffStatus, 4 * sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess && csum != nullptr && chunks > 0) {
    e = cudaMemcpyAsync(csum, s + kOffCsum, size_t(chunks) * 2 * sizeof(unsigned long long),
                        cudaMemcpyDeviceToHost, st);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  return static_cast<int>(e);
}

__attribute__((visibility("default"))) uint32_t ppb_noalloc_max_chunks(void) {
  return PPB_NOALLOC_MAX_CHUNKS;
}

__attribute__((visibility("default"))) uint64_t ppb_noalloc_scratch_bytes(void) {
  return PPB_NOALLOC_SCRATCH_BYTES;
}

__attribute__((visibility("default"))) const char* ppb_noalloc_strerror(int code) {
  switch (code) {
    case 0:
      return "ok";
    case PPB_NOALLOC_E_ARGUMENT:
      return "invalid argument (null pointer, zero size, unknown op, unit/chunk mismatch, or a "
             "scatter whose source or unit size is not 16-byte aligned)";
    case PPB_NOALLOC_E_TOO_LARGE:
      return "request exceeds the static scratch: more than 4096 chunks, chunk_bytes >= 4 GiB "
             "or more than 2^32-1 units";
    case PPB_NOALLOC_E_SETUP:
      return "setup failed: scratch symbol or kernel attributes unavailable on this device";
    default:
      return code > 0 ? cudaGetErrorString(static_cast<cudaError_t>(code)) : "unknown error";
  }
}

}  // extern "C"
