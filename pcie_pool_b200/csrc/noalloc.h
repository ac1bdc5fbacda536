// Allocation-free C entry point for the landing kernel.
//
// This interface has no counterpart in the reference project.  It runs the
// same `land_kernel` as PoolEngine (copy or paged-KV unit scatter, with
// per-chunk checksums) over a source that is already in device memory, but
// every piece of kernel scratch -- lane descriptor, chunk table, per-chunk
// arrival counters, checksums, status words, the ready counter -- lives in
// one file-scope `static __device__ __align__(256)` array of
// PPB_NOALLOC_SCRATCH_BYTES bytes.  No call makes cudaMalloc, cudaFree,
// cudaMallocAsync or any other allocating routine; the descriptors are
// written on the device by a small setup kernel, so no host staging either.
//
// Limits and rules:
//   * At most PPB_NOALLOC_MAX_CHUNKS chunks per call (ceil(src_bytes /
//     chunk_bytes)); chunk_bytes < 4 GiB.  A larger request is rejected with
//     PPB_NOALLOC_E_TOO_LARGE before any CUDA call.
//   * The first call on a device does the setup (cudaGetSymbolAddress of the
//     scratch array with that device current, kernel attributes, occupancy
//     query).  Make that first call -- or ppb_noalloc_setup() -- before any
//     stream capture.
//   * The scratch is one per device.  Calls that overlap on one device (two
//     streams, two threads, or a second call before ppb_noalloc_result of the
//     first) race on it; serialise them.
//   * Everything that must start at zero (arrival counters, checksums, status)
//     is cleared by the setup kernel of each call, on the caller's stream.
//   * src, dst and the unit address table are device memory owned by the
//     caller and stay valid until the work on `stream` completes.
#pragma once

#include <cstdint>

#define PPB_NOALLOC_MAX_CHUNKS 4096u
#define PPB_NOALLOC_SCRATCH_BYTES (256u * 1024u)

#define PPB_NOALLOC_OP_COPY 0
#define PPB_NOALLOC_OP_SCATTER_UNITS 1

// Return codes: 0 success; negative = rejected by argument checks (no CUDA
// call was made); positive = a cudaError_t from the CUDA runtime.
#define PPB_NOALLOC_E_ARGUMENT (-1)
#define PPB_NOALLOC_E_TOO_LARGE (-2)
#define PPB_NOALLOC_E_SETUP (-3)

#ifdef __cplusplus
extern "C" {
#endif

// Resolve the scratch array for `device` (idempotent).
int ppb_noalloc_setup(int device);

// Queue one landing on `stream` (a cudaStream_t, may be null for the legacy
// default stream) of `device`:
//   COPY:          dst[i] = src[i] for i < src_bytes (dst_bytes >= src_bytes)
//   SCATTER_UNITS: unit u (bytes [u*unit_bytes, (u+1)*unit_bytes) of src)
//                  -> unit_addrs[u]; src_bytes and chunk_bytes are multiples
//                  of unit_bytes; dst/dst_bytes are unused.  src and
//                  unit_bytes must be 16-byte aligned (checked here); the
//                  unit table is device memory, so its entries are checked on
//                  the device: a null or misaligned address makes the call
//                  land nothing and report status 3 with detail = unit index.
// Chunk c covers src bytes [c*chunk_bytes, min(src_bytes, (c+1)*chunk_bytes)).
// `ctas` CTAs share the chunks (clamped to the device's resident maximum);
// timeout_ns bounds every device-side wait (0 = 10 s).
int ppb_noalloc_land(int device, int op, const void* src, uint64_t src_bytes, void* dst,
                     uint64_t dst_bytes, const uint64_t* unit_addrs, uint32_t unit_bytes,
                     uint64_t chunk_bytes, uint32_t ctas, int checksum, uint64_t timeout_ns,
                     void* stream);

// Wait for `stream` and copy back the status words {code, lane, chunk, detail}
// and the first `chunks` per-chunk checksums {sum, weighted} (2*chunks words;
// csum may be null).  Status code 0 = ok, 1/2 = a wait ran out, 3 = bad
// argument (op, or a unit address; then nothing was written).
int ppb_noalloc_result(int device, int* status4, unsigned long long* csum, uint32_t chunks,
                       void* stream);

uint32_t ppb_noalloc_max_chunks(void);
uint64_t ppb_noalloc_scratch_bytes(void);
const char* ppb_noalloc_strerror(int code);

#ifdef __cplusplus
}
#endif
