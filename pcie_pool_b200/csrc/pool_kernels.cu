// Fused lane kernels for sm_100a (see pool_kernels.h for the protocol).
//
// Data path per CTA: a kStages-deep ring of kTileBytes shared-memory stages.
// One elected thread issues 1-D TMA bulk copies (cp.async.bulk, never the
// cluster-multicast form) from the source -- for landing that is the relay GPU's
// staging slot reached through the peer mapping over NVLink -- into shared
// memory, tracked by per-stage mbarriers with complete_tx.  All threads fold
// the tile into the chunk checksum straight from shared memory, then the
// elected thread writes the tile out with a bulk shared->global store.
//
// Synchronisation with the copy engines uses two monotonically increasing
// 32-bit counters per lane (ready / free) compared wrap-around safely; every
// wait is bounded and ends in an error status, never a trap.
#include <atomic>

#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include "device_utils.cuh"
#include "fp8_e4m3.cuh"
#include "pool_kernels.h"

namespace ppb {
namespace {

using namespace dev;

struct Tile {
  const uint8_t* src;
  uint8_t* dst;
  uint64_t pos;  // byte position inside the chunk stream (checksum index)
  uint32_t n;
};

__device__ __forceinline__ void record_error(int* status, int code, int lane, int chunk,
                                             int detail) {
  if (atomicCAS(status, 0, code) == 0) {
    status[1] = lane;
    status[2] = chunk;
    status[3] = detail;
  }
  __threadfence_system();
}

__device__ __forceinline__ int find_lane(const LaneKernelParams& p, LaneDesc& out) {
  for (uint32_t i = 0; i < p.num_lanes; ++i) {
    const LaneDesc d = p.lanes[i];
    if (blockIdx.x >= d.cta_begin && blockIdx.x < d.cta_begin + d.cta_count) {
      out = d;
      return static_cast<int>(i);
    }
  }
  return -1;
}

// Byte-granular fallback for ragged or misaligned pieces.  Threads of the CTA
// stride over [0, n); checksum contributions are accumulated per byte, which
// equals the word definition because the checksum is linear in the words.
__device__ void copy_generic(const uint8_t* src, uint8_t* dst, uint64_t n, uint64_t pos,
                             bool store, bool do_csum, Csum& cs) {
  for (uint64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const uint8_t b = ld_cg_u8(src + i);
    if (store) dst[i] = b;
    if (do_csum) {
      const uint64_t at = pos + i;
      const unsigned long long v = static_cast<unsigned long long>(b) << (8u * (at & 3u));
      cs.s += v;
      cs.w += (at / 4u + 1u) * v;
    }
  }
}

// Pipelined bulk-copy loop over the tiles j, j+G, j+2G, ... of one chunk.
// `q` is the CTA's running tile counter: stage = q % kStages and the mbarrier
// phase parity = (q / kStages) & 1.  Returns false on a copy timeout.
struct NoXform {
  static constexpr bool kActive = false;
  __device__ void operator()(uint8_t*, const Tile&, uint32_t) const {}
};

template <class Geom, class Xform = NoXform>
__device__ bool run_tiles(const Geom& geom, uint32_t ntiles, uint32_t j, uint32_t G, bool store,
                          bool do_csum, uint32_t& q, uint64_t* bars, uint8_t* smem,
                          Csum& cs, uint64_t timeout_ns, const Xform& xform = Xform{}) {
  const uint32_t my_n = ntiles > j ? (ntiles - j + G - 1) / G : 0;
  if (my_n == 0) return true;
  const uint32_t base = q;
  if (threadIdx.x == 0) {
    if (store) bulk_wait_read<0>();  // earlier stores no longer read any stage
    for (uint32_t k = 0; k < my_n && k < static_cast<uint32_t>(kStages); ++k) {
      const Tile t = geom(j + k * G);
      const uint32_t s = (base + k) % kStages;
      mbar_arrive_expect_tx(&bars[s], t.n);
      bulk_g2s(smem + size_t(s) * kTileBytes, t.src, t.n, &bars[s]);
    }
  }
  bool ok = true;
  uint32_t k = 0;
  for (; k < my_n; ++k) {
    const uint32_t s = (base + k) % kStages;
    const uint32_t parity = ((base + k) / kStages) & 1u;
    const Tile t = geom(j + k * G);
    const bool got = mbar_wait(&bars[s], parity, globaltimer_ns() + timeout_ns);
    if (!__syncthreads_and(got)) {
      ok = false;
      break;
    }
    uint8_t* stage = smem + size_t(s) * kTileBytes;
    if (do_csum) {
      const uint4* v = reinterpret_cast<const uint4*>(stage);
      const uint32_t nv = t.n >> 4;
      const uint64_t w0 = t.pos >> 2;
      for (uint32_t i = threadIdx.x; i < nv; i += blockDim.x) csum_vec(cs, v[i], w0 + 4ull * i);
    }
    if constexpr (Xform::kActive) {
      if (do_csum) __syncthreads();  // the checksum reads the tile as it arrived
      xform(stage, t, j + k * G);
      // generic-proxy writes of the stage become visible to the bulk store
      fence_proxy_async_smem();
    }
    __syncthreads();  // every reader is done with this stage
    if (threadIdx.x == 0) {
      if (store) {
        bulk_s2g(t.dst, stage, t.n);
        bulk_commit();
      }
      if (k + kStages < my_n) {
        if (store) bulk_wait_read<0>();
        const Tile nt = geom(j + (k + kStages) * G);
        mbar_arrive_expect_tx(&bars[s], nt.n);
        bulk_g2s(stage, nt.src, nt.n, &bars[s]);
      }
    }
  }
  if (!ok) {
    // Give the copies already in flight a bounded chance to land before the
    // CTA leaves, so no bulk copy targets shared memory of an exited CTA.
    const uint32_t issued = my_n < k + kStages ? my_n : k + kStages;
    for (uint32_t r = k; r < issued; ++r) {
      const uint32_t s = (base + r) % kStages;
      mbar_wait(&bars[s], ((base + r) / kStages) & 1u, globaltimer_ns() + timeout_ns);
    }
    q = base + issued;
    return false;
  }
  q = base + my_n;
  return true;
}

struct CopyGeom {
  const uint8_t* src;
  uint8_t* dst;
  uint32_t body;
  __device__ Tile operator()(uint32_t k) const {
    const uint32_t off = k * kTileBytes;
    const uint32_t n = body - off < kTileBytes ? body - off : kTileBytes;
    return Tile{src + off, dst ? dst + off : nullptr, off, n};
  }
};

// Fixed-size units at scattered device addresses (paged-KV block lanes).
// `scatter` = true: chunk stream -> unit addresses; false: gather.
struct UnitGeom {
  const uint8_t* stream_src;  // scatter: staged chunk; gather: unused
  uint8_t* stream_dst;        // gather: staging slot; scatter: unused
  const uint64_t* unit_addr;  // already offset to the chunk's first unit
  uint32_t unit_bytes;
  uint32_t tiles_per_unit;
  bool scatter;
  __device__ Tile operator()(uint32_t k) const {
    const uint32_t u = k / tiles_per_unit;
    const uint32_t sub = (k - u * tiles_per_unit) * kTileBytes;
    const uint32_t n = unit_bytes - sub < kTileBytes ? unit_bytes - sub : kTileBytes;
    const uint64_t pos = uint64_t(u) * unit_bytes + sub;
    uint8_t* ua = reinterpret_cast<uint8_t*>(unit_addr[u]) + sub;
    if (scatter) return Tile{stream_src + pos, ua, pos, n};
    return Tile{ua, stream_dst ? stream_dst + pos : nullptr, pos, n};
  }
};

// Variable ranges, pre-split on the host to at most kTileBytes each.
struct RangeGeom {
  const uint8_t* stream_src;
  uint8_t* stream_dst;
  const uint64_t* range_addr;  // offset to the chunk's first range
  const uint32_t* range_bytes;
  const uint64_t* range_pos;   // position of each range inside the chunk stream
  bool scatter;
  __device__ Tile operator()(uint32_t k) const {
    const uint64_t pos = range_pos[k];
    const uint32_t n = range_bytes[k];
    uint8_t* ra = reinterpret_cast<uint8_t*>(range_addr[k]);
    if (scatter) return Tile{stream_src + pos, ra, pos, n};
    return Tile{ra, stream_dst ? stream_dst + pos : nullptr, pos, n};
  }
};

// Streamed optimizer: tile k of a chunk is updated in its staging slot.
struct AdamGeom {
  uint8_t* slot;
  __device__ Tile operator()(uint32_t k) const {
    const uint32_t off = k * kAdamTileBytes;
    return Tile{slot + off, slot + off, off, kAdamTileBytes};
  }
};

// AdamW on one staged tile: [master | exp_avg | exp_avg_sq] fp32 in shared
// memory, bf16 gradient read from global memory, updated state written back
// into the stage (the bulk store returns it to the slot) and the bf16
// parameter written to global memory.  Thread t owns parameters 4t..4t+3 and
// 1024+4t..1024+4t+3 of the tile (float4 / 8-byte vector accesses).
struct AdamXform {
  static constexpr bool kActive = true;
  const uint16_t* grads;
  uint16_t* params;
  uint64_t nparams;
  uint32_t tile0;  // first tile of the chunk
  AdamCoeffs c;
  __device__ void operator()(uint8_t* stage, const Tile&, uint32_t k) const {
    float* M = reinterpret_cast<float*>(stage);
    float* A = M + kAdamTileParams;
    float* V = A + kAdamTileParams;
    const uint64_t base = uint64_t(tile0 + k) * kAdamTileParams;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const uint32_t i0 = r * (kAdamTileParams / 2) + 4u * threadIdx.x;
      const uint64_t gi = base + i0;
      if (gi >= nparams) continue;
      if (gi + 4 <= nparams) {
        const uint2 graw = *reinterpret_cast<const uint2*>(grads + gi);
        const __nv_bfloat162* gh = reinterpret_cast<const __nv_bfloat162*>(&graw);
        const float2 g01 = __bfloat1622float2(gh[0]);
        const float2 g23 = __bfloat1622float2(gh[1]);
        float4 m = *reinterpret_cast<float4*>(M + i0);
        float4 a = *reinterpret_cast<float4*>(A + i0);
        float4 v = *reinterpret_cast<float4*>(V + i0);
        m.x = adamw_update(a.x, v.x, m.x, g01.x, c);
        m.y = adamw_update(a.y, v.y, m.y, g01.y, c);
        m.z = adamw_update(a.z, v.z, m.z, g23.x, c);
        m.w = adamw_update(a.w, v.w, m.w, g23.y, c);
        *reinterpret_cast<float4*>(M + i0) = m;
        *reinterpret_cast<float4*>(A + i0) = a;
        *reinterpret_cast<float4*>(V + i0) = v;
        __nv_bfloat162 p01 = __floats2bfloat162_rn(m.x, m.y);
        __nv_bfloat162 p23 = __floats2bfloat162_rn(m.z, m.w);
        uint2 praw;
        praw.x = *reinterpret_cast<uint32_t*>(&p01);
        praw.y = *reinterpret_cast<uint32_t*>(&p23);
        *reinterpret_cast<uint2*>(params + gi) = praw;
      } else {
        for (uint32_t e = 0; e < 4 && gi + e < nparams; ++e) {
          const float g = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(grads + gi + e));
          const float p = adamw_update(A[i0 + e], V[i0 + e], M[i0 + e], g, c);
          M[i0 + e] = p;
          const __nv_bfloat16 pb = __float2bfloat16_rn(p);
          params[gi + e] = *reinterpret_cast<const uint16_t*>(&pb);
        }
      }
    }
  }
};

__device__ __forceinline__ bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// Contiguous copy of one chunk (bulk body + generic ragged tail).
__device__ bool move_contiguous(const uint8_t* src, uint8_t* dst, uint32_t bytes, uint32_t j,
                                uint32_t G, bool store, bool do_csum, uint32_t& q,
                                uint64_t* bars, uint8_t* smem, Csum& cs, uint64_t timeout_ns) {
  const bool fast = aligned16(src) && (!store || aligned16(dst));
  if (!fast) {
    // Misaligned chunk: split evenly across the group with the byte path.
    const uint64_t per = (uint64_t(bytes) + G - 1) / G;
    const uint64_t b0 = per * j;
    if (b0 < bytes) {
      const uint64_t n = bytes - b0 < per ? bytes - b0 : per;
      copy_generic(src + b0, store ? dst + b0 : nullptr, n, b0, store, do_csum, cs);
    }
    return true;
  }
  const uint32_t body = bytes & ~15u;
  const uint32_t ntiles = (body + kTileBytes - 1) / kTileBytes;
  if (!run_tiles(CopyGeom{src, store ? dst : nullptr, body}, ntiles, j, G, store, do_csum, q,
                 bars, smem, cs, timeout_ns))
    return false;
  if (body != bytes && j == 0) {
    copy_generic(src + body, store ? dst + body : nullptr, bytes - body, body, store, do_csum,
                 cs);
  }
  return true;
}

// ---- bf16 -> fp8 e4m3 with one fp32 scale per 128x128 block ------------------
// scale = amax / 448 (IEEE division, 1.0 for an all-zero block); q = e4m3(x /
// scale) with round-to-nearest-even and saturation to +-448 (the hardware
// cvt.rn.satfinite.e4m3x2.f32 conversion), the quotient taken as if rounded
// to fp32 (fp8_e4m3.cuh: estimate by the reciprocal, divide only near a
// rounding boundary).  256 threads cover one block: two
// threads per row, 64 columns (128 bytes) each.
__device__ __forceinline__ void fp8_load_half_row(uint4 (&v)[8], const uint8_t* p) {
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = ld_cg_v4(p + 16u * i);
}

// red: 2 x (kLaneThreads / 32) floats.  The block maximum goes through one of
// two halves by block parity, so one barrier per block suffices: a half is
// rewritten two blocks later, after a barrier that every reader has passed.
// The next block's loads are issued before that barrier, so their latency
// (HBM, or NVLink for a relay's ring) overlaps the reduction and the
// quantization of the current block.
__device__ bool land_fp8_chunk(const LaneKernelParams& p, const ChunkDesc& c,
                               const uint8_t* src, uint32_t j, uint32_t G, bool do_csum,
                               Csum& cs, float* red) {
  const QuantTensor T = p.tensors[c.tensor];
  const uint32_t C = T.cols;
  const uint32_t ncb = C / 128u;
  const uint32_t row0 = c.unit0;
  const uint64_t row_bytes = uint64_t(C) * 2u;
  const uint32_t nrows = static_cast<uint32_t>(c.bytes / row_bytes);
  const uint32_t nrb = (nrows + 127u) / 128u;
  const uint32_t nblocks = nrb * ncb;
  const uint32_t r = threadIdx.x >> 1;
  const uint32_t half = threadIdx.x & 1u;
  auto row_of = [&](uint32_t b) { return (b / ncb) * 128u + r; };
  auto offset_of = [&](uint32_t b) {
    const uint32_t rb = b / ncb;
    return uint64_t(rb * 128u + r) * row_bytes + (uint64_t(b - rb * ncb) * 128u + half * 64u) * 2u;
  };
  uint4 v[8];
  if (j < nblocks && row_of(j) < nrows) fp8_load_half_row(v, src + offset_of(j));
  uint32_t parity = 0;
  for (uint32_t b = j; b < nblocks; b += G, parity ^= 1u) {
    const uint32_t rb = b / ncb;
    const uint32_t cb = b - rb * ncb;
    const uint32_t row_local = rb * 128u + r;
    const bool valid = row_local < nrows;
    const uint64_t byte_off = offset_of(b);
    float amax = 0.f;
    if (valid) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (do_csum) csum_vec(cs, v[i], (byte_off >> 2) + 4u * i);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[i]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    float* rd = red + parity * (kLaneThreads / 32);
    if ((threadIdx.x & 31) == 0) rd[threadIdx.x >> 5] = amax;
    uint4 nv[8];
    const uint32_t nb = b + G;
    const bool nvalid = nb < nblocks && row_of(nb) < nrows;
    if (nvalid) fp8_load_half_row(nv, src + offset_of(nb));
    __syncthreads();
    float bmax = 0.f;
#pragma unroll
    for (int w = 0; w < kLaneThreads / 32; ++w) bmax = fmaxf(bmax, rd[w]);
    const float scale = bmax > 0.f ? __fdiv_rn(bmax, 448.0f) : 1.0f;
    const float rcp = __frcp_rn(scale);
    const bool exact_only = isinf(rcp);
    if (valid) {
      uint32_t packed[16];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[i]);
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const float2 f0 = __bfloat1622float2(h[e]);
          const float2 f1 = __bfloat1622float2(h[e + 1]);
          const uint32_t lo = e4m3x2_quotient(f0.x, f0.y, scale, rcp, exact_only);
          const uint32_t hi = e4m3x2_quotient(f1.x, f1.y, scale, rcp, exact_only);
          packed[i * 2 + e / 2] = lo | (hi << 16);
        }
      }
      uint8_t* qrow = T.q + uint64_t(row0 + row_local) * C + uint64_t(cb) * 128u + half * 64u;
      uint4* qo = reinterpret_cast<uint4*>(qrow);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        qo[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
    }
    if (threadIdx.x == 0) T.scales[uint64_t(row0 / 128u + rb) * ncb + cb] = scale;
    if (nvalid) {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = nv[i];
    }
  }
  // the next chunk's first block reuses the halves from parity 0: wait until
  // every thread has read this chunk's last maximum
  __syncthreads();
  return true;
}

// ---- landing kernel (H2D) -------------------------------------------------------

__global__ void __launch_bounds__(kLaneThreads, 1) land_kernel(const LaneKernelParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + size_t(kStages) * kTileBytes);
  __shared__ unsigned long long red[2 * (kLaneThreads / 32)];
  __shared__ float fred[2 * (kLaneThreads / 32)];
  __shared__ int s_ok;

  LaneDesc L;
  const int lane = find_lane(p, L);
  if (lane < 0) return;
  const uint32_t j = blockIdx.x - L.cta_begin;
  const uint32_t G = L.cta_count;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  uint32_t q = 0;
  const bool do_csum = p.checksum != 0;

  for (uint32_t ci = 0; ci < L.chunk_count; ++ci) {
    const uint32_t cidx = L.chunk_begin + ci;
    const ChunkDesc c = p.chunks[cidx];
    if (threadIdx.x == 0) {
      unsigned long long* tr = p.trace ? p.trace + uint64_t(kTraceWords) * cidx : nullptr;
      if (tr && j == 0) tr[0] = globaltimer_ns();
      const bool ok = wait_flag_geq(L.ready, c.seq, globaltimer_ns() + p.timeout_ns);
      if (ok) fence_proxy_async_global();
      if (tr && j == 0) tr[1] = globaltimer_ns();
      s_ok = ok ? 1 : 0;
    }
    __syncthreads();
    if (!s_ok) {
      if (threadIdx.x == 0) {
        record_error(p.status, kStatusReadyTimeout, lane, static_cast<int>(cidx), int(c.seq));
        // Unblock the producer (and a round trip's copy-out) for every
        // remaining chunk of this lane.
        if (L.freec) st_release_sys(L.freec, c.seq + 0x40000000u);
        if (L.donec) st_release_sys(L.donec, c.seq + 0x40000000u);
      }
      return;
    }
    const uint8_t* src =
        L.in_place ? (p.dev + c.dev_off) : (L.ring + uint64_t(c.slot) * L.slot_bytes);
    const bool store = !L.in_place;
    Csum cs{0ull, 0ull};
    bool ok = true;
    switch (p.op) {
      case kOpCopy:
        ok = move_contiguous(src, p.dev + c.dev_off, c.bytes, j, G, store, do_csum, q, bars, smem,
                             cs, p.timeout_ns);
        break;
      case kOpScatterUnits: {
        const uint32_t tpu = (p.unit_bytes + kTileBytes - 1) / kTileBytes;
        const uint32_t nunits = c.bytes / p.unit_bytes;
        ok = run_tiles(UnitGeom{src, nullptr, p.unit_addr + c.unit0, p.unit_bytes, tpu, true},
                       nunits * tpu, j, G, store, do_csum, q, bars, smem, cs, p.timeout_ns);
        break;
      }
      case kOpScatterRanges:
        ok = run_tiles(RangeGeom{src, nullptr, p.range_addr + c.unit0, p.range_bytes + c.unit0,
                                 p.range_pos + c.unit0, true},
                       c.count, j, G, store, do_csum, q, bars, smem, cs, p.timeout_ns);
        break;
      case kOpFp8Quant:
        ok = land_fp8_chunk(p, c, src, j, G, do_csum, cs, fred);
        break;
      case kOpAdamW:
        ok = !L.in_place &&
             run_tiles(AdamGeom{const_cast<uint8_t*>(src)}, c.bytes / kAdamTileBytes, j, G, true, do_csum,
                       q, bars, smem, cs, p.timeout_ns,
                       AdamXform{p.grads, p.params_out, p.nparams, c.unit0, p.adam});
        break;
      default:
        ok = false;
    }
    if (!ok) {
      if (threadIdx.x == 0) {
        const bool timed_out = p.op <= kOpScatterRanges || p.op == kOpAdamW;
        record_error(p.status, timed_out ? kStatusCopyTimeout : kStatusBadArgument, lane,
                     static_cast<int>(cidx), int(c.seq));
        if (L.freec) st_release_sys(L.freec, c.seq + 0x40000000u);
        if (L.donec) st_release_sys(L.donec, c.seq + 0x40000000u);
      }
      return;
    }
    if (do_csum) csum_block_commit(cs, p.csum + 2ull * cidx, red);
    if (L.donec && threadIdx.x == 0) {
      // round trip: the updated tiles must sit in the slot before the
      // copy-out stream is told to read them
      bulk_wait_all<0>();
      fence_proxy_async_global();
      fence_sys();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      const uint32_t old = G > 1 ? atom_add_acq_rel_gpu(p.done + cidx, 1u) : 0u;
      if (old == G - 1) {
        if (p.trace) {
          p.trace[uint64_t(kTraceWords) * cidx + 2] = globaltimer_ns();
          p.trace[uint64_t(kTraceWords) * cidx + 3] = G;
        }
        if (L.donec) {
          st_release_sys(L.donec, c.seq);
        } else if (L.freec) {
          st_release_sys(L.freec, c.seq);
        }
      }
    }
  }
  if (threadIdx.x == 0) bulk_wait_all<0>();
}

// ---- push kernel (D2H) ------------------------------------------------------------

__global__ void __launch_bounds__(kLaneThreads, 1) push_kernel(const LaneKernelParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + size_t(kStages) * kTileBytes);
  __shared__ unsigned long long red[2 * (kLaneThreads / 32)];
  __shared__ int s_ok;

  LaneDesc L;
  const int lane = find_lane(p, L);
  if (lane < 0) return;
  const uint32_t j = blockIdx.x - L.cta_begin;
  const uint32_t G = L.cta_count;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  uint32_t q = 0;
  const bool do_csum = p.checksum != 0;

  for (uint32_t ci = 0; ci < L.chunk_count; ++ci) {
    const uint32_t cidx = L.chunk_begin + ci;
    const ChunkDesc c = p.chunks[cidx];
    if (!L.in_place) {
      if (threadIdx.x == 0) {
        unsigned long long* tr = p.trace ? p.trace + uint64_t(kTraceWords) * cidx : nullptr;
        if (tr && j == 0) tr[0] = globaltimer_ns();
        s_ok = wait_flag_geq(L.freec, c.seq - L.slots, globaltimer_ns() + p.timeout_ns) ? 1 : 0;
        if (tr && j == 0) tr[1] = globaltimer_ns();
      }
      __syncthreads();
      if (!s_ok) {
        if (threadIdx.x == 0) {
          record_error(p.status, kStatusFreeTimeout, lane, static_cast<int>(cidx), int(c.seq));
          st_release_sys(L.ready, c.seq + 0x40000000u);
        }
        return;
      }
    }
    uint8_t* slot = L.in_place ? nullptr : (L.ring + uint64_t(c.slot) * L.slot_bytes);
    const bool store = !L.in_place;
    Csum cs{0ull, 0ull};
    bool ok = true;
    switch (p.op) {
      case kOpCopy:
        ok = move_contiguous(p.dev + c.dev_off, slot, c.bytes, j, G, store, do_csum, q, bars,
                             smem, cs, p.timeout_ns);
        break;
      case kOpGatherUnits: {
        const uint32_t tpu = (p.unit_bytes + kTileBytes - 1) / kTileBytes;
        const uint32_t nunits = c.bytes / p.unit_bytes;
        ok = run_tiles(UnitGeom{nullptr, slot, p.unit_addr + c.unit0, p.unit_bytes, tpu, false},
                       nunits * tpu, j, G, store, do_csum, q, bars, smem, cs, p.timeout_ns);
        break;
      }
      case kOpGatherRanges:
        ok = run_tiles(RangeGeom{nullptr, slot, p.range_addr + c.unit0, p.range_bytes + c.unit0,
                                 p.range_pos + c.unit0, false},
                       c.count, j, G, store, do_csum, q, bars, smem, cs, p.timeout_ns);
        break;
      default:
        ok = false;
    }
    if (!ok) {
      if (threadIdx.x == 0) {
        record_error(p.status, p.op == kOpCopy || p.op == kOpGatherUnits || p.op == kOpGatherRanges
                                   ? kStatusCopyTimeout
                                   : kStatusBadArgument,
                     lane, static_cast<int>(cidx), int(c.seq));
        if (!L.in_place) st_release_sys(L.ready, c.seq + 0x40000000u);
      }
      return;
    }
    if (do_csum) csum_block_commit(cs, p.csum + 2ull * cidx, red);
    if (threadIdx.x == 0 && store) {
      // Our bulk stores into the slot must be performed before the chunk is
      // published to the copy engine of the relay.
      bulk_wait_all<0>();
      fence_proxy_async_global();
      fence_sys();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      const uint32_t old = G > 1 ? atom_add_acq_rel_gpu(p.done + cidx, 1u) : 0u;
      if (old == G - 1) {
        if (p.trace) {
          p.trace[uint64_t(kTraceWords) * cidx + 2] = globaltimer_ns();
          p.trace[uint64_t(kTraceWords) * cidx + 3] = G;
        }
        if (!L.in_place) st_release_sys(L.ready, c.seq);
      }
    }
  }
  if (threadIdx.x == 0) bulk_wait_all<0>();
}

// Per-device "attributes set" flags.  Launchers run from several host threads
// (PoolEngine under its lock, the allocation-free entry point without it);
// setting the attribute twice is harmless, the flag only has to be race-free.
std::atomic<bool> g_attr_set[64];

cudaError_t prepare_attrs() {
  int dev = 0;
  cudaError_t rc = cudaGetDevice(&dev);
  if (rc != cudaSuccess) return rc;
  if (dev >= 0 && dev < 64 && g_attr_set[dev].load(std::memory_order_acquire)) return cudaSuccess;
  rc = cudaFuncSetAttribute(land_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            static_cast<int>(kLaneSmemBytes));
  if (rc != cudaSuccess) return rc;
  rc = cudaFuncSetAttribute(push_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            static_cast<int>(kLaneSmemBytes));
  if (rc != cudaSuccess) return rc;
  if (dev >= 0 && dev < 64) g_attr_set[dev].store(true, std::memory_order_release);
  return cudaSuccess;
}

}  // namespace

cudaError_t launch_land(const LaneKernelParams& p, int grid, cudaStream_t stream) {
  cudaError_t rc = prepare_attrs();
  if (rc != cudaSuccess) return rc;
  land_kernel<<<grid, kLaneThreads, kLaneSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_push(const LaneKernelParams& p, int grid, cudaStream_t stream) {
  cudaError_t rc = prepare_attrs();
  if (rc != cudaSuccess) return rc;
  push_kernel<<<grid, kLaneThreads, kLaneSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

int lane_kernel_max_ctas(int device) {
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  int per_sm = 0;
  if (prepare_attrs() == cudaSuccess) {
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, land_kernel, kLaneThreads,
                                                  kLaneSmemBytes);
  }
  cudaSetDevice(prev);
  return per_sm * sms;
}

}  // namespace ppb
