// Device-side building blocks for the sm_100a data-movement kernels:
// mbarrier + bulk-copy (TMA, non-tensor, never multicast) wrappers,
// system-scope flag operations with bounded spins, and the chunk checksum.
//
// Every wait in this file is bounded by a %globaltimer deadline; on expiry the
// caller records an error status and returns instead of trapping.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace ppb {
namespace dev {

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- system-scope flags -----------------------------------------------------

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;"
               : "=r"(old)
               : "l"(p), "r"(v)
               : "memory");
  return old;
}

__device__ __forceinline__ void fence_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

// (int32)(a - b) >= 0 : wrap-around safe "a has reached b".
__device__ __forceinline__ bool seq_reached(uint32_t a, uint32_t b) {
  return static_cast<int32_t>(a - b) >= 0;
}

// Spin until *flag has reached `target` (wrap-around compare).  Returns false
// when `deadline_ns` (absolute %globaltimer value) passes first.
__device__ __forceinline__ bool wait_flag_geq(const uint32_t* flag, uint32_t target,
                                              uint64_t deadline_ns) {
  uint32_t backoff = 32;
  uint32_t polls = 0;
  while (true) {
    if (seq_reached(ld_acquire_sys(flag), target)) return true;
    if ((++polls & 15u) == 0u && globaltimer_ns() > deadline_ns) return false;
    __nanosleep(backoff);
    if (backoff < 1024) backoff <<= 1;
  }
}

// ---- mbarrier ----------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase; false on deadline expiry.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t deadline_ns) {
  uint32_t polls = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++polls & 63u) == 0u && globaltimer_ns() > deadline_ns) return false;
  }
  return true;
}

// ---- bulk copies (TMA engine, 1-D, no multicast) -----------------------------
// Global -> shared, completion signalled on an mbarrier through complete_tx.
// Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Shared -> global through a bulk async-group.
__device__ __forceinline__ void bulk_s2g(void* gmem_dst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gmem_dst),
               "r"(smem_u32(smem_src)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until at most N bulk groups are still incomplete (writes performed).
template <int N>
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- plain vector access that bypasses L1 (data written by other agents) -----

__device__ __forceinline__ uint4 ld_cg_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ uint8_t ld_cg_u8(const void* p) {
  uint16_t v;
  asm volatile("ld.global.cg.u8 %0, [%1];" : "=h"(v) : "l"(p) : "memory");
  return static_cast<uint8_t>(v);
}

// ---- chunk checksum ------------------------------------------------------------
// The chunk is read as little-endian 32-bit words w_i (the final partial word
// zero-padded).  checksum = (sum_i w_i, sum_i (i+1) * w_i), both mod 2^64,
// with i the word index inside the chunk.  The position weight makes the sum
// sensitive to reordered or misplaced words; both halves combine with plain
// 64-bit adds, so partial sums from any number of threads/CTAs merge exactly.
struct Csum {
  unsigned long long s;
  unsigned long long w;
};

__device__ __forceinline__ void csum_word(Csum& c, uint32_t word, uint64_t word_index) {
  c.s += word;
  c.w += (word_index + 1ull) * static_cast<unsigned long long>(word);
}

__device__ __forceinline__ void csum_vec(Csum& c, uint4 v, uint64_t first_word) {
  csum_word(c, v.x, first_word);
  csum_word(c, v.y, first_word + 1);
  csum_word(c, v.z, first_word + 2);
  csum_word(c, v.w, first_word + 3);
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide reduction of a checksum pair, then one atomic add per CTA.
// `scratch` needs 2 * (blockDim.x / 32) entries.
__device__ __forceinline__ void csum_block_commit(Csum c, unsigned long long* out,
                                                  unsigned long long* scratch) {
  c.s = warp_sum(c.s);
  c.w = warp_sum(c.w);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  if (lane == 0) {
    scratch[2 * warp] = c.s;
    scratch[2 * warp + 1] = c.w;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long s = 0, w = 0;
    for (int i = 0; i < nwarps; ++i) {
      s += scratch[2 * i];
      w += scratch[2 * i + 1];
    }
    if (s | w) {
      atomicAdd(out, s);
      atomicAdd(out + 1, w);
    }
  }
  __syncthreads();
}

}  // namespace dev
}  // namespace ppb
