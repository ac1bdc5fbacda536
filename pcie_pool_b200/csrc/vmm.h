// Device buffers shared between processes through CUDA virtual memory
// management (VMM): the allocation is created exportable as a POSIX file
// descriptor, the descriptor travels to another process (SCM_RIGHTS over an
// AF_UNIX socket), and that process imports it and maps it into its own
// address space.  Unlike a legacy CUDA IPC handle, the exported object is an
// ordinary file descriptor: it can be passed, duplicated and closed with the
// usual POSIX rules, and the memory lives until every mapping and descriptor
// is gone.
#pragma once

#include <cstdint>

namespace ppb {

struct VmmBuffer {
  uint64_t ptr = 0;    // device address in this process
  uint64_t size = 0;   // mapped bytes (a multiple of the allocation granularity)
  int fd = -1;         // exported descriptor (owner only; -1 for imports)
  int device = -1;
};

// Allocate `bytes` (rounded up to the granularity) on `device`, map it
// read/write for `device`, and export a POSIX descriptor.
VmmBuffer vmm_alloc(int device, uint64_t bytes);
// Import a descriptor exported by vmm_alloc (possibly in another process) and
// map `size` bytes for `device`.  The descriptor stays owned by the caller.
VmmBuffer vmm_import(int fd, int device, uint64_t size);
// Unmap and release a buffer mapped by vmm_alloc / vmm_import in this process.
void vmm_release(uint64_t ptr);
// Allocation granularity of `device` (bytes).
uint64_t vmm_granularity(int device);

}  // namespace ppb
