// noalloc.cu - the tensor-core batched matmul, launched without allocating any device memory.
//
// Some callers of this library cannot allocate device memory when they run a kernel: a host
// application whose memory pool already owns the GPU's memory (a cudaMalloc would fail or fragment
// it), or code on a latency-critical path, where cudaMalloc/cudaFree may synchronise the whole
// device.  The tensor-core bmm kernel needs 16 bytes of scratch beyond its inputs and outputs (the
// status word its bounded pipeline waits write on time-out); the allocating path gets that from a
// small per-executable device tensor.  Here the scratch is a fixed array in this library's own
// device memory instead, so a call allocates nothing.

#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "emmy_launch.h"
#include "internal.h"

// Largest scratch one call may use.  Every GPU that loads this library holds it until the process exits.
#define EMMY_NOALLOC_SCRATCH_BYTES 256
#define EMMY_NOALLOC_MAX_DEVICES 64

static __device__ __align__(256) unsigned char g_noalloc_scratch[EMMY_NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_setup_mu;
void* g_scratch_addr[EMMY_NOALLOC_MAX_DEVICES] = {};
}  // namespace

extern "C" int emmy_bmm_bf16_noalloc(void* function, const void* tmap_a, const void* tmap_b, uint64_t a,
                                     uint64_t b, uint64_t c, uint32_t grid, uint32_t block,
                                     uint32_t dyn_smem, uint32_t scratch_bytes, void* stream) {
  if (!function || !tmap_a || !tmap_b || !a || !b || !c || grid == 0 || block == 0)
    return emmy_internal_fail(EMMY_ERR_BAD_ARG, "emmy_bmm_bf16_noalloc: null handle/pointer or empty launch");
  if (scratch_bytes > EMMY_NOALLOC_SCRATCH_BYTES)
    return emmy_internal_fail(EMMY_ERR_BAD_ARG,
                              "emmy_bmm_bf16_noalloc: the kernel needs %u bytes of scratch, more than the "
                              "%d bytes this entry point reserves",
                              scratch_bytes, EMMY_NOALLOC_SCRATCH_BYTES);
  int dev = -1;
  cudaError_t rc = cudaGetDevice(&dev);
  if (rc != cudaSuccess || dev < 0 || dev >= EMMY_NOALLOC_MAX_DEVICES)
    return emmy_internal_fail(EMMY_ERR_NOT_INIT, "emmy_bmm_bf16_noalloc: no current device (%s)",
                              cudaGetErrorString(rc));
  void* scratch = nullptr;
  {
    // Set-up, once per device, with that device current: the host-side name of the array is only a
    // stand-in, so the kernel gets the device address the runtime reports for it.
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_addr[dev]) {
      rc = cudaGetSymbolAddress(&g_scratch_addr[dev], g_noalloc_scratch);
      if (rc != cudaSuccess) {
        g_scratch_addr[dev] = nullptr;
        return emmy_internal_fail(EMMY_ERR_NOT_INIT, "emmy_bmm_bf16_noalloc: cudaGetSymbolAddress failed: %s",
                                  cudaGetErrorString(rc));
      }
    }
    scratch = g_scratch_addr[dev];
  }
  // The array keeps the previous call's contents; the status word must start at zero.
  rc = cudaMemsetAsync(scratch, 0, scratch_bytes ? scratch_bytes : 16, static_cast<cudaStream_t>(stream));
  if (rc != cudaSuccess)
    return emmy_internal_fail(EMMY_ERR_BAD_ARG, "emmy_bmm_bf16_noalloc: clearing the scratch failed: %s",
                              cudaGetErrorString(rc));
  uint64_t pa = a, pb = b, pc = c;
  uint64_t ps = reinterpret_cast<uint64_t>(scratch);
  void* args[6] = {&pa, &pb, &pc, const_cast<void*>(tmap_a), const_cast<void*>(tmap_b), &ps};
  const uint32_t g3[3] = {grid, 1, 1};
  const uint32_t b3[3] = {block, 1, 1};
  const uint32_t one[3] = {1, 1, 1};
  return emmy_launch(function, g3, b3, one, dyn_smem, stream, args, 6);
}
