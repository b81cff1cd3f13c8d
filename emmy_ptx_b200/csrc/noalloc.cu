// noalloc.cu - the tensor-core batched matmul, launched without allocating any device memory.
//
// Some callers of this library cannot allocate device memory when they run a kernel: a host
// application whose memory pool already owns the GPU's memory (a cudaMalloc would fail or fragment
// it), or code on a latency-critical path, where cudaMalloc/cudaFree may synchronise the whole
// device.  The tensor-core bmm kernel needs 16 bytes of scratch beyond its inputs and outputs (the
// status word its bounded pipeline waits write on time-out); the allocating path gets that from a
// small per-executable device tensor.  Here the scratch is a fixed array in this library's own
// device memory instead, so a call allocates nothing, and emmy_bmm_bf16_noalloc_status reads the
// status word back.

#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "emmy_launch.h"
#include "internal.h"

// Largest scratch one call may use.  Every GPU that loads this library holds it until the process exits.
#define EMMY_NOALLOC_SCRATCH_BYTES 256
#define EMMY_NOALLOC_MAX_CONTEXTS 64

static __device__ __align__(256) unsigned char g_noalloc_scratch[EMMY_NOALLOC_SCRATCH_BYTES];

namespace {
// Device addresses of the array, one per CUDA context the library has run in.  Keyed on the
// context's process-unique id, so a context that was reset and created again (the array reloaded
// at a new address) gets a fresh look-up instead of a stale address.
std::mutex g_setup_mu;
unsigned long long g_ctx_ids[EMMY_NOALLOC_MAX_CONTEXTS] = {};
void* g_scratch_addr[EMMY_NOALLOC_MAX_CONTEXTS] = {};
int g_n_ctx = 0;

int runtime_fail(cudaError_t rc, const char* what) {
  return emmy_internal_fail(EMMY_ERR_RUNTIME_BASE + static_cast<int>(rc), "%s failed: %s (%d)", what,
                            cudaGetErrorString(rc), static_cast<int>(rc));
}

// The array's device address in the context emmy_init() selected, looked up once per context with
// that context current.  The host-side name of the array is only a stand-in, never a device address.
int scratch_address(const char* who, void** out) {
  unsigned long long ctx = 0;
  if (int rc = emmy_internal_ready(&ctx)) return rc;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  for (int i = 0; i < g_n_ctx; ++i) {
    if (g_ctx_ids[i] == ctx) {
      *out = g_scratch_addr[i];
      return 0;
    }
  }
  if (g_n_ctx == EMMY_NOALLOC_MAX_CONTEXTS)
    return emmy_internal_fail(EMMY_ERR_BAD_ARG, "%s: more than %d CUDA contexts", who, EMMY_NOALLOC_MAX_CONTEXTS);
  void* addr = nullptr;
  cudaError_t rc = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
  if (rc != cudaSuccess) return runtime_fail(rc, "cudaGetSymbolAddress");
  g_ctx_ids[g_n_ctx] = ctx;
  g_scratch_addr[g_n_ctx] = addr;
  ++g_n_ctx;
  *out = addr;
  return 0;
}
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
  void* scratch = nullptr;
  if (int rc = scratch_address("emmy_bmm_bf16_noalloc", &scratch)) return rc;
  // The array keeps the previous call's contents; the status word must start at zero.
  cudaError_t rc = cudaMemsetAsync(scratch, 0, scratch_bytes ? scratch_bytes : 16, static_cast<cudaStream_t>(stream));
  if (rc != cudaSuccess) return runtime_fail(rc, "cudaMemsetAsync (clearing the scratch)");
  uint64_t pa = a, pb = b, pc = c;
  uint64_t ps = reinterpret_cast<uint64_t>(scratch);
  void* args[6] = {&pa, &pb, &pc, const_cast<void*>(tmap_a), const_cast<void*>(tmap_b), &ps};
  const uint32_t g3[3] = {grid, 1, 1};
  const uint32_t b3[3] = {block, 1, 1};
  const uint32_t one[3] = {1, 1, 1};
  return emmy_launch(function, g3, b3, one, dyn_smem, stream, args, 6);
}

extern "C" int emmy_bmm_bf16_noalloc_status(uint32_t* word, void* stream) {
  if (!word) return emmy_internal_fail(EMMY_ERR_BAD_ARG, "emmy_bmm_bf16_noalloc_status: null word pointer");
  void* scratch = nullptr;
  if (int rc = scratch_address("emmy_bmm_bf16_noalloc_status", &scratch)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Ordered after the calls already queued on `stream`; the wait makes the word valid on return.
  cudaError_t rc = cudaMemcpyAsync(word, scratch, sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
  if (rc != cudaSuccess) return runtime_fail(rc, "cudaMemcpyAsync (reading the status word)");
  rc = cudaStreamSynchronize(s);
  if (rc != cudaSuccess) return runtime_fail(rc, "cudaStreamSynchronize");
  return 0;
}
