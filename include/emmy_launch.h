/*
 * emmy_launch.h - C ABI of the B200 launcher for kernels emitted by the emmy_ptx_b200 backend.
 *
 * It replaces the reference's ctypes path over nvcuda.dll (tools/localrun.py:32-105,
 * tools/oracle.py:37-157, tools/bench.py:32-83): the same driver-API steps (load a module from
 * PTX, look up an entry, raise the dynamic shared-memory limit, launch, time with events, copy)
 * behind plain pointers and sizes, plus TMA descriptor encoding and one NCCL all-reduce.
 *
 * Conventions
 *  - Every function returns 0 on success.  Non-zero values are the CUresult of the failing
 *    driver call, EMMY_ERR_NCCL_BASE + ncclResult_t for NCCL, EMMY_ERR_RUNTIME_BASE + cudaError_t
 *    for the CUDA runtime calls of the no-allocation entry points, or one of the EMMY_ERR_* codes.
 *    emmy_last_error() returns a description of the last failure on the calling thread.
 *    Nothing in this library calls exit() or abort().
 *  - Device pointers are CUdeviceptr values (uint64_t) owned by the caller; module, function,
 *    event and communicator handles are owned by the library.
 *  - One CUDA context per device: the device's primary context (the one the CUDA runtime and
 *    PyTorch use), selected by emmy_init().  Multi-GPU runs use one process per GPU; a process
 *    that drives several devices calls emmy_init(d) before working on device d.
 *  - libcuda.so.1 and libnccl.so.2 are opened on first use, so the library itself loads on a
 *    host without a GPU.
 */
#ifndef EMMY_LAUNCH_H
#define EMMY_LAUNCH_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EMMY_ERR_NO_DRIVER 10001   /* libcuda.so.1 could not be opened or lacks a symbol */
#define EMMY_ERR_NOT_INIT 10002    /* emmy_init() has not succeeded on this thread */
#define EMMY_ERR_BAD_ARG 10003     /* null handle, zero size, misaligned pointer, ... */
#define EMMY_ERR_NO_NCCL 10004     /* libnccl.so.2 could not be opened or lacks a symbol */
#define EMMY_ERR_NCCL_BASE 20000   /* + ncclResult_t */
#define EMMY_ERR_RUNTIME_BASE 30000 /* + cudaError_t (CUDA runtime calls) */

/* ABI version of this header (bumped on incompatible change). */
int emmy_version(void);

/* Copies the last error message of this thread into buf (always NUL-terminated). */
int emmy_last_error(char* buf, size_t n);

/* Opens the driver and selects device `device`: its primary context (retained on the first call
 * for that device) becomes current, and every later call runs in it until emmy_init selects
 * another device.  Replaces cuInit/cuDeviceGet/cuCtxCreate in tools/localrun.py:33-46. */
int emmy_init(int device);

/* cuDeviceGetAttribute for the initialised device. */
int emmy_device_attribute(int attr, int* value);

/* Loads a module from NUL-terminated PTX (JIT-compiled by the driver for this GPU).  On failure
 * the JIT error log is copied into log (if non-null).  Replaces cuModuleLoadData(Ex)
 * (tools/localrun.py:92, tools/oracle.py:131). */
int emmy_module_load_ptx(const char* ptx, void** module, char* log, size_t log_size);

/* Loads a module from a cubin image (ptxas output). */
int emmy_module_load_image(const void* image, void** module);

int emmy_module_unload(void* module);

/* cuModuleGetFunction (tools/localrun.py:94). */
int emmy_get_function(void* module, const char* entry, void** function);

/* CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, needed above 48 KiB (tools/localrun.py:96-98). */
int emmy_set_max_dyn_smem(void* function, int bytes);

/* The preferred shared-memory share of the L1/shared split, in percent (-1 = no preference).
 * Kernels meant to share SMs (a pre-pass beside a large-shared-memory kernel) ask for the same
 * split.  No reference counterpart. */
int emmy_set_smem_carveout(void* function, int percent);

/* cuFuncGetAttribute (registers, local memory, max threads, ...). */
int emmy_func_attribute(void* function, int attr, int* value);

/* cuLaunchKernelEx.  args[i] points at the value of parameter i (nargs of them); cluster may be
 * null or {1,1,1} for no cluster; stream 0 is the legacy default stream.  Replaces
 * cuLaunchKernel (tools/localrun.py:101-103). */
int emmy_launch(void* function, const uint32_t grid[3], const uint32_t block[3],
                const uint32_t cluster[3], uint32_t dyn_smem, void* stream,
                void** args, uint32_t nargs);

/* Launch flags for the _ex variants. */
#define EMMY_LAUNCH_PDL 1u  /* programmatic dependent launch (CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_
                               STREAM_SERIALIZATION): the kernel may start while the previous work
                               in the stream finishes; it must run griddepcontrol.wait before its
                               first global memory access, as every generic kernel this backend
                               emits does (launch record "pdl": true) */

/* emmy_launch with flags (EMMY_LAUNCH_*); unknown bits are refused with EMMY_ERR_BAD_ARG.
 * No reference counterpart: the reference launches with cuLaunchKernel only. */
int emmy_launch_ex(void* function, const uint32_t grid[3], const uint32_t block[3],
                   const uint32_t cluster[3], uint32_t dyn_smem, void* stream,
                   void** args, uint32_t nargs, uint32_t flags);

/* Launch with every parameter a 64-bit value (the emitted kernels' ABI: .param .u64 p_<arg> in
 * arg_order, tools/localrun.py:175-184).  Each pointer must be a multiple of align[i] bytes
 * (align may be null); a misaligned pointer is refused with EMMY_ERR_BAD_ARG before launch. */
int emmy_launch_u64(void* function, const uint32_t grid[3], const uint32_t block[3],
                    uint32_t dyn_smem, void* stream, const uint64_t* params,
                    const uint32_t* align, uint32_t nparams);

/* emmy_launch_u64 with flags (EMMY_LAUNCH_*). */
int emmy_launch_u64_ex(void* function, const uint32_t grid[3], const uint32_t block[3],
                       uint32_t dyn_smem, void* stream, const uint64_t* params,
                       const uint32_t* align, uint32_t nparams, uint32_t flags);

/* cuTensorMapEncodeTiled into a 128-byte, 64-byte-aligned buffer.  dtype is a
 * CUtensorMapDataType, strides are the rank-1 byte strides of dims 1..rank-1. */
int emmy_tmap_encode_tiled(void* tmap, int dtype, uint32_t rank, uint64_t global_address,
                           const uint64_t* dims, const uint64_t* strides_bytes,
                           const uint32_t* box, const uint32_t* elem_strides,
                           int interleave, int swizzle, int l2_promotion, int oob_fill);

/* Events and synchronisation (tools/bench.py:66-83). */
int emmy_event_create(void** event);
int emmy_event_destroy(void* event);
int emmy_event_record(void* event, void* stream);
int emmy_event_synchronize(void* event);
int emmy_event_elapsed_ms(void* start, void* stop, float* ms);
int emmy_stream_synchronize(void* stream);
int emmy_ctx_synchronize(void);

/* An event with CUevent_flags (1 blocking sync, 2 no timing); a non-blocking stream of the
 * context; a stream waiting on an event.  A module whose entries run on two streams (an
 * overlapped pre-pass) forks and joins through these.  No reference counterpart: the reference
 * launches one kernel on one stream (tools/localrun.py:98-105). */
int emmy_event_create_flags(void** event, unsigned int flags);
int emmy_stream_create(void** stream);
int emmy_stream_destroy(void* stream);
int emmy_stream_wait_event(void* stream, void* event);

/* Memory (caller-owned device pointers). */
int emmy_mem_alloc(uint64_t* dptr, size_t bytes);
int emmy_mem_free(uint64_t dptr);

/* Cross-process device memory for the peer exchange of the multi-GPU sum (one process per GPU):
 * emmy_ipc_get_handle exports an allocation made by emmy_mem_alloc as a 64-byte handle, which the
 * caller passes to the other ranks; emmy_ipc_open maps a peer's allocation into this process
 * (cuIpcOpenMemHandle with lazy peer access over NVLink) and emmy_ipc_close unmaps it.  No
 * counterpart in the reference, which runs on one GPU (the replacement for its role here is one
 * ncclAllReduce). */
int emmy_ipc_get_handle(uint64_t dptr, char handle[64]);
int emmy_ipc_open(const char handle[64], uint64_t* dptr);
int emmy_ipc_close(uint64_t dptr);
int emmy_memset_d32_async(uint64_t dptr, uint32_t value, size_t count, void* stream);
int emmy_memcpy_htod_async(uint64_t dst, const void* src, size_t bytes, void* stream);
int emmy_memcpy_dtoh_async(void* dst, uint64_t src, size_t bytes, void* stream);

/* NCCL: one communicator per process (one process per GPU).  The 128-byte unique id made by
 * rank 0 is shared with the other ranks by the caller.  dtype 0 = float32, 1 = int32. */
int emmy_nccl_available(void);
int emmy_nccl_get_unique_id(char uid[128]);
int emmy_nccl_init(int rank, int nranks, const char uid[128]);
int emmy_allreduce_sum(uint64_t buf, size_t count, int dtype, void* stream);
int emmy_nccl_destroy(void);

/* Runs the tensor-core batched matmul (a launch record of kind "tcgen05_gemm", the one-CTA-per-tile kernel
 * that compile option gemm_pair=false builds: parameters A, B, C, the two TMA descriptors, then a scratch
 * pointer; the default CTA-pair kernel needs a cluster launch and is not taken here) without allocating
 * device memory, for callers that cannot
 * allocate when they launch: a host whose own pool already owns the GPU's memory, or a latency-critical
 * path where cudaMalloc/cudaFree may synchronise the device.  No counterpart in the reference.
 *  - function: the kernel, loaded with emmy_module_load_ptx / emmy_get_function; tmap_a / tmap_b: its
 *    descriptors from emmy_tmap_encode_tiled; a, b, c: device pointers; grid, block, dyn_smem: from the
 *    launch record; scratch_bytes: the record's scratch need (16 for the status word), at most 256 —
 *    larger values are refused with EMMY_ERR_BAD_ARG.
 *  - The scratch is a fixed 256-byte array in this library's device memory, held on every GPU that loads
 *    the library until the process exits.  The first call on a device looks up its address (with that
 *    device current); make that first call before any stream capture.
 *  - Every call uses the same array and clears it first; calls that overlap on the GPU race on it.
 *  - Needs emmy_init() on the calling thread first (EMMY_ERR_NOT_INIT otherwise).
 *  - A kernel whose bounded pipeline wait timed out returns early with C incomplete and a non-zero
 *    status word; read it with emmy_bmm_bf16_noalloc_status. */
int emmy_bmm_bf16_noalloc(void* function, const void* tmap_a, const void* tmap_b, uint64_t a, uint64_t b,
                          uint64_t c, uint32_t grid, uint32_t block, uint32_t dyn_smem,
                          uint32_t scratch_bytes, void* stream);

/* Reads the status word of the last emmy_bmm_bf16_noalloc call queued on `stream` into *word
 * (0 = every wait completed; otherwise the code of the wait that timed out).  It queues one 4-byte
 * device-to-host copy from the fixed array on `stream` and waits for that stream, so the word is
 * valid on return; it allocates nothing.  With calls in flight on other streams the word may be
 * theirs (the array is shared).  No counterpart in the reference. */
int emmy_bmm_bf16_noalloc_status(uint32_t* word, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* EMMY_LAUNCH_H */
