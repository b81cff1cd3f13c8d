// emmy_launch.cpp - C ABI launcher over libcuda (driver API) and NCCL, see include/emmy_launch.h.
//
// The driver and NCCL are opened with dlopen on first use: the library links only libdl, so it
// loads (and its symbols can be checked) on a machine without a GPU driver.  Every entry point
// returns a status code; the message for the last failure is kept per thread.

#include "emmy_launch.h"
#include "internal.h"

#include <cuda.h>
#include <dlfcn.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

// ---- driver entry points ---------------------------------------------------------------------
struct Driver {
  void* lib = nullptr;
  CUresult (*Init)(unsigned int);
  CUresult (*DeviceGet)(CUdevice*, int);
  CUresult (*DeviceGetAttribute)(int*, CUdevice_attribute, CUdevice);
  CUresult (*PrimaryCtxRetain)(CUcontext*, CUdevice);
  CUresult (*CtxSetCurrent)(CUcontext);
  CUresult (*CtxGetCurrent)(CUcontext*);
  CUresult (*CtxGetId)(CUcontext, unsigned long long*);  // optional (CUDA 12.0+)
  CUresult (*CtxSynchronize)(void);
  CUresult (*ModuleLoadDataEx)(CUmodule*, const void*, unsigned int, CUjit_option*, void**);
  CUresult (*ModuleLoadData)(CUmodule*, const void*);
  CUresult (*ModuleUnload)(CUmodule);
  CUresult (*ModuleGetFunction)(CUfunction*, CUmodule, const char*);
  CUresult (*FuncSetAttribute)(CUfunction, CUfunction_attribute, int);
  CUresult (*FuncGetAttribute)(int*, CUfunction_attribute, CUfunction);
  CUresult (*LaunchKernelEx)(const CUlaunchConfig*, CUfunction, void**, void**);
  CUresult (*EventCreate)(CUevent*, unsigned int);
  CUresult (*EventDestroy)(CUevent);
  CUresult (*EventRecord)(CUevent, CUstream);
  CUresult (*EventSynchronize)(CUevent);
  CUresult (*EventElapsedTime)(float*, CUevent, CUevent);
  CUresult (*StreamSynchronize)(CUstream);
  CUresult (*StreamCreate)(CUstream*, unsigned int);
  CUresult (*StreamDestroy)(CUstream);
  CUresult (*StreamWaitEvent)(CUstream, CUevent, unsigned int);
  CUresult (*MemAlloc)(CUdeviceptr*, size_t);
  CUresult (*MemFree)(CUdeviceptr);
  CUresult (*MemsetD32Async)(CUdeviceptr, unsigned int, size_t, CUstream);
  CUresult (*MemcpyHtoDAsync)(CUdeviceptr, const void*, size_t, CUstream);
  CUresult (*MemcpyDtoHAsync)(void*, CUdeviceptr, size_t, CUstream);
  CUresult (*TensorMapEncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  CUresult (*GetErrorString)(CUresult, const char**);
  CUresult (*IpcGetMemHandle)(CUipcMemHandle*, CUdeviceptr);
  CUresult (*IpcOpenMemHandle)(CUdeviceptr*, CUipcMemHandle, unsigned int);
  CUresult (*IpcCloseMemHandle)(CUdeviceptr);
};

Driver g_drv;
std::mutex g_mu;
bool g_loaded = false;
// The selected device: every call after emmy_init(d) runs in d's primary context.  Each device's
// primary context is retained once, on its first emmy_init, and kept for the process's lifetime.
constexpr int kMaxDevices = 64;
CUcontext g_ctxs[kMaxDevices] = {};
CUdevice g_devs[kMaxDevices] = {};
CUcontext g_ctx = nullptr;
CUdevice g_dev = 0;

template <typename T>
bool sym(void* lib, T& fn, const char* name) {
  fn = reinterpret_cast<T>(dlsym(lib, name));
  return fn != nullptr;
}

int load_driver() {
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_loaded) return 0;
  void* lib = dlopen("libcuda.so.1", RTLD_NOW | RTLD_GLOBAL);
  if (!lib) return fail(EMMY_ERR_NO_DRIVER, "cannot open libcuda.so.1: %s", dlerror());
  Driver d;
  d.lib = lib;
  bool ok = sym(lib, d.Init, "cuInit") && sym(lib, d.DeviceGet, "cuDeviceGet") &&
            sym(lib, d.DeviceGetAttribute, "cuDeviceGetAttribute") &&
            sym(lib, d.PrimaryCtxRetain, "cuDevicePrimaryCtxRetain") &&
            sym(lib, d.CtxSetCurrent, "cuCtxSetCurrent") &&
            sym(lib, d.CtxGetCurrent, "cuCtxGetCurrent") &&
            sym(lib, d.CtxSynchronize, "cuCtxSynchronize") &&
            sym(lib, d.ModuleLoadDataEx, "cuModuleLoadDataEx") &&
            sym(lib, d.ModuleLoadData, "cuModuleLoadData") &&
            sym(lib, d.ModuleUnload, "cuModuleUnload") &&
            sym(lib, d.ModuleGetFunction, "cuModuleGetFunction") &&
            sym(lib, d.FuncSetAttribute, "cuFuncSetAttribute") &&
            sym(lib, d.FuncGetAttribute, "cuFuncGetAttribute") &&
            sym(lib, d.LaunchKernelEx, "cuLaunchKernelEx") &&
            sym(lib, d.EventCreate, "cuEventCreate") &&
            sym(lib, d.EventDestroy, "cuEventDestroy_v2") &&
            sym(lib, d.EventRecord, "cuEventRecord") &&
            sym(lib, d.EventSynchronize, "cuEventSynchronize") &&
            sym(lib, d.EventElapsedTime, "cuEventElapsedTime") &&
            sym(lib, d.StreamSynchronize, "cuStreamSynchronize") &&
            sym(lib, d.StreamCreate, "cuStreamCreate") &&
            sym(lib, d.StreamDestroy, "cuStreamDestroy_v2") &&
            sym(lib, d.StreamWaitEvent, "cuStreamWaitEvent") &&
            sym(lib, d.MemAlloc, "cuMemAlloc_v2") && sym(lib, d.MemFree, "cuMemFree_v2") &&
            sym(lib, d.MemsetD32Async, "cuMemsetD32Async") &&
            sym(lib, d.MemcpyHtoDAsync, "cuMemcpyHtoDAsync_v2") &&
            sym(lib, d.MemcpyDtoHAsync, "cuMemcpyDtoHAsync_v2") &&
            sym(lib, d.TensorMapEncodeTiled, "cuTensorMapEncodeTiled") &&
            sym(lib, d.GetErrorString, "cuGetErrorString") &&
            sym(lib, d.IpcGetMemHandle, "cuIpcGetMemHandle") &&
            sym(lib, d.IpcOpenMemHandle, "cuIpcOpenMemHandle_v2") &&
            sym(lib, d.IpcCloseMemHandle, "cuIpcCloseMemHandle");
  if (!ok) return fail(EMMY_ERR_NO_DRIVER, "libcuda.so.1 lacks a required symbol: %s", dlerror());
  if (!sym(lib, d.CtxGetId, "cuCtxGetId")) d.CtxGetId = nullptr;
  g_drv = d;
  g_loaded = true;
  return 0;
}

int cu(CUresult rc, const char* what) {
  if (rc == CUDA_SUCCESS) return 0;
  const char* msg = nullptr;
  if (g_loaded && g_drv.GetErrorString) g_drv.GetErrorString(rc, &msg);
  return fail(static_cast<int>(rc), "%s failed: %s (%d)", what, msg ? msg : "unknown error",
              static_cast<int>(rc));
}

// Every call after emmy_init runs in the device's primary context, whatever thread it is on.
int ready() {
  if (!g_loaded || !g_ctx) return fail(EMMY_ERR_NOT_INIT, "emmy_init() has not been called");
  CUcontext cur = nullptr;
  if (g_drv.CtxGetCurrent(&cur) != CUDA_SUCCESS || cur != g_ctx)
    return cu(g_drv.CtxSetCurrent(g_ctx), "cuCtxSetCurrent");
  return 0;
}

// ---- NCCL -----------------------------------------------------------------------------------
typedef struct { char internal[128]; } NcclUid;
typedef void* NcclComm;
struct Nccl {
  void* lib = nullptr;
  int (*GetUniqueId)(NcclUid*);
  int (*CommInitRank)(NcclComm*, int, NcclUid, int);
  int (*AllReduce)(const void*, void*, size_t, int, int, NcclComm, CUstream);
  int (*CommDestroy)(NcclComm);
  const char* (*GetErrorString)(int);
};
Nccl g_nccl;
bool g_nccl_loaded = false;
NcclComm g_comm = nullptr;

int load_nccl() {
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_nccl_loaded) return 0;
  // reuse an already-loaded libnccl (e.g. PyTorch's) when there is one
  void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
  if (!lib) lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!lib) return fail(EMMY_ERR_NO_NCCL, "cannot open libnccl.so.2: %s", dlerror());
  Nccl n;
  n.lib = lib;
  bool ok = sym(lib, n.GetUniqueId, "ncclGetUniqueId") && sym(lib, n.CommInitRank, "ncclCommInitRank") &&
            sym(lib, n.AllReduce, "ncclAllReduce") && sym(lib, n.CommDestroy, "ncclCommDestroy") &&
            sym(lib, n.GetErrorString, "ncclGetErrorString");
  if (!ok) return fail(EMMY_ERR_NO_NCCL, "libnccl.so.2 lacks a required symbol: %s", dlerror());
  g_nccl = n;
  g_nccl_loaded = true;
  return 0;
}

int nc(int rc, const char* what) {
  if (rc == 0) return 0;
  const char* msg = g_nccl.GetErrorString ? g_nccl.GetErrorString(rc) : "unknown";
  return fail(EMMY_ERR_NCCL_BASE + rc, "%s failed: %s (%d)", what, msg, rc);
}

}  // namespace

int emmy_internal_ready(unsigned long long* context_id) {
  if (int rc = ready()) return rc;
  if (context_id) {
    // A context's id is unique for the process's lifetime: a primary context that was reset and
    // created again gets a new one, so a cache keyed on it never serves a stale device address.
    unsigned long long id = 0;
    if (g_drv.CtxGetId && g_drv.CtxGetId(g_ctx, &id) == CUDA_SUCCESS)
      *context_id = id;
    else
      *context_id = static_cast<unsigned long long>(reinterpret_cast<uintptr_t>(g_ctx));
  }
  return 0;
}

int emmy_internal_fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

extern "C" {

int emmy_version(void) { return 1; }

int emmy_last_error(char* buf, size_t n) {
  if (!buf || n == 0) return EMMY_ERR_BAD_ARG;
  std::snprintf(buf, n, "%s", g_err.c_str());
  return 0;
}

int emmy_init(int device) {
  if (device < 0 || device >= kMaxDevices) return fail(EMMY_ERR_BAD_ARG, "device %d out of range", device);
  if (int rc = load_driver()) return rc;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_ctxs[device]) {
    if (int rc = cu(g_drv.Init(0), "cuInit")) return rc;
    CUdevice dev;
    if (int rc = cu(g_drv.DeviceGet(&dev, device), "cuDeviceGet")) return rc;
    CUcontext ctx;
    if (int rc = cu(g_drv.PrimaryCtxRetain(&ctx, dev), "cuDevicePrimaryCtxRetain")) return rc;
    g_ctxs[device] = ctx;
    g_devs[device] = dev;
  }
  if (int rc = cu(g_drv.CtxSetCurrent(g_ctxs[device]), "cuCtxSetCurrent")) return rc;
  g_ctx = g_ctxs[device];
  g_dev = g_devs[device];
  return 0;
}

int emmy_device_attribute(int attr, int* value) {
  if (!value) return fail(EMMY_ERR_BAD_ARG, "null value pointer");
  if (int rc = ready()) return rc;
  return cu(g_drv.DeviceGetAttribute(value, static_cast<CUdevice_attribute>(attr), g_dev),
            "cuDeviceGetAttribute");
}

int emmy_module_load_ptx(const char* ptx, void** module, char* log, size_t log_size) {
  if (!ptx || !module) return fail(EMMY_ERR_BAD_ARG, "null ptx or module pointer");
  if (int rc = ready()) return rc;
  static thread_local char errlog[16384];
  errlog[0] = 0;
  CUjit_option opts[2] = {CU_JIT_ERROR_LOG_BUFFER, CU_JIT_ERROR_LOG_BUFFER_SIZE_BYTES};
  void* vals[2] = {errlog, reinterpret_cast<void*>(static_cast<uintptr_t>(sizeof(errlog)))};
  CUmodule mod = nullptr;
  CUresult r = g_drv.ModuleLoadDataEx(&mod, ptx, 2, opts, vals);
  if (log && log_size) std::snprintf(log, log_size, "%s", errlog);
  if (r != CUDA_SUCCESS) {
    int rc = cu(r, "cuModuleLoadDataEx");
    g_err += "\n";
    g_err += errlog;
    return rc;
  }
  *module = mod;
  return 0;
}

int emmy_module_load_image(const void* image, void** module) {
  if (!image || !module) return fail(EMMY_ERR_BAD_ARG, "null image or module pointer");
  if (int rc = ready()) return rc;
  CUmodule mod = nullptr;
  if (int rc = cu(g_drv.ModuleLoadData(&mod, image), "cuModuleLoadData")) return rc;
  *module = mod;
  return 0;
}

int emmy_module_unload(void* module) {
  if (!module) return fail(EMMY_ERR_BAD_ARG, "null module");
  if (int rc = ready()) return rc;
  return cu(g_drv.ModuleUnload(static_cast<CUmodule>(module)), "cuModuleUnload");
}

int emmy_get_function(void* module, const char* entry, void** function) {
  if (!module || !entry || !function) return fail(EMMY_ERR_BAD_ARG, "null argument");
  if (int rc = ready()) return rc;
  CUfunction fn = nullptr;
  if (int rc = cu(g_drv.ModuleGetFunction(&fn, static_cast<CUmodule>(module), entry),
                  "cuModuleGetFunction"))
    return rc;
  *function = fn;
  return 0;
}

int emmy_set_max_dyn_smem(void* function, int bytes) {
  if (!function) return fail(EMMY_ERR_BAD_ARG, "null function");
  if (int rc = ready()) return rc;
  return cu(g_drv.FuncSetAttribute(static_cast<CUfunction>(function),
                                   CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, bytes),
            "cuFuncSetAttribute(MAX_DYNAMIC_SHARED_SIZE_BYTES)");
}

int emmy_set_smem_carveout(void* function, int percent) {
  if (!function) return fail(EMMY_ERR_BAD_ARG, "null function");
  if (percent < -1 || percent > 100) return fail(EMMY_ERR_BAD_ARG, "carveout outside -1..100");
  if (int rc = ready()) return rc;
  return cu(g_drv.FuncSetAttribute(static_cast<CUfunction>(function),
                                   CU_FUNC_ATTRIBUTE_PREFERRED_SHARED_MEMORY_CARVEOUT, percent),
            "cuFuncSetAttribute(PREFERRED_SHARED_MEMORY_CARVEOUT)");
}

int emmy_func_attribute(void* function, int attr, int* value) {
  if (!function || !value) return fail(EMMY_ERR_BAD_ARG, "null argument");
  if (int rc = ready()) return rc;
  return cu(g_drv.FuncGetAttribute(value, static_cast<CUfunction_attribute>(attr),
                                   static_cast<CUfunction>(function)),
            "cuFuncGetAttribute");
}

int emmy_launch(void* function, const uint32_t grid[3], const uint32_t block[3],
                const uint32_t cluster[3], uint32_t dyn_smem, void* stream, void** args,
                uint32_t nargs) {
  return emmy_launch_ex(function, grid, block, cluster, dyn_smem, stream, args, nargs, 0);
}

int emmy_launch_ex(void* function, const uint32_t grid[3], const uint32_t block[3],
                   const uint32_t cluster[3], uint32_t dyn_smem, void* stream, void** args,
                   uint32_t nargs, uint32_t flags) {
  if (!function || !grid || !block) return fail(EMMY_ERR_BAD_ARG, "null function/grid/block");
  if (flags & ~static_cast<uint32_t>(EMMY_LAUNCH_PDL)) return fail(EMMY_ERR_BAD_ARG, "unknown launch flags 0x%x", flags);
  if (nargs && !args) return fail(EMMY_ERR_BAD_ARG, "null args with nargs > 0");
  if (int rc = ready()) return rc;
  CUlaunchConfig cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDimX = grid[0];
  cfg.gridDimY = grid[1];
  cfg.gridDimZ = grid[2];
  cfg.blockDimX = block[0];
  cfg.blockDimY = block[1];
  cfg.blockDimZ = block[2];
  cfg.sharedMemBytes = dyn_smem;
  cfg.hStream = static_cast<CUstream>(stream);
  CUlaunchAttribute attr[2];
  std::memset(attr, 0, sizeof(attr));
  unsigned n_attr = 0;
  if (cluster && (cluster[0] > 1 || cluster[1] > 1 || cluster[2] > 1)) {
    attr[n_attr].id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
    attr[n_attr].value.clusterDim.x = cluster[0];
    attr[n_attr].value.clusterDim.y = cluster[1];
    attr[n_attr].value.clusterDim.z = cluster[2];
    ++n_attr;
  }
  if (flags & EMMY_LAUNCH_PDL) {
    // the kernel executes griddepcontrol.wait before touching global memory, so it may be
    // scheduled while the previous work in the stream is still finishing
    attr[n_attr].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
    attr[n_attr].value.programmaticStreamSerializationAllowed = 1;
    ++n_attr;
  }
  if (n_attr) {
    cfg.attrs = attr;
    cfg.numAttrs = n_attr;
  }
  return cu(g_drv.LaunchKernelEx(&cfg, static_cast<CUfunction>(function), args, nullptr),
            "cuLaunchKernelEx");
}

int emmy_launch_u64(void* function, const uint32_t grid[3], const uint32_t block[3],
                    uint32_t dyn_smem, void* stream, const uint64_t* params,
                    const uint32_t* align, uint32_t nparams) {
  return emmy_launch_u64_ex(function, grid, block, dyn_smem, stream, params, align, nparams, 0);
}

int emmy_launch_u64_ex(void* function, const uint32_t grid[3], const uint32_t block[3],
                       uint32_t dyn_smem, void* stream, const uint64_t* params,
                       const uint32_t* align, uint32_t nparams, uint32_t flags) {
  if (nparams > 256) return fail(EMMY_ERR_BAD_ARG, "too many parameters (%u)", nparams);
  if (nparams && !params) return fail(EMMY_ERR_BAD_ARG, "null params");
  void* args[256];
  uint64_t vals[256];
  for (uint32_t i = 0; i < nparams; ++i) {
    vals[i] = params[i];
    if (align && align[i] > 1 && (params[i] % align[i]) != 0)
      return fail(EMMY_ERR_BAD_ARG, "parameter %u (0x%llx) is not %u-byte aligned", i,
                  static_cast<unsigned long long>(params[i]), align[i]);
    args[i] = &vals[i];
  }
  const uint32_t one[3] = {1, 1, 1};
  return emmy_launch_ex(function, grid, block, one, dyn_smem, stream, args, nparams, flags);
}

int emmy_tmap_encode_tiled(void* tmap, int dtype, uint32_t rank, uint64_t global_address,
                           const uint64_t* dims, const uint64_t* strides_bytes,
                           const uint32_t* box, const uint32_t* elem_strides, int interleave,
                           int swizzle, int l2_promotion, int oob_fill) {
  if (!tmap || !dims || !box || !elem_strides || (rank > 1 && !strides_bytes))
    return fail(EMMY_ERR_BAD_ARG, "null tensor-map argument");
  if (reinterpret_cast<uintptr_t>(tmap) % 64) return fail(EMMY_ERR_BAD_ARG, "tensor map not 64-byte aligned");
  if (rank < 1 || rank > 5) return fail(EMMY_ERR_BAD_ARG, "tensor rank %u out of range", rank);
  if (global_address % 16) return fail(EMMY_ERR_BAD_ARG, "tensor base not 16-byte aligned");
  if (int rc = load_driver()) return rc;
  return cu(g_drv.TensorMapEncodeTiled(
                static_cast<CUtensorMap*>(tmap), static_cast<CUtensorMapDataType>(dtype), rank,
                reinterpret_cast<void*>(global_address), dims, strides_bytes, box, elem_strides,
                static_cast<CUtensorMapInterleave>(interleave), static_cast<CUtensorMapSwizzle>(swizzle),
                static_cast<CUtensorMapL2promotion>(l2_promotion),
                static_cast<CUtensorMapFloatOOBfill>(oob_fill)),
            "cuTensorMapEncodeTiled");
}

int emmy_event_create(void** event) {
  if (!event) return fail(EMMY_ERR_BAD_ARG, "null event pointer");
  if (int rc = ready()) return rc;
  CUevent ev;
  if (int rc = cu(g_drv.EventCreate(&ev, CU_EVENT_DEFAULT), "cuEventCreate")) return rc;
  *event = ev;
  return 0;
}

int emmy_event_destroy(void* event) {
  if (int rc = ready()) return rc;
  return cu(g_drv.EventDestroy(static_cast<CUevent>(event)), "cuEventDestroy");
}

int emmy_event_record(void* event, void* stream) {
  if (int rc = ready()) return rc;
  return cu(g_drv.EventRecord(static_cast<CUevent>(event), static_cast<CUstream>(stream)),
            "cuEventRecord");
}

int emmy_event_synchronize(void* event) {
  if (int rc = ready()) return rc;
  return cu(g_drv.EventSynchronize(static_cast<CUevent>(event)), "cuEventSynchronize");
}

int emmy_event_elapsed_ms(void* start, void* stop, float* ms) {
  if (!ms) return fail(EMMY_ERR_BAD_ARG, "null ms pointer");
  if (int rc = ready()) return rc;
  return cu(g_drv.EventElapsedTime(ms, static_cast<CUevent>(start), static_cast<CUevent>(stop)),
            "cuEventElapsedTime");
}

int emmy_event_create_flags(void** event, unsigned int flags) {
  if (!event) return fail(EMMY_ERR_BAD_ARG, "null event pointer");
  if (flags & ~0x3u) return fail(EMMY_ERR_BAD_ARG, "unknown event flags");
  if (int rc = ready()) return rc;
  CUevent ev;
  if (int rc = cu(g_drv.EventCreate(&ev, flags), "cuEventCreate")) return rc;
  *event = ev;
  return 0;
}

int emmy_stream_create(void** stream) {
  if (!stream) return fail(EMMY_ERR_BAD_ARG, "null stream pointer");
  if (int rc = ready()) return rc;
  CUstream s;
  if (int rc = cu(g_drv.StreamCreate(&s, CU_STREAM_NON_BLOCKING), "cuStreamCreate")) return rc;
  *stream = s;
  return 0;
}

int emmy_stream_destroy(void* stream) {
  if (!stream) return fail(EMMY_ERR_BAD_ARG, "null stream");
  if (int rc = ready()) return rc;
  return cu(g_drv.StreamDestroy(static_cast<CUstream>(stream)), "cuStreamDestroy");
}

int emmy_stream_wait_event(void* stream, void* event) {
  if (!event) return fail(EMMY_ERR_BAD_ARG, "null event");
  if (int rc = ready()) return rc;
  return cu(g_drv.StreamWaitEvent(static_cast<CUstream>(stream), static_cast<CUevent>(event), 0),
            "cuStreamWaitEvent");
}

int emmy_stream_synchronize(void* stream) {
  if (int rc = ready()) return rc;
  return cu(g_drv.StreamSynchronize(static_cast<CUstream>(stream)), "cuStreamSynchronize");
}

int emmy_ctx_synchronize(void) {
  if (int rc = ready()) return rc;
  return cu(g_drv.CtxSynchronize(), "cuCtxSynchronize");
}

int emmy_mem_alloc(uint64_t* dptr, size_t bytes) {
  if (!dptr || bytes == 0) return fail(EMMY_ERR_BAD_ARG, "null pointer or zero size");
  if (int rc = ready()) return rc;
  CUdeviceptr p;
  if (int rc = cu(g_drv.MemAlloc(&p, bytes), "cuMemAlloc")) return rc;
  *dptr = p;
  return 0;
}

int emmy_mem_free(uint64_t dptr) {
  if (int rc = ready()) return rc;
  return cu(g_drv.MemFree(static_cast<CUdeviceptr>(dptr)), "cuMemFree");
}

int emmy_ipc_get_handle(uint64_t dptr, char handle[64]) {
  if (!dptr || !handle) return fail(EMMY_ERR_BAD_ARG, "null device pointer or handle buffer");
  if (int rc = ready()) return rc;
  CUipcMemHandle h;
  if (int rc = cu(g_drv.IpcGetMemHandle(&h, static_cast<CUdeviceptr>(dptr)), "cuIpcGetMemHandle")) return rc;
  std::memcpy(handle, h.reserved, sizeof(h.reserved));
  return 0;
}

int emmy_ipc_open(const char handle[64], uint64_t* dptr) {
  if (!handle || !dptr) return fail(EMMY_ERR_BAD_ARG, "null handle or result pointer");
  if (int rc = ready()) return rc;
  CUipcMemHandle h;
  std::memcpy(h.reserved, handle, sizeof(h.reserved));
  CUdeviceptr p = 0;
  // peer access to the exporting device is enabled on first use of the mapping
  if (int rc = cu(g_drv.IpcOpenMemHandle(&p, h, CU_IPC_MEM_LAZY_ENABLE_PEER_ACCESS), "cuIpcOpenMemHandle"))
    return rc;
  *dptr = p;
  return 0;
}

int emmy_ipc_close(uint64_t dptr) {
  if (!dptr) return fail(EMMY_ERR_BAD_ARG, "null device pointer");
  if (int rc = ready()) return rc;
  return cu(g_drv.IpcCloseMemHandle(static_cast<CUdeviceptr>(dptr)), "cuIpcCloseMemHandle");
}

int emmy_memset_d32_async(uint64_t dptr, uint32_t value, size_t count, void* stream) {
  if (int rc = ready()) return rc;
  return cu(g_drv.MemsetD32Async(dptr, value, count, static_cast<CUstream>(stream)),
            "cuMemsetD32Async");
}

int emmy_memcpy_htod_async(uint64_t dst, const void* src, size_t bytes, void* stream) {
  if (!src && bytes) return fail(EMMY_ERR_BAD_ARG, "null host source");
  if (int rc = ready()) return rc;
  return cu(g_drv.MemcpyHtoDAsync(dst, src, bytes, static_cast<CUstream>(stream)),
            "cuMemcpyHtoDAsync");
}

int emmy_memcpy_dtoh_async(void* dst, uint64_t src, size_t bytes, void* stream) {
  if (!dst && bytes) return fail(EMMY_ERR_BAD_ARG, "null host destination");
  if (int rc = ready()) return rc;
  return cu(g_drv.MemcpyDtoHAsync(dst, src, bytes, static_cast<CUstream>(stream)),
            "cuMemcpyDtoHAsync");
}

int emmy_nccl_available(void) { return load_nccl() == 0 ? 1 : 0; }

int emmy_nccl_get_unique_id(char uid[128]) {
  if (!uid) return fail(EMMY_ERR_BAD_ARG, "null uid buffer");
  if (int rc = load_nccl()) return rc;
  NcclUid id;
  if (int rc = nc(g_nccl.GetUniqueId(&id), "ncclGetUniqueId")) return rc;
  std::memcpy(uid, id.internal, 128);
  return 0;
}

int emmy_nccl_init(int rank, int nranks, const char uid[128]) {
  if (!uid || nranks < 1 || rank < 0 || rank >= nranks)
    return fail(EMMY_ERR_BAD_ARG, "bad rank %d / nranks %d", rank, nranks);
  if (int rc = ready()) return rc;
  if (int rc = load_nccl()) return rc;
  if (g_comm) return fail(EMMY_ERR_BAD_ARG, "NCCL communicator already initialised");
  NcclUid id;
  std::memcpy(id.internal, uid, 128);
  NcclComm comm = nullptr;
  if (int rc = nc(g_nccl.CommInitRank(&comm, nranks, id, rank), "ncclCommInitRank")) return rc;
  g_comm = comm;
  return 0;
}

int emmy_allreduce_sum(uint64_t buf, size_t count, int dtype, void* stream) {
  if (!g_comm) return fail(EMMY_ERR_NOT_INIT, "emmy_nccl_init() has not been called");
  if (dtype != 0 && dtype != 1) return fail(EMMY_ERR_BAD_ARG, "dtype must be 0 (f32) or 1 (i32)");
  if (int rc = ready()) return rc;
  // ncclDataType_t: ncclInt32 = 2, ncclFloat32 = 7; ncclRedOp_t: ncclSum = 0
  const int nccl_type = dtype == 0 ? 7 : 2;
  void* p = reinterpret_cast<void*>(buf);
  return nc(g_nccl.AllReduce(p, p, count, nccl_type, 0, g_comm, static_cast<CUstream>(stream)),
            "ncclAllReduce");
}

int emmy_nccl_destroy(void) {
  if (!g_comm) return 0;
  int rc = nc(g_nccl.CommDestroy(g_comm), "ncclCommDestroy");
  g_comm = nullptr;
  return rc;
}

}  // extern "C"
