"""ctypes binding of ``libemmy_launch.so`` (declared in ``include/emmy_launch.h``).

This is the only route by which the backend touches the GPU: module loading, launches, events,
copies and the NCCL all-reduce all go through the C ABI.  There is no fallback: if the library is
missing, every call raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libemmy_launch.so"

c_u32p = ctypes.POINTER(ctypes.c_uint32)
c_u64p = ctypes.POINTER(ctypes.c_uint64)
vp = ctypes.c_void_p
LAUNCH_PDL = 1          # EMMY_LAUNCH_PDL in include/emmy_launch.h

# name -> argtypes (all functions return int)
SIGNATURES = {
    "emmy_version": [],
    "emmy_last_error": [ctypes.c_char_p, ctypes.c_size_t],
    "emmy_init": [ctypes.c_int],
    "emmy_device_attribute": [ctypes.c_int, ctypes.POINTER(ctypes.c_int)],
    "emmy_module_load_ptx": [ctypes.c_char_p, ctypes.POINTER(vp), ctypes.c_char_p, ctypes.c_size_t],
    "emmy_module_load_image": [vp, ctypes.POINTER(vp)],
    "emmy_module_unload": [vp],
    "emmy_get_function": [vp, ctypes.c_char_p, ctypes.POINTER(vp)],
    "emmy_set_max_dyn_smem": [vp, ctypes.c_int],
    "emmy_set_smem_carveout": [vp, ctypes.c_int],
    "emmy_func_attribute": [vp, ctypes.c_int, ctypes.POINTER(ctypes.c_int)],
    "emmy_launch": [vp, c_u32p, c_u32p, c_u32p, ctypes.c_uint32, vp, ctypes.POINTER(vp), ctypes.c_uint32],
    "emmy_launch_u64": [vp, c_u32p, c_u32p, ctypes.c_uint32, vp, c_u64p, c_u32p, ctypes.c_uint32],
    "emmy_launch_ex": [vp, c_u32p, c_u32p, c_u32p, ctypes.c_uint32, vp, ctypes.POINTER(vp), ctypes.c_uint32,
                       ctypes.c_uint32],
    "emmy_launch_u64_ex": [vp, c_u32p, c_u32p, ctypes.c_uint32, vp, c_u64p, c_u32p, ctypes.c_uint32,
                           ctypes.c_uint32],
    "emmy_tmap_encode_tiled": [vp, ctypes.c_int, ctypes.c_uint32, ctypes.c_uint64, c_u64p, c_u64p, c_u32p,
                               c_u32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int],
    "emmy_event_create": [ctypes.POINTER(vp)],
    "emmy_event_destroy": [vp],
    "emmy_event_record": [vp, vp],
    "emmy_event_synchronize": [vp],
    "emmy_event_elapsed_ms": [vp, vp, ctypes.POINTER(ctypes.c_float)],
    "emmy_stream_synchronize": [vp],
    "emmy_event_create_flags": [ctypes.POINTER(vp), ctypes.c_uint],
    "emmy_stream_create": [ctypes.POINTER(vp)],
    "emmy_stream_destroy": [vp],
    "emmy_stream_wait_event": [vp, vp],
    "emmy_ctx_synchronize": [],
    "emmy_mem_alloc": [c_u64p, ctypes.c_size_t],
    "emmy_mem_free": [ctypes.c_uint64],
    "emmy_ipc_get_handle": [ctypes.c_uint64, ctypes.c_char_p],
    "emmy_ipc_open": [ctypes.c_char_p, c_u64p],
    "emmy_ipc_close": [ctypes.c_uint64],
    "emmy_memset_d32_async": [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_size_t, vp],
    "emmy_memcpy_htod_async": [ctypes.c_uint64, vp, ctypes.c_size_t, vp],
    "emmy_memcpy_dtoh_async": [vp, ctypes.c_uint64, ctypes.c_size_t, vp],
    "emmy_nccl_available": [],
    "emmy_nccl_get_unique_id": [ctypes.c_char_p],
    "emmy_nccl_init": [ctypes.c_int, ctypes.c_int, ctypes.c_char_p],
    "emmy_allreduce_sum": [ctypes.c_uint64, ctypes.c_size_t, ctypes.c_int, vp],
    "emmy_nccl_destroy": [],
    "emmy_bmm_bf16_noalloc": [vp, vp, vp, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint32,
                              ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, vp],
    "emmy_bmm_bf16_noalloc_status": [ctypes.POINTER(ctypes.c_uint32), vp],
}

# CUfunction_attribute values used by the runtime
ATTR_NUM_REGS = 4
ATTR_LOCAL_SIZE_BYTES = 3
ATTR_MAX_THREADS = 0
# CUdevice_attribute
DEV_MULTIPROCESSOR_COUNT = 16
DEV_L2_CACHE_SIZE = 38


class EmmyError(RuntimeError):
    """A failing C-ABI call: ``code`` is the returned status, the message the library's."""

    def __init__(self, code: int, what: str, msg: str):
        super().__init__(f"{what}: status {code}: {msg}")
        self.code = code


_lock = threading.Lock()
_lib = None


def load_library(path: Path | None = None):
    """Open ``libemmy_launch.so`` (building it first if it is missing and nvcc is present)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = Path(path or LIB_PATH)
        if not p.exists():
            from . import build
            build.build()
        lib = ctypes.CDLL(str(p))
        for name, args in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        _lib = lib
        return lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(4096)
    load_library().emmy_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(code: int, what: str) -> None:
    if code != 0:
        raise EmmyError(code, what, last_error())


def dims3(v) -> ctypes.Array:
    v = [int(x) for x in (list(v) + [1, 1, 1])[:3]]
    return (ctypes.c_uint32 * 3)(*v)


class Device:
    """The launcher bound to one CUDA device (its primary context)."""

    _inited: dict[int, "Device"] = {}
    _active: int | None = None          # the device the library has selected (emmy_init)

    def __init__(self, index: int = 0):
        self.lib = load_library()
        self.index = index
        self.launches = 0
        self._use()

    def _use(self) -> None:
        """Select this device in the library before a call that runs in its context, so that objects
        bound to different devices in one process each reach their own."""
        if Device._active != self.index:
            check(self.lib.emmy_init(self.index), f"emmy_init({self.index})")
            Device._active = self.index

    @classmethod
    def get(cls, index: int = 0) -> "Device":
        dev = cls._inited.get(index)
        if dev is None:
            dev = cls(index)
            cls._inited[index] = dev
        dev._use()
        return dev

    def attribute(self, attr: int) -> int:
        self._use()
        v = ctypes.c_int()
        check(self.lib.emmy_device_attribute(attr, ctypes.byref(v)), "emmy_device_attribute")
        return v.value

    def load_ptx(self, ptx: str):
        self._use()
        mod = vp()
        log = ctypes.create_string_buffer(16384)
        check(self.lib.emmy_module_load_ptx(ptx.encode("ascii"), ctypes.byref(mod), log, len(log)),
              "emmy_module_load_ptx")
        return mod

    def load_image(self, image: bytes):
        self._use()
        mod = vp()
        buf = ctypes.create_string_buffer(image, len(image))
        check(self.lib.emmy_module_load_image(ctypes.cast(buf, vp), ctypes.byref(mod)), "emmy_module_load_image")
        return mod

    def unload(self, mod) -> None:
        self._use()
        check(self.lib.emmy_module_unload(mod), "emmy_module_unload")

    def function(self, mod, entry: str):
        self._use()
        fn = vp()
        check(self.lib.emmy_get_function(mod, entry.encode(), ctypes.byref(fn)), f"emmy_get_function({entry})")
        return fn

    def func_attribute(self, fn, attr: int) -> int:
        self._use()
        v = ctypes.c_int()
        check(self.lib.emmy_func_attribute(fn, attr, ctypes.byref(v)), "emmy_func_attribute")
        return v.value

    def set_max_dyn_smem(self, fn, nbytes: int) -> None:
        self._use()
        check(self.lib.emmy_set_max_dyn_smem(fn, int(nbytes)), "emmy_set_max_dyn_smem")

    def set_carveout(self, fn, percent: int) -> None:
        self._use()
        check(self.lib.emmy_set_smem_carveout(fn, int(percent)), "emmy_set_smem_carveout")

    def launch_u64(self, fn, grid, block, dyn_smem: int, stream: int, params, align=None, pdl: bool = False) -> None:
        """Launch a kernel whose parameters are all 64-bit values.  ``pdl`` launches it as a
        programmatic dependent of the stream's previous work (the kernel must begin with
        ``griddepcontrol.wait``, as the launch record's ``pdl`` says)."""
        self._use()
        n = len(params)
        p = (ctypes.c_uint64 * n)(*[int(x) for x in params])
        a = (ctypes.c_uint32 * n)(*[int(x) for x in align]) if align is not None else None
        check(self.lib.emmy_launch_u64_ex(fn, dims3(grid), dims3(block), int(dyn_smem), vp(stream or 0), p, a, n,
                                          LAUNCH_PDL if pdl else 0), "emmy_launch_u64_ex")
        self.launches += 1

    def launch(self, fn, grid, block, dyn_smem: int, stream: int, arg_ptrs, cluster=(1, 1, 1),
               pdl: bool = False) -> None:
        self._use()
        n = len(arg_ptrs)
        args = (vp * n)(*arg_ptrs)
        check(self.lib.emmy_launch_ex(fn, dims3(grid), dims3(block), dims3(cluster), int(dyn_smem),
                                      vp(stream or 0), args, n, LAUNCH_PDL if pdl else 0), "emmy_launch_ex")
        self.launches += 1

    def tmap_encode_tiled(self, out_buf, dtype: int, gaddr: int, dims, strides_bytes, box, elem_strides=None,
                          swizzle: int = 0, l2promo: int = 2, oob_fill: int = 0, interleave: int = 0) -> None:
        rank = len(dims)
        d = (ctypes.c_uint64 * rank)(*dims)
        s = (ctypes.c_uint64 * max(rank - 1, 1))(*(list(strides_bytes) or [0]))
        bx = (ctypes.c_uint32 * rank)(*box)
        es = (ctypes.c_uint32 * rank)(*(elem_strides or [1] * rank))
        check(self.lib.emmy_tmap_encode_tiled(out_buf, dtype, rank, int(gaddr), d, s, bx, es, interleave,
                                              swizzle, l2promo, oob_fill), "emmy_tmap_encode_tiled")

    def memset_d32(self, dptr: int, value: int, count: int, stream: int) -> None:
        self._use()
        check(self.lib.emmy_memset_d32_async(int(dptr), value & 0xFFFFFFFF, int(count), vp(stream or 0)),
              "emmy_memset_d32_async")

    def mem_alloc(self, nbytes: int) -> int:
        """A device allocation of its own (cuMemAlloc), e.g. memory to export to other processes."""
        self._use()
        p = ctypes.c_uint64(0)
        check(self.lib.emmy_mem_alloc(ctypes.byref(p), int(nbytes)), "emmy_mem_alloc")
        return int(p.value)

    def mem_free(self, dptr: int) -> None:
        self._use()
        check(self.lib.emmy_mem_free(int(dptr)), "emmy_mem_free")

    def ipc_handle(self, dptr: int) -> bytes:
        """The 64-byte inter-process handle of an allocation from :meth:`mem_alloc`."""
        self._use()
        buf = ctypes.create_string_buffer(64)
        check(self.lib.emmy_ipc_get_handle(int(dptr), buf), "emmy_ipc_get_handle")
        return buf.raw[:64]

    def ipc_open(self, handle: bytes) -> int:
        """Map another process's exported allocation (over NVLink peer access); its device address."""
        self._use()
        if len(handle) != 64:
            raise ValueError("an IPC handle is 64 bytes")
        p = ctypes.c_uint64(0)
        check(self.lib.emmy_ipc_open(ctypes.create_string_buffer(handle, 64), ctypes.byref(p)), "emmy_ipc_open")
        return int(p.value)

    def ipc_close(self, dptr: int) -> None:
        self._use()
        check(self.lib.emmy_ipc_close(int(dptr)), "emmy_ipc_close")

    def htod(self, dst: int, src_ptr: int, nbytes: int, stream: int) -> None:
        self._use()
        check(self.lib.emmy_memcpy_htod_async(int(dst), vp(src_ptr), int(nbytes), vp(stream or 0)),
              "emmy_memcpy_htod_async")

    def dtoh(self, dst_ptr: int, src: int, nbytes: int, stream: int) -> None:
        self._use()
        check(self.lib.emmy_memcpy_dtoh_async(vp(dst_ptr), int(src), int(nbytes), vp(stream or 0)),
              "emmy_memcpy_dtoh_async")

    def sync(self, stream: int | None = None) -> None:
        self._use()
        if stream is None:
            check(self.lib.emmy_ctx_synchronize(), "emmy_ctx_synchronize")
        else:
            check(self.lib.emmy_stream_synchronize(vp(stream)), "emmy_stream_synchronize")

    # events
    def event(self):
        self._use()
        ev = vp()
        check(self.lib.emmy_event_create(ctypes.byref(ev)), "emmy_event_create")
        return ev

    def sync_event(self):
        """An event for ordering only (no timing)."""
        self._use()
        ev = vp()
        check(self.lib.emmy_event_create_flags(ctypes.byref(ev), 2), "emmy_event_create_flags")
        return ev

    def stream(self) -> int:
        """A new non-blocking stream (its handle)."""
        self._use()
        s = vp()
        check(self.lib.emmy_stream_create(ctypes.byref(s)), "emmy_stream_create")
        return s.value

    def destroy_stream(self, stream: int) -> None:
        self._use()
        check(self.lib.emmy_stream_destroy(vp(stream)), "emmy_stream_destroy")

    def wait_event(self, stream: int, ev) -> None:
        self._use()
        check(self.lib.emmy_stream_wait_event(vp(stream or 0), ev), "emmy_stream_wait_event")

    def record(self, ev, stream: int) -> None:
        self._use()
        check(self.lib.emmy_event_record(ev, vp(stream or 0)), "emmy_event_record")

    def elapsed_ms(self, a, b) -> float:
        self._use()
        check(self.lib.emmy_event_synchronize(b), "emmy_event_synchronize")
        ms = ctypes.c_float()
        check(self.lib.emmy_event_elapsed_ms(a, b, ctypes.byref(ms)), "emmy_event_elapsed_ms")
        return ms.value

    def destroy_event(self, ev) -> None:
        self._use()
        check(self.lib.emmy_event_destroy(ev), "emmy_event_destroy")

    # NCCL
    def nccl_unique_id(self) -> bytes:
        buf = ctypes.create_string_buffer(128)
        check(self.lib.emmy_nccl_get_unique_id(buf), "emmy_nccl_get_unique_id")
        return buf.raw[:128]

    def nccl_init(self, rank: int, nranks: int, uid: bytes) -> None:
        self._use()
        check(self.lib.emmy_nccl_init(rank, nranks, ctypes.create_string_buffer(uid, 128)), "emmy_nccl_init")

    def allreduce_sum(self, dptr: int, count: int, dtype: str, stream: int) -> None:
        self._use()
        code = {"f32": 0, "i32": 1}[dtype]
        check(self.lib.emmy_allreduce_sum(int(dptr), int(count), code, vp(stream or 0)), "emmy_allreduce_sum")

    def bmm_noalloc(self, fn, tmap_a: int, tmap_b: int, a: int, b: int, c: int, grid: int, block: int,
                    dyn_smem: int, scratch_bytes: int, stream: int) -> None:
        """The tensor-core bmm through the entry point that allocates nothing (its scratch is a fixed
        array inside the library)."""
        self._use()
        check(self.lib.emmy_bmm_bf16_noalloc(fn, vp(tmap_a), vp(tmap_b), int(a), int(b), int(c), int(grid),
                                             int(block), int(dyn_smem), int(scratch_bytes), vp(stream or 0)),
              "emmy_bmm_bf16_noalloc")
        self.launches += 1

    def bmm_noalloc_status(self, stream: int) -> int:
        """The status word of the last no-allocation bmm queued on ``stream`` (0 = every bounded wait
        completed); waits for the stream."""
        self._use()
        word = ctypes.c_uint32(0)
        check(self.lib.emmy_bmm_bf16_noalloc_status(ctypes.byref(word), vp(stream or 0)),
              "emmy_bmm_bf16_noalloc_status")
        return int(word.value)

    def nccl_destroy(self) -> None:
        self._use()
        check(self.lib.emmy_nccl_destroy(), "emmy_nccl_destroy")
