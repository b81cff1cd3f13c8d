"""Run compiled modules: load the PTX through the C ABI and launch each entry on torch tensors.

``Executable`` is the successor of the reference's launch harness (tools/localrun.py:137-206,
tools/bench.py:86-115): it loads a module once, then each call zeroes the outputs a kernel's
record lists (``zero_outputs``, tools/stress.py:106-111), checks every pointer's alignment against
what the emitted code assumes, encodes TMA descriptors for tensor-core kernels, and launches
the entries in order on the caller's stream.  Buffers are caller-owned tensors on the device.

An entry whose record says ``"stream": 1`` runs on the Executable's side stream instead, so that it
overlaps the main stream's next entries; ``"after": [entry, ...]`` names entries it must follow
(on the other stream: a fork or join through an event).  The side stream always rejoins the caller's
stream before the call returns, so callers (and CUDA-graph capture) see one stream.
"""
from __future__ import annotations

import ctypes

from .compiler import CompiledModule, compile_ir
from .launcher import Device
from .data import torch_dtype

_TMAP_DTYPE = {"u8": 0, "u32": 2, "i32": 3, "f16": 6, "f32": 7, "f64": 8, "bf16": 9}   # CUtensorMapDataType (cuda.h)
_SWIZZLE = {"none": 0, "32B": 1, "64B": 2, "128B": 3}


class _TmapBlob:
    """A 128-byte CUtensorMap in a host buffer, at a 64-byte-aligned address."""

    def __init__(self):
        self.buf = ctypes.create_string_buffer(128 + 64)
        self.addr = (ctypes.addressof(self.buf) + 63) & ~63


class Executable:
    """A compiled module loaded on one device."""

    def __init__(self, compiled: CompiledModule | str, device: int | None = None):
        import torch
        if isinstance(compiled, str):
            compiled = compile_ir(compiled)
        self.compiled = compiled
        self.index = torch.cuda.current_device() if device is None else device
        self.dev = Device.get(self.index)
        self.module = self.dev.load_ptx(compiled.ptx)
        self.funcs = []
        for rec in compiled.kernels:
            fn = self.dev.function(self.module, rec["entry"])
            if rec.get("dyn_smem", 0) > 48 * 1024:
                self.dev.set_max_dyn_smem(fn, rec["dyn_smem"])
            if rec.get("carveout") is not None:
                self.dev.set_carveout(fn, rec["carveout"])
            self.funcs.append(fn)
        self._tmap_cache: dict = {}
        # device scratch some lowerings need between their entries (e.g. the attention's f16 copy of V),
        # allocated once per Executable and passed to the entries by name
        self.scratch: dict = {}
        for rec in compiled.kernels:
            for spec in rec.get("scratch", []):
                if spec["name"] not in self.scratch:
                    self.scratch[spec["name"]] = self._device_tensor(tuple(spec["shape"]), torch_dtype(spec["dtype"]))
                    if spec.get("zeroed"):
                        # a self-zeroing accumulator: zero once here, every launch leaves it zero
                        self.scratch[spec["name"]].zero_()
        self.side = None
        names = [rec["entry"] for rec in compiled.kernels]
        for i, rec in enumerate(compiled.kernels):
            for dep in rec.get("after", []):
                if dep not in names[:i]:
                    raise ValueError(f"entry {rec['entry']!r} follows {dep!r}, which is not an earlier entry")
        if any(rec.get("stream") for rec in compiled.kernels):
            self.side = self.dev.stream()
            self._fork = self.dev.sync_event()
            self._events = {rec["entry"]: self.dev.sync_event() for rec in compiled.kernels}
        self.err = None
        if any(spec.get("kind") == "errword" for rec in compiled.kernels for spec in rec.get("extra", [])):
            self.err = self._device_tensor((4,), torch.int32)
            self.err.zero_()

    def _device_tensor(self, shape, dtype):
        """Device memory the Executable owns (scratch between entries, the error word)."""
        import torch
        return torch.empty(shape, dtype=dtype, device=f"cuda:{self.index}")

    def error_code(self) -> int:
        """The error word a tensor-core kernel writes when one of its bounded waits times out
        (0 = no error).  Read after synchronising."""
        return 0 if self.err is None else int(self.err[0].item())

    def check(self) -> None:
        code = self.error_code()
        if code:
            raise RuntimeError(f"kernel reported error code {code} (a pipeline wait timed out)")

    @property
    def records(self) -> list[dict]:
        return self.compiled.kernels

    def registers(self, i: int = 0) -> int:
        from .launcher import ATTR_NUM_REGS
        return self.dev.func_attribute(self.funcs[i], ATTR_NUM_REGS)

    def _tmap(self, spec: dict, t) -> ctypes.Array:
        key = (spec["name"], t.data_ptr(), tuple(t.shape))
        hit = self._tmap_cache.get(key)
        if hit is not None:
            return hit
        blob = _TmapBlob()
        dims = spec["dims"]
        strides = spec["strides"]
        self.dev.tmap_encode_tiled(ctypes.c_void_p(blob.addr), _TMAP_DTYPE[spec["dtype"]], t.data_ptr(), dims, strides,
                                   spec["box"], swizzle=_SWIZZLE[spec.get("swizzle", "128B")],
                                   l2promo=spec.get("l2promo", 2))
        self._tmap_cache[key] = blob
        return blob

    def zero_outputs(self, i: int, tensors: dict, stream: int) -> None:
        """Zero the outputs entry ``i`` accumulates into (its record's ``zero_outputs``)."""
        for name in self.records[i].get("zero_outputs", []):
            t = tensors[name]
            nbytes = t.numel() * t.element_size()
            if nbytes % 4:
                raise ValueError(f"zeroed output {name!r} is not a whole number of 32-bit words")
            self.dev.memset_d32(t.data_ptr(), 0, nbytes // 4, stream)

    def launch(self, i: int, tensors: dict, stream: int, grid=None, zero: bool = True) -> None:
        """Launch entry ``i`` with its parameters taken from ``tensors`` by name."""
        if self.scratch:
            tensors = {**self.scratch, **tensors}
        rec = self.records[i]
        fn = self.funcs[i]
        if grid is not None and (rec.get("self_zeroing") or rec.get("exchange")) and list(grid) != list(rec["grid"]):
            # the last block is the one whose ticket is grid - 1 of the compiled grid
            raise ValueError(f"kernel {rec['entry']!r} counts its blocks: launch it with its compiled grid "
                             f"{rec['grid']}, not {list(grid)}")
        if zero:
            self.zero_outputs(i, tensors, stream)
        g = grid or rec["grid"]
        if not g or not rec["block"]:
            raise ValueError(f"kernel {rec['entry']!r} has no launch geometry (no meta.json record)")
        if 0 in list(g)[:3]:
            return                   # an empty input: no blocks to run (CUDA refuses a zero-sized grid)
        if rec.get("tmaps") or rec.get("extra"):
            args = []
            keep = []
            for name in rec["params"]:
                ptr = tensors[name].data_ptr()
                al = int(rec.get("align", {}).get(name, 1))
                if al > 1 and ptr % al:
                    raise ValueError(f"{name!r} must be {al}-byte aligned for kernel {rec['entry']!r}")
                v = ctypes.c_uint64(ptr)
                keep.append(v)
                args.append(ctypes.cast(ctypes.byref(v), ctypes.c_void_p).value)
            for spec in rec.get("tmaps", []):
                blob = self._tmap(spec, tensors[spec["tensor"]])
                keep.append(blob)
                args.append(blob.addr)
            for spec in rec.get("extra", []):
                if spec.get("kind") == "errword":
                    v = ctypes.c_uint64(self.err.data_ptr())
                else:
                    if "value" in spec:
                        ptr = int(spec["value"])
                    else:
                        t = tensors[spec["name"]]
                        ptr = int(t) if isinstance(t, int) else t.data_ptr()   # a raw device address, or a tensor
                    v = ctypes.c_uint64(ptr)
                keep.append(v)
                args.append(ctypes.cast(ctypes.byref(v), ctypes.c_void_p).value)
            self.dev.launch(fn, g, rec["block"], rec.get("dyn_smem", 0), stream, args,
                            cluster=rec.get("cluster", (1, 1, 1)))
            return
        ptrs, align = [], []
        for name in rec["params"]:
            t = tensors[name]
            ptrs.append(t.data_ptr() if hasattr(t, "data_ptr") else int(t))
            align.append(int(rec.get("align", {}).get(name, 1)))
        self.dev.launch_u64(fn, g, rec["block"], rec.get("dyn_smem", 0), stream, ptrs, align,
                            pdl=bool(rec.get("pdl")))

    def __call__(self, tensors: dict, stream: int | None = None) -> None:
        """Run every entry of the module once, in order, on ``stream`` (default: torch's current)."""
        self.run(tensors, stream)

    def run(self, tensors: dict, stream: int | None = None, zero: bool = True) -> None:
        """Launch every entry once in module order: on ``stream`` or, for ``"stream": 1`` records, on
        the side stream, forked from ``stream`` at the first such entry and joined back at the end.
        ``zero=False`` skips the output zeroing (for replaying kernels only)."""
        import torch
        if stream is None:
            stream = torch.cuda.current_stream(self.index).cuda_stream
        if self.side is None:
            for i in range(len(self.records)):
                self.launch(i, tensors, stream, zero=zero)
            return
        on = {}
        last_side = None
        for i, rec in enumerate(self.records):
            s = self.side if rec.get("stream") else stream
            if s == self.side and last_side is None:
                # the side stream starts after everything queued on the caller's stream so far
                self.dev.record(self._fork, stream)
                self.dev.wait_event(self.side, self._fork)
            for dep in rec.get("after", []):
                if on[dep] != s:
                    self.dev.wait_event(s, self._events[dep])
            self.launch(i, tensors, s, zero=zero)
            on[rec["entry"]] = s
            self.dev.record(self._events[rec["entry"]], s)
            if s == self.side:
                last_side = rec["entry"]
        if last_side is not None:
            self.dev.wait_event(stream, self._events[last_side])

    @property
    def launches(self) -> int:
        return self.dev.launches

    def close(self) -> None:
        if self.module is not None:
            self.dev.unload(self.module)
            self.module = None
        if self.side is not None:
            for ev in [self._fork, *self._events.values()]:
                self.dev.destroy_event(ev)
            self.dev.destroy_stream(self.side)
            self.side = None
