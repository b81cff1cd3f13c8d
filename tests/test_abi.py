"""The C-ABI library loads without a GPU and exports every function include/*.h declares."""
import ctypes
import re
from pathlib import Path

from emmy_ptx_b200 import launcher

ROOT = Path(__file__).resolve().parents[1]


def _declared() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names.update(re.findall(r"^\s*int\s+(emmy_\w+)\s*\(", text, flags=re.M))
    return names


def test_library_exports_every_declared_symbol():
    lib = launcher.load_library()
    declared = _declared()
    assert declared, "no declarations found"
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_the_header():
    assert _declared() <= set(launcher.SIGNATURES) | {"emmy_launch_u64"}


def test_calls_without_a_driver_fail_cleanly():
    lib = launcher.load_library()
    assert lib.emmy_version() == 1
    # no emmy_init: every device call reports "not initialised" (or no driver) instead of crashing
    rc = lib.emmy_ctx_synchronize()
    assert rc != 0
    assert launcher.last_error()


def test_launch_flags_are_checked_before_the_driver():
    lib = launcher.load_library()
    grid = (ctypes.c_uint32 * 3)(1, 1, 1)
    block = (ctypes.c_uint32 * 3)(32, 1, 1)
    fake_fn = ctypes.c_void_p(0x1000)        # never reaches the driver: the flag check fails first
    rc = lib.emmy_launch_ex(fake_fn, grid, block, None, 0, None, None, 0, 0x80)
    assert rc != 0
    assert "unknown launch flags" in launcher.last_error()


def test_stream_and_event_arguments_are_checked_before_the_driver():
    lib = launcher.load_library()
    vp = ctypes.c_void_p
    ev = vp()
    assert lib.emmy_event_create_flags(ctypes.byref(ev), 8) != 0          # unknown CUevent flag
    assert "unknown event flags" in launcher.last_error()
    assert lib.emmy_event_create_flags(None, 2) != 0
    assert lib.emmy_stream_create(None) != 0
    assert lib.emmy_stream_destroy(None) != 0
    assert lib.emmy_stream_wait_event(None, None) != 0
    assert lib.emmy_set_smem_carveout(None, 50) != 0
    assert lib.emmy_set_smem_carveout(vp(0x1000), 101) != 0              # outside -1..100
    assert "carveout" in launcher.last_error()


def test_device_index_is_checked_before_the_driver():
    lib = launcher.load_library()
    for bad in (-1, 64):
        assert lib.emmy_init(bad) == 10003                                # EMMY_ERR_BAD_ARG
        assert "out of range" in launcher.last_error()


class _FakeLib:
    """Records which device the library has selected when each context-bound call arrives."""

    def __init__(self):
        self.selected = None
        self.calls = []

    def emmy_init(self, index):
        self.selected = index
        return 0

    def __getattr__(self, name):
        def call(*args):
            self.calls.append((name, self.selected))
            return 0
        return call


def test_each_device_object_selects_its_own_device(monkeypatch):
    fake = _FakeLib()
    monkeypatch.setattr(launcher, "load_library", lambda: fake)
    monkeypatch.setattr(launcher.Device, "_inited", {})
    monkeypatch.setattr(launcher.Device, "_active", None)
    d0 = launcher.Device.get(0)
    d1 = launcher.Device.get(1)
    d0.memset_d32(0x1000, 0, 4, 0)                # after d1 was selected: must switch back to 0
    d1.memset_d32(0x2000, 0, 4, 0)
    d1.sync()
    d0.sync(0)
    assert fake.calls == [("emmy_memset_d32_async", 0), ("emmy_memset_d32_async", 1),
                          ("emmy_ctx_synchronize", 1), ("emmy_stream_synchronize", 0)]
    assert launcher.Device.get(0) is d0 and fake.selected == 0
