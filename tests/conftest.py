import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def _spread_cpu_suite(config):
    """The CPU suite (``-m "not gpu"``) is mostly emulator work, PTX run instruction by instruction on
    numpy: a quarter of an hour in one process, a few minutes over the cores.  When the mark expression is
    exactly ``not gpu``, no ``-n`` was given, pytest-xdist is installed and ``EMMY_TESTS_SERIAL`` is not
    ``1``, the run is distributed over up to 8 worker processes (xdist's own configure step, which runs
    after this one, starts them).  GPU runs stay in one process: their tests share one device and some
    spawn processes of their own."""
    if hasattr(config, "workerinput") or os.environ.get("EMMY_TESTS_SERIAL") == "1":
        return
    if (config.getoption("markexpr", "") or "").strip() != "not gpu":
        return
    if not config.pluginmanager.hasplugin("xdist") or config.getoption("collectonly", False):
        return
    if config.getoption("numprocesses", None) or config.getoption("dist", "no") != "no":
        return
    if config.getoption("usepdb", False):
        return
    workers = max(1, min(8, os.cpu_count() or 1))
    if workers > 1:
        config.option.numprocesses = workers
        config.option.dist = "load"
        config.option.tx = ["popen"] * workers


def pytest_configure(config):
    _spread_cpu_suite(config)
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")
    config.addinivalue_line("markers", "gpu_optin: opt-in variants not yet run on a B200 (skipped without a "
                                       "GPU); run with -m gpu_optin")
