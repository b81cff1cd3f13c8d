"""The integration notes stay true to the code: every compile option they list is read by the package,
and every option the package reads is listed; every C-ABI function is mapped."""
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _options_read() -> set[str]:
    names = set()
    for f in (ROOT / "emmy_ptx_b200").rglob("*.py"):
        names.update(re.findall(r'(?:opts|options)\.get\("([a-z0-9_]+)"', f.read_text()))
    return names


def _options_documented() -> set[str]:
    text = (ROOT / "INTEGRATION.md").read_text()
    section = text.split("## 5. Compile options", 1)[1]
    names = set()
    for row in section.splitlines():
        if row.startswith("| `"):
            names.update(re.findall(r"`([a-z0-9_]+)`", row.split("|")[1]))
    return names


def test_compile_options_are_documented():
    read, documented = _options_read(), _options_documented()
    assert read <= documented, sorted(read - documented)
    assert documented <= read, sorted(documented - read)


def test_every_abi_function_is_mapped():
    header = (ROOT / "include" / "emmy_launch.h").read_text()
    text = (ROOT / "INTEGRATION.md").read_text()
    missing = [f for f in sorted(set(re.findall(r"\bint (emmy_\w+)\(", header))) if f not in text]
    assert not missing, missing
