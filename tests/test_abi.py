"""The C ABI library builds, loads without a GPU, and exports every symbol
include/b2moe.h declares (no compute calls are made here)."""
import re
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _declared():
    names = set()
    for h in sorted((ROOT / "include").glob("*.h")):
        names |= set(re.findall(r"\b(b2_[a-z0-9_]+)\s*\(", h.read_text()))
    return sorted(names)


def test_header_matches_binding_list():
    from final_b200._lib import EXPORTED
    assert sorted(EXPORTED) == _declared()


def test_library_loads_and_exports():
    from final_b200 import build
    lib_path = build.build()
    from final_b200 import _lib
    lib = _lib.load(lib_path)
    for name in _declared():
        assert hasattr(lib, name), name
    assert lib.b2_version().startswith(b"b2moe")
    assert lib.b2_status_string(3) == b"token count exceeds capacity"


def test_library_is_sm100a_only():
    """The shared object carries sm_100a device code (checked via cuobjdump's
    ELF listing of our own build, names only)."""
    from final_b200 import build
    lib_path = build.build()
    out = subprocess.run(["cuobjdump", "--list-elf", str(lib_path)], capture_output=True,
                         text=True)
    if out.returncode != 0:
        import pytest
        pytest.skip("cuobjdump unavailable")
    assert "sm_100a" in out.stdout
    assert "sm_90" not in out.stdout and "sm_80" not in out.stdout


def test_no_fallback_without_library(tmp_path):
    """Loading from a path without the .so raises instead of falling back."""
    import pytest
    from final_b200 import _lib
    saved = _lib._lib
    _lib._lib = None
    try:
        with pytest.raises(ImportError):
            _lib.load(tmp_path / "libb2moe.so")
    finally:
        _lib._lib = saved
