"""The C ABI library builds, loads without a GPU, and exports every symbol
include/b2moe.h declares (no compute calls are made here)."""
import re
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


def test_library_is_built_for_sm100a_only():
    """The build compiles device code for sm_100a alone (one -gencode, no PTX
    for other targets); the GPU-side check of the loaded code's architecture
    is tests/test_moe_gpu.py::test_device_code_is_sm100."""
    from final_b200 import build
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


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


def test_new_entry_points_reject_bad_arguments():
    """Argument checks that return before any device work (no GPU needed)."""
    import ctypes as C
    from final_b200 import _lib
    lib = _lib.load()
    n = C.c_int(0)
    assert lib.b2_ep_profile_timeline(None, 0, None, None, C.byref(n)) == _lib.B2_ERR_INVALID
    assert lib.b2_lfm2_set_timeout(None, 1.0) == _lib.B2_ERR_INVALID
    d = _lib.Lfm2Desc(vocab=300, hidden=256, num_layers=5, num_heads=4, num_kv_heads=2,
                      dense_inter=384, moe_inter=128, num_experts=8, top_k=4,
                      num_dense_layers=2, max_batch=2, max_seq=8)
    h = C.c_void_p()
    uid = C.create_string_buffer(128)
    fn = _lib.WEIGHT_FN(lambda ctx, name, numel: None)
    # world / rank / mode out of range, no id, experts not divisible among owners
    for world, rank, mode, u in ((0, 0, 1, uid), (2, 2, 1, uid), (2, 0, 7, uid),
                                 (2, 0, 1, None), (3, 0, 0, uid)):
        assert lib.b2_lfm2_create_ep(C.byref(d), fn, None, 1, world, rank, u, mode, None,
                                     C.byref(h)) == _lib.B2_ERR_INVALID
    assert not h.value
