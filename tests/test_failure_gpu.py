"""Failure detection on the GPU without a GPU fault.

The expert-parallel exchange waits on the device for sequence-number flags
that peers write over NVLink.  Every such wait is bounded: when the flag never
arrives the kernel records status 0x105 and returns, so the context stays
usable and the host learns of the lost peer from the status word.  Here the
"peer" is a flag that nothing ever sets; no kernel traps, faults or spins
without a limit.
"""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV_TIMEOUT_PEER = 0x105


def _vp(t):
    return C.c_void_p(t.data_ptr())


def test_flag_wait_times_out_and_context_survives(cuda_dev):
    from final_b200 import _lib, gemm_nt
    lib = _lib.load()
    flags = torch.zeros(4, dtype=torch.int64, device=cuda_dev)
    idx = torch.tensor([0, 1, 2, 3], dtype=torch.int32, device=cuda_dev)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    s = torch.cuda.current_stream().cuda_stream
    flags[:2] = 7  # two flags arrived, two never will
    _lib.check(lib.b2_flag_wait(_vp(flags), _vp(idx), 4, 7, 0.2, _vp(status), C.c_void_p(s)),
               "b2_flag_wait")
    torch.cuda.synchronize()
    assert int(status.item()) == DEV_TIMEOUT_PEER
    # the context is still usable: a GEMM runs and is right
    A = torch.randn(128, 256, device=cuda_dev).to(torch.bfloat16)
    B = torch.randn(64, 256, device=cuda_dev).to(torch.bfloat16)
    got = gemm_nt(A, B, dtype="bf16")
    torch.cuda.synchronize()
    want = A.double() @ B.double().T
    assert ((got.double() - want).abs().max() / want.abs().max()).item() < 1e-4


def test_flag_wait_returns_when_flags_arrive(cuda_dev):
    from final_b200 import _lib
    lib = _lib.load()
    flags = torch.full((40,), 9, dtype=torch.int64, device=cuda_dev)
    idx = torch.arange(40, dtype=torch.int32, device=cuda_dev)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    s = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.b2_flag_wait(_vp(flags), _vp(idx), 40, 9, 5.0, _vp(status), C.c_void_p(s)),
               "b2_flag_wait")
    torch.cuda.synchronize()
    assert int(status.item()) == 0


def test_flag_wait_rejects_bad_arguments(cuda_dev):
    from final_b200 import _lib
    lib = _lib.load()
    status = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    assert lib.b2_flag_wait(None, None, 2, 1, 0.1, _vp(status), None) == _lib.B2_ERR_INVALID
    flags = torch.zeros(1, dtype=torch.int64, device=cuda_dev)
    idx = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    assert lib.b2_flag_wait(_vp(flags), _vp(idx), 1, 1, 0.0, _vp(status), None) == \
        _lib.B2_ERR_INVALID
    assert lib.b2_flag_wait(_vp(flags), _vp(idx), 2000, 1, 0.1, _vp(status), None) == \
        _lib.B2_ERR_INVALID
