"""b2_moe_route_noalloc -- the routing step for callers that may not allocate
device memory after start-up (a server that plans every device byte up
front; a host whose allocator is owned elsewhere) -- must give exactly what
the allocating entry point b2_moe_forward_ex reports for the same input.

Called through the C ABI twice in a row, on two different inputs (larger
first, then smaller), so that whatever the shared static scratch keeps from
the first call cannot leak into the second.  Routing is integer / index work
plus fp32 weights computed in the reference's exact operation order, so the
tolerance is zero: every output must be bit-identical.

This file is collected last on purpose (its name sorts after every other
test file) and must pass both alone in a fresh process and after the others.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from moe_cases import build_case

pytestmark = pytest.mark.gpu


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _reference_entry(inp, dev):
    """Routing outputs of the existing, allocating entry point."""
    from final_b200 import SparseMoeBlock
    layer = SparseMoeBlock(_t(inp["gate"], dev), _t(inp["w1"], dev), _t(inp["w2"], dev),
                           _t(inp["w3"], dev), _t(inp["bias"], dev),
                           max_tokens=inp["x"].shape[0], top_k=inp["K"])
    out = layer.forward_traced(_t(inp["x"], dev))
    torch.cuda.synchronize()
    assert layer.device_status() == 0
    layer.close()
    return {k: out[k].cpu() for k in ("topk_idx", "topk_w", "counts", "offsets", "token_slot")}


def _noalloc_entry(inp, dev):
    from final_b200 import _lib
    lib = _lib.load()
    x, gate, bias = _t(inp["x"], dev), _t(inp["gate"], dev), _t(inp["bias"], dev)
    T, H = inp["x"].shape
    E, K = inp["gate"].shape[0], inp["K"]
    out = {
        "topk_idx": torch.full((T, K), -7, dtype=torch.int32, device=dev),
        "topk_w": torch.full((T, K), -7.0, dtype=torch.float32, device=dev),
        "counts": torch.full((E,), -7, dtype=torch.int32, device=dev),
        "offsets": torch.full((E,), -7, dtype=torch.int32, device=dev),
        "token_slot": torch.full((T, K), -7, dtype=torch.int32, device=dev),
    }
    p = lambda t: C.c_void_p(t.data_ptr())
    rc = lib.b2_moe_route_noalloc(p(x), p(gate), p(bias), T, H, E, K, C.c_float(1.0),
                                  p(out["topk_idx"]), p(out["topk_w"]), p(out["counts"]),
                                  p(out["offsets"]), p(out["token_slot"]),
                                  C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.b2_status_string(rc)
    torch.cuda.synchronize()
    return {k: v.cpu() for k, v in out.items()}


def test_route_noalloc_matches_allocating_entry_point(cuda_dev):
    for case in ("zipf", "small"):  # 512 tokens, then 40 tokens
        inp = build_case(case)
        want = _reference_entry(inp, cuda_dev)
        got = _noalloc_entry(inp, cuda_dev)
        for k in ("topk_idx", "counts", "offsets", "token_slot"):
            assert torch.equal(got[k], want[k]), f"{case}: {k}"
        assert torch.equal(got["topk_w"].view(torch.int32), want["topk_w"].view(torch.int32)), case


def test_route_noalloc_rejects_oversize(cuda_dev):
    from final_b200 import _lib
    lib = _lib.load()
    big = 65536 + 32
    x = torch.zeros(1, device=cuda_dev)
    rc = lib.b2_moe_route_noalloc(C.c_void_p(x.data_ptr()), C.c_void_p(x.data_ptr()), None,
                                  big, 2048, 32, 4, C.c_float(1.0), C.c_void_p(x.data_ptr()),
                                  C.c_void_p(x.data_ptr()), C.c_void_p(x.data_ptr()),
                                  C.c_void_p(x.data_ptr()), C.c_void_p(x.data_ptr()), None)
    assert rc == _lib.B2_ERR_CAPACITY
