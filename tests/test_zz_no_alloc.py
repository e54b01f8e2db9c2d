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
    bias = None if inp["bias"] is None else _t(inp["bias"], dev)
    layer = SparseMoeBlock(_t(inp["gate"], dev), _t(inp["w1"], dev), _t(inp["w2"], dev),
                           _t(inp["w3"], dev), bias,
                           max_tokens=inp["x"].shape[0], top_k=inp["K"])
    out = layer.forward_traced(_t(inp["x"], dev))
    torch.cuda.synchronize()
    assert layer.device_status() == 0
    layer.close()
    return {k: out[k].cpu() for k in ("topk_idx", "topk_w", "counts", "offsets", "token_slot")}


def _noalloc_entry(inp, dev, stream=None):
    from final_b200 import _lib
    lib = _lib.load()
    x, gate = _t(inp["x"], dev), _t(inp["gate"], dev)
    bias = None if inp["bias"] is None else _t(inp["bias"], dev)
    T, H = inp["x"].shape
    E, K = inp["gate"].shape[0], inp["K"]
    out = {
        "topk_idx": torch.full((T, K), -7, dtype=torch.int32, device=dev),
        "topk_w": torch.full((T, K), -7.0, dtype=torch.float32, device=dev),
        "counts": torch.full((E,), -7, dtype=torch.int32, device=dev),
        "offsets": torch.full((E,), -7, dtype=torch.int32, device=dev),
        "token_slot": torch.full((T, K), -7, dtype=torch.int32, device=dev),
    }
    p = lambda t: None if t is None else C.c_void_p(t.data_ptr())
    s = stream if stream is not None else torch.cuda.current_stream()
    s.wait_stream(torch.cuda.current_stream())
    rc = lib.b2_moe_route_noalloc(p(x), p(gate), p(bias), T, H, E, K, C.c_float(1.0),
                                  p(out["topk_idx"]), p(out["topk_w"]), p(out["counts"]),
                                  p(out["offsets"]), p(out["token_slot"]),
                                  C.c_void_p(s.cuda_stream))
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


def test_route_noalloc_without_bias_on_own_stream(cuda_dev):
    """No expert bias (NULL), issued on a stream of the caller's own: the same
    bits as the allocating entry point run without bias."""
    inp = dict(build_case("hot_expert"))
    inp["bias"] = None
    want = _reference_entry(inp, cuda_dev)
    got = _noalloc_entry(inp, cuda_dev, stream=torch.cuda.Stream(cuda_dev))
    for k in ("topk_idx", "counts", "offsets", "token_slot"):
        assert torch.equal(got[k], want[k]), k
    assert torch.equal(got["topk_w"].view(torch.int32), want["topk_w"].view(torch.int32))


def test_route_noalloc_zero_tokens_clears_counts(cuda_dev):
    """T = 0 launches no kernel but still reports zero counts and offsets."""
    from final_b200 import _lib
    lib = _lib.load()
    g = torch.zeros(32, 256, device=cuda_dev)
    counts = torch.full((32,), -7, dtype=torch.int32, device=cuda_dev)
    offsets = torch.full((32,), -7, dtype=torch.int32, device=cuda_dev)
    rc = lib.b2_moe_route_noalloc(None, C.c_void_p(g.data_ptr()), None, 0, 256, 32, 4,
                                  C.c_float(1.0), None, None, C.c_void_p(counts.data_ptr()),
                                  C.c_void_p(offsets.data_ptr()), None, None)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(counts.abs().sum()) == 0 and int(offsets.abs().sum()) == 0


def test_route_noalloc_argument_statuses(cuda_dev):
    """Which limit gives which status, all returned before any device work:
    sizes beyond the fixed scratch give B2_ERR_CAPACITY, shapes the kernels do
    not support and a misaligned x give B2_ERR_INVALID."""
    from final_b200 import _lib
    lib = _lib.load()
    buf = torch.zeros(1 << 16, device=cuda_dev)
    p = C.c_void_p(buf.data_ptr())
    mis = C.c_void_p(buf.data_ptr() + 4)

    def call(x, T, H, E, K):
        return lib.b2_moe_route_noalloc(x, p, None, T, H, E, K, C.c_float(1.0), p, p, p, p, p,
                                        None)

    assert call(p, 64, 8192, 32, 4) == _lib.B2_ERR_CAPACITY      # hidden above 4096
    assert call(p, 65537, 256, 32, 4) == _lib.B2_ERR_CAPACITY    # tokens above 65536
    assert call(p, 64, 256, 33, 4) == _lib.B2_ERR_INVALID        # experts above 32
    assert call(p, 64, 256, 32, 9) == _lib.B2_ERR_INVALID        # top-k above 8
    assert call(p, 64, 256, 4, 5) == _lib.B2_ERR_INVALID         # top-k above experts
    assert call(p, 64, 200, 32, 4) == _lib.B2_ERR_INVALID        # hidden not a multiple of 64
    assert call(mis, 64, 256, 32, 4) == _lib.B2_ERR_INVALID      # x not 16-byte aligned
    torch.cuda.synchronize()
