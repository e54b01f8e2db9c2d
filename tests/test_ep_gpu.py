"""Expert-parallel MoE on GPUs, through the C ABI of include/b2moe_ep.h.

Every rank's output must be bit-identical to the single-GPU layer's output for
the same tokens: rows meet the same expert in the same kernels, and the
combine order does not change.  The several-rank tests run one process per
GPU at 2, 4 and 8 ranks and skip the rank counts the box has too few GPUs for
(the host-side exchange logic is covered on CPU by tests/test_ep_plan.py)."""
import os
import socket

import numpy as np
import pytest
import torch

from moe_cases import build_case

pytestmark = pytest.mark.gpu


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _single_gpu_y(inp, dev):
    from final_b200 import SparseMoeBlock
    layer = SparseMoeBlock(_t(inp["gate"], dev), _t(inp["w1"], dev), _t(inp["w2"], dev),
                           _t(inp["w3"], dev), _t(inp["bias"], dev),
                           max_tokens=inp["x"].shape[0], top_k=inp["K"])
    y = layer.forward(_t(inp["x"], dev))
    torch.cuda.synchronize()
    layer.close()
    return y.cpu()


@pytest.mark.parametrize("pipeline", ["fused", "staged"])
@pytest.mark.parametrize("mode", ["owner", "balanced"])
def test_ep_one_rank_matches_single_gpu(cuda_dev, mode, pipeline):
    from final_b200.ep import ExpertParallelMoE
    inp = build_case("zipf")
    want = _single_gpu_y(inp, cuda_dev)
    ep = ExpertParallelMoE(_t(inp["gate"], cuda_dev), _t(inp["w1"], cuda_dev),
                           _t(inp["w2"], cuda_dev), _t(inp["w3"], cuda_dev),
                           _t(inp["bias"], cuda_dev), max_tokens=inp["x"].shape[0],
                           top_k=inp["K"], mode=mode, world=1, rank=0, pipeline=pipeline)
    y = ep.forward(_t(inp["x"], cuda_dev))
    torch.cuda.synchronize()
    assert ep.device_status() == 0
    assert torch.equal(y.cpu(), want)
    plan = ep.last_plan()
    assert plan["recv_rows"] == inp["x"].shape[0] * inp["K"]
    # a second forward with fewer tokens reuses the communicator and buffers
    y2 = ep.forward(_t(inp["x"][:100], cuda_dev))
    torch.cuda.synchronize()
    assert torch.equal(y2.cpu(), _single_gpu_y({**inp, "x": inp["x"][:100]}, cuda_dev))
    ep.close()


def _rank_main(rank, world, port, mode, q, pipeline="fused"):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "oracle"), os.path.join(root, "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist
    from moe_cases import build_case as bc
    from final_b200.ep import ExpertParallelMoE
    import datetime
    dev = torch.device(f"cuda:{rank}")
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        inp = bc("zipf")
        shard = np.array_split(np.arange(inp["x"].shape[0]), world)[rank]
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        ep = ExpertParallelMoE(t(inp["gate"]), t(inp["w1"]), t(inp["w2"]), t(inp["w3"]),
                               t(inp["bias"]), max_tokens=len(shard), top_k=inp["K"], mode=mode,
                               timeout_s=60.0, pipeline=pipeline)
        y = ep.forward(t(inp["x"][shard]))
        # the other pipeline on the same layer and tokens: the same bits
        ep.set_pipeline("staged" if pipeline == "fused" else "fused")
        y2 = ep.forward(t(inp["x"][shard]))
        torch.cuda.synchronize()
        assert torch.equal(y, y2), f"rank {rank}: pipelines differ"
        status = ep.device_status()
        plan = ep.last_plan()
        ep.close()
        q.put((rank, y.cpu().numpy(), status, plan["recv_rows"]))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("pipeline", ["fused", "staged"])
@pytest.mark.parametrize("mode", ["owner", "balanced"])
def test_ep_ranks_match_single_gpu(cuda_dev, mode, pipeline, world):
    """world ranks (one per GPU) over the same 512 tokens: the concatenated
    outputs are bit-identical to the single-GPU layer's, with 32 / world
    experts per GPU in owner placement."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs (host-side exchange logic is tested on CPU)")
    import torch.multiprocessing as mp
    inp = build_case("zipf")
    want = _single_gpu_y(inp, cuda_dev).numpy()
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, mode, q, pipeline))
             for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        r, y, status, rows = q.get(timeout=300)
        assert status == 0
        got[r] = y
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    y = np.concatenate([got[r] for r in range(world)])
    assert np.array_equal(y.view(np.uint32), want.view(np.uint32))


def _config4_inputs(routing, dev, T=65536, seed=4321):
    """Config 4 (65536 tokens, H 2048, E 32, top-4, I 1792): x and the router
    from the oracle's seeded generator (host), expert weights drawn on the
    device from a seeded torch generator (identical on every GPU)."""
    import oracle
    H, E, I = 2048, 32, 1792
    x = oracle.randn((T, H), seed, oracle.S_X)
    if routing == "zipf":
        gate = np.zeros((E, H), dtype=np.float32)
        oracle.inject_logits(x, gate, oracle.zipf_logits(T, E, seed))
        bias = None
    else:
        gate = oracle.randn((E, H), seed, oracle.S_GATE, 0.02)
        bias = oracle.randn((E,), seed, oracle.S_BIAS, 0.02)
    gen = torch.Generator(device=dev).manual_seed(seed)
    w1 = torch.randn(E, I, H, device=dev, generator=gen) * 0.02
    w3 = torch.randn(E, I, H, device=dev, generator=gen) * 0.02
    w2 = torch.randn(E, H, I, device=dev, generator=gen) * 0.02
    return x, gate, bias, w1, w2, w3


def _config4_rank_main(rank, world, port, mode, routing, outdir, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "oracle"), os.path.join(root, "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime
    import torch.distributed as dist
    from final_b200.ep import ExpertParallelMoE
    dev = torch.device(f"cuda:{rank}")
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        x, gate, bias, w1, w2, w3 = _config4_inputs(routing, dev)
        shard = np.array_split(np.arange(x.shape[0]), world)[rank]
        t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        ep = ExpertParallelMoE(t(gate), w1, w2, w3, t(bias), max_tokens=len(shard), top_k=4,
                               mode=mode, timeout_s=60.0)
        del w1, w2, w3
        xs = t(x[shard])
        y = ep.forward(xs)
        y2 = ep.forward(xs)  # a second forward reuses the buffers and flags
        torch.cuda.synchronize()
        status = ep.device_status()
        plan = ep.last_plan()
        ep.close()
        path = os.path.join(outdir, f"y{rank}.npy")
        np.save(path, y.cpu().numpy())
        q.put((rank, path, status, plan["recv_rows"], bool(torch.equal(y, y2))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("routing", ["uniform", "zipf"])
def test_ep_ranks_config4_owner(cuda_dev, routing, world, tmp_path):
    """Config 4 (65536 tokens) sharded as 32 / world experts per GPU (owner
    placement: 16, 8, 4 experts per GPU on 2, 4, 8 GPUs), 65536 / world tokens
    per rank: every rank's y is bit-identical to the single-GPU layer's y for
    the same tokens (the single-GPU layer itself is checked against the oracle
    at this size by test_moe_gpu.test_moe_config4_one_gpu)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs (host-side exchange logic is tested on CPU)")
    import torch.multiprocessing as mp
    from final_b200 import SparseMoeBlock
    x, gate, bias, w1, w2, w3 = _config4_inputs(routing, cuda_dev)
    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(cuda_dev)
    layer = SparseMoeBlock(t(gate), w1, w2, w3, t(bias), max_tokens=x.shape[0], top_k=4)
    del w1, w2, w3
    want = layer.forward(t(x)).cpu().numpy()
    torch.cuda.synchronize()
    layer.close()
    torch.cuda.empty_cache()
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_config4_rank_main,
                         args=(r, world, port, "owner", routing, str(tmp_path), q))
             for r in range(world)]
    for p in procs:
        p.start()
    got, rows = {}, {}
    for _ in range(world):
        r, path, status, nrows, same = q.get(timeout=600)
        assert status == 0
        assert same, f"rank {r}: second forward differs"
        got[r] = np.load(path)
        rows[r] = nrows
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert sum(rows.values()) == x.shape[0] * 4
    y = np.concatenate([got[r] for r in range(world)])
    assert np.array_equal(y.view(np.uint32), want.view(np.uint32))
