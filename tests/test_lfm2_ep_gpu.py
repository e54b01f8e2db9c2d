"""The expert-parallel model (b2_lfm2_create_ep) on GPUs.

Every rank runs its own batch through the whole model; only the MoE layers
exchange expert rows.  Its logits must be bit-identical to the single-GPU
model's (b2_lfm2_create) on the same ids: the dense blocks are the same
kernels, and each expert row meets the same grouped GEMMs and the same
k-ordered combine wherever it is computed.  The one-rank cases run on any
B200 box; the two-rank cases need two GPUs and are skipped on a one-GPU box.
"""
import os
import socket

import numpy as np
import pytest
import torch

import lfm2_cases as lc

pytestmark = pytest.mark.gpu

CFG = lc.TINY


def _overrides(cfg):
    return dict(vocab=cfg["vocab"], hidden=cfg["H"], num_layers=cfg["layers"],
                num_heads=cfg["HQ"], num_kv_heads=cfg["HKV"], dense_inter=cfg["I_DENSE"],
                moe_inter=cfg["I_MOE"], num_experts=cfg["E"], top_k=cfg["K"],
                num_dense_layers=cfg["NUM_DENSE"], layer_types=cfg["TYPES"])


def _model(W, cfg, dev, **ep):
    from final_b200.lfm2 import LFM2Model
    fetched = []

    def get(name, n):
        if name == "lm_head.weight":
            return None
        fetched.append(name)
        return W(name)
    with torch.cuda.device(dev):
        m = LFM2Model(get, weights_on_host=True, max_batch=cfg["batch"], max_seq=cfg["seq"],
                      device=dev, **_overrides(cfg), **ep)
    return m, fetched


def _ids(rank):
    return lc.token_ids(CFG["batch"], CFG["seq"], CFG["vocab"], CFG["seed"] + 100 * rank)


def _single_logits(dev, ranks):
    W = lc.Weights(CFG["seed"], CFG["vocab"], CFG)
    m, _ = _model(W, CFG, dev)
    out = [m.forward(torch.from_numpy(_ids(r))).cpu() for r in ranks]
    torch.cuda.synchronize()
    assert m.device_status() == 0
    m.close()
    return out


@pytest.mark.parametrize("mode", ["owner", "balanced"])
def test_ep_model_one_rank_matches_single_gpu(cuda_dev, mode):
    want = _single_logits(cuda_dev, [0, 1])
    W = lc.Weights(CFG["seed"], CFG["vocab"], CFG)
    m, fetched = _model(W, CFG, cuda_dev, expert_parallel=mode, world=1, rank=0)
    for r in (0, 1):  # two forwards reuse the shared communicator and buffers
        got = m.forward(torch.from_numpy(_ids(r))).cpu()
        assert torch.equal(got, want[r]), r
    torch.cuda.synchronize()
    assert m.device_status() == 0
    # a rank without tokens still runs the exchanges; nothing else happens
    m.forward_gpu(torch.empty(0, dtype=torch.int32, device=cuda_dev),
                  torch.empty(0, device=cuda_dev), 0, CFG["seq"])
    torch.cuda.synchronize()
    assert m.device_status() == 0
    m.close()
    n_exp = sum(".experts." in n for n in fetched)
    assert n_exp == (CFG["layers"] - CFG["NUM_DENSE"]) * CFG["E"] * 3


def test_ep_model_rejects_bad_arguments(cuda_dev):
    from final_b200 import _lib
    W = lc.Weights(CFG["seed"], CFG["vocab"], CFG)
    with pytest.raises(_lib.B2Error):
        _model(W, CFG, cuda_dev, expert_parallel="owner", world=3, rank=0, uid=b"\0" * 128)
    with pytest.raises(_lib.B2Error):
        _model(W, CFG, cuda_dev, expert_parallel="balanced", world=2, rank=2, uid=b"\0" * 128)


def _rank_main(rank, world, port, mode, empty_rank, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "oracle"), os.path.join(root, "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime
    import torch.distributed as dist
    import lfm2_cases as lcc
    dev = torch.device(f"cuda:{rank}")
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        W = lcc.Weights(CFG["seed"], CFG["vocab"], CFG)
        m, fetched = _model(W, CFG, dev, expert_parallel=mode)
        m.lib.b2_lfm2_set_timeout(m._h, 60.0)
        if rank == empty_rank:
            m.forward_gpu(torch.empty(0, dtype=torch.int32, device=dev),
                          torch.empty(0, device=dev), 0, CFG["seq"])
            logits = None
        else:
            logits = m.forward(torch.from_numpy(_ids(rank))).cpu().numpy()
        torch.cuda.synchronize()
        status = m.device_status()
        m.close()
        q.put((rank, logits, status, sum(".experts." in n for n in fetched)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode,empty_rank", [("owner", -1), ("balanced", -1), ("balanced", 1)])
def test_ep_model_two_ranks_match_single_gpu(cuda_dev, mode, empty_rank):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs (the exchange plan is tested on CPU)")
    import torch.multiprocessing as mp
    want = _single_logits(cuda_dev, [0, 1])
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, mode, empty_rank, q))
             for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        r, logits, status, n_exp = q.get(timeout=300)
        assert status == 0
        moe_layers = CFG["layers"] - CFG["NUM_DENSE"]
        assert n_exp == moe_layers * 3 * (CFG["E"] // 2 if mode == "owner" else CFG["E"])
        got[r] = logits
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in (0, 1):
        if r == empty_rank:
            assert got[r] is None
        else:
            assert np.array_equal(got[r].view(np.uint32), want[r].numpy().view(np.uint32)), r
