"""final_b200 -- B200-native (sm_100a) MoE expert-FFN and dense-GEMM hot path
of the LFM2-8B-A1B inference engine, behind the reference's operator API.

Compute lives in ``lib/libb2moe.so`` (hand-written tcgen05 / TMA CUDA, C ABI
in include/b2moe.h, b2moe_ep.h, b2mlp.h, b2lfm2.h).  This package is the
Python side of that boundary: ctypes bindings plus host mirrors of the
reference's SparseMoeBlock, MLP, Attention, ShortConv, RMSNorm and LFM2Model.
"""
from ._lib import B2Error, load  # noqa: F401
from .lfm2 import Attention, LFM2Model, ShortConv, embed, rmsnorm, rope_tables  # noqa: F401
from .mlp import MLP  # noqa: F401
from .moe import SparseMoeBlock, gemm_nt, launch_count, to_bf16  # noqa: F401

__all__ = ["SparseMoeBlock", "MLP", "Attention", "ShortConv", "LFM2Model", "rmsnorm",
           "rope_tables", "embed", "gemm_nt", "to_bf16", "launch_count", "B2Error", "load"]
