"""final_b200 -- B200-native (sm_100a) MoE expert-FFN and dense-GEMM hot path
of the LFM2-8B-A1B inference engine, behind the reference's operator API.

Compute lives in ``lib/libb2moe.so`` (hand-written tcgen05 / TMA CUDA, C ABI
in include/b2moe.h).  This package is the Python side of that boundary:
ctypes bindings plus host mirrors of the reference's SparseMoeBlock and MLP.
"""
from ._lib import B2Error, load  # noqa: F401
from .mlp import MLP  # noqa: F401
from .moe import SparseMoeBlock, gemm_nt, launch_count, to_bf16  # noqa: F401

__all__ = ["SparseMoeBlock", "MLP", "gemm_nt", "to_bf16", "launch_count", "B2Error", "load"]
