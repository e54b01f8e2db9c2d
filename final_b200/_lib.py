"""ctypes binding of the C ABI declared in include/b2moe.h.

The CUDA library is mandatory: importing this module on a machine where
``final_b200/lib/libb2moe.so`` is missing raises immediately -- there is no
CPU fallback for any entry point.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libb2moe.so"

B2_OK, B2_ERR_INVALID, B2_ERR_CUDA, B2_ERR_CAPACITY, B2_ERR_DEVICE, B2_ERR_NO_DEVICE, B2_ERR_COMM = range(7)
B2_BF16, B2_TF32, B2_F32 = 0, 1, 2

# Every symbol include/*.h declares (checked by tests/test_abi.py).
EXPORTED = (
    "b2_moe_create", "b2_moe_destroy", "b2_moe_forward", "b2_moe_forward_ex",
    "b2_moe_get_status", "b2_moe_tile_rows", "b2_moe_profile_enable", "b2_moe_profile_read", "b2_moe_device_bytes", "b2_gemm_nt", "b2_convert_f32_to_bf16",
    "b2_gemm_plan", "b2_gemm_nt_config",
    "b2_kernel_launch_count", "b2_status_string", "b2_version", "b2_moe_route_noalloc",
    "b2_device_code_version", "b2_moe_dispatch_slots",
    # include/b2moe_ep.h
    "b2_ep_plan_compute", "b2_ep_unique_id", "b2_ep_create", "b2_ep_forward",
    "b2_ep_set_timeout", "b2_ep_last_plan", "b2_ep_layer", "b2_ep_destroy", "b2_flag_wait",
    "b2_ep_profile_timeline", "b2_ep_set_pipeline", "b2_ep_fused_schedule",
    # include/b2mlp.h
    "b2_mlp_create", "b2_mlp_forward", "b2_mlp_get_status", "b2_mlp_device_bytes",
    "b2_mlp_destroy",
    # include/b2lfm2.h
    "b2_rmsnorm", "b2_add_rmsnorm", "b2_rope_tables", "b2_embed",
    "b2_attn_create", "b2_attn_forward", "b2_attn_destroy",
    "b2_conv_create", "b2_conv_forward", "b2_conv_destroy",
    "b2_lfm2_create", "b2_lfm2_create_ep", "b2_lfm2_set_timeout", "b2_lfm2_forward",
    "b2_lfm2_forward_ex", "b2_lfm2_get_status", "b2_lfm2_device_bytes", "b2_lfm2_destroy",
    # include/b2loader.h
    "b2_loader_open", "b2_loader_num_tensors", "b2_loader_name", "b2_loader_tensor",
    "b2_loader_weight", "b2_loader_close",
)

EP_MAX_WORLD = 64
EP_MAX_SEGMENTS = 256
B2_EP_OWNER, B2_EP_BALANCED = 0, 1


class B2Error(RuntimeError):
    def __init__(self, status: int, what: str, lib=None):
        msg = lib.b2_status_string(status).decode() if lib is not None else str(status)
        super().__init__(f"{what}: {msg} (status {status})")
        self.status = status


class MoeDesc(C.Structure):
    _fields_ = [("hidden", C.c_int), ("inter", C.c_int), ("num_experts", C.c_int),
                ("top_k", C.c_int), ("max_tokens", C.c_int), ("routed_scale", C.c_float),
                ("use_bias", C.c_int), ("dtype", C.c_int)]


class MlpDesc(C.Structure):
    _fields_ = [("hidden", C.c_int), ("inter", C.c_int), ("max_tokens", C.c_int),
                ("dtype", C.c_int)]


class AttnDesc(C.Structure):
    _fields_ = [("hidden", C.c_int), ("num_heads", C.c_int), ("num_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("max_tokens", C.c_int), ("eps", C.c_float)]


class ConvDesc(C.Structure):
    _fields_ = [("hidden", C.c_int), ("kernel", C.c_int), ("max_tokens", C.c_int)]


class Lfm2Desc(C.Structure):
    _fields_ = [("vocab", C.c_int), ("hidden", C.c_int), ("num_layers", C.c_int),
                ("num_heads", C.c_int), ("num_kv_heads", C.c_int), ("dense_inter", C.c_int),
                ("moe_inter", C.c_int), ("num_experts", C.c_int), ("top_k", C.c_int),
                ("num_dense_layers", C.c_int), ("max_batch", C.c_int), ("max_seq", C.c_int),
                ("eps", C.c_float), ("rope_theta", C.c_float), ("routed_scale", C.c_float),
                ("use_expert_bias", C.c_int), ("layer_types", C.c_int * 64), ("dtype", C.c_int)]


# const float *(*)(void *ctx, const char *name, int64_t numel)
WEIGHT_FN = C.CFUNCTYPE(C.c_void_p, C.c_void_p, C.c_char_p, C.c_int64)


class MoeTrace(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "logits", "topk_idx", "topk_w", "counts", "offsets", "mtile_offsets",
        "token_slot", "sorted_token", "sorted_w")]


class EpPlan(C.Structure):
    _fields_ = [("send_off", C.c_int64 * EP_MAX_WORLD), ("send_cnt", C.c_int64 * EP_MAX_WORLD),
                ("recv_off", C.c_int64 * EP_MAX_WORLD), ("recv_cnt", C.c_int64 * EP_MAX_WORLD),
                ("recv_rows", C.c_int64), ("num_segments", C.c_int32),
                ("seg_off", C.c_int32 * EP_MAX_SEGMENTS), ("seg_cnt", C.c_int32 * EP_MAX_SEGMENTS),
                ("seg_expert", C.c_int32 * EP_MAX_SEGMENTS),
                ("seg_source", C.c_int32 * EP_MAX_SEGMENTS)]

    def to_dict(self, world: int) -> dict:
        n = self.num_segments
        return {"send_off": list(self.send_off[:world]), "send_cnt": list(self.send_cnt[:world]),
                "recv_off": list(self.recv_off[:world]), "recv_cnt": list(self.recv_cnt[:world]),
                "recv_rows": int(self.recv_rows), "seg_off": list(self.seg_off[:n]),
                "seg_cnt": list(self.seg_cnt[:n]), "seg_expert": list(self.seg_expert[:n]),
                "seg_source": list(self.seg_source[:n])}


_lib = None


def load(path: Path | None = None):
    """Load (once) and type the library; raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise ImportError(
            f"{p} is missing: build it with `python -m final_b200.build` "
            "(the MoE / GEMM path has no CPU fallback)")
    lib = C.CDLL(str(p))
    vp, i, sz = C.c_void_p, C.c_int, C.c_size_t
    lib.b2_moe_create.argtypes = [C.POINTER(MoeDesc), vp, vp, vp, vp, vp, i, vp, C.POINTER(vp)]
    lib.b2_moe_destroy.argtypes = [vp]
    lib.b2_moe_forward.argtypes = [vp, vp, vp, i, vp]
    lib.b2_moe_forward_ex.argtypes = [vp, vp, vp, i, C.POINTER(MoeTrace), vp]
    lib.b2_moe_get_status.argtypes = [vp, vp, C.POINTER(i)]
    lib.b2_moe_profile_enable.argtypes = [vp, i]
    lib.b2_moe_profile_read.argtypes = [vp, C.POINTER(C.c_float), C.POINTER(i)]
    lib.b2_moe_device_bytes.argtypes = [vp]
    lib.b2_moe_device_bytes.restype = sz
    lib.b2_gemm_nt.argtypes = [vp, vp, vp, i, i, i, i, i, vp, vp]
    lib.b2_convert_f32_to_bf16.argtypes = [vp, vp, sz, vp]
    lib.b2_gemm_plan.argtypes = [i, i, i, i, i, C.POINTER(i), C.POINTER(i), C.POINTER(i)]
    lib.b2_gemm_plan.restype = i
    lib.b2_gemm_nt_config.argtypes = [vp, vp, vp, i, i, i, i, i, i, i, i, vp, vp]
    lib.b2_gemm_nt_config.restype = i
    lib.b2_moe_route_noalloc.argtypes = [vp, vp, vp, i, i, i, i, C.c_float, vp, vp, vp, vp, vp, vp]
    lib.b2_ep_plan_compute.argtypes = [i, i, i, i, vp, C.POINTER(EpPlan)]
    lib.b2_ep_unique_id.argtypes = [vp]
    lib.b2_ep_create.argtypes = [C.POINTER(MoeDesc), i, i, vp, i, vp, vp, vp, vp, vp, i, vp,
                                 C.POINTER(vp)]
    lib.b2_ep_forward.argtypes = [vp, vp, vp, i, vp]
    lib.b2_ep_set_timeout.argtypes = [vp, C.c_double]
    lib.b2_ep_set_pipeline.argtypes = [vp, i]
    lib.b2_ep_fused_schedule.argtypes = [i, i, i, i, vp, i, vp, C.POINTER(i), C.POINTER(i)]
    lib.b2_flag_wait.argtypes = [vp, vp, i, C.c_uint64, C.c_double, vp, vp]
    lib.b2_ep_last_plan.argtypes = [vp, C.POINTER(EpPlan)]
    lib.b2_ep_profile_timeline.argtypes = [vp, i, C.POINTER(i), C.POINTER(C.c_float),
                                           C.POINTER(i)]
    lib.b2_ep_layer.argtypes = [vp]
    lib.b2_ep_layer.restype = vp
    lib.b2_ep_destroy.argtypes = [vp]
    lib.b2_mlp_create.argtypes = [C.POINTER(MlpDesc), vp, vp, vp, i, vp, C.POINTER(vp)]
    lib.b2_mlp_forward.argtypes = [vp, vp, vp, i, vp]
    lib.b2_mlp_get_status.argtypes = [vp, vp, C.POINTER(i)]
    lib.b2_mlp_device_bytes.argtypes = [vp]
    lib.b2_mlp_device_bytes.restype = sz
    lib.b2_mlp_destroy.argtypes = [vp]
    f = C.c_float
    lib.b2_rmsnorm.argtypes = [vp, vp, vp, i, i, f, vp]
    lib.b2_add_rmsnorm.argtypes = [vp, vp, vp, vp, vp, i, i, f, vp]
    lib.b2_rope_tables.argtypes = [vp, vp, i, i, f]
    lib.b2_embed.argtypes = [vp, vp, vp, i, i, i, vp, vp]
    lib.b2_attn_create.argtypes = [C.POINTER(AttnDesc), vp, vp, vp, vp, vp, vp, i, vp,
                                   C.POINTER(vp)]
    lib.b2_attn_forward.argtypes = [vp, vp, vp, vp, vp, i, i, vp]
    lib.b2_attn_destroy.argtypes = [vp]
    lib.b2_conv_create.argtypes = [C.POINTER(ConvDesc), vp, vp, vp, i, vp, C.POINTER(vp)]
    lib.b2_conv_forward.argtypes = [vp, vp, vp, i, i, vp]
    lib.b2_conv_destroy.argtypes = [vp]
    lib.b2_lfm2_create.argtypes = [C.POINTER(Lfm2Desc), WEIGHT_FN, vp, i, vp, C.POINTER(vp)]
    lib.b2_lfm2_create_ep.argtypes = [C.POINTER(Lfm2Desc), WEIGHT_FN, vp, i, i, i, vp, i, vp,
                                      C.POINTER(vp)]
    lib.b2_lfm2_set_timeout.argtypes = [vp, C.c_double]
    lib.b2_lfm2_forward.argtypes = [vp, vp, i, i, vp, vp]
    lib.b2_lfm2_forward_ex.argtypes = [vp, vp, i, i, vp, vp, vp]
    lib.b2_lfm2_get_status.argtypes = [vp, vp, C.POINTER(i)]
    lib.b2_lfm2_device_bytes.argtypes = [vp]
    lib.b2_lfm2_device_bytes.restype = sz
    lib.b2_lfm2_destroy.argtypes = [vp]
    for name in ("b2_rmsnorm", "b2_add_rmsnorm", "b2_rope_tables", "b2_embed", "b2_attn_create",
                 "b2_attn_forward", "b2_attn_destroy", "b2_conv_create", "b2_conv_forward",
                 "b2_conv_destroy", "b2_lfm2_create", "b2_lfm2_create_ep", "b2_lfm2_set_timeout",
                 "b2_lfm2_forward", "b2_lfm2_forward_ex", "b2_lfm2_get_status",
                 "b2_lfm2_destroy"):
        getattr(lib, name).restype = i
    lib.b2_loader_open.argtypes = [C.c_char_p, C.POINTER(vp)]
    lib.b2_loader_open.restype = i
    lib.b2_loader_num_tensors.argtypes = [vp]
    lib.b2_loader_num_tensors.restype = C.c_int64
    lib.b2_loader_name.argtypes = [vp, C.c_int64]
    lib.b2_loader_name.restype = C.c_char_p
    lib.b2_loader_tensor.argtypes = [vp, C.c_char_p, C.POINTER(vp), C.POINTER(C.c_int64),
                                     C.POINTER(C.c_int64), C.POINTER(i)]
    lib.b2_loader_tensor.restype = i
    lib.b2_loader_weight.argtypes = [vp, C.c_char_p, C.c_int64]
    lib.b2_loader_weight.restype = vp
    lib.b2_loader_close.argtypes = [vp]
    lib.b2_loader_close.restype = i
    lib.b2_kernel_launch_count.restype = C.c_uint64
    lib.b2_moe_tile_rows.restype = i
    lib.b2_status_string.argtypes = [i]
    lib.b2_status_string.restype = C.c_char_p
    lib.b2_version.restype = C.c_char_p
    lib.b2_device_code_version.argtypes = [C.POINTER(i)]
    lib.b2_moe_dispatch_slots.argtypes = [vp, vp, i, vp, vp, vp, vp]
    lib.b2_device_code_version.restype = i
    for name in ("b2_moe_create", "b2_moe_destroy", "b2_moe_forward", "b2_moe_forward_ex",
                 "b2_moe_get_status", "b2_gemm_nt", "b2_convert_f32_to_bf16",
                 "b2_moe_profile_enable", "b2_moe_profile_read", "b2_moe_route_noalloc",
                 "b2_moe_dispatch_slots",
                 "b2_ep_plan_compute", "b2_ep_unique_id", "b2_ep_create", "b2_ep_forward",
                 "b2_ep_set_timeout", "b2_ep_last_plan", "b2_ep_destroy", "b2_flag_wait",
                 "b2_ep_profile_timeline", "b2_ep_set_pipeline", "b2_ep_fused_schedule",
                 "b2_mlp_create", "b2_mlp_forward", "b2_mlp_get_status", "b2_mlp_destroy"):
        getattr(lib, name).restype = i
    _lib = lib
    return lib


def check(status: int, what: str) -> None:
    if status != B2_OK:
        raise B2Error(status, what, _lib)
