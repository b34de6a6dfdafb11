"""ctypes binding of the shrimp_b200 C ABI (include/shrimp_b200.h).

The library is mandatory: importing the model on a machine without the built
library, or calling it with CPU tensors, raises instead of falling back.
"""

from __future__ import annotations

import ctypes as C
from functools import lru_cache

from .build import lib_path

MAX_BLOCKS = 32
SB_OK = 0
SB_ERR_INVALID_ARG = 1
SB_ERR_UNSUPPORTED = 2
SB_ERR_CUDA = 3
SB_ERR_WORKSPACE = 4

DT_F32, DT_F16, DT_BF16, DT_I64, DT_I32, DT_U8, DT_I16, DT_U16 = range(8)

EXPORTED = (
    "sb_abi_version",
    "sb_last_error",
    "sb_forward_workspace_bytes",
    "sb_forward_policy_value",
    "sb_plan_groups",
    "sb_evaluate_workspace_bytes",
    "sb_evaluate_payload",
    "sb_build_gather_index",
    "sb_build_pair_u8",
    "sb_hex_conv",
    "sb_hex_conv_noalloc",
    "sb_hex_conv_ln",
    "sb_hex_conv_workspace_bytes",
    "sb_hex_conv_plan",
    "sb_hex_conv_planned",
    "sb_hex_conv_ln_planned",
    "sb_attn_pair",
    "sb_pack_hex_conv_weight",
    "sb_pack_linear_weight",
    "sb_decode_binned",
    "sb_legal_prefix_softmax",
    "sb_raytap_conv",
    "sb_offset_attention",
)

_P = C.c_void_p


class ConvBlockW(C.Structure):
    _fields_ = [(n, _P) for n in ("w1", "b1", "ln1_w", "ln1_b", "w2", "b2", "ln2_w", "ln2_b", "gamma")]


class AttnBlockW(C.Structure):
    _fields_ = [
        (n, _P)
        for n in (
            "ln1_w", "ln1_b", "wqkv", "bqkv", "wo", "bo", "gamma_attn", "ln2_w", "ln2_b",
            "w1", "b1", "w2", "b2", "gamma_mlp", "bias_table",
        )
    ]


class Net(C.Structure):
    _fields_ = [
        ("channels", C.c_int),
        ("heads", C.c_int),
        ("num_blocks", C.c_int),
        ("layout", C.c_char * (MAX_BLOCKS + 1)),
        ("stem_w", _P), ("stem_b", _P), ("stem_ln_w", _P), ("stem_ln_b", _P),
        ("tokens", _P), ("tokens_ln16", _P),
        ("ln_final_w", _P), ("ln_final_b", _P),
        ("policy_conv_w", _P), ("policy_conv_b", _P),
        ("policy_head_w", _P), ("policy_head_b", _P),
        ("value_red_wT", _P), ("value_red_b", _P), ("value_head_wT", _P), ("value_head_b", _P),
        ("ml_red_wT", _P), ("ml_red_b", _P), ("ml_head_wT", _P), ("ml_head_b", _P),
        ("lut", _P),
        ("conv", ConvBlockW * MAX_BLOCKS),
        ("attn", AttnBlockW * MAX_BLOCKS),
    ]


class Inputs(C.Structure):
    _fields_ = [
        ("feats", _P), ("feats_dtype", C.c_int),
        ("nbr", _P), ("nbr_dtype", C.c_int),
        ("mask", _P), ("mask_dtype", C.c_int),
        ("coords", _P), ("coords_dtype", C.c_int),
        ("batch", C.c_int), ("npad", C.c_int),
    ]


class Outputs(C.Structure):
    _fields_ = [(n, _P) for n in ("policy", "value_logits", "value", "ml_logits", "moves_left", "status")]


class Payload(C.Structure):
    _fields_ = [
        ("node_feats", _P), ("feats_dtype", C.c_int),
        ("node_qr", _P), ("nbr", _P), ("row_offsets", _P), ("legal_counts", _P), ("prior_offsets", _P),
        ("batch", C.c_int),
    ]


class Reply(C.Structure):
    _fields_ = [(n, _P) for n in ("values", "priors", "moves_left", "priors_logits", "status")]


class Group(C.Structure):
    _fields_ = [("start", C.c_int), ("end", C.c_int), ("pad_to", C.c_int)]


class NativeError(RuntimeError):
    pass


@lru_cache(maxsize=1)
def lib() -> C.CDLL:
    path = lib_path()
    if not path.exists():
        raise NativeError(
            f"shrimp_b200 native library missing at {path}; build it with `python -m hexo_bot_b200.build`"
        )
    h = C.CDLL(str(path))
    sz = C.c_size_t
    i32 = C.c_int
    f32 = C.c_float
    sig = {
        "sb_abi_version": ([], i32),
        "sb_last_error": ([C.c_char_p, sz], i32),
        "sb_forward_workspace_bytes": ([C.POINTER(Net), i32, i32, C.POINTER(sz)], i32),
        "sb_forward_policy_value": ([C.POINTER(Net), C.POINTER(Inputs), C.POINTER(Outputs), _P, sz, _P], i32),
        "sb_plan_groups": ([_P, i32, i32, C.c_double, C.c_double, C.POINTER(Group), C.POINTER(i32)], i32),
        "sb_evaluate_workspace_bytes": ([C.POINTER(Net), C.POINTER(Group), i32, C.POINTER(sz)], i32),
        "sb_evaluate_payload": ([C.POINTER(Net), C.POINTER(Payload), C.POINTER(Group), i32, C.POINTER(Reply), _P, sz,
                                 _P], i32),
        "sb_build_gather_index": ([_P, i32, i32, i32, _P, _P, _P], i32),
        "sb_build_pair_u8": ([_P, i32, _P, i32, i32, i32, _P, _P, _P], i32),
        "sb_hex_conv": ([_P, _P, _P, _P, _P, i32, i32, i32, i32, _P, _P, sz, _P], i32),
        "sb_hex_conv_noalloc": ([_P, _P, _P, _P, _P, i32, i32, i32, i32, _P, _P], i32),
        "sb_hex_conv_ln": ([_P, _P, _P, _P, _P, _P, _P, f32, i32, i32, i32, i32, i32, _P, _P, sz, _P], i32),
        "sb_hex_conv_workspace_bytes": ([i32, i32, C.POINTER(sz)], i32),
        "sb_hex_conv_plan": ([_P, _P, i32, i32, _P, sz, C.POINTER(i32), _P], i32),
        "sb_hex_conv_planned": ([_P, _P, sz, i32, _P, _P, i32, i32, i32, i32, _P, _P], i32),
        "sb_hex_conv_ln_planned": ([_P, _P, sz, i32, _P, _P, _P, _P, f32, i32, i32, i32, i32, i32, _P, _P], i32),
        "sb_attn_pair": ([_P, _P, _P, _P, _P, _P, i32, i32, i32, i32, _P, _P], i32),
        "sb_pack_hex_conv_weight": ([_P, i32, i32, i32, i32, _P, _P], i32),
        "sb_pack_linear_weight": ([_P, i32, i32, _P, _P], i32),
        "sb_decode_binned": ([_P, i32, f32, f32, _P, _P], i32),
        "sb_legal_prefix_softmax": ([_P, i32, i32, _P, _P, _P, _P], i32),
        "sb_raytap_conv": ([_P, _P, i32, _P, _P, i32, i32, i32, _P, _P, sz, _P], i32),
        "sb_offset_attention": ([_P, _P, _P, _P, i32, _P, i32, i32, i32, i32, _P, _P], i32),
    }
    for name, (args, res) in sig.items():
        fn = getattr(h, name)
        fn.argtypes = args
        fn.restype = res
    return h


def last_error() -> str:
    buf = C.create_string_buffer(512)
    lib().sb_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(status: int, what: str) -> None:
    if status != SB_OK:
        raise NativeError(f"{what} failed (status {status}): {last_error()}")
