"""ctypes binding of the C ABI in include/bt_b200.h.

The shared library is built in-tree (``python -m breezetoken_b200.build``)
and loaded from ``breezetoken_b200/lib``.  There is no fallback: if the
library is missing or fails to load, every B200 entry point raises.
"""

from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libbt_b200.so"

BT_OK, BT_ERR_INVALID, BT_ERR_UNSUPPORTED, BT_ERR_CUDA, BT_ERR_TIMEOUT = range(5)
BT_F32, BT_BF16 = 0, 1
BT_STATUS_WORDS = 8

_SITES = {
    1: "GEMV producer waiting for a consumed stage",
    2: "GEMV producer waiting for its last copies",
    3: "GEMV consumer waiting for a stage",
    4: "token id outside the vocabulary",
    5: "attended length outside the cache",
    6: "RoPE position outside the table",
}


def describe_status(rec) -> str:
    """Human-readable form of a device status record [code, site, block, a, b, c, ...]."""
    code, site, block, a, b, c = (list(rec) + [0] * 6)[:6]
    what = "bounded wait expired" if code == BT_ERR_TIMEOUT else "invalid input"
    return f"{what} at {_SITES.get(site, f'site {site}')} (block {block}, detail {a}, {b}, {c})"


class B200Error(RuntimeError):
    """A failed call into the B200 library (carries the BT_* status code)."""

    def __init__(self, code: int, msg: str) -> None:
        super().__init__(f"[bt status {code}] {msg}")
        self.code = code


class BtMoeShared(C.Structure):
    _fields_ = [("gate", C.c_void_p), ("up", C.c_void_p), ("down", C.c_void_p), ("gate_inp", C.c_void_p),
                ("ffn", C.c_int64)]


class BtQwen35Dims(C.Structure):
    _fields_ = [
        (n, C.c_int32)
        for n in (
            "hidden", "n_layers", "n_heads", "n_kv", "head_dim", "rope_dim", "ffn", "vocab",
            "ssm_inner", "ssm_state", "ssm_heads", "conv_k", "max_ctx", "batch",
        )
    ] + [("eps", C.c_float), ("l2_eps", C.c_float)]


class BtQwen35Layer(C.Structure):
    _fields_ = [
        ("is_attn", C.c_int32),
        ("pad_", C.c_int32),
        ("norm_in", C.c_void_p),
        ("norm_post", C.c_void_p),
        ("norm_next", C.c_void_p),
        ("w_in", C.c_void_p),
        ("w_out", C.c_void_p),
        ("w_gu", C.c_void_p),
        ("w_down", C.c_void_p),
        ("conv_w", C.c_void_p),
        ("a_log", C.c_void_p),
        ("dt_bias", C.c_void_p),
        ("ssm_norm", C.c_void_p),
        ("q_norm", C.c_void_p),
        ("k_norm", C.c_void_p),
        ("conv_state", C.c_void_p),
        ("rec_state", C.c_void_p),
        ("k_cache", C.c_void_p),
        ("v_cache", C.c_void_p),
    ]


class BtQwen35Model(C.Structure):
    _fields_ = [
        ("dims", BtQwen35Dims),
        ("embed", C.c_void_p),
        ("rope_cos", C.c_void_p),
        ("rope_sin", C.c_void_p),
        ("layers", C.POINTER(BtQwen35Layer)),
    ]


class BtQwen35Runtime(C.Structure):
    _fields_ = [
        (n, C.c_void_p)
        for n in (
            "pos", "token", "history", "logits", "h0", "h1", "delta", "proj", "mix", "act", "workspace", "trace",
            "status",
        )
    ]


_P = C.c_void_p
_I64 = C.c_int64
_SIGS: dict[str, tuple[object, list]] = {
    "bt_last_error": (C.c_char_p, []),
    "bt_version": (C.c_int, []),
    "bt_sm_count": (C.c_int, []),
    "bt_q8_row_bytes": (_I64, [_I64]),
    "bt_repack_q8_0": (C.c_int, [_P, _P, _I64, _I64, _I64, _I64, _P]),
    "bt_dequant_q8_rows": (C.c_int, [_P, _P, _I64, _I64, _P]),
    "bt_dequant_iq3_s": (C.c_int, [_P, _P, _I64, _I64, _P]),
    "bt_linear_q8": (C.c_int, [_P, _P, _P, _I64, _I64, C.c_int, _P]),
    "bt_linear_kn": (C.c_int, [_P, C.c_int, _P, _P, _I64, _I64, _P]),
    "bt_bf16_planes": (C.c_int, [_P, _P, _I64, _I64, _P]),
    "bt_conv_silu": (C.c_int, [_P, _P, _P, _P, _I64, _I64, _I64, _P]),
    "bt_conv_silu_scan": (C.c_int, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _P]),
    "bt_linear_rows": (C.c_int, [_P, C.c_int, _P, _P, _I64, _I64, _I64, _P]),
    "bt_linear_rows_timeouts": (C.c_int, []),
    "bt_launch_count": (C.c_longlong, []),
    "bt_rms_norm": (C.c_int, [_P, _P, _P, _I64, _I64, C.c_float, _P]),
    "bt_fused_add_rms_norm": (C.c_int, [_P, _P, _P, _P, _P, _I64, _I64, C.c_float, _P]),
    "bt_silu_mul": (C.c_int, [_P, _P, _P, _I64, _P]),
    "bt_rope": (C.c_int, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P]),
    "bt_attention_workspace_bytes": (_I64, [_I64, _I64, _I64, _I64, C.c_int]),
    "bt_attention_decode": (
        C.c_int,
        [_P, _P, _P, C.c_int, _P, _P, _I64, _I64, _I64, _I64, _I64, C.c_float, C.c_int, _P, _P],
    ),
    "bt_attention_layer": (
        C.c_int,
        [_P, _I64, _P, _P, _P, _P, _I64, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, C.c_float, C.c_float,
         C.c_int, _P, _P, _P],
    ),
    "bt_attention_decode_noalloc": (
        C.c_int,
        [_P, _P, _P, C.c_int, _P, _P, _I64, _I64, _I64, _I64, _I64, C.c_float, C.c_int, _P],
    ),
    "bt_gdn_decode": (C.c_int, [_P, _P, _P, C.c_int, _P, _P, _P, _P, _I64, _I64, _I64, _I64, C.c_float, C.c_float, _P]),
    "bt_gdn_decode_strided": (C.c_int, [_P, _P, _P, C.c_int, _I64, _I64, _I64, _P, _I64, _P, _I64, _P, _P, _I64, _I64,
                                        _I64, _I64, _I64, C.c_float, C.c_float, _P]),
    "bt_gdn_gated_step": (C.c_int, [_P, _I64, _P, _I64, _P, _P, _P, _P, _I64, _P, _P, _I64, _I64, _I64, _I64,
                                    C.c_float, C.c_float, C.c_float, _P]),
    "bt_gdn_gated_scan": (C.c_int, [_P, _I64, _P, _I64, _P, _P, _P, _P, _I64, _P, _P, _I64, _I64, _I64, _I64, _I64,
                                    C.c_float, C.c_float, C.c_float, _P]),
    "bt_gdn_prefill": (C.c_int, [_P, _P, _P, C.c_int, _I64, _I64, _I64, _I64, _I64, _I64, _P, _I64, _I64, _P, _I64,
                                 _I64, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, C.c_float, C.c_float, _P]),
    "bt_add_rms_norm_planes": (C.c_int, [_P, _P, _P, _P, _P, _P, _I64, _I64, C.c_float, _P]),
    "bt_argmax_workspace_bytes": (_I64, [_I64]),
    "bt_iq3s_row_bytes": (_I64, [_I64]),
    "bt_repack_iq3_s": (C.c_int, [_P, _P, _I64, _I64, _P]),
    "bt_moe_route": (C.c_int, [_P, _I64, _I64, C.c_int, _P, _P, _P]),
    "bt_moe_workspace_bytes": (_I64, [_I64, _I64, _I64, _I64, C.c_int]),
    "bt_moe_experts_iq3s": (
        C.c_int,
        [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _P, C.c_int, _P, _P, _P],
    ),
    "bt_moe_layer_workspace_bytes": (_I64, [_I64, _I64, _I64, _I64, _I64, C.c_int]),
    "bt_moe_layer_iq3s": (
        C.c_int,
        [_P, _P, _P, C.POINTER(BtMoeShared), _P, _I64, _I64, _I64, _I64, _P, _P, C.c_int, _P, _P, _P],
    ),
    "bt_argmax": (C.c_int, [_P, _I64, _I64, _P, _P, _P]),
    "bt_moe_layer_iq3s_add_norm": (C.c_int, [_P, _P, _P, C.POINTER(BtMoeShared), _P, _I64, _I64, _I64, _I64, _P, _P,
                                             C.c_int, _P, _P,
                                             C.c_float, _P, _P, _P, _P, _P, _P]),
    "bt_moe_route_sort_iq3s": (C.c_int, [_P, _P, _I64, _I64, _I64, _I64, C.c_int, _I64, _P, _P, _P, _P]),
    "bt_moe_layer_iq3s_add_norm_prepared": (C.c_int, [_P, _P, _P, C.POINTER(BtMoeShared), _P, _I64, _I64, _I64, _I64,
                                                      _P, _P, C.c_int, _P, _P, C.c_float, _P, _P, _P, _P, _P, _P]),
    "bt_qwen35_kernels_per_step": (C.c_int, [C.POINTER(BtQwen35Model)]),
    "bt_qwen35_proj_elems": (_I64, [C.POINTER(BtQwen35Dims)]),
    "bt_qwen35_workspace_bytes": (_I64, [C.POINTER(BtQwen35Dims)]),
    "bt_qwen35_step": (C.c_int, [C.POINTER(BtQwen35Model), C.POINTER(BtQwen35Runtime), C.c_int, _P]),
    "bt_qwen35_graph_create": (
        C.c_int,
        [C.POINTER(BtQwen35Model), C.POINTER(BtQwen35Runtime), C.c_int, _P, C.POINTER(C.c_void_p)],
    ),
    "bt_graph_launch": (C.c_int, [_P, _P]),
    "bt_graph_destroy": (C.c_int, [_P]),
}

#: every symbol include/bt_b200.h declares
EXPORTED = tuple(_SIGS)

_lib: C.CDLL | None = None
_lock = threading.Lock()


def load() -> C.CDLL:
    """Load (once) and return the library; raises B200Error if it is missing."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = Path(os.environ.get("BT_B200_LIB", LIB_PATH))
        if not path.is_file():
            raise B200Error(
                BT_ERR_UNSUPPORTED,
                f"B200 library not built ({path}); run `python -m breezetoken_b200.build`",
            )
        lib = C.CDLL(str(path))
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(rc: int, what: str) -> None:
    if rc != BT_OK:
        msg = load().bt_last_error().decode(errors="replace")
        raise B200Error(rc, f"{what}: {msg}")


def call(name: str, *args) -> None:
    """Call a status-returning entry point and raise on failure."""
    check(getattr(load(), name)(*args), name)
