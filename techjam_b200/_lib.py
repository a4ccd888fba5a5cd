"""ctypes binding of ``libtj.so`` (declarations in ``include/tj.h``).

The library is loaded from this package directory only.  If it is missing the
import of any compute entry point raises -- there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import threading
from ctypes import POINTER, c_char_p, c_float, c_int, c_size_t, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libtj.so")

TJ_OK = 0
TJ_ERR_DEVICE = 4
STATUS_NAMES = {0: "TJ_OK", 1: "TJ_ERR_INVALID", 2: "TJ_ERR_UNSUPPORTED", 3: "TJ_ERR_CUDA",
                4: "TJ_ERR_DEVICE", 5: "TJ_ERR_NO_DEVICE", 6: "TJ_ERR_NCCL"}
ROUTE_EXACT, ROUTE_POLY, ROUTE_AUTO = 0, 1, 2
EPI_QKV, EPI_GELU, EPI_RESID, EPI_PLAIN16 = 0, 1, 2, 3
KERNEL_CLASSES = ("prep", "layernorm", "gemm_qkv", "attention", "gemm_out", "gemm_ffn_in", "gemm_ffn_out",
                  "layernorm_final", "poly")

LAYER_FIELDS = ("norm1_weight", "norm1_bias", "q_weight", "q_bias", "k_weight", "k_bias", "v_weight", "v_bias",
                "out_weight", "out_bias", "norm2_weight", "norm2_bias", "ffn_in_weight", "ffn_in_bias",
                "ffn_out_weight", "ffn_out_bias")


class TjConfig(ctypes.Structure):
    _fields_ = [("d_model", c_int), ("num_heads", c_int), ("ffn_dim", c_int), ("num_layers", c_int),
                ("causal", c_int), ("layer_norm_eps", c_float)]


class TjLayerParams(ctypes.Structure):
    _fields_ = [(name, c_void_p) for name in LAYER_FIELDS]


class TjError(RuntimeError):
    """A libtj entry point returned a non-zero TjStatus."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


# name -> (restype, argtypes); mirrors include/tj.h
SIGNATURES = {
    "tj_version": (c_int, []),
    "tj_last_error": (c_char_p, []),
    "tj_model_create": (c_int, [POINTER(TjConfig), POINTER(c_void_p)]),
    "tj_model_destroy": (c_int, [c_void_p]),
    "tj_model_load_layer": (c_int, [c_void_p, c_int, POINTER(TjLayerParams), c_void_p]),
    "tj_model_load_final_norm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p]),
    "tj_workspace_bytes": (c_int, [c_void_p, c_int, c_int, c_int, POINTER(c_size_t)]),
    "tj_forward": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_size_t,
                           c_void_p]),
    "tj_forward_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "tj_device_error": (c_int, [c_void_p, POINTER(c_int)]),
    "tj_set_wait_limit": (c_int, [ctypes.c_ulonglong]),
    "tj_set_pdl": (c_int, [c_int]),
    "tj_attention_shard_f16": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p,
                                       c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "tj_copy_valid_rows": (c_int, [c_void_p, c_void_p, POINTER(c_int), c_int, c_int, c_size_t, c_void_p]),
    "tj_wait_selftest": (c_int, [c_void_p, c_void_p, c_void_p]),
    "tj_profile_begin": (c_int, [c_void_p, c_int]),
    "tj_profile_end": (c_int, [c_void_p, POINTER(ctypes.c_double), POINTER(ctypes.c_longlong)]),
    "tj_profile_collect": (c_int, [c_void_p, POINTER(ctypes.c_double), POINTER(ctypes.c_longlong)]),
    "tj_launch_count": (c_int, [c_void_p, POINTER(ctypes.c_longlong)]),
    "tj_prepare_mask": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                c_void_p]),
    "tj_layernorm": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_void_p, c_int,
                             c_void_p, c_void_p, c_void_p, c_void_p]),
    "tj_gemm_f16": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                            c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                            c_void_p]),
    "tj_nccl_unique_id": (c_int, [c_void_p]),
    "tj_comm_create": (c_int, [c_void_p, c_int, c_int, c_int, POINTER(c_void_p)]),
    "tj_comm_destroy": (c_int, [c_void_p]),
    "tj_workspace_bytes_seqshard": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, POINTER(c_size_t)]),
    "tj_seqshard_route": (c_int, [c_void_p, c_int, POINTER(c_int)]),
    "tj_forward_seqshard": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p,
                                    c_size_t, c_void_p]),
    "tj_poly_workspace_bytes": (c_int, [c_int, c_int, c_int, c_int, POINTER(c_size_t)]),
    "tj_poly_attention_f16": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                      c_void_p, c_size_t, c_void_p, c_void_p]),
    "tj_attention_f16": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                                 c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
}

_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load ``libtj.so`` once; raise if it has not been built."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m techjam_b200.build` "
                                   "(techjam_b200 has no CPU fallback)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
        return _lib


def check(status: int) -> None:
    if status != TJ_OK:
        msg = load().tj_last_error()
        raise TjError(status, msg.decode() if msg else "")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))
