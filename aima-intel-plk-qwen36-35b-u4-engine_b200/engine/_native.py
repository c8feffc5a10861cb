"""ctypes binding to ``libiq36_b200.so`` (C ABI declared in include/iq36_b200.h).

The library is the only compute path: if it is missing or fails to load, every
op raises. There is no CPU or PyTorch fallback.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, Structure, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t
from ctypes import c_uint64, c_void_p
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parents[1]
LIB_PATH = PKG_DIR / "libiq36_b200.so"

F32, F16, BF16 = 0, 1, 2


class Iq36Error(RuntimeError):
    """A C-ABI entry point returned a non-zero status."""

    def __init__(self, name: str, status: int, text: str):
        super().__init__(f"{name} failed with status {status}: {text}")
        self.status = status


class U4Matrix(Structure):
    _fields_ = [("weight", c_void_p), ("scale", c_void_p), ("zp", c_void_p), ("rows", c_int32)]


class U4Projection(Structure):
    _fields_ = [("m", U4Matrix), ("out", c_void_p), ("out_dtype", c_int32),
                ("accumulate", c_int32)]


class ExpertBankC(Structure):
    _fields_ = [("gate_up_weight", c_void_p), ("gate_up_scale", c_void_p),
                ("gate_up_zp", c_void_p), ("down_weight", c_void_p),
                ("down_scale", c_void_p), ("down_zp", c_void_p), ("num_experts", c_int32),
                ("hidden", c_int32), ("intermediate", c_int32), ("group", c_int32)]


class TpCommC(Structure):
    """iq36_tp_comm: every rank's exchange buffers as mapped in this process."""
    _fields_ = [("rank", c_int32), ("world", c_int32), ("hidden", c_int32),
                ("peer_recv", c_void_p * 8), ("peer_flags", c_void_p * 8),
                ("peer_keys", c_void_p * 8), ("local_recv", c_void_p),
                ("local_flags", c_void_p), ("local_keys", c_void_p), ("counter", c_void_p)]


# name -> (restype, argtypes)
_P = c_void_p
_SIGS: dict[str, tuple] = {
    "iq36_version": (c_char_p, []),
    "iq36_status_string": (c_char_p, [c_int]),
    "iq36_set_pdl": (None, [c_int]),
    "iq36_wait_timeouts": (c_int, [POINTER(c_int32), c_int32]),
    "iq36_u4_gemv": (c_int, [_P, c_int32, c_int32, POINTER(U4Matrix), _P, c_int32, _P]),
    "iq36_u4_gemv_multi": (c_int, [_P, _P, _P, c_float, c_int32, c_int32, c_int32,
                                   POINTER(U4Projection), _P]),
    "iq36_router_logits": (c_int, [_P, _P, _P, c_float, c_int32, c_int32, _P, c_int32, _P, _P,
                                   _P, _P]),
    "iq36_router_select": (c_int, [_P, c_int32, c_int32, c_int32, _P, _P, _P]),
    "iq36_moe_decode": (c_int, [_P, _P, _P, c_float, _P, _P, c_int32, POINTER(ExpertBankC),
                                POINTER(ExpertBankC), _P, _P, c_int32, c_int32, _P, c_size_t, _P]),
    "iq36_moe_decode_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32]),
    "iq36_moe_decode_sharded": (c_int, [_P, _P, _P, c_float, _P, _P, c_int32,
                                        POINTER(ExpertBankC), c_int32, POINTER(ExpertBankC), _P,
                                        _P, c_int32, c_int32, _P, c_size_t, _P]),
    "iq36_moe_block_decode": (c_int, [_P, _P, _P, c_int32, POINTER(ExpertBankC),
                                      POINTER(ExpertBankC), _P, _P, _P, _P, c_int32, _P,
                                      c_size_t, _P]),
    "iq36_moe_block_decode_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32]),
    "iq36_moe_layer_decode": (c_int, [_P, c_int32, _P, c_float, _P, _P, c_int32,
                                      POINTER(ExpertBankC), POINTER(ExpertBankC), _P, _P, _P, _P,
                                      _P, c_size_t, _P]),
    "iq36_moe_layer_decode_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32]),
    "iq36_moe_layer_decode_partial": (c_int, [_P, c_int32, _P, c_float, _P, _P, c_int32,
                                              POINTER(ExpertBankC), POINTER(ExpertBankC), _P, _P,
                                              _P, _P, _P, _P, c_size_t, _P]),
    "iq36_tp_comm_bytes": (c_size_t, [c_int32, c_int32]),
    "iq36_tp_comm_alloc": (c_int, [c_size_t, POINTER(c_void_p)]),
    "iq36_tp_comm_free": (c_int, [_P]),
    "iq36_ipc_get_handle": (c_int, [_P, _P]),
    "iq36_ipc_open_handle": (c_int, [_P, POINTER(c_void_p)]),
    "iq36_ipc_close_handle": (c_int, [_P]),
    "iq36_tp_allreduce_residual": (c_int, [POINTER(TpCommC), _P, _P, _P]),
    "iq36_tp_argmax": (c_int, [POINTER(TpCommC), _P, c_int32, c_int32, _P, _P, _P]),
    "iq36_tp_argmax_workspace_bytes": (c_size_t, []),
    "iq36_lm_head_cert_table_bytes": (c_size_t, [c_int32, c_int32, c_int32]),
    "iq36_lm_head_cert_table": (c_int, [POINTER(U4Matrix), c_int32, c_int32, _P, _P]),
    "iq36_lm_head_top1_certified_workspace_bytes": (c_size_t, [c_int32, c_int32]),
    "iq36_lm_head_top1_certified": (c_int, [_P, _P, _P, c_float, c_int32, c_int32,
                                            POINTER(U4Matrix), _P, _P, c_int32, _P, _P, _P, _P,
                                            c_size_t, _P]),
    "iq36_moe_prefill": (c_int, [_P, c_int32, _P, _P, c_int32, POINTER(ExpertBankC), _P, c_int32,
                                 _P, c_size_t, _P]),
    "iq36_moe_layer_prefill": (c_int, [_P, c_int32, c_int32, _P, c_float, _P, _P, c_int32,
                                       POINTER(ExpertBankC), POINTER(ExpertBankC), _P, _P, _P,
                                       _P, c_size_t, _P]),
    "iq36_moe_layer_prefill_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32, c_int32,
                                                          c_int32]),
    "iq36_u4_gemm": (c_int, [_P, c_int32, _P, c_float, c_int32, c_int32, c_int32,
                             POINTER(U4Matrix), _P, c_int32, c_int32, _P, c_size_t, _P]),
    "iq36_u4_gemm_workspace_bytes": (c_size_t, [c_int32, c_int32]),
    "iq36_u4_gemm_multi": (c_int, [_P, c_int32, _P, c_float, c_int32, c_int32, c_int32, c_int32,
                                   POINTER(U4Projection), _P, c_size_t, _P]),
    "iq36_moe_combine": (c_int, [_P, _P, c_int32, c_int32, c_int32, _P, c_int32, _P]),
    "iq36_moe_prefill_rows": (c_int, [_P, c_int32, c_int32, _P, _P, _P, POINTER(ExpertBankC),
                                      _P, _P, c_size_t, _P]),
    "iq36_moe_prefill_rows_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32, c_int32]),
    "iq36_moe_prefill_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32, c_int32,
                                                    c_int32]),
    "iq36_paged_gqa_decode": (c_int, [_P, _P, _P, _P, c_int32, _P, c_int32, c_int32, c_int32,
                                      c_int32, c_float, _P, _P, c_int32, _P, c_size_t, _P]),
    "iq36_paged_gqa_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32, c_int32]),
    "iq36_paged_gqa_decode_noalloc": (c_int, [_P, _P, _P, _P, c_int32, _P, c_int32, c_int32,
                                              c_int32, c_int32, c_float, _P, _P, c_int32, _P]),
    "iq36_rms_norm": (c_int, [_P, c_int32, c_int32, _P, c_int32, c_float, _P, c_int32, _P]),
    "iq36_attn_prep": (c_int, [_P, _P, _P, _P, _P, c_float, _P, c_int32, c_int32, c_int32,
                               c_int32, c_float, _P, c_int32, _P, _P, _P, _P, _P]),
    "iq36_attn_prep_batch": (c_int, [_P, _P, _P, _P, _P, c_float, _P, c_int32, c_int32, c_int32,
                                     c_int32, c_int32, c_float, _P, c_int32, _P, _P, _P, _P, _P]),
    "iq36_attn_prefill": (c_int, [_P, _P, _P, _P, c_int32, c_int32, _P, c_int32, c_int32,
                                  c_int32, c_int32, c_float, _P, _P, c_int32, _P]),
    "iq36_delta_prep": (c_int, [_P, c_int32, _P, _P, _P, _P, _P, _P, c_int32, _P, _P, _P, _P]),
    "iq36_delta_step": (c_int, [_P, _P, _P, _P, _P, _P, c_float, c_int32, c_int32, c_int32, _P,
                                _P]),
    "iq36_delta_prefill": (c_int, [_P, c_int32, c_int32, c_int32, c_int32, _P, _P, _P, _P,
                                   c_int32, _P, _P, _P, _P, _P, c_float, _P, _P, c_size_t, _P]),
    "iq36_delta_prefill_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32]),
    "iq36_embed": (c_int, [_P, c_int32, c_int32, _P, _P, _P]),
    "iq36_embed_batch": (c_int, [_P, c_int32, c_int32, _P, c_int32, _P, _P]),
    "iq36_decode_positions": (c_int, [_P, _P, c_int32, _P]),
    "iq36_argmax": (c_int, [_P, c_int32, _P, _P, c_size_t, _P]),
    "iq36_u4_layout_from_group_major": (c_int, [_P, _P, c_int32, c_int32, _P, _P, _P]),
    "iq36_u4_layout_to_group_major": (c_int, [_P, _P, c_int32, c_int32, _P, _P, _P]),
    "iq36_argmax_workspace_bytes": (c_size_t, []),
    "iq36_synth_fill": (c_int, [_P, c_int64, c_int32, c_uint64, c_uint64, c_float, c_float, _P]),
    "iq36_synth_tensor_id": (c_uint64, [c_int32, c_int32, c_int32]),
    "iq36_synth_tensor_spec": (None, [c_int32, c_int32, POINTER(c_int32), POINTER(c_float),
                                      POINTER(c_float)]),
}

_LIB: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Load the library once (raises if it has not been built)."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python {PKG_DIR / 'build.py'}` "
                "(there is no fallback path)")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = handle
    return _LIB


def call(name: str, *args) -> None:
    """Call an int-returning entry point and raise Iq36Error on failure."""
    st = getattr(lib(), name)(*args)
    if st != 0:
        text = lib().iq36_status_string(st).decode()
        raise Iq36Error(name, st, text)


def wait_timeouts(reset: bool = True) -> int:
    """Bounded device waits that gave up on the current device (see the header)."""
    n = c_int32(0)
    call("iq36_wait_timeouts", ctypes.byref(n), 1 if reset else 0)
    return int(n.value)


def exported_symbols() -> list[str]:
    return list(_SIGS)
