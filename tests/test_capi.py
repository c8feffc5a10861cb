"""CPU tests of the C ABI: the library loads, exports every declared symbol,
and rejects bad arguments on the host before any launch (no GPU needed:
validation precedes every CUDA call)."""

import ctypes
import re
from pathlib import Path

import pytest

from conftest import ROOT

HEADERS = sorted((ROOT / "include").glob("*.h"))


def _declared_functions() -> set[str]:
    names = set()
    for h in HEADERS:
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^[ \t]*(?:const[ \t]+)?[A-Za-z_][\w \t\*]*?\b(iq36_\w+)[ \t]*\(", text, re.M):
            # IQ36_HD marks header-only inline helpers (iq36_synth.h), not symbols.
            if "IQ36_HD" in m.group(0) or m.group(0).strip().startswith("return"):
                continue
            names.add(m.group(1))
    return names


@pytest.fixture(scope="module")
def native():
    from engine import _native
    return _native


def test_headers_declare_api():
    names = _declared_functions()
    assert "iq36_u4_gemv" in names and "iq36_paged_gqa_decode" in names
    assert "iq36_moe_prefill" in names and "iq36_router_select" in names


def test_library_exports_every_declared_symbol(native):
    lib = native.lib()
    missing = [n for n in sorted(_declared_functions()) if not hasattr(lib, n)]
    assert not missing, f"symbols declared in include/*.h but not exported: {missing}"
    assert set(native.exported_symbols()) >= _declared_functions()


def test_library_is_sm100a_only(native):
    # The version string names the single compiled target.
    assert b"sm_100a" in native.lib().iq36_version()


def _status(native, name, *args):
    return getattr(native.lib(), name)(*args)


def test_u4_gemv_rejects_bad_shapes_on_host(native):
    m = native.U4Matrix(16, 16, 16, 64)  # fake non-null, 16-aligned pointers
    # group 96 unsupported
    assert _status(native, "iq36_u4_gemv", 16, 2048, 96, ctypes.byref(m), 16, 0, None) == -2
    # K not a multiple of G
    assert _status(native, "iq36_u4_gemv", 16, 2000, 128, ctypes.byref(m), 16, 0, None) == -2
    # null x
    assert _status(native, "iq36_u4_gemv", None, 2048, 128, ctypes.byref(m), 16, 0, None) == -1
    # misaligned weight
    m2 = native.U4Matrix(17, 16, 16, 64)
    assert _status(native, "iq36_u4_gemv", 16, 2048, 128, ctypes.byref(m2), 16, 0, None) == -3
    # accumulate into fp16 is not allowed
    p = native.U4Projection(m, 16, native.F16, 1)
    assert _status(native, "iq36_u4_gemv_multi", 16, None, None, 0.0, 2048, 128, 1,
                   ctypes.byref(p), None) == -1
    # arity 5
    arr = (native.U4Projection * 5)()
    assert _status(native, "iq36_u4_gemv_multi", 16, None, None, 0.0, 2048, 128, 5, arr,
                   None) == -1


def test_router_select_rejects_bad_k(native):
    assert _status(native, "iq36_router_select", 16, 1, 256, 0, 16, 16, None) == -2
    assert _status(native, "iq36_router_select", 16, 1, 256, 17, 16, 16, None) == -2
    assert _status(native, "iq36_router_select", 16, 1, 512, 8, 16, 16, None) == -2


def test_paged_gqa_rejects_bad_shapes(native):
    ws = native.lib().iq36_paged_gqa_workspace_bytes(4096, 16, 2, 256)
    assert ws > 0
    # head_dim 128 unsupported; GQA ratio must be 8; workspace too small
    args = [16, 16, 16, 16, 4096, None, 16, 2, 128, 16, 0.0625, None, 16, 0, 256, ws, None]
    assert _status(native, "iq36_paged_gqa_decode", *args) == -2
    args[8] = 256
    args[6] = 12
    assert _status(native, "iq36_paged_gqa_decode", *args) == -2
    args[6] = 16
    args[15] = 8
    assert _status(native, "iq36_paged_gqa_decode", *args) == -4


def test_moe_decode_rejects_bad_bank(native):
    bank = native.ExpertBankC(16, 16, 16, 16, 16, 16, 256, 2048, 500, 128)  # I % G != 0
    assert _status(native, "iq36_moe_decode", 16, None, None, 0.0, 16, 16, 8, ctypes.byref(bank),
                   None, None, 16, 1, 0, 256, 1 << 20, None) == -2
    bank = native.ExpertBankC(16, 16, 16, 16, 16, 16, 256, 2048, 512, 128)
    assert _status(native, "iq36_moe_decode", 16, None, None, 0.0, 16, 16, 8, ctypes.byref(bank),
                   None, None, 16, 1, 0, 256, 8, None) == -4
    # fp32 input without a norm weight
    assert _status(native, "iq36_moe_decode", None, 16, None, 0.0, 16, 16, 8, ctypes.byref(bank),
                   None, None, 16, 1, 0, 256, 1 << 20, None) == -1


def test_status_strings(native):
    for st in range(-7, 1):
        assert native.lib().iq36_status_string(st)


def test_synth_spec_matches_oracle_header():
    from engine import _native as n
    kind, lo, hi = ctypes.c_int32(), ctypes.c_float(), ctypes.c_float()
    n.lib().iq36_synth_tensor_spec(1, 0, ctypes.byref(kind), ctypes.byref(lo), ctypes.byref(hi))
    assert kind.value == 2 and abs(lo.value - 1.0) < 1e-7
    assert n.lib().iq36_synth_tensor_id(-1, 2, 1) == (2 << 4) | 1
    assert n.lib().iq36_synth_tensor_id(3, 27, 0) == (4 << 16) | (27 << 4)


def test_prompt_path_entries_reject_bad_arguments_on_host(native):
    lib = native.lib()
    # DeltaNet over a prompt: head_dim 64 unsupported, nv % nk != 0, workspace too small
    ws = lib.iq36_delta_prefill_workspace_bytes(64, 16, 32)
    assert ws > 0 and lib.iq36_delta_prefill_workspace_bytes(0, 16, 32) == 0
    base = [16, 64, 16, 32, 128, 16, 16, 16, 16, 256, 16, 16, 16, 16, 16, 1e-6, 16, 256, ws, None]
    bad = list(base)
    bad[4] = 64
    assert _status(native, "iq36_delta_prefill", *bad) == -2
    bad = list(base)
    bad[2] = 12
    assert _status(native, "iq36_delta_prefill", *bad) == -2
    bad = list(base)
    bad[18] = ws - 1
    assert _status(native, "iq36_delta_prefill", *bad) == -4
    bad = list(base)
    bad[0] = None
    assert _status(native, "iq36_delta_prefill", *bad) == -1
    # prompt attention: 12 query heads over 2 KV heads (group must be 8); bad dtype
    args = [16, 16, 16, 16, 16, 64, 16, 64, 12, 2, 256, 0.0625, None, 16, 1, None]
    assert _status(native, "iq36_attn_prefill", *args) == -2
    args[8], args[14] = 16, 7
    assert _status(native, "iq36_attn_prefill", *args) == -1
    # batched attention pre-step: zero tokens
    assert _status(native, "iq36_attn_prep_batch", 16, 16, 16, 16, 16, 1e-6, 16, 0, 16, 2, 256,
                   64, 1e7, 16, 16, 16, 16, 16, 16, None) == -2
    # MoE layer over a prompt: null residual; workspace query
    assert lib.iq36_moe_layer_prefill_workspace_bytes(4096, 8, 256, 2048, 512) > 0
    assert lib.iq36_moe_layer_prefill_workspace_bytes(0, 8, 256, 2048, 512) == 0
    bank = native.ExpertBankC(16, 16, 16, 16, 16, 16, 256, 2048, 512, 128)
    assert _status(native, "iq36_moe_layer_prefill", None, 64, 2048, 16, 1e-6, 16, 16, 8,
                   ctypes.byref(bank), None, 16, 16, 16, 256, 1 << 30, None) == -1
    # expert-parallel owner side: null rows; no assignments is a no-op; rows missing
    assert _status(native, "iq36_moe_prefill_rows", None, 4, 8, 16, 16, 16, ctypes.byref(bank),
                   16, 16, 1 << 30, None) == -1
    assert _status(native, "iq36_moe_prefill_rows", 16, 4, 0, 16, 16, 16, ctypes.byref(bank),
                   16, 16, 1 << 30, None) == 0
    assert _status(native, "iq36_moe_prefill_rows", 16, 0, 8, 16, 16, 16, ctypes.byref(bank),
                   16, 16, 1 << 30, None) == -2
    assert lib.iq36_moe_prefill_rows_workspace_bytes(4096, 128, 2048, 512) > 0
    # embedding rows: T out of range
    assert _status(native, "iq36_embed_batch", 16, 1000, 2048, 16, 0, 16, None) == -2
