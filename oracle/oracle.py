"""numpy/ctypes front end of the CPU checker.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / reference arm, never by the product package.

``port()`` loads the CPU restatement (oracle/_build/liboracle_port.so, built
by oracle/Makefile on first use); ``ref()`` loads the reference's own CPU
functions compiled from the reference checkout (oracle/_ref/libiq36_ref.so),
or returns None where that library was not built.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import POINTER, Structure, c_float, c_int, c_int32, c_int64, c_uint64, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_LIB = HERE / "_build" / "liboracle_port.so"
REF_LIB = HERE / "_ref" / "libiq36_ref.so"

_port = None
_ref = None


def build(ref: bool = True) -> None:
    """Build the restatement (always) and the reference library (when the
    reference checkout is present)."""
    targets = ["port"]
    if ref and Path(os.environ.get("IQ36_REFERENCE", "/root/reference")).exists():
        targets.append("ref")
    env = dict(os.environ)
    if "IQ36_REFERENCE" in env:
        env["REF"] = env["IQ36_REFERENCE"]
    subprocess.run(["make", "-s", *targets], cwd=HERE, check=True, env=env)


class ModelConfig(Structure):
    _fields_ = [(n, c_int32) for n in (
        "hidden", "layers", "attn_interval", "nq", "nkv", "head_dim", "rope_dim", "nk", "nv",
        "dk", "conv", "experts", "topk", "inter", "shared_inter", "vocab", "group")] + [
        ("rope_base", c_float), ("eps", c_float), ("fc_group", c_int32)]


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "arrays passed to the oracle must be contiguous"
    return a.ctypes.data_as(c_void_p)


def port() -> ctypes.CDLL:
    global _port
    if _port is None:
        if not PORT_LIB.exists():
            build(ref=False)
        lib = ctypes.CDLL(str(PORT_LIB))
        lib.orc_model_create.restype = c_void_p
        lib.orc_model_create.argtypes = [POINTER(ModelConfig), c_uint64, c_int]
        lib.orc_model_destroy.argtypes = [c_void_p]
        lib.orc_model_step.argtypes = [c_void_p, c_int, c_int, c_void_p, c_int]
        lib.orc_model_step.restype = c_int
        lib.orc_model_feed.argtypes = [c_void_p, c_int, c_int, c_int]
        lib.orc_model_feed.restype = c_int
        lib.orc_model_step_trace.argtypes = [c_void_p, c_int, c_int, c_void_p, c_int, c_void_p,
                                             c_void_p, c_void_p]
        lib.orc_model_step_trace.restype = c_int
        lib.orc_synth_fill.argtypes = [c_void_p, c_int64, c_int, c_uint64, c_uint64, c_float,
                                       c_float]
        lib.orc_argmax.restype = c_int
        lib.orc_argmax.argtypes = [c_void_p, c_int64]
        _port = lib
    return _port


def ref() -> ctypes.CDLL | None:
    global _ref
    if _ref is None and REF_LIB.exists():
        lib = ctypes.CDLL(str(REF_LIB))
        lib.ref_sigmoid_scalar.restype = c_float
        lib.ref_sigmoid_scalar.argtypes = [c_float]
        _ref = lib
    return _ref


# ---------------------------------------------------------------------------
# fp16 helpers (numpy float16 is IEEE binary16 with round-to-nearest-even)

def f16_bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a.astype(np.float16)).view(np.uint16)


def bf16_bits(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a.astype(np.float32)).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------
# restated ops (port)

def synth_fill(count: int, kind: int, seed: int, tensor: int, lo: float, hi: float = 0.0):
    dt = {0: np.uint8, 1: np.uint16, 2: np.uint16, 3: np.float32, 4: np.float32}[kind]
    out = np.empty(count, dtype=dt)
    port().orc_synth_fill(_p(out), count, kind, c_uint64(seed), c_uint64(tensor), lo, hi)
    return out


def u4_gemv(x_f16: np.ndarray, w: np.ndarray, scale: np.ndarray, zp: np.ndarray, group: int,
            precise: bool = True, threads: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x_f16.astype(np.float16)).view(np.uint16)
    n, k = w.shape[0], w.shape[1] * 2
    out = np.empty(n, dtype=np.float32)
    port().orc_u4_gemv(_p(x), c_int(k), c_int(group), _p(np.ascontiguousarray(w)),
                       _p(np.ascontiguousarray(scale.view(np.uint16))),
                       _p(np.ascontiguousarray(zp)), c_int64(n), _p(out), c_int(int(precise)),
                       c_int(threads))
    return out


def lm_head_top1_certified(x_f16: np.ndarray, w: np.ndarray, scale: np.ndarray, zp: np.ndarray,
                           seed_token: int, capacity_chunks: int, group: int = 128):
    """Certified greedy top-1 of a u4 LM head, restated in fp64 (numpy).

    Follows the reference's certificate (engine/gpu/opencl/
    iq36_lm_head_affine_q4_group128_component.cl:126-217: a per-row upper
    bound sum_g |s_g| ||q_g - zp_g||_2 ||x_g||_2 compared against the seed's
    exact value, rows at or above it become candidates; :219-300: candidates
    evaluated exactly, the top-1 taken with the lowest id on ties; the full
    head when the candidates overflow the capacity), at the granularity of
    16-row chunks: the seed is the largest logit of seed_token's chunk.
    Returns (token, evaluated_chunks, fp64 logits of every row)."""
    rows, k = w.shape[0], w.shape[1] * 2
    ng = k // group
    q = np.empty((rows, k), np.float64)
    q[:, 0::2] = w & 15
    q[:, 1::2] = w >> 4
    zz = np.empty(zp.size * 2, np.float64)
    zz[0::2] = zp & 15
    zz[1::2] = zp >> 4
    d = q.reshape(rows, ng, group) - zz.reshape(rows, ng)[:, :, None]
    x = x_f16.astype(np.float64).reshape(ng, group)
    sc = scale.astype(np.float64)
    logits = (np.einsum("rgk,gk->rg", d, x) * sc).sum(axis=1)
    upper = (np.abs(sc) * np.sqrt((d * d).sum(axis=2)) * np.sqrt((x * x).sum(axis=1))).sum(axis=1)
    nchunks = rows // 16
    seed_chunk = min(max(seed_token, 0), rows - 1) // 16
    seed = logits[seed_chunk * 16:seed_chunk * 16 + 16].max()
    flagged = np.unique(np.nonzero(upper >= seed)[0] // 16)
    chunks = flagged if flagged.size <= capacity_chunks else np.arange(nchunks)
    cand = (chunks[:, None] * 16 + np.arange(16)[None, :]).reshape(-1)
    best = cand[np.argmax(logits[cand])]  # first maximum = lowest id among sorted candidates
    return int(best), int(chunks.size), logits


def f16_linear(x_f16: np.ndarray, w_f16: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x_f16.astype(np.float16)).view(np.uint16)
    e, h = w_f16.shape
    out = np.empty(e, dtype=np.float32)
    port().orc_f16_linear(_p(x), c_int(h), _p(np.ascontiguousarray(w_f16).view(np.uint16)),
                          c_int(e), _p(out))
    return out


def router_select(logits: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    l2 = np.ascontiguousarray(logits.reshape(-1, logits.shape[-1]).astype(np.float32))
    t, e = l2.shape
    ids = np.empty((t, k), dtype=np.int32)
    wts = np.empty((t, k), dtype=np.float32)
    port().orc_router_select(_p(l2), c_int(t), c_int(e), c_int(k), _p(ids), _p(wts))
    return ids, wts


def swiglu(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(gate, dtype=np.float32)
    u = np.ascontiguousarray(up, dtype=np.float32)
    out = np.empty_like(g)
    port().orc_swiglu(_p(g), _p(u), c_int64(g.size), _p(out))
    return out


def moe_decode(x_f16, ids, weights, bank: dict, shared: dict | None, shared_logit, group,
               precise=True, threads=0) -> np.ndarray:
    """bank/shared: dicts of numpy arrays gu_w, gu_s, gu_z, d_w, d_s, d_z."""
    x = np.ascontiguousarray(x_f16.astype(np.float16)).view(np.uint16)
    h = x.size
    i = bank["gu_w"].shape[1] // 2
    out = np.empty(h, dtype=np.float32)
    sl = np.array([shared_logit if shared_logit is not None else 0.0], dtype=np.float32)
    s = shared or {}

    def arr(d, key, view=None):
        if key not in d:
            return None
        a = np.ascontiguousarray(d[key])
        return _p(a.view(np.uint16) if view else a)

    ids32 = np.ascontiguousarray(ids, dtype=np.int32)
    w32 = np.ascontiguousarray(weights, dtype=np.float32)
    port().orc_moe_decode(
        _p(x), _p(ids32), _p(w32), c_int(ids32.size), arr(bank, "gu_w"), arr(bank, "gu_s", 1),
        arr(bank, "gu_z"), arr(bank, "d_w"), arr(bank, "d_s", 1), arr(bank, "d_z"),
        arr(s, "gu_w"), arr(s, "gu_s", 1), arr(s, "gu_z"), arr(s, "d_w"), arr(s, "d_s", 1),
        arr(s, "d_z"), _p(sl), c_int(h), c_int(i), c_int(group), _p(out), c_int(int(precise)),
        c_int(threads))
    return out


def paged_gqa(q_f16, k_cache_f16, v_cache_f16, block_table, ctx, scale, gate_f16=None,
              threads=0) -> np.ndarray:
    q = np.ascontiguousarray(q_f16.astype(np.float16)).view(np.uint16)
    kc = np.ascontiguousarray(k_cache_f16.astype(np.float16)).view(np.uint16)
    vc = np.ascontiguousarray(v_cache_f16.astype(np.float16)).view(np.uint16)
    nq, d = q_f16.shape
    bs, nkv = k_cache_f16.shape[1], k_cache_f16.shape[2]
    bt = np.ascontiguousarray(block_table, dtype=np.int32)
    g = None if gate_f16 is None else np.ascontiguousarray(gate_f16.astype(np.float16)).view(np.uint16)
    out = np.empty((nq, d), dtype=np.float32)
    port().orc_paged_gqa(_p(q), _p(kc), _p(vc), _p(bt), c_int(ctx), c_int(nq), c_int(nkv),
                         c_int(d), c_int(bs), c_float(scale), _p(g), _p(out), c_int(threads))
    return out


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x2 = np.ascontiguousarray(x.reshape(-1, x.shape[-1]), dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty_like(x2)
    port().orc_rms_norm(_p(x2), c_int(x2.shape[0]), c_int(x2.shape[1]), _p(w), c_int(w.size),
                        c_float(eps), _p(out))
    return out.reshape(x.shape)


def attn_prep(q_full_f16, k_f16, v_f16, qn_w, kn_w, eps, pos, rope_dim=64, base=1e7):
    nq = q_full_f16.size // 512
    nkv = k_f16.size // 256
    d = 256
    qo = np.empty(nq * d, np.float32)
    go = np.empty(nq * d, np.float32)
    kn = np.empty(nkv * d, np.float32)
    vn = np.empty(nkv * d, np.float32)
    port().orc_attn_prep(_p(f16_bits(q_full_f16.ravel())), _p(f16_bits(k_f16.ravel())),
                         _p(f16_bits(v_f16.ravel())), _p(np.ascontiguousarray(qn_w, np.float32)),
                         _p(np.ascontiguousarray(kn_w, np.float32)), c_float(eps), c_int(pos),
                         c_int(nq), c_int(nkv), c_int(d), c_int(rope_dim), c_float(base),
                         _p(qo), _p(go), _p(kn), _p(vn))
    return qo, go, kn, vn


def delta_prep(qkv_f16, conv_state, conv_w, a_f16, b_f16, a_log, dt_bias):
    c = qkv_f16.size
    nv = a_log.size
    st = np.ascontiguousarray(conv_state, dtype=np.float32).copy()
    act = np.empty(c, np.float32)
    g = np.empty(nv, np.float32)
    beta = np.empty(nv, np.float32)
    port().orc_delta_prep(_p(f16_bits(qkv_f16.ravel())), c_int(c), _p(st),
                          _p(np.ascontiguousarray(conv_w, np.float32)), _p(f16_bits(a_f16)),
                          _p(f16_bits(b_f16)), _p(np.ascontiguousarray(a_log, np.float32)),
                          _p(np.ascontiguousarray(dt_bias, np.float32)), c_int(nv), _p(act),
                          _p(g), _p(beta))
    return act, g, beta, st


def delta_step(act, g, beta, state, z_f16, norm_w, eps, nk, nv, d=128):
    st = np.ascontiguousarray(state, dtype=np.float32).copy()
    out = np.empty(nv * d, np.float32)
    port().orc_delta_step(_p(np.ascontiguousarray(act, np.float32)),
                          _p(np.ascontiguousarray(g, np.float32)),
                          _p(np.ascontiguousarray(beta, np.float32)), _p(st),
                          _p(f16_bits(z_f16.ravel())), _p(np.ascontiguousarray(norm_w, np.float32)),
                          c_float(eps), c_int(nk), c_int(nv), c_int(d), _p(out))
    return out, st


def moe_prefill(x_bf16_bits, tokens, ids, weights, bank: dict, group, threads=0) -> np.ndarray:
    t, h = x_bf16_bits.shape
    k = ids.shape[1]
    i = bank["gu_w"].shape[1] // 2
    toks = np.ascontiguousarray(tokens, dtype=np.int32)
    out = np.empty((toks.size, h), np.float32)
    port().orc_moe_prefill(
        _p(np.ascontiguousarray(x_bf16_bits, np.uint16)), _p(toks), c_int(toks.size), c_int(h),
        _p(np.ascontiguousarray(ids, np.int32)), _p(np.ascontiguousarray(weights, np.float32)),
        c_int(k), _p(np.ascontiguousarray(bank["gu_w"])),
        _p(np.ascontiguousarray(bank["gu_s"]).view(np.uint16)),
        _p(np.ascontiguousarray(bank["gu_z"])), _p(np.ascontiguousarray(bank["d_w"])),
        _p(np.ascontiguousarray(bank["d_s"]).view(np.uint16)),
        _p(np.ascontiguousarray(bank["d_z"])), c_int(i), c_int(group), _p(out), c_int(threads))
    return out


class OracleModel:
    """CPU restatement of the synthetic config-4 model (weights regenerated
    from the shared generator)."""

    def __init__(self, cfg: dict, seed: int, max_ctx: int):
        self.cfg = ModelConfig(**cfg)
        self.vocab = cfg["vocab"]
        self.h = port().orc_model_create(ctypes.byref(self.cfg), c_uint64(seed), max_ctx)

    def step(self, token: int, pos: int, want_logits: bool = True, threads: int = 0):
        logits = np.empty(self.vocab, np.float32) if want_logits else None
        tok = port().orc_model_step(self.h, token, pos, _p(logits), threads)
        return tok, logits

    def step_trace(self, token: int, pos: int, threads: int = 0):
        """step() plus its trace: the fp32 residual entering every layer and
        leaving the last ([layers + 1, hidden]), the routed ids [layers, topk]
        and the router logits [layers, experts]."""
        c = self.cfg
        logits = np.empty(self.vocab, np.float32)
        hidden = np.empty((c.layers + 1, c.hidden), np.float32)
        ids = np.empty((c.layers, c.topk), np.int32)
        router = np.empty((c.layers, c.experts), np.float32)
        tok = port().orc_model_step_trace(self.h, token, pos, _p(logits), threads, _p(hidden),
                                          _p(ids), _p(router))
        return tok, logits, hidden, ids, router

    def feed(self, token: int, pos: int, threads: int = 0) -> None:
        """A step without the LM head (a prompt token whose logits are not needed)."""
        port().orc_model_feed(self.h, token, pos, threads)

    def close(self):
        if self.h:
            port().orc_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
