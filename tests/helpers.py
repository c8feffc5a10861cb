"""Seeded synthetic inputs (BASELINE config distributions) and tolerances.

Tolerance for floating-point parity: max relative error
<= 2e-3, read as max|gpu - oracle| / max|oracle| over the output vector, plus
the reference's component gate cosine >= 0.999 and relL2 <= 2e-3
(reference benchmarks/.../acceptance-matrix.json:365-369). Router ids must be
bit-exact.
"""

from __future__ import annotations

import numpy as np

MAX_REL = 2e-3
MIN_COS = 0.999
MAX_RELL2 = 2e-3


def max_rel_err(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def cosine(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / max(np.linalg.norm(a) * np.linalg.norm(b), 1e-300))


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def assert_close(gpu, ref, what: str, max_rel: float = MAX_REL):
    mre, cs, rl = max_rel_err(gpu, ref), cosine(gpu, ref), rel_l2(gpu, ref)
    assert np.all(np.isfinite(np.asarray(gpu, np.float64))), f"{what}: non-finite output"
    assert mre <= max_rel and cs >= MIN_COS and rl <= MAX_RELL2, (
        f"{what}: max_rel={mre:.3e} (<= {max_rel}) cos={cs:.6f} relL2={rl:.3e}")
    return mre


def make_u4(rng: np.random.Generator, rows: int, k: int, group: int = 128):
    """u4 codes uniform 0..15 packed two per byte (low nibble = even k), fp16
    scales uniform [0.005, 0.02], u4 zero points uniform 0..15."""
    ng = k // group
    w = rng.integers(0, 256, size=(rows, k // 2), dtype=np.uint8)
    s = rng.uniform(0.005, 0.02, size=(rows, ng)).astype(np.float16)
    z = rng.integers(0, 256, size=(rows * ng // 2,), dtype=np.uint8)
    return w, s, z


def make_bank(rng, experts: int, hidden: int, inter: int, group: int = 128) -> dict:
    gw, gs, gz = make_u4(rng, experts * 2 * inter, hidden, group)
    dw, ds, dz = make_u4(rng, experts * hidden, inter, group)
    return {
        "gu_w": gw.reshape(experts, 2 * inter, hidden // 2),
        "gu_s": gs.reshape(experts, 2 * inter, hidden // group),
        "gu_z": gz.reshape(experts, -1),
        "d_w": dw.reshape(experts, hidden, inter // 2),
        "d_s": ds.reshape(experts, hidden, inter // group),
        "d_z": dz.reshape(experts, -1),
    }


def zipf_router_logits(rng: np.random.Generator, tokens: int, experts: int = 256,
                       s: float = 1.1, span: float = 2.0) -> np.ndarray:
    """BASELINE config 3 router logits: N(0,1) plus a per-expert bias from a
    Zipf(s) ranking (a seeded permutation assigns ranks), scaled to [-span, span]."""
    ranks = rng.permutation(experts) + 1
    w = ranks.astype(np.float64) ** (-s)
    bias = -span + 2 * span * (w - w.min()) / (w.max() - w.min())
    return (rng.standard_normal((tokens, experts)) + bias[None, :]).astype(np.float32)


def bank_to_torch(bank: dict, device, group: int = 128):
    import torch
    from engine.ops import ExpertBank

    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(device) for k, v in bank.items()}
    return ExpertBank(t["gu_w"], t["gu_s"], t["gu_z"], t["d_w"], t["d_s"], t["d_z"], group)


def u4_to_torch(w, s, z, device, group: int = 128):
    import torch
    from engine.ops import U4Weight

    return U4Weight(torch.from_numpy(w).to(device), torch.from_numpy(s).to(device),
                    torch.from_numpy(z).to(device), group)


def dequant_u4(w, s, z, group: int = 128) -> np.ndarray:
    """Dense fp32 [rows, K] of a u4 matrix (for small reference checks)."""
    rows, kb = w.shape
    k = kb * 2
    q = np.empty((rows, k), np.int32)
    q[:, 0::2] = w & 15
    q[:, 1::2] = w >> 4
    zz = np.empty(z.size * 2, np.int32)
    zz[0::2] = z & 15
    zz[1::2] = z >> 4
    zz = zz.reshape(rows, k // group)
    sc = s.astype(np.float32)
    return ((q.reshape(rows, k // group, group) - zz[:, :, None]) * sc[:, :, None]).reshape(rows, k)
