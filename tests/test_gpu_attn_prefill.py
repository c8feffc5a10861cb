"""Batched attention pre-step and causal prompt attention against the oracle.

The oracle is the per-token path: oracle.attn_prep at each prompt position,
and oracle.paged_gqa (the decode attention) for each prompt token over the
context up to and including its own position. Cases: a prompt into an empty
cache, a prompt appended after 1000 cached tokens, a single token, ragged
16-token tiles, and a sample of rows of a 2048-token prompt. Tolerance:
tests/helpers.py (max rel 2e-3), 1e-3 for the roped q/k as in the decode test.
"""

import numpy as np
import pytest

from helpers import assert_close
from oracle import oracle

pytestmark = pytest.mark.gpu


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def test_attn_prep_batch_matches_per_token_oracle(cuda):
    import torch
    from engine.ops import attn_prep_batch
    rng = np.random.default_rng(21)
    T, p0, nq, nkv = 37, 5, 16, 2
    qf = rng.standard_normal((T, 2 * nq * 256)).astype(np.float16)
    k = rng.standard_normal((T, nkv * 256)).astype(np.float16)
    v = rng.standard_normal((T, nkv * 256)).astype(np.float16)
    qn = rng.uniform(0.9, 1.1, 256).astype(np.float32)
    kn = rng.uniform(0.9, 1.1, 256).astype(np.float32)
    nblk = 8
    bt = rng.permutation(nblk).astype(np.int32)
    kc = torch.zeros((nblk, 16, nkv, 256), dtype=torch.float16, device=cuda)
    vc = torch.zeros_like(kc)
    qo = torch.empty((T, nq * 256), dtype=torch.float16, device=cuda)
    go = torch.empty_like(qo)
    attn_prep_batch(_t(qf, cuda), _t(k, cuda), _t(v, cuda), _t(qn, cuda), _t(kn, cuda), 1e-6,
                    torch.tensor([p0], dtype=torch.int32, device=cuda), _t(bt, cuda), kc, vc, qo,
                    go)
    qo_h, go_h = qo.float().cpu().numpy(), go.float().cpu().numpy()
    kc_h, vc_h = kc.float().cpu().numpy(), vc.float().cpu().numpy()
    for t in range(T):
        pos = p0 + t
        rq, rg, rk, rv = oracle.attn_prep(qf[t], k[t], v[t], qn, kn, 1e-6, pos)
        assert_close(qo_h[t], rq, f"q t={t}", max_rel=1e-3)
        np.testing.assert_array_equal(go_h[t], rg)
        blk = bt[pos // 16]
        assert_close(kc_h[blk, pos % 16].ravel(), rk, f"k t={t}", max_rel=1e-3)
        np.testing.assert_array_equal(vc_h[blk, pos % 16].ravel(), rv)


def _prefill_case(rng, p0, T, extra_blocks=2):
    ctx = p0 + T
    nblk = (ctx + 15) // 16 + extra_blocks
    q = rng.standard_normal((T, 16, 256)).astype(np.float16)
    kc = rng.standard_normal((nblk, 16, 2, 256)).astype(np.float16)
    vc = rng.standard_normal((nblk, 16, 2, 256)).astype(np.float16)
    bt = rng.permutation(nblk).astype(np.int32)
    gate = rng.standard_normal((T, 16, 256)).astype(np.float16)
    return q, kc, vc, bt, gate


@pytest.mark.parametrize("p0,T,out_f16", [(0, 1, True), (0, 100, True), (1000, 45, False),
                                          (0, 257, True)])
def test_attn_prefill_matches_per_token_decode_oracle(cuda, p0, T, out_f16):
    import torch
    from engine.ops import attn_prefill
    rng = np.random.default_rng(p0 * 13 + T)
    q, kc, vc, bt, gate = _prefill_case(rng, p0, T)
    out = attn_prefill(_t(q, cuda), _t(kc, cuda), _t(vc, cuda), _t(bt, cuda),
                       torch.tensor([p0], dtype=torch.int32, device=cuda), 1 / 16,
                       gate=_t(gate, cuda),
                       out_dtype=torch.float16 if out_f16 else torch.float32)
    got = out.float().cpu().numpy()
    for t in range(T):
        ref = oracle.paged_gqa(q[t], kc, vc, bt, p0 + t + 1, 1 / 16, gate[t])
        assert_close(got[t], ref, f"prefill attention t={t}")


def test_attn_prefill_long_prompt_sampled_rows(cuda):
    import torch
    from engine.ops import attn_prefill
    rng = np.random.default_rng(99)
    T = 2048
    q, kc, vc, bt, _ = _prefill_case(rng, 0, T)
    out = attn_prefill(_t(q, cuda), _t(kc, cuda), _t(vc, cuda), _t(bt, cuda),
                       torch.zeros(1, dtype=torch.int32, device=cuda), 1 / 16, gate=None,
                       out_dtype=torch.float32)
    got = out.cpu().numpy()
    for t in (0, 15, 16, 63, 64, 1000, 2031, 2047):
        ref = oracle.paged_gqa(q[t], kc, vc, bt, t + 1, 1 / 16, None)
        assert_close(got[t], ref, f"prefill attention t={t}")


def test_attn_prefill_rejects_bad_group(cuda):
    import torch
    from engine import _native as N
    from engine.ops import attn_prefill
    q = torch.zeros((4, 12, 256), dtype=torch.float16, device=cuda)  # 12 q heads, 2 kv heads
    kc = torch.zeros((2, 16, 2, 256), dtype=torch.float16, device=cuda)
    bt = torch.arange(2, dtype=torch.int32, device=cuda)
    with pytest.raises(N.Iq36Error):
        attn_prefill(q, kc, kc, bt, torch.zeros(1, dtype=torch.int32, device=cuda), 1 / 16)
