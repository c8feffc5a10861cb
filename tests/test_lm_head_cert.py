"""Certified greedy top-1 of the LM head (the reference's bound-and-candidate
certificate, engine/gpu/opencl/iq36_lm_head_affine_q4_group128_component.cl:
126-300).

CPU: the oracle's fp64 restatement returns the plain argmax on random heads
(where the bound prunes nothing) and on planted heads (where it prunes all but
a few chunks), ties included. GPU: iq36_lm_head_top1_certified returns the
full head's argmax bit for bit and writes, for every evaluated chunk, the same
logits as the full head; on planted heads it evaluates the oracle's number of
chunks.
"""

import numpy as np
import pytest

from helpers import make_u4
from oracle import oracle


def planted_head(rng, rows, k, x, plants, base_scale=0.01):
    """Random u4 head whose rows `plants` (row -> scale multiplier) carry codes
    8 + 7 sign(x) against zero point 8: logits far above every other row's
    Cauchy-Schwarz bound once the multiplier is large enough."""
    w, s, z = make_u4(rng, rows, k)
    s[:] = np.float16(base_scale)
    ng = k // 128
    code = np.where(x.astype(np.float32) >= 0, 15, 1).astype(np.uint8)
    packed = (code[0::2] | (code[1::2] << 4)).astype(np.uint8)
    zn = np.empty(z.size * 2, np.uint8)
    zn[0::2] = z & 15
    zn[1::2] = z >> 4
    zn = zn.reshape(rows, ng)
    for r, mult in plants.items():
        w[r] = packed
        s[r] = np.float16(base_scale * mult)
        zn[r] = 8
    zf = zn.reshape(-1)
    z = (zf[0::2] | (zf[1::2] << 4)).astype(np.uint8)
    return w, s, z


def _x(rng, k):
    return rng.standard_normal(k).astype(np.float16)


# --------------------------------------------------------------------- CPU


def test_oracle_cert_random_head_is_argmax():
    rng = np.random.default_rng(11)
    for seed_tok in (0, 777, 4095):
        w, s, z = make_u4(rng, 4096, 1024)
        x = _x(rng, 1024)
        tok, ev, logits = oracle.lm_head_top1_certified(x, w, s, z, seed_tok, 64)
        assert tok == int(np.argmax(logits))
        assert ev == 4096 // 16  # random rows: the bound prunes nothing


def test_oracle_cert_planted_prunes_and_agrees():
    rng = np.random.default_rng(12)
    k = 1024
    x = _x(rng, k)
    # one planted winner: only its chunk survives
    w, s, z = planted_head(rng, 4096, k, x, {1000: 4.0})
    tok, ev, logits = oracle.lm_head_top1_certified(x, w, s, z, 1000, 64)
    assert tok == 1000 == int(np.argmax(logits)) and ev == 1
    # a stronger row elsewhere than the seed's: both chunks, the stronger wins
    w, s, z = planted_head(rng, 4096, k, x, {1000: 4.0, 3000: 5.0})
    tok, ev, logits = oracle.lm_head_top1_certified(x, w, s, z, 1000, 64)
    assert tok == 3000 == int(np.argmax(logits)) and ev == 2
    # an exact tie in two chunks: the lower id
    w, s, z = planted_head(rng, 4096, k, x, {2500: 4.0, 70: 4.0})
    tok, ev, _ = oracle.lm_head_top1_certified(x, w, s, z, 2500, 64)
    assert tok == 70 and ev == 2
    # candidates over capacity: the full head
    tok, ev, _ = oracle.lm_head_top1_certified(x, w, s, z, 2500, 1)
    assert tok == 70 and ev == 4096 // 16


# --------------------------------------------------------------------- GPU


def _gpu_case(w, s, z, x, seed_tok, capacity, use_norm=False, rng=None):
    import torch
    from engine import ops
    from helpers import u4_to_torch

    dev = torch.device("cuda:0")
    W = u4_to_torch(w, s, z, dev)
    full = torch.empty(W.rows, dtype=torch.float32, device=dev)
    if use_norm:
        x32 = torch.from_numpy(x.astype(np.float32) * 3.0).to(dev)
        nw = torch.from_numpy(rng.uniform(0.5, 1.5, x.size).astype(np.float32)).to(dev)
        ops.u4_matvec_multi(None, [W], [full], x_f32=x32, norm_weight=nw, norm_eps=1e-6)
        kw = dict(x_f32=x32, norm_weight=nw, norm_eps=1e-6)
    else:
        xd = torch.from_numpy(x).to(dev)
        ops.u4_matvec_multi(xd, [W], [full])
        kw = dict(x=xd)
    ref_tok = torch.empty(1, dtype=torch.int32, device=dev)
    ops.argmax(full, ref_tok)
    table = ops.lm_head_cert_table(W)
    logits = torch.full((W.rows,), float("nan"), dtype=torch.float32, device=dev)
    tok = torch.empty(1, dtype=torch.int32, device=dev)
    ev = torch.empty(1, dtype=torch.int32, device=dev)
    seed = torch.tensor([seed_tok], dtype=torch.int32, device=dev)
    ops.lm_head_top1_certified(W, table, seed, logits, tok, capacity_chunks=capacity,
                               evaluated=ev, **kw)
    torch.cuda.synchronize()
    done = ~torch.isnan(logits)
    # every row of an evaluated chunk carries the full head's logit, bit for bit
    assert torch.equal(logits[done], full[done])
    assert int(done.sum()) % 16 == 0
    return int(tok), int(ref_tok), int(ev), int(done.sum()) // 16


@pytest.mark.gpu
@pytest.mark.parametrize("rows,k,use_norm", [(248320, 2048, True), (4096, 1024, False)])
def test_gpu_cert_random_head_equals_full_argmax(rows, k, use_norm):
    rng = np.random.default_rng(21)
    w, s, z = make_u4(rng, rows, k)
    x = _x(rng, k)
    tok, ref_tok, ev, done = _gpu_case(w, s, z, x, 12345 % rows, 1024, use_norm, rng)
    assert tok == ref_tok
    assert ev == done


@pytest.mark.gpu
def test_gpu_cert_planted_heads():
    rng = np.random.default_rng(22)
    rows, k = 16384, 2048
    x = _x(rng, k)
    cases = [({5000: 4.0}, 5000, 64), ({5000: 4.0, 12000: 5.0}, 5000, 64),
             ({9000: 4.0, 33: 4.0}, 9000, 64), ({9000: 4.0, 33: 4.0}, 9000, 1),
             ({5000: 4.0}, 77, 64)]
    for plants, seed_tok, cap in cases:
        w, s, z = planted_head(rng, rows, k, x, plants)
        o_tok, o_ev, _ = oracle.lm_head_top1_certified(x, w, s, z, seed_tok, cap)
        tok, ref_tok, ev, done = _gpu_case(w, s, z, x, seed_tok, cap)
        assert tok == ref_tok == o_tok, (plants, seed_tok, cap)
        assert ev == done
        if seed_tok in plants:
            assert ev == o_ev, (plants, seed_tok, cap, ev, o_ev)


@pytest.mark.gpu
def test_gpu_runtime_certified_head_same_tokens(cuda):
    """The decode graph with the certified head generates the full head's
    tokens (4-layer model, vocab 4096, shared weights)."""
    from engine.runtime import ModelConfig, Qwen36Runtime
    cfg = ModelConfig(layers=4, experts=16, vocab=4096)
    full = Qwen36Runtime(cfg, seed=31, max_ctx=64, device=cuda)
    cert = Qwen36Runtime(cfg, max_ctx=64, device=cuda, weights=full.w, lm_head="certified")
    full.capture()
    cert.capture()
    prompt = [5, 17, 900, 4000, 2, 3]
    a, _ = full.generate(prompt, 10)
    b, _ = cert.generate(prompt, 10)
    assert a == b
    assert 1 <= int(cert.lm_evaluated.item()) <= cfg.vocab // 16
