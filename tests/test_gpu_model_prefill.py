"""Batched prefill (the whole prompt per launch) against the CPU oracle.

The MoE block over T tokens (iq36_moe_layer_prefill) is checked per token
against the oracle's MoE FFN (selection bit-exact on the kernel's logits,
logits within the reference's 1e-4 router gate); the batched model prefill
is checked end to end against the oracle model fed the prompt token by token:
greedy token after the prompt equal, KL divergence of the next-token
distribution <= 0.005, then a greedy decode continuation from the state the
batched prefill left (DeltaNet states, KV cache, position). Reduced counts (4
layers = 3 DeltaNet + 1 attention, 16 experts, vocab 4096) with the full
per-layer dimensions of BASELINE config 4.
"""

import numpy as np
import pytest

from helpers import assert_close, bank_to_torch
from oracle import oracle

pytestmark = pytest.mark.gpu

KLD_MAX = 0.005


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _kld(p_logits, q_logits) -> float:
    p = np.exp(p_logits - p_logits.max())
    p /= p.sum()
    q = np.exp(q_logits - q_logits.max())
    q /= q.sum()
    return float(np.sum(p * (np.log(p + 1e-30) - np.log(q + 1e-30))))


def test_moe_layer_prefill_matches_oracle(cuda, config1):
    import torch
    from engine.ops import moe_layer_prefill
    c = config1
    T = 40
    rng = np.random.default_rng(12)
    rb, sb = bank_to_torch(c["bank"], cuda), bank_to_torch(c["shared"], cuda)
    res0 = (rng.standard_normal((T, 2048)) * 3).astype(np.float32)
    nw = rng.uniform(0.9, 1.1, 2048).astype(np.float32)
    res = _t(res0.copy(), cuda)
    ids = torch.empty((T, 8), dtype=torch.int32, device=cuda)
    wts = torch.empty((T, 8), dtype=torch.float32, device=cuda)
    logits = torch.empty((T, 256), dtype=torch.float32, device=cuda)
    moe_layer_prefill(res, _t(nw, cuda), _t(c["w_router"], cuda), _t(c["w_sg"], cuda), rb, sb,
                      ids, wts, logits)
    got = res.cpu().numpy()
    g_logits, g_ids, g_wts = logits.cpu().numpy(), ids.cpu().numpy(), wts.cpu().numpy()
    # the decode step's router (fused norm from the fp32 residual, one token per
    # call, CUDA-core FMAs) agrees with the tensor-core prompt router up to the
    # fp32 summation order: the reference's router gate, max-abs <= 1e-4
    from engine import _native as N
    from engine.ops import _stream
    dl = torch.empty(256, dtype=torch.float32, device=cuda)
    dsl = torch.empty(1, dtype=torch.float32, device=cuda)
    r0, wr, wsg, nwd = _t(res0, cuda), _t(c["w_router"], cuda), _t(c["w_sg"], cuda), _t(nw, cuda)
    for t in (0, 17, T - 1):
        N.call("iq36_router_logits", None, r0[t].data_ptr(), nwd.data_ptr(), 1e-6, 1, 2048,
               wr.data_ptr(), 256, wsg.data_ptr(), dl.data_ptr(), dsl.data_ptr(), _stream(cuda))
        assert np.max(np.abs(g_logits[t] - dl.cpu().numpy())) <= 1e-4
    sh0 = {k: v[0] for k, v in c["shared"].items()}
    for t in range(T):
        x16 = oracle.rms_norm(res0[t], nw, 1e-6).astype(np.float16)
        ref_logits = oracle.f16_linear(x16, c["w_router"])
        assert np.max(np.abs(g_logits[t] - ref_logits)) <= 1e-4
        oid, ow = oracle.router_select(g_logits[t][None], 8)
        np.testing.assert_array_equal(g_ids[t], oid[0])  # bit-exact selection
        np.testing.assert_array_equal(g_wts[t], ow[0])
        ref_sl = oracle.f16_linear(x16, c["w_sg"])[0]
        ref = oracle.moe_decode(x16, oid[0], ow[0], c["bank"], sh0, ref_sl, 128)
        assert_close(got[t] - res0[t], ref, f"moe layer prefill t={t}")


def _small_cfg():
    from engine.runtime import ModelConfig
    return ModelConfig(layers=4, experts=16, vocab=4096)


@pytest.mark.parametrize("prompt_len,chunk,fc_group", [(40, 8192, 0), (40, 16, 0), (1, 8192, 0),
                                                      (40, 8192, 64)])
def test_batched_prefill_matches_oracle_then_decodes(cuda, prompt_len, chunk, fc_group):
    """fc_group 64: the attention and DeltaNet projections at the reference
    checkpoint's group size (prompt GEMMs and decode GEMVs at group 64; experts
    and LM head stay at 128)."""
    from engine.runtime import ModelConfig, Qwen36Runtime
    cfg = ModelConfig(layers=4, experts=16, vocab=4096, fc_group=fc_group)
    seed = 4242
    rt = Qwen36Runtime(cfg, seed=seed, max_ctx=96, device=cuda)
    rt.capture()
    orc = oracle.OracleModel(cfg.as_dict(), seed, 96)
    rng = np.random.default_rng(prompt_len)
    prompt = rng.integers(0, cfg.vocab, prompt_len).tolist()
    rt.prefill_batched(prompt, chunk=chunk)
    tok = ol = None
    for pos, t in enumerate(prompt):
        tok, ol = orc.step(t, pos)
    k = _kld(ol, rt.logits.cpu().numpy())
    assert k <= KLD_MAX, f"after prompt: KLD {k}"
    assert int(rt.token.item()) == tok
    assert int(rt.pos.item()) == prompt_len and int(rt.ctx.item()) == prompt_len + 1
    pos = prompt_len
    for _ in range(4):
        g_tok = int(rt.token.item())
        rt.step()
        o_tok, ol = orc.step(g_tok, pos)
        k = _kld(ol, rt.logits.cpu().numpy())
        assert k <= KLD_MAX, f"decode pos {pos} after batched prefill: KLD {k}"
        assert int(rt.token.item()) == o_tok, f"greedy token differs at pos {pos}"
        pos += 1
    orc.close()


def _close_stats(got, ref, what):
    """State after a 33-token prompt through two different summation orders
    (GEMM vs GEMV, grouped vs per-token MoE with fp16 contributions): the
    residual streams drift apart by ~1e-3, and a router near-tie can route one
    token differently, so the check is on aggregate agreement."""
    from helpers import cosine, rel_l2
    cs, rl = cosine(got, ref), rel_l2(got, ref)
    assert cs >= 0.9999 and rl <= 1e-2, f"{what}: cos={cs:.6f} relL2={rl:.3e}"


def test_batched_prefill_state_equals_token_serial(cuda):
    """Same prompt through the batched path and through the decode graph one
    token at a time: recurrent states, conv states and the KV cache agree."""
    import torch
    from engine.runtime import Qwen36Runtime
    cfg = _small_cfg()
    rt = Qwen36Runtime(cfg, seed=99, max_ctx=64, device=cuda)
    rt.capture()
    prompt = np.random.default_rng(5).integers(0, cfg.vocab, 33).tolist()
    rt.prefill(prompt)
    serial = {"logits": rt.logits.clone(), "token": int(rt.token.item()),
              "rec": {l: s.clone() for l, s in rt.rec_state.items()},
              "conv": {l: s.clone() for l, s in rt.conv_state.items()},
              "kv": {l: (k.clone(), v.clone()) for l, (k, v) in rt.kv.items()}}
    rt.reset()
    rt.prefill_batched(prompt)
    torch.cuda.synchronize(cuda)
    assert int(rt.token.item()) == serial["token"]
    assert _kld(serial["logits"].cpu().numpy(), rt.logits.cpu().numpy()) <= KLD_MAX
    for l in rt.rec_state:
        _close_stats(rt.rec_state[l].cpu().numpy(), serial["rec"][l].cpu().numpy(),
                     f"recurrent state layer {l}")
        _close_stats(rt.conv_state[l].cpu().numpy(), serial["conv"][l].cpu().numpy(),
                     f"conv state layer {l}")
    for l, (k, v) in rt.kv.items():
        n = len(prompt)
        bt = rt.block_table.cpu().numpy()
        rows = [(bt[p // 16], p % 16) for p in range(n)]
        kb = np.stack([k[b, s].float().cpu().numpy() for b, s in rows])
        ks = np.stack([serial["kv"][l][0][b, s].float().cpu().numpy() for b, s in rows])
        vb = np.stack([v[b, s].float().cpu().numpy() for b, s in rows])
        vs = np.stack([serial["kv"][l][1][b, s].float().cpu().numpy() for b, s in rows])
        _close_stats(kb, ks, f"K cache layer {l}")
        _close_stats(vb, vs, f"V cache layer {l}")


def test_batched_prefill_rejects_prompt_past_the_cache(cuda):
    from engine.runtime import Qwen36Runtime
    rt = Qwen36Runtime(_small_cfg(), seed=3, max_ctx=32, device=cuda)
    with pytest.raises(ValueError):
        rt.prefill_batched(list(range(33)))
    with pytest.raises(ValueError):
        rt.prefill_batched([])
