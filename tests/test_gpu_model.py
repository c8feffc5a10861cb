"""End-to-end batch-1 decode of the synthetic model against the CPU oracle.

Reduced counts (4 layers = 3 DeltaNet + 1 attention, 16 experts, vocab 4096)
with the full per-layer dimensions of BASELINE config 4. Bar (north star):
greedy tokens equal at every position and per-position KL divergence of the
next-token distribution <= 0.005. The GPU runs the captured CUDA graph.
"""

import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu

KLD_MAX = 0.005


def _kld(p_logits, q_logits) -> float:
    p = np.exp(p_logits - p_logits.max())
    p /= p.sum()
    q = np.exp(q_logits - q_logits.max())
    q /= q.sum()
    return float(np.sum(p * (np.log(p + 1e-30) - np.log(q + 1e-30))))


def _small_cfg():
    from engine.runtime import ModelConfig
    return ModelConfig(layers=4, experts=16, vocab=4096)


@pytest.mark.parametrize("graph", [False, True])
def test_decode_matches_oracle(cuda, graph):
    from engine.runtime import Qwen36Runtime
    cfg = _small_cfg()
    seed = 4242
    rt = Qwen36Runtime(cfg, seed=seed, max_ctx=64, device=cuda)
    if graph:
        rt.capture()
    orc = oracle.OracleModel(cfg.as_dict(), seed, 64)
    rng = np.random.default_rng(0)
    prompt = rng.integers(0, cfg.vocab, 6).tolist()
    kept = rt.prefill(prompt, keep_logits=True)
    worst = 0.0
    tok = None
    for pos, t in enumerate(prompt):
        tok, ol = orc.step(t, pos)
        k = _kld(ol, kept[pos].cpu().numpy())
        worst = max(worst, k)
        assert k <= KLD_MAX, f"prefill pos {pos}: KLD {k}"
    assert int(rt.token.item()) == tok
    # greedy continuation
    pos = len(prompt)
    for _ in range(6):
        g_tok = int(rt.token.item())
        rt.step()
        o_tok, ol = orc.step(g_tok, pos)
        k = _kld(ol, rt.logits.cpu().numpy())
        worst = max(worst, k)
        assert k <= KLD_MAX, f"decode pos {pos}: KLD {k}"
        assert int(rt.token.item()) == o_tok, f"greedy token differs at pos {pos}"
        pos += 1
    orc.close()
    print(f"worst per-position KLD {worst:.2e}")


def test_graph_replay_is_deterministic(cuda):
    from engine.runtime import Qwen36Runtime
    cfg = _small_cfg()
    rt = Qwen36Runtime(cfg, seed=7, max_ctx=64, device=cuda)
    rt.capture()
    prompt = [1, 2, 3, 4]
    rt.prefill(prompt)
    a = rt.logits.clone()
    rt.reset()
    rt.prefill(prompt)
    assert (rt.logits == a).all()
