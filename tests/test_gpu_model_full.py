"""Full-size parity: the BASELINE config-4 model that bench.py times
(40 layers = 10 x (3 DeltaNet + 1 GQA), 256 experts + 1 shared, vocab
248,320, the bench's weight seed) against the CPU checker.

The reference's loop being restated is the prompt feed followed by greedy
decoding (engine/service/iq36_server/runtime.py:533-545). Its acceptance bars
are the per-component gate (cosine >= 0.999, relL2 <= 2e-3,
acceptance-matrix.json:365-369), greedy agreement and per-position KL
divergence <= 0.005 (BENCHMARKS.md:111-119, measured on the trained model).

Why the strict gate is layer-wise. On this random-init 40-layer model two
implementations that differ only in float summation order drift apart
end to end: a 1-ulp fp16 difference in one layer's output moves a later
router past a near-tie, a different expert joins the top 8, and the
residual stream diverges by a few percent from there on. The checker run
against itself with fp64 instead of fp32 GEMV accumulation (the control
below) differs by KLD up to ~3e-2 per position, with routing differences in
up to half the layers, while the 4-layer model's two paths agree to ~1e-5.
So:
  * every layer is checked with TEACHER FORCING: the GPU layer gets the
    checker's own residual as its input at every position, and its output
    (and routed ids) must match the checker's within the per-op bar; the
    layer's KV cache / DeltaNet state evolves from those same inputs;
  * end to end, the free-running GPU (batched prefill, then back-to-back
    CUDA-graph replays with no host synchronisation, so every read a kernel
    issues before its griddepcontrol.wait runs with its predecessors still
    in flight) must agree with the checker's greedy token wherever the
    checker's top-1 margin exceeds the measured drift, and its KL divergence
    must stay within the checker-vs-checker control's;
  * the 4096-token batched prefill is checked layer by layer against the
    token-serial decode path, each batched layer fed the serial path's
    residuals.
"""

import os

import numpy as np
import pytest

from helpers import assert_close, cosine, rel_l2
from oracle import oracle

pytestmark = pytest.mark.gpu

SEED = 1234      # bench.py's weight seed
PROMPT = 64      # 4 full 16-token pages before the first decoded token
STEPS = 16       # greedy decode steps after the prompt


def _kld(p_logits, q_logits) -> float:
    p = np.exp(p_logits - p_logits.max())
    p /= p.sum()
    q = np.exp(q_logits - q_logits.max())
    q /= q.sum()
    return float(np.sum(p * (np.log(p + 1e-30) - np.log(q + 1e-30))))


def _near_tie(ids_a, ids_b, ref_logits, tol) -> bool:
    """A routing difference is a near-tie when the reference router logits of
    the experts that differ lie within tol of each other (tol: twice the
    observed logit difference between the two sides). For the same set in a
    different order, the swapped experts must be within tol; for different
    sets, every expert selected by one side only must be within tol of one
    selected by the other side only."""
    a, b = [int(i) for i in ids_a], [int(i) for i in ids_b]
    only_a, only_b = set(a) - set(b), set(b) - set(a)
    lg = lambda x: float(ref_logits[x])
    if not only_a:
        return all(abs(lg(x) - lg(y)) <= tol for x, y in zip(a, b) if x != y)
    return all(min(abs(lg(x) - lg(y)) for y in only_b) <= tol for x in only_a)


@pytest.fixture(scope="module")
def full(cuda):
    import torch
    from engine.runtime import ModelConfig, Qwen36Runtime
    cfg = ModelConfig()
    rt = Qwen36Runtime(cfg, seed=SEED, max_ctx=PROMPT + STEPS + 32, device=cuda)
    gen = torch.Generator().manual_seed(4096)
    prompt = torch.randint(0, cfg.vocab, (PROMPT,), generator=gen, dtype=torch.int32).tolist()
    rt.capture()
    rt.prefill_batched(prompt)
    toks = torch.empty(STEPS + 1, dtype=torch.int32, device=cuda)
    logs = torch.empty(STEPS + 1, cfg.vocab, dtype=torch.float32, device=cuda)
    toks[0:1].copy_(rt.token)
    logs[0].copy_(rt.logits)
    for i in range(STEPS):          # back to back: no host sync in this loop
        rt.step()
        toks[i + 1:i + 2].copy_(rt.token)
        logs[i + 1].copy_(rt.logits)
    torch.cuda.synchronize(cuda)
    toks, logs = toks.cpu().numpy(), logs.cpu().numpy()
    seq = prompt + [int(t) for t in toks[:STEPS]]   # the token fed at each position

    # the checker over the same tokens (teacher-forced on the GPU's), with traces
    orc = oracle.OracleModel(cfg.as_dict(), SEED, PROMPT + STEPS + 8)
    trace = []
    try:
        for pos, t in enumerate(seq):
            trace.append(orc.step_trace(t, pos))   # (token, logits, hidden, ids, router)
    finally:
        orc.close()
    # control: the checker with fp64 instead of fp32 accumulation, same tokens
    prev = os.environ.get("IQ36_ORACLE_PRECISE")
    os.environ["IQ36_ORACLE_PRECISE"] = "1"
    try:
        ctl = oracle.OracleModel(cfg.as_dict(), SEED, PROMPT + STEPS + 8)
        ctl_logits = []
        for pos, t in enumerate(seq):
            if pos < PROMPT - 1:
                ctl.feed(t, pos)
            else:
                ctl_logits.append(ctl.step(t, pos)[1])
        ctl.close()
    finally:
        if prev is None:
            del os.environ["IQ36_ORACLE_PRECISE"]
        else:
            os.environ["IQ36_ORACLE_PRECISE"] = prev
    yield {"cfg": cfg, "rt": rt, "prompt": prompt, "seq": seq, "toks": toks, "logs": logs,
           "trace": trace, "ctl": ctl_logits}
    del rt
    torch.cuda.empty_cache()


def test_layerwise_teacher_forced_decode(full):
    """Every layer at every position (prompt fed token by token, then the
    decoded tokens), given the checker's residual as input: output within the
    per-op bar, routed ids bit-exact except near-ties; the embedding row bit
    for bit; the LM head on the checker's final residual within the bar."""
    import torch
    from engine import ops
    cfg, rt, seq, trace = full["cfg"], full["rt"], full["seq"], full["trace"]
    W = rt.w
    rt.reset()
    ties, worst, worst_router = 0, 0.0, 0.0
    for pos, tok in enumerate(seq):
        _, o_logits, hid, o_ids, o_router = trace[pos]
        rt.pos.fill_(pos)
        rt.ctx.fill_(pos + 1)
        rt.token.fill_(tok)
        ops.embed(W.embed, rt.token, rt.hres)
        np.testing.assert_array_equal(rt.hres.cpu().numpy(), hid[0])
        for l in range(cfg.layers):
            rt.hres.copy_(torch.from_numpy(hid[l]))
            rt.enqueue_layer(l)
            out = rt.hres.cpu().numpy()
            ids = rt.b_ids.cpu().numpy()
            # router logits: the per-op bar, given the layer's (teacher-forced)
            # input; the attention / DeltaNet half of the layer feeds them
            dl = float(np.max(np.abs(rt.b_logits_r.cpu().numpy() - o_router[l])))
            worst_router = max(worst_router, dl / float(np.max(np.abs(o_router[l]))))
            assert dl <= 2e-3 * float(np.max(np.abs(o_router[l]))), (
                f"position {pos} layer {l}: router logits differ by {dl:.3e}")
            if not np.array_equal(ids, o_ids[l]):
                assert _near_tie(ids, o_ids[l], o_router[l], 2 * dl + 1e-6), (
                    f"position {pos} layer {l}: routed ids {ids} vs checker {o_ids[l]}")
                ties += 1
                continue
            d_gpu, d_ref = out - hid[l], hid[l + 1] - hid[l]
            worst = max(worst, assert_close(d_gpu, d_ref, f"position {pos} layer {l}"))
        rt.hres.copy_(torch.from_numpy(hid[cfg.layers]))
        ops.u4_matvec_multi(None, [W.lm_head], [rt.logits], x_f32=rt.hres,
                            norm_weight=W.final_norm, norm_eps=cfg.eps)
        assert_close(rt.logits.cpu().numpy(), o_logits, f"position {pos} LM head")
    n = len(seq) * cfg.layers
    print(f"layer-wise: {n} layer steps, worst max_rel {worst:.2e}, worst router logit "
          f"difference {worst_router:.2e} of the largest, near-ties {ties}")


def test_end_to_end_free_running(full):
    """Batched prefill + back-to-back graph decode against the checker: greedy
    agreement wherever the checker's margin exceeds the drift the control
    shows, and KL divergence within the checker-vs-checker control's."""
    trace, logs, toks, ctl = full["trace"], full["logs"], full["toks"], full["ctl"]
    k_gpu, k_ctl, undecided, ctl_flips = [], [], [], 0
    for i in range(STEPS + 1):
        o_tok, o_logits = trace[PROMPT - 1 + i][0], trace[PROMPT - 1 + i][1]
        k_gpu.append(_kld(o_logits, logs[i]))
        k_ctl.append(_kld(o_logits, ctl[i]))
        ctl_flips += int(np.argmax(ctl[i])) != o_tok
        top2 = np.partition(o_logits, -2)[-2:]
        # logit drift of the control at this position bounds what a summation
        # order can move; a margin above twice that must be kept
        drift = float(np.max(np.abs(ctl[i] - o_logits)))
        if float(top2[1] - top2[0]) > 2 * drift:
            assert int(toks[i]) == o_tok, f"greedy token differs at position {PROMPT - 1 + i}"
        elif int(toks[i]) != o_tok:
            undecided.append(PROMPT - 1 + i)
    mg, mc = float(np.mean(k_gpu)), float(np.mean(k_ctl))
    print(f"end to end: mean KLD gpu {mg:.2e} (max {max(k_gpu):.2e}), checker fp64 control "
          f"{mc:.2e} (max {max(k_ctl):.2e}); greedy disagreements at undecided positions "
          f"{undecided}, the control's own {ctl_flips}")
    assert mg <= 0.005 or mg <= 3.0 * mc + 0.005, (mg, mc)


def test_graph_back_to_back_equals_eager_synced(full):
    """The same prompt and steps run eagerly with a device sync after every
    step give the same tokens and logits bit for bit as the back-to-back
    graph replays."""
    import torch
    rt, prompt = full["rt"], full["prompt"]
    rt.reset()
    rt.prefill_batched(prompt)
    torch.cuda.synchronize(rt.dev)
    assert int(rt.token.item()) == int(full["toks"][0])
    np.testing.assert_array_equal(rt.logits.cpu().numpy(), full["logs"][0])
    for i in range(STEPS):
        rt.enqueue_step()
        torch.cuda.synchronize(rt.dev)
        assert int(rt.token.item()) == int(full["toks"][i + 1]), f"step {i}"
        np.testing.assert_array_equal(rt.logits.cpu().numpy(), full["logs"][i + 1])


def test_prompt_4096_batched_layerwise_equals_token_serial(full):
    """A 4096-token prompt through the decode graph token by token (recording
    every layer's input residual and routed ids), then through the batched
    prefill one layer at a time, each batched layer fed the serial path's
    residuals: per layer, the batched output agrees with the serial output
    (rows whose routing differs at a near-tie excluded and counted), and the
    DeltaNet states, conv states and KV pages the two paths leave agree."""
    import torch
    from engine.runtime import Qwen36Runtime
    cfg, rt0 = full["cfg"], full["rt"]
    T, L, H, k = 4096, cfg.layers, cfg.hidden, cfg.topk
    rt = Qwen36Runtime(cfg, max_ctx=T + 32, device=rt0.dev, weights=rt0.w)
    E = cfg.experts
    rt.trace = torch.zeros(L + 1, H, dtype=torch.float32, device=rt.dev)
    rt.trace_ids = torch.zeros(L, k, dtype=torch.int32, device=rt.dev)
    rt.trace_router = torch.zeros(L, E, dtype=torch.float32, device=rt.dev)
    rt.capture()
    gen = torch.Generator().manual_seed(4097)
    prompt = torch.randint(0, cfg.vocab, (T,), generator=gen, dtype=torch.int32)
    rec = torch.empty(T, L + 1, H, dtype=torch.float32, device=rt.dev)
    rec_ids = torch.empty(T, L, k, dtype=torch.int32, device=rt.dev)
    rec_router = torch.empty(T, L, E, dtype=torch.float32, device=rt.dev)
    toks = prompt.pin_memory()
    for t in range(T):
        rt.token.copy_(toks[t:t + 1], non_blocking=True)
        rt.step()
        rec[t].copy_(rt.trace)
        rec_ids[t].copy_(rt.trace_ids)
        rec_router[t].copy_(rt.trace_router)
    torch.cuda.synchronize(rt.dev)
    serial_rec = {l: s.clone() for l, s in rt.rec_state.items()}
    serial_conv = {l: s.clone() for l, s in rt.conv_state.items()}
    serial_kv = {l: (a.clone(), b.clone()) for l, (a, b) in rt.kv.items()}
    rt.reset()
    B = rt._prefill_buffers(T)
    excluded, worst_router = 0, 0.0
    for l in range(L):
        B["h"][:T].copy_(rec[:, l])
        rt.enqueue_prefill_layer(l, T)
        # router logits of the batched layer against the serial path's, per row
        ls = rec_router[:, l]
        dl = (B["logits_r"][:T] - ls).abs().amax(dim=1)
        scale = float(ls.abs().max())
        worst_router = max(worst_router, float(dl.max()) / scale)
        assert float(dl.max()) <= 2e-3 * scale, f"layer {l}: router logits differ by {dl.max():.3e}"
        same = (B["ids"][:T] == rec_ids[:, l]).all(dim=1)
        diff_rows = (~same).nonzero().flatten().tolist()
        if diff_rows:
            bi, si = B["ids"][:T][diff_rows].cpu().numpy(), rec_ids[diff_rows, l].cpu().numpy()
            lsr, dlr = ls[diff_rows].cpu().numpy(), dl[diff_rows].cpu().numpy()
            for j, t in enumerate(diff_rows):
                assert _near_tie(bi[j], si[j], lsr[j], 2 * float(dlr[j]) + 1e-6), (
                    f"layer {l} token {t}: routed ids {bi[j]} vs serial {si[j]}")
        excluded += len(diff_rows)
        d_b = (B["h"][:T] - rec[:, l])[same].double()
        d_s = (rec[:, l + 1] - rec[:, l])[same].double()
        cs = float((d_b * d_s).sum() / (d_b.norm() * d_s.norm()))
        rl = float((d_b - d_s).norm() / d_s.norm())
        assert cs >= 0.999 and rl <= 2e-3, f"layer {l}: cos={cs:.6f} relL2={rl:.3e}"
    torch.cuda.synchronize(rt.dev)

    def close(got, ref, what):
        got, ref = got.double().cpu().numpy(), ref.double().cpu().numpy()
        cs, rl = cosine(got, ref), rel_l2(got, ref)
        assert cs >= 0.9999 and rl <= 1e-2, f"{what}: cos={cs:.6f} relL2={rl:.3e}"

    for l, s in rt.rec_state.items():
        close(s, serial_rec[l], f"recurrent state {l}")
        close(rt.conv_state[l], serial_conv[l], f"conv state {l}")
    for l, (a, b) in rt.kv.items():
        close(a, serial_kv[l][0], f"K cache {l}")
        close(b, serial_kv[l][1], f"V cache {l}")
    print(f"4096-token prompt: {excluded} of {T * L} (token, layer) routings differ at near-ties; "
          f"worst router logit difference {worst_router:.2e} of the largest")
