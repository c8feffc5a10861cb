"""GPU parity of each hot-path operator against the CPU oracle.

Every case calls the CUDA library through its C ABI (engine.ops wraps the
ctypes calls) and compares with oracle/ on the same seeded inputs:
floating point within max relative error 2e-3 (tests/helpers.py), router ids
and top-1 ids bit-exact, synthetic weights bit-exact.
"""

import numpy as np
import pytest

from helpers import (assert_close, bank_to_torch, make_bank, make_u4, max_rel_err, u4_to_torch)
from oracle import oracle

pytestmark = pytest.mark.gpu


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _np(t):
    return t.detach().float().cpu().numpy()


# ---------------------------------------------------------------------------
# (1) u4 GEMV


@pytest.mark.parametrize("n,k,g,out", [
    (1024, 2048, 128, "f32"),
    (1024, 2048, 64, "f32"),    # the locked model's group size
    (1000, 2048, 128, "f16"),   # ragged rows, fp16 output (fixed-FC output type)
    (2048, 4096, 128, "f32"),   # o_proj / out_proj shape
    (32, 2048, 128, "f16"),     # DeltaNet a/b projections
    (2048, 512, 128, "f32"),    # expert down shape (K = 512, 4 groups)
    (16384, 4096, 128, "f32"),  # many chunks per CTA with a 2-stage ring (wraps)
    (248320, 2048, 128, "f32"), # LM head: ~105 chunks per CTA, ring wraps ~20 times
])
def test_u4_gemv_matches_oracle(cuda, n, k, g, out):
    import torch
    from engine.ops import u4_matvec
    rng = np.random.default_rng(n * 7 + k + g)
    w, s, z = make_u4(rng, n, k, g)
    x = rng.standard_normal(k).astype(np.float16)
    dt = torch.float32 if out == "f32" else torch.float16
    y = u4_matvec(_t(x, cuda), u4_to_torch(w, s, z, cuda, g), out_dtype=dt)
    ref = oracle.u4_gemv(x, w, s, z, g, precise=True)
    assert_close(_np(y), ref, f"u4_gemv {n}x{k} g{g}")


def test_u4_gemv_deterministic(cuda):
    from engine.ops import u4_matvec
    rng = np.random.default_rng(1)
    w, s, z = make_u4(rng, 1024, 2048)
    x = _t(rng.standard_normal(2048).astype(np.float16), cuda)
    wt = u4_to_torch(w, s, z, cuda)
    a, b = _np(u4_matvec(x, wt)), _np(u4_matvec(x, wt))
    np.testing.assert_array_equal(a, b)


def test_u4_gemv_multi_with_fused_rmsnorm_and_accumulate(cuda):
    import torch
    from engine.ops import u4_matvec_multi
    rng = np.random.default_rng(2)
    h = 2048
    mats = [make_u4(rng, r, h) for r in (8192, 4096, 32, 32)]
    hres = (rng.standard_normal(h) * 3).astype(np.float32)
    nw = rng.uniform(0.9, 1.1, h).astype(np.float32)
    x16 = oracle.rms_norm(hres, nw, 1e-6).astype(np.float16)
    outs = [torch.empty(m[0].shape[0], dtype=torch.float16, device=cuda) for m in mats]
    u4_matvec_multi(None, [u4_to_torch(*m, cuda) for m in mats], outs, x_f32=_t(hres, cuda),
                    norm_weight=_t(nw, cuda))
    for i, (m, o) in enumerate(zip(mats, outs)):
        assert_close(_np(o), oracle.u4_gemv(x16, *m, 128), f"multi proj {i}")
    # accumulate into an fp32 residual: res += f16(W x)
    wo = make_u4(rng, h, 4096)
    xo = rng.standard_normal(4096).astype(np.float16)
    res0 = rng.standard_normal(h).astype(np.float32)
    res = _t(res0.copy(), cuda)
    u4_matvec_multi(_t(xo, cuda), [u4_to_torch(*wo, cuda)], [res], accumulate=[True])
    ref = res0 + oracle.u4_gemv(xo, *wo, 128).astype(np.float16).astype(np.float32)
    assert_close(_np(res), ref, "accumulate")


# ---------------------------------------------------------------------------
# (4) router


def test_router_logits_and_select(cuda):
    from engine.ops import router_logits, router_select
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((256, 2048)) * 0.02).astype(np.float16)
    wsg = (rng.standard_normal((1, 2048)) * 0.02).astype(np.float16)
    x = rng.standard_normal(2048).astype(np.float16)
    lg, sl = router_logits(_t(x, cuda), _t(w, cuda), _t(wsg, cuda))
    ref = oracle.f16_linear(x, w)
    # reference router-logit gate: max-abs <= 1e-4 (engine/tests/router_topk_compare.cpp:19-25)
    assert np.max(np.abs(_np(lg)[0] - ref)) <= 1e-4
    assert abs(_np(sl)[0] - oracle.f16_linear(x, wsg)[0]) <= 1e-4
    # selection on identical logits: bit-exact ids and weights
    ids, wts = router_select(lg, 8)
    oid, ow = oracle.router_select(_np(lg), 8)
    np.testing.assert_array_equal(_np(ids).astype(np.int32), oid)
    np.testing.assert_array_equal(_np(wts), ow)
    # ids from GPU logits equal ids from the fp64 oracle logits (margin check)
    oid2, _ = oracle.router_select(ref[None], 8)
    np.testing.assert_array_equal(_np(ids).astype(np.int32), oid2)


def test_router_select_ties_and_batches(cuda):
    from engine.ops import router_select
    g = np.load(__import__("conftest").ROOT / "tests" / "golden" / "ref_golden.npz")
    lg = g["router_logits"]
    ids, wts = router_select(_t(lg, cuda), 8)
    np.testing.assert_array_equal(_np(ids).astype(np.int32), g["router_ids"])
    np.testing.assert_array_equal(_np(wts), g["router_norm"])
    # prefill-shaped batch: 4096 tokens, N(0,1) + skewed per-expert bias
    rng = np.random.default_rng(4)
    big = (rng.standard_normal((4096, 256)) + rng.uniform(-2, 2, 256)).astype(np.float32)
    big[::97, 17] = big[::97, 3]  # plant ties
    ids, wts = router_select(_t(big, cuda), 8)
    oid, ow = oracle.router_select(big, 8)
    np.testing.assert_array_equal(_np(ids).astype(np.int32), oid)
    np.testing.assert_array_equal(_np(wts), ow)


# ---------------------------------------------------------------------------
# (2a) MoE decode block


def test_moe_block_decode_config1(cuda, config1):
    from engine.ops import moe_block_decode
    c = config1
    rb, sb = bank_to_torch(c["bank"], cuda), bank_to_torch(c["shared"], cuda)
    out, ids, wts, logits = moe_block_decode(_t(c["x"], cuda), _t(c["w_router"], cuda),
                                             _t(c["w_sg"], cuda), rb, sb, k=8)
    ref_logits = oracle.f16_linear(c["x"], c["w_router"])
    oid, ow = oracle.router_select(ref_logits[None], 8)
    np.testing.assert_array_equal(_np(ids).astype(np.int32), oid[0])  # bit-exact ids
    np.testing.assert_allclose(_np(wts), ow[0], rtol=1e-6)
    sl = oracle.f16_linear(c["x"], c["w_sg"])[0]
    bank0 = {k: v.reshape(v.shape[0], *v.shape[1:]) for k, v in c["bank"].items()}
    sh0 = {k: v[0] for k, v in c["shared"].items()}
    ref = oracle.moe_decode(c["x"], oid[0], ow[0], bank0, sh0, sl, 128)
    assert_close(_np(out), ref, "moe block config 1")


def test_moe_layer_decode_matches_oracle(cuda, config1):
    """RMSNorm -> router -> top-8 (inside the expert kernels) -> experts ->
    residual += f16(out), as the reference's MoE FFN layer."""
    import torch
    from engine.ops import moe_layer_decode
    c = config1
    rng = np.random.default_rng(11)
    rb, sb = bank_to_torch(c["bank"], cuda), bank_to_torch(c["shared"], cuda)
    res0 = (rng.standard_normal(2048) * 3).astype(np.float32)
    nw = rng.uniform(0.9, 1.1, 2048).astype(np.float32)
    res = _t(res0.copy(), cuda)
    ids = torch.empty(8, dtype=torch.int32, device=cuda)
    wts = torch.empty(8, dtype=torch.float32, device=cuda)
    logits = torch.empty(256, dtype=torch.float32, device=cuda)
    sl = torch.empty(1, dtype=torch.float32, device=cuda)
    moe_layer_decode(res, _t(nw, cuda), _t(c["w_router"], cuda), _t(c["w_sg"], cuda), rb, sb,
                     ids, wts, logits, sl)
    x16 = oracle.rms_norm(res0, nw, 1e-6).astype(np.float16)
    ref_logits = oracle.f16_linear(x16, c["w_router"])
    assert np.max(np.abs(_np(logits) - ref_logits)) <= 1e-4
    oid, ow = oracle.router_select(_np(logits)[None], 8)
    np.testing.assert_array_equal(_np(ids).astype(np.int32), oid[0])  # bit-exact selection
    np.testing.assert_array_equal(_np(wts), ow[0])
    np.testing.assert_array_equal(oid, oracle.router_select(ref_logits[None], 8)[0])
    ref_sl = oracle.f16_linear(x16, c["w_sg"])[0]
    sh0 = {k: v[0] for k, v in c["shared"].items()}
    ref = oracle.moe_decode(x16, oid[0], ow[0], c["bank"], sh0, ref_sl, 128)
    assert_close(_np(res), res0 + ref.astype(np.float16).astype(np.float32), "moe layer")


def _moe_layer_four_launches(res, nw, w_router, w_sg, rb, sb, k, stream):
    """The layer composed from the separate entry points (router logits on the
    normalised residual, top-k selection, routed + shared experts adding into
    the residual): the four-launch form of iq36_moe_layer_decode."""
    import ctypes
    import torch
    from engine import _native as N
    dev = res.device
    logits = torch.empty(256, dtype=torch.float32, device=dev)
    sl = torch.empty(1, dtype=torch.float32, device=dev)
    ids = torch.empty(k, dtype=torch.int32, device=dev)
    wts = torch.empty(k, dtype=torch.float32, device=dev)
    N.call("iq36_router_logits", None, res.data_ptr(), nw.data_ptr(), 1e-6, 1, 2048,
           w_router.data_ptr(), 256, w_sg.data_ptr(), logits.data_ptr(), sl.data_ptr(), stream)
    N.call("iq36_router_select", logits.data_ptr(), 1, 256, k, ids.data_ptr(), wts.data_ptr(),
           stream)
    ws = torch.empty(N.lib().iq36_moe_decode_workspace_bytes(k, 2048, 512), dtype=torch.uint8,
                     device=dev)
    r, s = rb.c(), sb.c()
    N.call("iq36_moe_decode", None, res.data_ptr(), nw.data_ptr(), 1e-6, ids.data_ptr(),
           wts.data_ptr(), k, ctypes.byref(r), ctypes.byref(s), sl.data_ptr(), res.data_ptr(),
           0, 1, ws.data_ptr(), ws.numel(), stream)
    return logits, ids, wts


def test_moe_layer_one_launch_equals_four_launches(cuda, config1):
    """The one-launch layer (grid barriers in the workspace) gives the same bits
    as the four separate launches, over several calls in a row that reuse one
    workspace (its barrier words must come back to rest after every call)."""
    import torch
    from engine.ops import moe_layer_decode, moe_layer_workspace
    c = config1
    rng = np.random.default_rng(12)
    rb, sb = bank_to_torch(c["bank"], cuda), bank_to_torch(c["shared"], cuda)
    nw = _t(rng.uniform(0.9, 1.1, 2048).astype(np.float32), cuda)
    wr, wsg = _t(c["w_router"], cuda), _t(c["w_sg"], cuda)
    res0 = (rng.standard_normal(2048) * 3).astype(np.float32)
    a = _t(res0.copy(), cuda)
    b = _t(res0.copy(), cuda)
    ws = moe_layer_workspace(8, 2048, 512, cuda)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    ids = torch.empty(8, dtype=torch.int32, device=cuda)
    wts = torch.empty(8, dtype=torch.float32, device=cuda)
    logits = torch.empty(256, dtype=torch.float32, device=cuda)
    sl = torch.empty(1, dtype=torch.float32, device=cuda)
    for step in range(6):
        moe_layer_decode(a, nw, wr, wsg, rb, sb, ids, wts, logits, sl, workspace=ws)
        l4, i4, w4 = _moe_layer_four_launches(b, nw, wr, wsg, rb, sb, 8, stream)
        torch.cuda.synchronize(cuda)
        assert torch.equal(logits, l4), f"call {step}: router logits differ"
        assert torch.equal(ids, i4) and torch.equal(wts, w4), f"call {step}: selection differs"
        assert torch.equal(a, b), f"call {step}: residual differs"
    # the grid-barrier counter took exactly two arrivals per CTA per call
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    bar = ws[-256:].view(torch.int64)
    assert int(bar[0].item()) == 6 * 2 * sms


def test_moe_decode_without_shared_and_accumulate(cuda, config1):
    import torch
    from engine.ops import moe_expert_ffn
    c = config1
    rb = bank_to_torch(c["bank"], cuda)
    ids = np.array([5, 250, 17, 17 + 64, 128, 3, 99, 200], np.int32)
    wts = np.array([0.3, 0.2, 0.15, 0.1, 0.1, 0.06, 0.05, 0.04], np.float32)
    res0 = np.random.default_rng(9).standard_normal(2048).astype(np.float32)
    res = _t(res0.copy(), cuda)
    moe_expert_ffn(_t(c["x"], cuda), _t(ids, cuda), _t(wts, cuda), rb, out=res, accumulate=True)
    ref = oracle.moe_decode(c["x"], ids, wts, c["bank"], None, None, 128)
    assert_close(_np(res), res0 + ref.astype(np.float16).astype(np.float32), "moe accumulate")
    out = moe_expert_ffn(_t(c["x"], cuda), _t(ids, cuda), _t(wts, cuda), rb,
                         out_dtype=torch.float32)
    assert_close(_np(out), ref, "moe no-shared")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_moe_decode_sharded_partials_sum_to_full(cuda, config1, world):
    """Expert-sharded decode emulated on one GPU: the per-shard partial sums
    (shared expert on shard 0) add up to the full block."""
    import ctypes
    import torch
    from engine import _native as N
    from engine.ops import moe_expert_ffn
    from engine.parallel_tp import shard_expert_bank
    c = config1
    rb, sb = bank_to_torch(c["bank"], cuda), bank_to_torch(c["shared"], cuda)
    ids = _t(np.array([5, 250, 17, 81, 128, 3, 99, 200], np.int32), cuda)
    wts = _t(np.array([0.3, 0.2, 0.15, 0.1, 0.1, 0.06, 0.05, 0.04], np.float32), cuda)
    sl = _t(np.array([0.7], np.float32), cuda)
    x = _t(c["x"], cuda)
    full = moe_expert_ffn(x, ids, wts, rb, sb, sl, out_dtype=torch.float32)
    total = torch.zeros_like(full)
    ws = torch.empty(N.lib().iq36_moe_decode_workspace_bytes(8, 2048, 512), dtype=torch.uint8,
                     device=cuda)
    for r in range(world):
        local, e0 = shard_expert_bank(rb, r, world)
        part = torch.empty_like(full)
        lb = local.c()
        sbc = sb.c()
        N.call("iq36_moe_decode_sharded", x.data_ptr(), None, None, 0.0, ids.data_ptr(),
               wts.data_ptr(), 8, ctypes.byref(lb), e0,
               ctypes.byref(sbc) if r == 0 else None, sl.data_ptr() if r == 0 else None,
               part.data_ptr(), 0, 0, ws.data_ptr(), ws.numel(),
               torch.cuda.current_stream(cuda).cuda_stream)
        total += part
    assert_close(_np(total), _np(full), f"sharded x{world}", max_rel=1e-5)


# ---------------------------------------------------------------------------
# (3) paged GQA decode


def _gqa_case(rng, ctx, n_blocks_extra=3):
    nblk = (ctx + 15) // 16
    total = nblk + n_blocks_extra
    q = rng.standard_normal((16, 256)).astype(np.float16)
    kc = rng.standard_normal((total, 16, 2, 256)).astype(np.float16)
    vc = rng.standard_normal((total, 16, 2, 256)).astype(np.float16)
    bt = rng.permutation(total)[:nblk].astype(np.int32)
    gate = rng.standard_normal((16, 256)).astype(np.float16)
    return q, kc, vc, bt, gate


@pytest.mark.parametrize("ctx", [1, 17, 1000, 2048, 8192, 32768])
def test_paged_gqa_matches_oracle(cuda, ctx):
    from engine.ops import paged_gqa_decode
    rng = np.random.default_rng(ctx)
    q, kc, vc, bt, gate = _gqa_case(rng, ctx)
    out = paged_gqa_decode(_t(q, cuda), _t(kc, cuda), _t(vc, cuda), _t(bt, cuda), ctx, 1 / 16,
                           gate=_t(gate, cuda))
    ref = oracle.paged_gqa(q, kc, vc, bt, ctx, 1 / 16, gate)
    assert_close(_np(out), ref, f"paged gqa ctx={ctx}")


def test_paged_gqa_131072_and_device_ctx(cuda):
    """Largest BASELINE context, and the graph-replay form (ctx read on device,
    launch sized for a larger capacity)."""
    import torch
    from engine.ops import paged_gqa_decode, paged_gqa_workspace
    ctx = 131072
    rng = np.random.default_rng(7)
    q, kc, vc, bt, gate = _gqa_case(rng, ctx, n_blocks_extra=0)
    dq, dk, dv, dbt = _t(q, cuda), _t(kc, cuda), _t(vc, cuda), _t(bt, cuda)
    out = paged_gqa_decode(dq, dk, dv, dbt, ctx, 1 / 16, gate=None)
    ref = oracle.paged_gqa(q, kc, vc, bt, ctx, 1 / 16, None)
    assert_close(_np(out), ref, "paged gqa 131072")
    ws = paged_gqa_workspace(ctx, device=cuda)
    for real in (ctx, 5000):
        cdev = torch.tensor([real], dtype=torch.int32, device=cuda)
        out2 = paged_gqa_decode(dq, dk, dv, dbt, ctx, 1 / 16, ctx_len_dev=cdev, workspace=ws)
        ref2 = ref if real == ctx else oracle.paged_gqa(q, kc, vc, bt, real, 1 / 16, None)
        assert_close(_np(out2), ref2, f"device ctx {real}")


# ---------------------------------------------------------------------------
# config-4 support ops


def test_synth_fill_bit_exact(cuda):
    import torch
    from engine.ops import synth_fill
    for kind, dt, lo, hi in ((0, torch.uint8, 0, 0), (1, torch.float16, 0.005, 0.02),
                             (2, torch.float16, 0.02, 0), (3, torch.float32, 0.9, 1.1),
                             (4, torch.float32, 1.0, 0)):
        n = 100003
        d = synth_fill(torch.empty(n, dtype=dt, device=cuda), kind, 1234, 77, lo, hi)
        h = oracle.synth_fill(n, kind, 1234, 77, lo, hi)
        got = d.cpu().numpy()
        if dt == torch.float16:
            got = got.view(np.uint16)
        np.testing.assert_array_equal(got, h)


def test_rms_norm_matches_oracle(cuda):
    import torch
    from engine.ops import rms_norm
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((3, 2048)) * 5).astype(np.float32)
    w = rng.uniform(0.9, 1.1, 2048).astype(np.float32)
    y = rms_norm(_t(x, cuda), _t(w, cuda), out_dtype=torch.float32)
    assert_close(_np(y), oracle.rms_norm(x, w, 1e-6), "rms_norm", max_rel=1e-5)


@pytest.mark.parametrize("rope_dim", [64, 256])
def test_attn_prep_matches_oracle(cuda, rope_dim):
    import torch
    from engine.ops import attn_prep
    rng = np.random.default_rng(6)
    qf = (rng.standard_normal(16 * 512) * 2).astype(np.float16)
    k = (rng.standard_normal(512) * 2).astype(np.float16)
    v = rng.standard_normal(512).astype(np.float16)
    qn = rng.uniform(0.9, 1.1, 256).astype(np.float32)
    kn = rng.uniform(0.9, 1.1, 256).astype(np.float32)
    for pos in (0, 1, 4095, 131071):
        nblk = pos // 16 + 2
        bt = rng.permutation(nblk).astype(np.int32)
        kc = torch.zeros((nblk, 16, 2, 256), dtype=torch.float16, device=cuda)
        vc = torch.zeros_like(kc)
        qo = torch.empty(16 * 256, dtype=torch.float16, device=cuda)
        go = torch.empty_like(qo)
        attn_prep(_t(qf, cuda), _t(k, cuda), _t(v, cuda), _t(qn, cuda), _t(kn, cuda), 1e-6,
                  torch.tensor([pos], dtype=torch.int32, device=cuda), _t(bt, cuda), kc, vc,
                  qo, go, rope_dim=rope_dim)
        rq, rg, rk, rv = oracle.attn_prep(qf, k, v, qn, kn, 1e-6, pos, rope_dim=rope_dim)
        assert_close(_np(qo), rq, f"q rope pos={pos}", max_rel=1e-3)
        np.testing.assert_array_equal(_np(go), rg)
        blk = bt[pos // 16]
        assert_close(_np(kc[blk, pos % 16]).ravel(), rk, f"k rope pos={pos}", max_rel=1e-3)
        np.testing.assert_array_equal(_np(vc[blk, pos % 16]).ravel(), rv)


def test_delta_prep_and_step_match_oracle(cuda):
    import torch
    from engine.ops import delta_prep, delta_step
    rng = np.random.default_rng(8)
    c, nv, nk, d = 8192, 32, 16, 128
    qkv = (rng.standard_normal(c) * 2).astype(np.float16)
    st = rng.standard_normal((c, 4)).astype(np.float16).astype(np.float32)
    cw = rng.uniform(-0.5, 0.5, (c, 4)).astype(np.float32)
    a = rng.standard_normal(nv).astype(np.float16)
    b = rng.standard_normal(nv).astype(np.float16)
    alog = rng.uniform(-2, 1, nv).astype(np.float32)
    dtb = rng.uniform(-1, 1, nv).astype(np.float32)
    dst = _t(st.copy(), cuda)
    act = torch.empty(c, dtype=torch.float16, device=cuda)
    g = torch.empty(nv, dtype=torch.float32, device=cuda)
    beta = torch.empty_like(g)
    delta_prep(_t(qkv, cuda), dst, _t(cw, cuda), _t(a, cuda), _t(b, cuda), _t(alog, cuda),
               _t(dtb, cuda), act, g, beta)
    ract, rg, rb, rst = oracle.delta_prep(qkv, st, cw, a, b, alog, dtb)
    assert max_rel_err(_np(act), ract) <= 2e-3
    assert_close(_np(g), rg, "gate", max_rel=1e-5)
    assert_close(_np(beta), rb, "beta", max_rel=1e-5)
    np.testing.assert_array_equal(_np(dst), rst)
    # recurrent step on the oracle's activation (so both see identical inputs)
    state0 = (rng.standard_normal((nv, d, d)) * 0.05).astype(np.float32)
    z = rng.standard_normal(nv * d).astype(np.float16)
    nw = rng.uniform(0.9, 1.1, d).astype(np.float32)
    dstate = _t(state0.copy(), cuda)
    out = torch.empty(nv * d, dtype=torch.float16, device=cuda)
    delta_step(_t(ract.astype(np.float16), cuda), _t(rg, cuda), _t(rb, cuda), dstate,
               _t(z, cuda), _t(nw, cuda), 1e-6, nk, nv, out)
    rout, rstate = oracle.delta_step(ract, rg, rb, state0, z, nw, 1e-6, nk, nv)
    assert_close(_np(out), rout, "delta out")
    assert_close(_np(dstate), rstate, "delta state", max_rel=1e-4)


def test_embed_and_argmax(cuda):
    import torch
    from engine.ops import argmax, embed
    rng = np.random.default_rng(10)
    table = rng.standard_normal((1000, 2048)).astype(np.float16)
    h = torch.empty(2048, dtype=torch.float32, device=cuda)
    embed(_t(table, cuda), torch.tensor([417], dtype=torch.int32, device=cuda), h)
    np.testing.assert_array_equal(_np(h), table[417].astype(np.float32))
    lg = rng.standard_normal(248320).astype(np.float32)
    lg[1000] = lg[200000] = lg.max() + 1.0  # tie: lowest id wins
    tok = torch.empty(1, dtype=torch.int32, device=cuda)
    argmax(_t(lg, cuda), tok)
    assert int(tok.item()) == 1000 == oracle.port().orc_argmax(
        lg.ctypes.data_as(__import__("ctypes").c_void_p), lg.size)
    lg2 = -np.abs(rng.standard_normal(5000)).astype(np.float32)  # all negative
    argmax(_t(lg2, cuda), tok)
    assert int(tok.item()) == int(np.argmax(lg2))
