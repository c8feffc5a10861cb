"""Batched u4 projections (iq36_u4_gemm, tcgen05) against the CPU oracle.

Each output row is the u4 GEMV of the matching input row, so the oracle runs
its GEMV per row. Shapes follow the batched prefill projections: DeltaNet and
attention in-projections (K = 2048, fused RMSNorm of the fp32 residual, fp16
out) and the out/o projections (K = 4096, fp16 in, fp32 residual update).
Tolerance: tests/helpers.py (max rel 2e-3).
"""

import numpy as np
import pytest

from helpers import assert_close, make_u4, u4_to_torch
from oracle import oracle

pytestmark = pytest.mark.gpu


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.mark.parametrize("T,N,G", [(300, 512, 128), (129, 256, 128), (1, 768, 128),
                                   (300, 512, 64), (129, 768, 64)])
def test_u4_gemm_fused_norm_f16_out(cuda, T, N, G):
    import torch
    from engine.ops import u4_gemm
    rng = np.random.default_rng(T * 31 + N + G)
    K = 2048
    w, s, z = make_u4(rng, N, K, G)
    x = (rng.standard_normal((T, K)) * 2).astype(np.float32)
    nw = rng.uniform(0.9, 1.1, K).astype(np.float32)
    out = u4_gemm(_t(x, cuda), u4_to_torch(w, s, z, cuda, G), out_dtype=torch.float16,
                  norm_weight=_t(nw, cuda))
    got = out.float().cpu().numpy()
    for t in range(T):
        x16 = oracle.rms_norm(x[t], nw, 1e-6).astype(np.float16)
        assert_close(got[t], oracle.u4_gemv(x16, w, s, z, G), f"gemm row {t}")


@pytest.mark.parametrize("G", [128, 64])
def test_u4_gemm_k4096_residual_accumulate(cuda, G):
    """K = 4096 at group 64 is 64 groups per row: the case the shared-memory
    scale staging of group 128 cannot hold."""
    from engine.ops import u4_gemm
    rng = np.random.default_rng(9 + G)
    T, K, N = 200, 4096, 512
    w, s, z = make_u4(rng, N, K, G)
    x = rng.standard_normal((T, K)).astype(np.float16)
    res0 = rng.standard_normal((T, N)).astype(np.float32)
    res = _t(res0.copy(), cuda)
    u4_gemm(_t(x, cuda), u4_to_torch(w, s, z, cuda, G), out=res, accumulate=True)
    got = res.cpu().numpy()
    for t in range(0, T, 7):
        ref = res0[t] + oracle.u4_gemv(x[t], w, s, z, G).astype(np.float16).astype(np.float32)
        assert_close(got[t], ref, f"gemm accumulate row {t}")


def test_u4_gemm_rejects_bad_shapes(cuda):
    import torch
    from engine import _native as N
    from engine.ops import u4_gemm
    rng = np.random.default_rng(1)
    w, s, z = make_u4(rng, 128, 2048)                  # N not a multiple of 256
    with pytest.raises(N.Iq36Error):
        u4_gemm(torch.zeros(4, 2048, dtype=torch.float16, device=cuda), u4_to_torch(w, s, z, cuda))


@pytest.mark.parametrize("G", [128, 64])
def test_u4_gemm_multi_matches_single_calls_and_oracle(cuda, G):
    """Three projections of one input in one launch (the DeltaNet in-projection
    shape family): each output equals its own iq36_u4_gemm bit for bit, and the
    oracle's GEMV per row; a fourth, fp32-accumulating output checks the
    residual form."""
    import torch
    from engine.ops import u4_gemm, u4_gemm_multi
    rng = np.random.default_rng(77)
    T, K = 200, 2048
    mats = [make_u4(rng, n, K, G) for n in (512, 256, 768)]
    ws = [u4_to_torch(w, s, z, cuda, G) for w, s, z in mats]
    x = (rng.standard_normal((T, K)) * 2).astype(np.float32)
    nw = rng.uniform(0.9, 1.1, K).astype(np.float32)
    outs = [torch.empty(T, w.rows, dtype=torch.float16, device=cuda) for w in ws]
    acc_w = u4_to_torch(*make_u4(rng, 256, K, G), cuda, G)
    res0 = rng.standard_normal((T, 256)).astype(np.float32)
    res = _t(res0.copy(), cuda)
    u4_gemm_multi(_t(x, cuda), ws + [acc_w], outs + [res], accumulate=[False] * 3 + [True],
                  norm_weight=_t(nw, cuda))
    for w, o in zip(ws, outs):
        single = u4_gemm(_t(x, cuda), w, out_dtype=torch.float16, norm_weight=_t(nw, cuda))
        assert torch.equal(single, o)
    got = [o.float().cpu().numpy() for o in outs]
    for t in (0, 77, T - 1):
        x16 = oracle.rms_norm(x[t], nw, 1e-6).astype(np.float16)
        for (w, s, z), g in zip(mats, got):
            assert_close(g[t], oracle.u4_gemv(x16, w, s, z, G), f"multi row {t}")
    single_res = _t(res0.copy(), cuda)
    u4_gemm(_t(x, cuda), acc_w, out=single_res, accumulate=True, norm_weight=_t(nw, cuda))
    assert torch.equal(single_res, res)


@pytest.mark.parametrize("T", [4160, 4296])
def test_u4_gemm_two_tile_units_bit_equal_one_tile(cuda, T):
    """At T = 4160 / 4296 and N = 12288 the GEMM runs units of two 128-row
    tiles that share each dequantised k-block, the last unit holding one tile
    (64 rows) or a partial second tile (72 rows). Each output row depends only
    on its input row, so every row equals, bit for bit, the same row from
    calls short enough to run one-tile units; sampled rows also match the
    oracle's GEMV."""
    import torch
    from engine.ops import u4_gemm
    rng = np.random.default_rng(T)
    K, N, G = 2048, 12288, 128
    w, s, z = make_u4(rng, N, K, G)
    wt = u4_to_torch(w, s, z, cuda, G)
    x = (rng.standard_normal((T, K)) * 2).astype(np.float32)
    nw = rng.uniform(0.9, 1.1, K).astype(np.float32)
    xt, nwt = _t(x, cuda), _t(nw, cuda)
    full = u4_gemm(xt, wt, out_dtype=torch.float16, norm_weight=nwt)
    for r0, r1 in ((0, 128), (3968, 4096), (4096, T)):
        part = u4_gemm(xt[r0:r1].contiguous(), wt, out_dtype=torch.float16, norm_weight=nwt)
        assert torch.equal(full[r0:r1], part), f"rows {r0}..{r1}: two-tile units differ"
    got = full.float().cpu().numpy()
    for t in (5, 4095, T - 1):
        x16 = oracle.rms_norm(x[t], nw, 1e-6).astype(np.float16)
        assert_close(got[t], oracle.u4_gemv(x16, w, s, z, G), f"gemm row {t}")
