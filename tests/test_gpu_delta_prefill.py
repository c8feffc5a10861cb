"""Batched DeltaNet prefill (iq36_delta_prefill) against the CPU oracle.

The oracle is the per-token restatement (oracle.delta_prep then
oracle.delta_step, token after token, conv and recurrent state carried), so
the batched kernels must reproduce the sequential recurrence of the reference's
linear-attention layer over a whole prompt. Cases: prompts shorter than the
conv width (state taken from the carried conv state), a ragged last chunk of
the 32-token staging, the full model head counts, a non-zero incoming state,
and prompts of 16 chunks and more, whose chunk scan runs as two segments. Tolerance: tests/helpers.py (max rel 2e-3 for the fp16 outputs; 1e-3
for the fp32 recurrent state after T tokens).
"""

import numpy as np
import pytest

from helpers import assert_close
from oracle import oracle

pytestmark = pytest.mark.gpu


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _case(rng, T, nk, nv, d=128, alog=(-2, 1)):
    c = (2 * nk + nv) * d
    return dict(
        qkv=(rng.standard_normal((T, c)) * 2).astype(np.float16),
        st=rng.standard_normal((c, 4)).astype(np.float16).astype(np.float32),
        cw=rng.uniform(-0.5, 0.5, (c, 4)).astype(np.float32),
        ab=rng.standard_normal((T, 2 * nv + 8)).astype(np.float16),  # a | b | pad
        alog=rng.uniform(alog[0], alog[1], nv).astype(np.float32),
        dtb=rng.uniform(-1, 1, nv).astype(np.float32),
        state=(rng.standard_normal((nv, d, d)) * 0.05).astype(np.float32),
        z=rng.standard_normal((T, nv * d)).astype(np.float16),
        nw=rng.uniform(0.9, 1.1, d).astype(np.float32),
    )


def _oracle(cs, T, nk, nv):
    st, state = cs["st"].copy(), cs["state"].copy()
    outs = []
    for t in range(T):
        a = cs["ab"][t, :nv]
        b = cs["ab"][t, nv:2 * nv]
        act, g, beta, st = oracle.delta_prep(cs["qkv"][t], st, cs["cw"], a, b, cs["alog"],
                                             cs["dtb"])
        out, state = oracle.delta_step(act, g, beta, state, cs["z"][t], cs["nw"], 1e-6, nk, nv)
        outs.append(out)
    return np.stack(outs), st, state


def _gpu(cs, T, nk, nv, dev):
    import torch
    from engine.ops import delta_prefill
    ab = _t(cs["ab"], dev)
    conv = _t(cs["st"], dev)
    state = _t(cs["state"], dev)
    out = torch.empty((T, nv * 128), dtype=torch.float16, device=dev)
    delta_prefill(_t(cs["qkv"], dev), conv, _t(cs["cw"], dev), ab[:, :nv], ab[:, nv:2 * nv],
                  _t(cs["alog"], dev), _t(cs["dtb"], dev), state, _t(cs["z"], dev),
                  _t(cs["nw"], dev), 1e-6, nk, nv, out)
    torch.cuda.synchronize(dev)
    return out.float().cpu().numpy(), conv.cpu().numpy(), state.cpu().numpy()


# 513 and 600 tokens (17 and 19 chunks) run the split scan: two segments at once,
# the second from a zero state and as the transition scan, joined afterwards;
# 513 leaves a one-token last chunk in the second segment.
@pytest.mark.parametrize("T,nk,nv", [(1, 2, 4), (3, 2, 4), (70, 2, 4), (40, 16, 32), (513, 4, 8),
                                     (600, 2, 4)])
def test_delta_prefill_matches_sequential_oracle(cuda, T, nk, nv):
    cs = _case(np.random.default_rng(T * 7 + nv), T, nk, nv)
    got, gconv, gstate = _gpu(cs, T, nk, nv, cuda)
    ref, rconv, rstate = _oracle(cs, T, nk, nv)
    for t in range(T):
        assert_close(got[t], ref[t], f"delta prefill out t={t}")
    np.testing.assert_array_equal(gconv, rconv)
    assert_close(gstate, rstate, "recurrent state", max_rel=1e-3)


def test_delta_prefill_split_scan_carries_the_state_across_the_cut(cuda):
    """Slow decay (log decay ~ -1e-3 per token): the state at the segment cut
    still weighs on every later token and on the final state, so the joined
    second segment (zero-start outputs + Z O_M, final state Z M + R) is
    checked where the cut matters. 600 tokens, 19 chunks, cut after 10."""
    T, nk, nv = 600, 2, 4
    cs = _case(np.random.default_rng(5), T, nk, nv, alog=(-9, -6))
    got, gconv, gstate = _gpu(cs, T, nk, nv, cuda)
    ref, rconv, rstate = _oracle(cs, T, nk, nv)
    for t in range(T):
        assert_close(got[t], ref[t], f"delta prefill out t={t}")
    np.testing.assert_array_equal(gconv, rconv)
    assert_close(gstate, rstate, "recurrent state", max_rel=1e-3)


@pytest.mark.parametrize("T", [45, 1000])
def test_delta_prefill_equals_token_serial_decode_path(cuda, T):
    """Prefill over T tokens == the decode kernels run T times (same fp32
    arithmetic, only the order of the sums over key rows differs). T = 1000:
    32 chunks with a ragged last one, the state carried through every chunk
    of the tensor-core scan; no bounded device wait expires."""
    import torch
    from engine import _native as N
    from engine.ops import delta_prep, delta_step
    import ctypes
    nk, nv = 16, 32
    before = ctypes.c_int32()
    N.call("iq36_wait_timeouts", ctypes.byref(before), 0)
    cs = _case(np.random.default_rng(11), T, nk, nv)
    got, gconv, gstate = _gpu(cs, T, nk, nv, cuda)
    c = cs["qkv"].shape[1]
    conv, state = _t(cs["st"], cuda), _t(cs["state"], cuda)
    ab, qkv, z = _t(cs["ab"], cuda), _t(cs["qkv"], cuda), _t(cs["z"], cuda)
    cw, alog, dtb, nw = (_t(cs[k], cuda) for k in ("cw", "alog", "dtb", "nw"))
    act = torch.empty(c, dtype=torch.float16, device=cuda)
    g = torch.empty(nv, dtype=torch.float32, device=cuda)
    beta = torch.empty_like(g)
    outs = torch.empty((T, nv * 128), dtype=torch.float16, device=cuda)
    for t in range(T):
        delta_prep(qkv[t], conv, cw, ab[t, :nv].contiguous(), ab[t, nv:2 * nv].contiguous(),
                   alog, dtb, act, g, beta)
        delta_step(act, g, beta, state, z[t], nw, 1e-6, nk, nv, outs[t])
    torch.cuda.synchronize(cuda)
    np.testing.assert_array_equal(gconv, conv.cpu().numpy())
    assert_close(got, outs.float().cpu().numpy(), "prefill vs decode path", max_rel=2e-3)
    assert_close(gstate, state.cpu().numpy(), "state prefill vs decode path", max_rel=1e-4)
    after = ctypes.c_int32()
    N.call("iq36_wait_timeouts", ctypes.byref(after), 0)
    assert after.value == before.value


def test_delta_prefill_rejects_bad_shapes(cuda):
    import torch
    from engine import _native as N
    from engine.ops import delta_prefill
    cs = _case(np.random.default_rng(3), 4, 2, 4)
    out = torch.empty((4, 4 * 128), dtype=torch.float16, device=cuda)
    with pytest.raises(N.Iq36Error):
        delta_prefill(_t(cs["qkv"], cuda), _t(cs["st"], cuda), _t(cs["cw"], cuda),
                      _t(cs["ab"], cuda)[:, :4], _t(cs["ab"], cuda)[:, 4:8], _t(cs["alog"], cuda),
                      _t(cs["dtb"], cuda), _t(cs["state"], cuda), _t(cs["z"], cuda),
                      _t(cs["nw"], cuda), 1e-6, 3, 4, out)  # nv % nk != 0
    assert N.lib().iq36_delta_prefill_workspace_bytes(0, 2, 4) == 0
