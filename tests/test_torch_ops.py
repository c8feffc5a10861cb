"""The boundary operators registered as PyTorch custom ops (torch.ops.iq36.*).

CPU: the schemas exist and their fake kernels propagate shapes and dtypes
under FakeTensorMode (no kernel runs). GPU: each custom op returns exactly
what the plain engine.ops function returns, and torch.library.opcheck accepts
the registrations (schema, fake kernel vs real kernel)."""

import numpy as np
import pytest
import torch

from engine import ops  # noqa: F401  (registers torch.ops.iq36.*)

OPS = ("u4_matvec", "router_topk", "moe_expert_ffn", "moe_expert_ffn_prefill",
       "paged_gqa_decode")


def test_ops_registered_with_schemas():
    for name in OPS:
        op = getattr(torch.ops.iq36, name)
        assert "iq36::" + name in str(op.default._schema)


def test_fake_kernels_propagate_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        x = torch.empty(2048, dtype=torch.float16)
        w = torch.empty(1024, 1024, dtype=torch.uint8)
        s = torch.empty(1024, 16, dtype=torch.float16)
        z = torch.empty(8192, dtype=torch.uint8)
        y = torch.ops.iq36.u4_matvec(x, w, s, z, 128, torch.float32)
        assert y.shape == (1024,) and y.dtype == torch.float32
        wr = torch.empty(256, 2048, dtype=torch.float16)
        ids, wts, lg = torch.ops.iq36.router_topk(x.view(1, -1), wr, 8)
        assert ids.shape == (1, 8) and ids.dtype == torch.int32 and lg.shape == (1, 256)
        q = torch.empty(16, 256, dtype=torch.float16)
        kc = torch.empty(64, 16, 2, 256, dtype=torch.float16)
        bt = torch.empty(64, dtype=torch.int32)
        o = torch.ops.iq36.paged_gqa_decode(q, kc, kc, bt, 1000, 0.0625, None, torch.float32)
        assert o.shape == (16, 256)
        xb = torch.empty(300, 2048, dtype=torch.bfloat16)
        gu = [torch.empty(16, 1024, 1024, dtype=torch.uint8),
              torch.empty(16, 1024, 16, dtype=torch.float16),
              torch.empty(16, 8192, dtype=torch.uint8),
              torch.empty(16, 2048, 256, dtype=torch.uint8),
              torch.empty(16, 2048, 4, dtype=torch.float16),
              torch.empty(16, 4096, dtype=torch.uint8)]
        pid = torch.empty(300, 8, dtype=torch.int32)
        pw = torch.empty(300, 8, dtype=torch.float32)
        out = torch.ops.iq36.moe_expert_ffn_prefill(xb, pid, pw, *gu, 128, torch.float32)
        assert out.shape == (300, 2048)
        d = torch.ops.iq36.moe_expert_ffn(x, pid[0], pw[0], *gu, None, None, None, None, None,
                                          None, None, 128, torch.float16)
        assert d.shape == (2048,) and d.dtype == torch.float16


@pytest.mark.gpu
def test_custom_ops_equal_plain_ops(cuda):
    from engine.ops import U4Weight, u4_matvec
    from helpers import bank_to_torch, make_bank, make_u4
    rng = np.random.default_rng(21)
    w, s, z = (torch.from_numpy(a).to(cuda) for a in make_u4(rng, 1024, 2048))
    x = torch.from_numpy(rng.standard_normal(2048).astype(np.float16)).to(cuda)
    a = torch.ops.iq36.u4_matvec(x, w, s, z, 128, torch.float32)
    b = u4_matvec(x, U4Weight(w, s, z, 128))
    assert torch.equal(a, b)
    torch.library.opcheck(torch.ops.iq36.u4_matvec.default, (x, w, s, z, 128, torch.float32))
    wr = torch.from_numpy((rng.standard_normal((256, 2048)) * 0.02).astype(np.float16)).to(cuda)
    ids, wts, lg = torch.ops.iq36.router_topk(x.view(1, -1), wr, 8)
    li, lw, ll = ops.router_topk(x.view(1, -1), wr, 8)
    assert torch.equal(ids, li) and torch.equal(wts, lw) and torch.equal(lg, ll)
    bank = bank_to_torch(make_bank(rng, 16, 2048, 512), cuda)
    t = [bank.gate_up_weight, bank.gate_up_scale, bank.gate_up_zp, bank.down_weight,
         bank.down_scale, bank.down_zp]
    ids16 = (ids[0] % 16).contiguous()
    got = torch.ops.iq36.moe_expert_ffn(x, ids16, wts[0].contiguous(), *t, None, None, None, None,
                                        None, None, None, 128, torch.float32)
    want = ops.moe_expert_ffn(x, ids16, wts[0].contiguous(), bank, out_dtype=torch.float32)
    assert torch.equal(got, want)
