"""Allocation-free paged GQA decode (iq36_paged_gqa_decode_noalloc).

Some callers of this library cannot allocate device memory for a workspace:
a graph-plugin host that hands an op only its input and output buffers, or a
service held to a fixed device-memory budget with no allocator reachable from
the op. For them the split-K partials of the paged GQA decode live in a static
device array inside the library. This file checks, through the C ABI, that the
allocation-free entry point returns exactly what the workspace entry point
returns (both run the same kernels with the same split count, so the outputs
are bit-identical) on two calls in a row (the array keeps the previous call's
contents, so the second call must not be affected by them), that the same
holds when the context length is read from device memory (the form a captured
decode graph uses), and that shapes beyond the array's stated maximum are
rejected before any launch.

It runs last in a pytest session (file name) and also passes on its own in a
fresh process.
"""

import ctypes

import numpy as np
import pytest

from helpers import assert_close
from oracle import oracle

pytestmark = pytest.mark.gpu


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _case(rng, ctx):
    nblk = (ctx + 15) // 16 + 2
    q = rng.standard_normal((16, 256)).astype(np.float16)
    kc = rng.standard_normal((nblk, 16, 2, 256)).astype(np.float16)
    vc = rng.standard_normal((nblk, 16, 2, 256)).astype(np.float16)
    bt = rng.permutation(nblk).astype(np.int32)
    gate = rng.standard_normal((16, 256)).astype(np.float16)
    return q, kc, vc, bt, gate


def _noalloc(lib, q, kc, vc, bt, ctx, ctx_dev, gate, out, stream):
    return lib.iq36_paged_gqa_decode_noalloc(
        q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), ctx,
        None if ctx_dev is None else ctx_dev.data_ptr(), 16, 2, 256, 16,
        ctypes.c_float(1 / 16), gate.data_ptr(), out.data_ptr(), 0, stream)


def test_noalloc_matches_workspace_entry_point_twice(cuda):
    import torch
    from engine import _native
    from engine.ops import paged_gqa_decode

    lib = _native.lib()
    rng = np.random.default_rng(2026)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    # Two calls in a row: a long context first (many splits), then a short one
    # (few splits) so stale partials of the first call are still in the array.
    for ctx in (8192, 1000):
        q, kc, vc, bt, gate = (_t(a, cuda) for a in _case(rng, ctx))
        ref = paged_gqa_decode(q, kc, vc, bt, ctx, 1 / 16, gate=gate, out_dtype=torch.float32)
        out = torch.full((16, 256), float("nan"), dtype=torch.float32, device=cuda)
        st = _noalloc(lib, q, kc, vc, bt, ctx, None, gate, out, stream)
        assert st == 0, lib.iq36_status_string(st)
        torch.cuda.synchronize(cuda)
        assert torch.equal(out, ref), f"noalloc ctx={ctx}: not bit-identical to the workspace call"


def test_noalloc_device_context_length(cuda):
    """Capacity 8192 on the host, 1000 live tokens in device memory: the split
    count comes from the capacity and the kernels read the live length. The
    first call (live length 8192) leaves partials of every split in the array;
    the second must ignore them."""
    import torch
    from engine import _native
    from engine.ops import paged_gqa_decode

    lib = _native.lib()
    rng = np.random.default_rng(77)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    cap = 8192
    arrs = _case(rng, cap)
    q, kc, vc, bt, gate = (_t(a, cuda) for a in arrs)
    for live in (cap, 1000):
        ctx_dev = torch.tensor([live], dtype=torch.int32, device=cuda)
        ref = paged_gqa_decode(q, kc, vc, bt, cap, 1 / 16, gate=gate, out_dtype=torch.float32,
                               ctx_len_dev=ctx_dev)
        out = torch.full((16, 256), float("nan"), dtype=torch.float32, device=cuda)
        st = _noalloc(lib, q, kc, vc, bt, cap, ctx_dev, gate, out, stream)
        assert st == 0, lib.iq36_status_string(st)
        torch.cuda.synchronize(cuda)
        assert torch.equal(out, ref), f"noalloc live={live}: not bit-identical"
    # and the live-length result is the attention over the first 1000 tokens
    q_np, kc_np, vc_np, bt_np, g_np = arrs
    want = oracle.paged_gqa(q_np, kc_np, vc_np, bt_np, 1000, 1 / 16, gate_f16=g_np)
    assert_close(out.cpu().numpy(), want, "noalloc live=1000 vs oracle")


def test_noalloc_rejects_shapes_beyond_its_maximum(cuda):
    import torch
    from engine import _native

    lib = _native.lib()
    buf = torch.zeros(1 << 20, dtype=torch.float16, device=cuda)
    bt = torch.zeros(64, dtype=torch.int32, device=cuda)
    p = buf.data_ptr()
    # 3 KV heads (24 query heads) exceed the static array's 2-head maximum
    st = lib.iq36_paged_gqa_decode_noalloc(p, p, p, bt.data_ptr(), 512, None, 24, 3, 256, 16,
                                           ctypes.c_float(1 / 16), None, p, 0, None)
    assert st == -4  # IQ36_ERR_WORKSPACE
