"""The boundary operators as PyTorch custom ops: ``torch.ops.iq36.*``.

The north star's host "calls a PyTorch extension over a thin C-ABI"; the
reference reserves ``engine/ops`` for those operators (reference
engine/ops/README.md:1-7: one operation per file, parameterised by layer
weights). Each op here is a ``torch.library.custom_op`` with a schema and a
fake (meta) kernel, so torch sees shapes and dtypes without running the
kernel (tracing, fake-tensor shape propagation, ``torch.library.opcheck``);
the real kernel is the same ctypes call into libiq36_b200.so as the plain
functions of ``engine.ops``. Weights travel as their tensors (codes, scales,
zero points) plus the group size, since a custom op takes only tensors and
scalars.

    iq36::u4_matvec(x, weight, scale, zp, group, out_dtype) -> y [rows]
    iq36::router_topk(x, w_router, k) -> (ids [T, k] i32, weights [T, k] f32, logits [T, E] f32)
    iq36::moe_expert_ffn(x, ids, weights, <routed bank>, <shared bank?>, shared_logit?, group,
                         out_dtype) -> out [H]
    iq36::moe_expert_ffn_prefill(x_bf16, ids, weights, <routed bank>, group, out_dtype)
                         -> out [T, H]
    iq36::paged_gqa_decode(q, k_cache, v_cache, block_table, ctx_len, scale, gate?, out_dtype)
                         -> out [n_q, D]
"""

from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor

from . import (ExpertBank, U4Weight, moe_expert_ffn, moe_expert_ffn_prefill, paged_gqa_decode,
               router_select, u4_matvec)
from . import router_logits as _router_logits


@torch.library.custom_op("iq36::u4_matvec", mutates_args=())
def u4_matvec_op(x: Tensor, weight: Tensor, scale: Tensor, zp: Tensor, group: int,
                 out_dtype: torch.dtype) -> Tensor:
    return u4_matvec(x, U4Weight(weight, scale, zp, group), out_dtype=out_dtype)


@u4_matvec_op.register_fake
def _(x, weight, scale, zp, group, out_dtype):
    return x.new_empty(weight.shape[0], dtype=out_dtype)


@torch.library.custom_op("iq36::router_topk", mutates_args=())
def router_topk_op(x: Tensor, w_router: Tensor, k: int) -> tuple[Tensor, Tensor, Tensor]:
    logits, _ = _router_logits(x, w_router)
    ids, wts = router_select(logits, k)
    return ids, wts, logits


@router_topk_op.register_fake
def _(x, w_router, k):
    t = x.numel() // x.shape[-1]
    return (x.new_empty(t, k, dtype=torch.int32), x.new_empty(t, k, dtype=torch.float32),
            x.new_empty(t, w_router.shape[0], dtype=torch.float32))


def _bank(gu_w, gu_s, gu_z, d_w, d_s, d_z, group) -> ExpertBank:
    return ExpertBank(gu_w, gu_s, gu_z, d_w, d_s, d_z, group)


@torch.library.custom_op("iq36::moe_expert_ffn", mutates_args=())
def moe_expert_ffn_op(x: Tensor, ids: Tensor, weights: Tensor, gu_w: Tensor, gu_s: Tensor,
                      gu_z: Tensor, d_w: Tensor, d_s: Tensor, d_z: Tensor,
                      s_gu_w: Optional[Tensor], s_gu_s: Optional[Tensor], s_gu_z: Optional[Tensor],
                      s_d_w: Optional[Tensor], s_d_s: Optional[Tensor], s_d_z: Optional[Tensor],
                      shared_logit: Optional[Tensor], group: int,
                      out_dtype: torch.dtype) -> Tensor:
    shared = None
    if s_gu_w is not None:
        shared = _bank(s_gu_w, s_gu_s, s_gu_z, s_d_w, s_d_s, s_d_z, group)
    return moe_expert_ffn(x, ids, weights, _bank(gu_w, gu_s, gu_z, d_w, d_s, d_z, group), shared,
                          shared_logit, out_dtype=out_dtype)


@moe_expert_ffn_op.register_fake
def _(x, ids, weights, gu_w, gu_s, gu_z, d_w, d_s, d_z, s_gu_w, s_gu_s, s_gu_z, s_d_w, s_d_s,
      s_d_z, shared_logit, group, out_dtype):
    return x.new_empty(gu_w.shape[2] * 2, dtype=out_dtype)


@torch.library.custom_op("iq36::moe_expert_ffn_prefill", mutates_args=())
def moe_expert_ffn_prefill_op(x: Tensor, ids: Tensor, weights: Tensor, gu_w: Tensor,
                              gu_s: Tensor, gu_z: Tensor, d_w: Tensor, d_s: Tensor, d_z: Tensor,
                              group: int, out_dtype: torch.dtype) -> Tensor:
    return moe_expert_ffn_prefill(x, ids, weights, _bank(gu_w, gu_s, gu_z, d_w, d_s, d_z, group),
                                  out_dtype=out_dtype)


@moe_expert_ffn_prefill_op.register_fake
def _(x, ids, weights, gu_w, gu_s, gu_z, d_w, d_s, d_z, group, out_dtype):
    return x.new_empty(x.shape[0], x.shape[1], dtype=out_dtype)


@torch.library.custom_op("iq36::paged_gqa_decode", mutates_args=())
def paged_gqa_decode_op(q: Tensor, k_cache: Tensor, v_cache: Tensor, block_table: Tensor,
                        ctx_len: int, scale: float, gate: Optional[Tensor],
                        out_dtype: torch.dtype) -> Tensor:
    return paged_gqa_decode(q, k_cache, v_cache, block_table, ctx_len, scale, gate=gate,
                            out_dtype=out_dtype)


@paged_gqa_decode_op.register_fake
def _(q, k_cache, v_cache, block_table, ctx_len, scale, gate, out_dtype):
    return q.new_empty(q.shape[-2], q.shape[-1], dtype=out_dtype)
