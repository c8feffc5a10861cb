"""Tensor-/expert-parallel decode across ranks (one process per GPU).

No counterpart in the reference (one Intel iGPU, no collectives). The north
star's decode split:

* column-parallel u4 GEMV (q/k/v, DeltaNet input projections, gate_up, LM
  head): each rank holds a contiguous block of output rows; the outputs are
  concatenated (all-gather) when a full vector is needed;
* row-parallel u4 GEMV (o_proj, out_proj, down): each rank holds a K slice of
  every row (whole quant groups) and the matching slice of x; the fp32
  partial sums are added across ranks (all-reduce);
* MoE decode, expert-sharded: each rank holds E/P experts; the router runs
  replicated (identical ids everywhere), each rank computes only the routed
  experts it owns (``iq36_moe_decode_sharded``), rank 0 adds the shared
  expert, and one all-reduce of the [H] fp32 partial sums completes the block;
* MoE decode, row-sharded inside every expert: each rank holds I/P
  intermediate rows of every expert (gate and up rows, the matching K slice
  of down) and computes all routed experts on them (``iq36_moe_decode``);
  one all-reduce of the [H] fp32 partial sums completes the block.

Sharding helpers work on host or device tensors (plain slicing and nibble
repacking); the collectives are torch.distributed (NCCL on GPUs, gloo on CPU).
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _native as N
from .ops import ExpertBank, U4Weight, _dtype_code, _ptr, _stream


def _split(n: int, world: int, rank: int, quantum: int = 1) -> tuple[int, int]:
    if n % (world * quantum):
        raise ValueError(f"{n} does not split into {world} parts of whole {quantum}s")
    step = n // world
    return rank * step, (rank + 1) * step


def shard_u4_rows(w: U4Weight, rank: int, world: int) -> U4Weight:
    """Contiguous block of output rows (column-parallel)."""
    r0, r1 = _split(w.rows, world, rank, 16)
    ng = w.k // w.group
    zp = _unpack_nibbles(w.zp).view(w.rows, ng)[r0:r1]
    return U4Weight(w.weight[r0:r1].contiguous(), w.scale[r0:r1].contiguous(),
                    _pack_nibbles(zp.reshape(-1)), w.group)


def shard_u4_k(w: U4Weight, rank: int, world: int) -> U4Weight:
    """K slice of every row in whole quant groups (row-parallel)."""
    ng = w.k // w.group
    g0, g1 = _split(ng, world, rank)
    k0, k1 = g0 * w.group, g1 * w.group
    zp = _unpack_nibbles(w.zp).view(w.rows, ng)[:, g0:g1]
    return U4Weight(w.weight[:, k0 // 2:k1 // 2].contiguous(), w.scale[:, g0:g1].contiguous(),
                    _pack_nibbles(zp.reshape(-1)), w.group)


def shard_expert_bank(b: ExpertBank, rank: int, world: int) -> tuple[ExpertBank, int]:
    """Experts [rank*E/P, (rank+1)*E/P); returns the local bank and its first id."""
    e0, e1 = _split(b.num_experts, world, rank)
    local = ExpertBank(*(getattr(b, f)[e0:e1].contiguous() for f in (
        "gate_up_weight", "gate_up_scale", "gate_up_zp", "down_weight", "down_scale",
        "down_zp")), b.group)
    return local, e0


def _unpack_nibbles(p: torch.Tensor) -> torch.Tensor:
    out = torch.empty(p.numel() * 2, dtype=torch.uint8, device=p.device)
    out[0::2] = p & 15
    out[1::2] = p >> 4
    return out


def _pack_nibbles(v: torch.Tensor) -> torch.Tensor:
    if v.numel() % 2:
        raise ValueError("odd nibble count")
    return (v[0::2] | (v[1::2] << 4)).contiguous()


def tp_u4_gemv_rowparallel(x_slice: torch.Tensor, w_kslice: U4Weight,
                           group: dist.ProcessGroup | None = None) -> torch.Tensor:
    """y = W x with W and x split along K across ranks: local partial + all-reduce."""
    from .ops import u4_matvec
    y = u4_matvec(x_slice, w_kslice, out_dtype=torch.float32)
    dist.all_reduce(y, group=group)
    return y


def tp_u4_gemv_colparallel(x: torch.Tensor, w_rows: U4Weight,
                           group: dist.ProcessGroup | None = None) -> torch.Tensor:
    """y = W x with W split by output rows: local block + all-gather."""
    from .ops import u4_matvec
    y = u4_matvec(x, w_rows, out_dtype=torch.float32)
    parts = [torch.empty_like(y) for _ in range(dist.get_world_size(group))]
    dist.all_gather(parts, y, group=group)
    return torch.cat(parts)


def shard_expert_bank_rows(b: ExpertBank, rank: int, world: int) -> ExpertBank:
    """Tensor parallel inside every expert: intermediate rows [rank*I/P,
    (rank+1)*I/P) of gate and of up (gate_up rows), and the matching K slice of
    down (whole quant groups). SwiGLU is elementwise over the intermediate
    rows, so the down partial sums of all ranks add up to the block."""
    e, i, g = b.num_experts, b.intermediate, b.group
    h = b.hidden
    i0, i1 = _split(i, world, rank, g)
    rows = torch.cat([torch.arange(i0, i1), torch.arange(i + i0, i + i1)]).to(
        b.gate_up_weight.device)
    ngh, ngi = h // g, i // g
    gu_z = _unpack_nibbles(b.gate_up_zp.reshape(-1)).view(e, 2 * i, ngh)[:, rows]
    d_z = _unpack_nibbles(b.down_zp.reshape(-1)).view(e, h, ngi)[:, :, i0 // g:i1 // g]
    return ExpertBank(b.gate_up_weight[:, rows].contiguous(), b.gate_up_scale[:, rows].contiguous(),
                      _pack_nibbles(gu_z.reshape(-1)).view(e, -1),
                      b.down_weight[:, :, i0 // 2:i1 // 2].contiguous(),
                      b.down_scale[:, :, i0 // g:i1 // g].contiguous(),
                      _pack_nibbles(d_z.reshape(-1)).view(e, -1), g)


def tp_moe_decode(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                  bank_rows: ExpertBank, shared_rows: ExpertBank | None,
                  shared_logit: torch.Tensor | None, group: dist.ProcessGroup | None = None,
                  workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Row-sharded batch-1 MoE block: every routed (and the shared) expert over
    this rank's intermediate rows as an fp32 partial sum, then one all-reduce."""
    dev = x.device
    k = ids.numel()
    h, i = bank_rows.hidden, bank_rows.intermediate
    partial = torch.empty(h, dtype=torch.float32, device=dev)
    if workspace is None:
        workspace = torch.empty(N.lib().iq36_moe_decode_workspace_bytes(k, h, i),
                                dtype=torch.uint8, device=dev)
    rb = bank_rows.c()
    sb = shared_rows.c() if shared_rows is not None else None
    N.call("iq36_moe_decode", x.data_ptr(), None, None, 0.0, ids.data_ptr(), weights.data_ptr(),
           k, ctypes.byref(rb), ctypes.byref(sb) if sb is not None else None,
           _ptr(shared_logit) if shared_rows is not None else None, partial.data_ptr(),
           _dtype_code(torch.float32), 0, workspace.data_ptr(), workspace.numel(), _stream(dev))
    dist.all_reduce(partial, group=group)
    return partial


def ep_moe_decode(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                  local_bank: ExpertBank, expert_lo: int, shared: ExpertBank | None,
                  shared_logit: torch.Tensor | None, group: dist.ProcessGroup | None = None,
                  workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Expert-sharded batch-1 MoE block: this rank's routed experts (+ the shared
    expert when given) as an fp32 partial sum, then one all-reduce."""
    dev = x.device
    k = ids.numel()
    h, i = local_bank.hidden, local_bank.intermediate
    partial = torch.empty(h, dtype=torch.float32, device=dev)
    if workspace is None:
        workspace = torch.empty(N.lib().iq36_moe_decode_workspace_bytes(k, h, i),
                                dtype=torch.uint8, device=dev)
    rb = local_bank.c()
    sb = shared.c() if shared is not None else None
    N.call("iq36_moe_decode_sharded", x.data_ptr(), None, None, 0.0, ids.data_ptr(),
           weights.data_ptr(), k, ctypes.byref(rb), expert_lo,
           ctypes.byref(sb) if sb is not None else None,
           _ptr(shared_logit) if shared is not None else None, partial.data_ptr(),
           _dtype_code(torch.float32), 0, workspace.data_ptr(), workspace.numel(), _stream(dev))
    dist.all_reduce(partial, group=group)
    return partial
