"""Expert-parallel grouped MoE prefill across ranks (one process per GPU).

No counterpart in the reference (it runs on one Intel iGPU); this
is the north star's expert-parallel prefill. Rank r owns the contiguous
experts [r*E/P, (r+1)*E/P) and its own token shard. Per call:

  1. every assignment (token t, rank slot j, expert e) goes to rank
     e // (E/P); a token row goes once to each rank that owns at least one of
     its experts (deduplicated), assignments are ordered stably by
     destination and carry (row in the destination's block, local expert id,
     router weight);
  2. the per-destination row and assignment counts are exchanged (one
     all-to-all of 2P ints, one host read), then the rows (bf16 [n, H]) and
     the assignment records (all-to-all with those split sizes, NCCL over
     NVLink on GPUs);
  3. the owner computes every received assignment's fp16 contribution
     fp16(weight * expert(x_row)) in one grouped launch over the received
     rows (iq36_moe_prefill_rows) — exactly the single-GPU contribution;
  4. the contributions return by the reverse all-to-all (fp16);
  5. the source sums the k contributions of each token in slot order in fp32
     (iq36_moe_combine, the single-GPU scatter kernel), so the result is
     bitwise the single-GPU result.

The local expert computation is a parameter (``expert_fn(x_rows, row_of,
local_ids, weights) -> contributions``), so the exchange logic can be tested
on CPU ranks (gloo) with a reference expert function; on GPUs it is
``iq36_moe_prefill_rows`` over the rank's expert bank.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

ExpertFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]


def gpu_expert_fn(local_bank) -> ExpertFn:
    """The rank's grouped-prefill kernel over its local expert bank."""
    from . import ops

    def fn(x_rows: torch.Tensor, row_of: torch.Tensor, local_ids: torch.Tensor,
           weights: torch.Tensor) -> torch.Tensor:
        return ops.moe_prefill_rows(x_rows.contiguous(), row_of.contiguous(),
                                    local_ids.contiguous(), weights.contiguous(), local_bank)
    return fn


def ep_moe_prefill(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, num_experts: int,
                   expert_fn: ExpertFn, group: dist.ProcessGroup | None = None) -> torch.Tensor:
    """Expert-parallel MoE over this rank's tokens x [T, H] with routing
    ids/weights [T, k] (global expert ids). Returns out [T, H] fp32."""
    world = dist.get_world_size(group)
    if num_experts % world:
        raise ValueError("num_experts must divide evenly across ranks")
    e_local = num_experts // world
    dev = x.device
    t_tokens, hidden = x.shape
    k = ids.shape[1]
    flat_e = ids.reshape(-1).to(torch.int64)
    flat_d = torch.div(flat_e, e_local, rounding_mode="floor")
    need = torch.zeros(t_tokens, world, dtype=torch.bool, device=dev)
    need.scatter_(1, flat_d.view(t_tokens, k), True)                # token t -> rank r
    send_counts = torch.stack([need.sum(0), torch.bincount(flat_d, minlength=world)], 1)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    counts = torch.cat([send_counts.reshape(-1), recv_counts.reshape(-1)]).tolist()
    s_rows, s_asg = counts[0:2 * world:2], counts[1:2 * world:2]
    r_rows, r_asg = counts[2 * world::2], counts[2 * world + 1::2]
    n_rows, n_asg = int(sum(r_rows)), int(sum(r_asg))

    # rows: destination-major, token order inside each destination's block
    pairs = torch.nonzero_static(need.t(), size=int(sum(s_rows)))    # [(r, t)], no host sync
    send_x = x.index_select(0, pairs[:, 1])
    row_in_block = need.to(torch.int64).cumsum(0) - 1                 # [T, P]
    # assignments: destination-major, stable
    order = torch.sort(flat_d, stable=True).indices
    d_of = flat_d.index_select(0, order)
    t_of = torch.div(order, k, rounding_mode="floor")
    send_meta = torch.stack([
        row_in_block[t_of, d_of].to(torch.int32),
        (flat_e.index_select(0, order) - d_of * e_local).to(torch.int32),
        weights.reshape(-1).index_select(0, order).to(torch.float32).view(torch.int32)], dim=1)
    recv_x = torch.empty(n_rows, hidden, dtype=x.dtype, device=dev)
    recv_meta = torch.empty(n_asg, 3, dtype=torch.int32, device=dev)
    dist.all_to_all_single(recv_x, send_x, r_rows, s_rows, group=group)
    dist.all_to_all_single(recv_meta, send_meta, r_asg, s_asg, group=group)
    # row indices are relative to each source's block of received rows
    starts = (torch.cumsum(recv_counts[:, 0], 0) - recv_counts[:, 0]).to(torch.int32)
    base = torch.repeat_interleave(starts, recv_counts[:, 1], output_size=n_asg)
    row_of = recv_meta[:, 0] + base
    y = expert_fn(recv_x, row_of, recv_meta[:, 1].contiguous(),
                  recv_meta[:, 2].contiguous().view(torch.float32))    # [n_asg, H]

    back = torch.empty(order.numel(), hidden, dtype=y.dtype, device=dev)
    dist.all_to_all_single(back, y.contiguous(), s_asg, r_asg, group=group)
    if back.is_cuda and back.dtype == torch.float16:
        from . import ops
        # inv[a] = row of assignment a in `back`; slot-order fp32 sums on device
        inv = torch.empty(order.numel(), dtype=torch.int32, device=dev)
        inv[order] = torch.arange(order.numel(), dtype=torch.int32, device=dev)
        return ops.moe_combine(back, inv, k)
    contrib = torch.empty_like(back, dtype=torch.float32)
    contrib.index_copy_(0, order, back.float())                    # back to assignment order
    contrib = contrib.view(t_tokens, k, hidden)
    out = contrib[:, 0].clone()
    for j in range(1, k):                                           # slot order, fp32
        out += contrib[:, j]
    return out
