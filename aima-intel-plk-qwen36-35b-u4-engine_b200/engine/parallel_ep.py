"""Expert-parallel grouped MoE prefill across ranks (one process per GPU).

No counterpart in the reference (it runs on one Intel iGPU); this
is the north star's expert-parallel prefill. Rank r owns the contiguous
experts [r*E/P, (r+1)*E/P) and its own token shard. Per call:

  1. every assignment (token t, rank slot j, expert e) goes to rank
     e // (E/P); assignments are ordered stably by destination;
  2. the per-destination counts are exchanged (all-to-all of P ints), then
     the token rows (bf16 [n, H]), local expert ids and router weights
     (all-to-all with those split sizes, NCCL over NVLink on GPUs);
  3. the owner runs the grouped prefill on its received rows, one
     assignment per row (k = 1), producing the fp16 contribution
     fp16(weight * expert(x)) — exactly the single-GPU contribution;
  4. the contributions return by the reverse all-to-all (fp16);
  5. the source sums the k contributions of each token in slot order in fp32
     (iq36_moe_combine, the single-GPU scatter kernel), so the result is
     bitwise the single-GPU result.

The local expert computation is a parameter (``expert_fn``), so the exchange
logic can be tested on CPU ranks (gloo) with a reference expert function;
on GPUs it is ``iq36_moe_prefill`` over the rank's expert bank.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

ExpertFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]


def gpu_expert_fn(local_bank) -> ExpertFn:
    """The rank's grouped-prefill kernel over its local expert bank."""
    from . import ops

    def fn(x_rows: torch.Tensor, local_ids: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        if x_rows.shape[0] == 0:
            return torch.empty(0, x_rows.shape[1], dtype=torch.float16, device=x_rows.device)
        return ops.moe_expert_ffn_prefill(x_rows.contiguous(), local_ids.view(-1, 1).contiguous(),
                                          weights.view(-1, 1).contiguous(), local_bank,
                                          out_dtype=torch.float16)
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
    dest = torch.div(flat_e, e_local, rounding_mode="floor")
    order = torch.sort(dest, stable=True).indices                  # assignment ids by dest
    send_counts = torch.bincount(dest, minlength=world).to(torch.int64)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    s_split = send_counts.tolist()
    r_split = recv_counts.tolist()
    n_recv = int(sum(r_split))

    send_x = x.index_select(0, torch.div(order, k, rounding_mode="floor"))
    # local expert id and router weight travel together as two int32 words
    send_meta = torch.stack([
        (flat_e.index_select(0, order) - dest.index_select(0, order) * e_local).to(torch.int32),
        weights.reshape(-1).index_select(0, order).to(torch.float32).view(torch.int32)], dim=1)
    recv_x = torch.empty(n_recv, hidden, dtype=x.dtype, device=dev)
    recv_meta = torch.empty(n_recv, 2, dtype=torch.int32, device=dev)
    dist.all_to_all_single(recv_x, send_x, r_split, s_split, group=group)
    dist.all_to_all_single(recv_meta, send_meta, r_split, s_split, group=group)
    recv_id = recv_meta[:, 0].contiguous()
    recv_w = recv_meta[:, 1].contiguous().view(torch.float32)

    y = expert_fn(recv_x, recv_id, recv_w)                           # [n_recv, H]

    back = torch.empty(order.numel(), hidden, dtype=y.dtype, device=dev)
    dist.all_to_all_single(back, y.contiguous(), s_split, r_split, group=group)
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
