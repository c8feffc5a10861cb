"""Tensor-parallel batch-1 decode of the synthetic model across 2/4/8 GPUs.

No counterpart in the reference (one Intel iGPU). The north star's decode
split, one process per GPU:

* column-parallel (output rows sharded): the attention q/k/v projections by
  KV head (a rank computes the 8 query heads of its KV head; with more ranks
  than KV heads, P/2 ranks share one), the DeltaNet input projections by
  head (key heads [r nk/P, (r+1) nk/P), value heads [r nv/P, ...): the
  recurrence of a value head needs only its own key head, so conv, gates,
  recurrence and gated norm stay local), the LM head by vocab rows;
* row-parallel (K sharded): the attention output projection over this
  rank's query heads, the DeltaNet output projection over its value heads,
  and the experts (each rank holds I/P intermediate rows of every routed and
  of the shared expert; at P = 8, I/P is below one quant group, so the
  experts are sharded instead: 32 per rank, the shared expert on rank 0);
* replicated: embedding, norms, router, the fp32 residual stream.

Each row-parallel sub-block ends with iq36_tp_allreduce_residual (one-shot
peer stores over NVLink into CUDA-IPC-mapped buffers, bounded flag waits):
two per layer, plus the LM head's (value, id) key merge (iq36_tp_argmax).
One decode step is captured as one CUDA graph per rank, as on one GPU.
"""

from __future__ import annotations

import ctypes
import math

import torch
import torch.distributed as dist

from . import _native as N
from . import ops
from .parallel_tp import _pack_nibbles, _unpack_nibbles, shard_expert_bank, shard_expert_bank_rows
from .runtime import ModelConfig, SyntheticWeights


# ---------------------------------------------------------------------------
# weight slicing

def u4_rows(w: ops.U4Weight, ranges: list[tuple[int, int]]) -> ops.U4Weight:
    """The listed row ranges of a u4 matrix, concatenated into one matrix."""
    ng = w.k // w.group
    zp = _unpack_nibbles(w.zp).view(w.rows, ng)
    pick = lambda t: torch.cat([t[a:b] for a, b in ranges]).contiguous()
    return ops.U4Weight(pick(w.weight), pick(w.scale), _pack_nibbles(pick(zp).reshape(-1)),
                        w.group)


def u4_cols(w: ops.U4Weight, k0: int, k1: int) -> ops.U4Weight:
    """Columns [k0, k1) of a u4 matrix (whole quant groups): the K slice of a
    row-parallel projection."""
    g = w.group
    if k0 % g or k1 % g:
        raise ValueError("a K slice must cover whole quant groups")
    ng = w.k // g
    zp = _unpack_nibbles(w.zp).view(w.rows, ng)[:, k0 // g:k1 // g]
    return ops.U4Weight(w.weight[:, k0 // 2:k1 // 2].contiguous(),
                        w.scale[:, k0 // g:k1 // g].contiguous(),
                        _pack_nibbles(zp.reshape(-1)), g)


class TPWeights:
    """Rank r's shard of the synthetic model (sliced from the full weights)."""

    def __init__(self, full: SyntheticWeights, rank: int, world: int):
        c = full.cfg
        self.cfg, self.rank, self.world = c, rank, world
        D, dk = c.head_dim, c.dk
        if c.nq % world or c.nk % world or c.nv % world or c.vocab % (16 * world):
            raise ValueError(f"the model does not shard over {world} ranks")
        self.kvh = rank * c.nkv // world                 # this rank's KV head
        self.nh = c.nq // world                          # query heads in its o_proj slice
        self.h_off = rank * self.nh - self.kvh * (c.nq // c.nkv)  # their offset in the KV head
        self.nk, self.nv = c.nk // world, c.nv // world
        kh0, vh0 = rank * self.nk, rank * self.nv
        self.expert_rows = c.inter % (world * c.group) == 0
        self.layers = []
        for l in range(c.layers):
            F = full.layers[l]
            L = {"in_norm": F["in_norm"], "post_norm": F["post_norm"], "router": F["router"],
                 "sgate": F["sgate"]}
            if c.is_attn(l):
                grp = c.nq // c.nkv
                q0 = self.kvh * grp * 2 * D
                L["q"] = u4_rows(F["q"], [(q0, q0 + grp * 2 * D)])
                L["k"] = u4_rows(F["k"], [(self.kvh * D, (self.kvh + 1) * D)])
                L["v"] = u4_rows(F["v"], [(self.kvh * D, (self.kvh + 1) * D)])
                L["o"] = u4_cols(F["o"], rank * self.nh * D, (rank + 1) * self.nh * D)
                L["qn"], L["kn"] = F["qn"], F["kn"]
            else:
                qr = (kh0 * dk, (kh0 + self.nk) * dk)
                kr = (c.nk * dk + kh0 * dk, c.nk * dk + (kh0 + self.nk) * dk)
                vr = (2 * c.nk * dk + vh0 * dk, 2 * c.nk * dk + (vh0 + self.nv) * dk)
                L["qkv"] = u4_rows(F["qkv"], [qr, kr, vr])
                L["z"] = u4_rows(F["z"], [(vh0 * dk, (vh0 + self.nv) * dk)])
                L["a"] = u4_rows(F["a"], [(vh0, vh0 + self.nv)])
                L["b"] = u4_rows(F["b"], [(vh0, vh0 + self.nv)])
                L["out"] = u4_cols(F["out"], vh0 * dk, (vh0 + self.nv) * dk)
                cw = F["conv_w"].view(-1, c.conv)
                L["conv_w"] = torch.cat([cw[a:b] for a, b in (qr, kr, vr)]).contiguous()
                L["a_log"] = F["a_log"][vh0:vh0 + self.nv].contiguous()
                L["dt_bias"] = F["dt_bias"][vh0:vh0 + self.nv].contiguous()
                L["dnorm"] = F["dnorm"]
            if self.expert_rows:
                L["bank"] = shard_expert_bank_rows(F["bank"], rank, world)
                L["shared"] = shard_expert_bank_rows(F["shared"], rank, world)
            else:
                L["bank"], L["expert_lo"] = shard_expert_bank(F["bank"], rank, world)
                L["shared"] = F["shared"] if rank == 0 else None
            self.layers.append(L)
        self.embed, self.final_norm = full.embed, full.final_norm
        self.vocab_lo = rank * (c.vocab // world)
        self.vocab_n = c.vocab // world
        self.lm_head = u4_rows(full.lm_head, [(self.vocab_lo, self.vocab_lo + self.vocab_n)])


# ---------------------------------------------------------------------------
# the exchange buffers

class TPComm:
    """This rank's exchange buffer, mapped by every rank through CUDA IPC
    (iq36_tp_comm of include/iq36_b200.h)."""

    def __init__(self, rank: int, world: int, hidden: int, device: torch.device,
                 group: dist.ProcessGroup | None = None):
        lib = N.lib()
        self.rank, self.world, self.hidden = rank, world, hidden
        nbytes = lib.iq36_tp_comm_bytes(world, hidden)
        base = ctypes.c_void_p()
        with torch.cuda.device(device):
            N.call("iq36_tp_comm_alloc", nbytes, ctypes.byref(base))
            self.base = base.value
            handle = (ctypes.c_char * 64)()
            N.call("iq36_ipc_get_handle", self.base, handle)
            handles = [None] * world
            dist.all_gather_object(handles, bytes(handle), group=group)
            self.peer_bases = []
            for q in range(world):
                if q == rank:
                    self.peer_bases.append(self.base)
                    continue
                p = ctypes.c_void_p()
                h = (ctypes.c_char * 64).from_buffer_copy(handles[q])
                N.call("iq36_ipc_open_handle", h, ctypes.byref(p))
                self.peer_bases.append(p.value)
        off_flags = 2 * world * hidden * 4
        off_keys = off_flags + 256
        off_counter = off_keys + 2 * world * 8
        c = N.TpCommC()
        c.rank, c.world, c.hidden = rank, world, hidden
        for q, b in enumerate(self.peer_bases):
            c.peer_recv[q] = b
            c.peer_flags[q] = b + off_flags
            c.peer_keys[q] = b + off_keys
        c.local_recv = self.base
        c.local_flags = self.base + off_flags
        c.local_keys = self.base + off_keys
        c.counter = self.base + off_counter
        self.c = c
        # every rank's buffer zeroed and mapped before the first exchange
        dist.barrier(group=group)

    def close(self, group: dist.ProcessGroup | None = None) -> None:
        if self.base is None:
            return
        dist.barrier(group=group)
        for q, b in enumerate(self.peer_bases):
            if q != self.rank:
                N.call("iq36_ipc_close_handle", b)
        dist.barrier(group=group)
        N.call("iq36_tp_comm_free", self.base)
        self.base = None


# ---------------------------------------------------------------------------
# the runtime

class TPRuntime:
    """Rank r of a tensor-parallel decode of one sequence (see module doc)."""

    def __init__(self, cfg: ModelConfig, rank: int, world: int, device: torch.device,
                 seed: int = 0, max_ctx: int = 4608, block_seed: int = 1,
                 full: SyntheticWeights | None = None, group: dist.ProcessGroup | None = None):
        self.cfg, self.rank, self.world, self.dev = cfg, rank, world, torch.device(device)
        self.group = group
        full = full or SyntheticWeights(cfg, seed, self.dev)
        self.w = TPWeights(full, rank, world)
        del full
        torch.cuda.empty_cache()
        self.comm = TPComm(rank, world, cfg.hidden, self.dev, group)
        c, dev, W = cfg, self.dev, self.w
        f16, f32, i32 = torch.float16, torch.float32, torch.int32
        self.max_ctx = max_ctx
        nblk = (max_ctx + 15) // 16
        gen = torch.Generator().manual_seed(block_seed)
        self.block_table = torch.randperm(nblk, generator=gen).to(torch.int32).to(dev)
        self.kv, self.conv_state, self.rec_state = {}, {}, {}
        ch = (2 * W.nk + W.nv) * c.dk
        for l in range(c.layers):
            if c.is_attn(l):
                self.kv[l] = (torch.zeros(nblk, 16, 1, c.head_dim, dtype=f16, device=dev),
                              torch.zeros(nblk, 16, 1, c.head_dim, dtype=f16, device=dev))
            else:
                self.conv_state[l] = torch.zeros(ch, c.conv, dtype=f32, device=dev)
                self.rec_state[l] = torch.zeros(W.nv, c.dk, c.dk, dtype=f32, device=dev)
        grp = c.nq // c.nkv
        h = c.hidden
        self.token = torch.zeros(1, dtype=i32, device=dev)
        self.pos = torch.zeros(1, dtype=i32, device=dev)
        self.ctx = torch.ones(1, dtype=i32, device=dev)
        self.hres = torch.zeros(h, dtype=f32, device=dev)
        self.partial = torch.zeros(h, dtype=f32, device=dev)
        self.b_qfull = torch.empty(grp * 2 * c.head_dim, dtype=f16, device=dev)
        self.b_k = torch.empty(c.head_dim, dtype=f16, device=dev)
        self.b_v = torch.empty(c.head_dim, dtype=f16, device=dev)
        self.b_q = torch.empty(grp * c.head_dim, dtype=f16, device=dev)
        self.b_gate = torch.empty(grp * c.head_dim, dtype=f16, device=dev)
        self.b_attn = torch.empty(grp * c.head_dim, dtype=f16, device=dev)
        self.b_qkv = torch.empty(ch, dtype=f16, device=dev)
        self.b_z = torch.empty(W.nv * c.dk, dtype=f16, device=dev)
        self.b_a = torch.empty(W.nv, dtype=f16, device=dev)
        self.b_b = torch.empty(W.nv, dtype=f16, device=dev)
        self.b_act = torch.empty(ch, dtype=f16, device=dev)
        self.b_g = torch.empty(W.nv, dtype=f32, device=dev)
        self.b_beta = torch.empty(W.nv, dtype=f32, device=dev)
        self.b_dout = torch.empty(W.nv * c.dk, dtype=f16, device=dev)
        self.b_logits_r = torch.empty(c.experts, dtype=f32, device=dev)
        self.b_slogit = torch.empty(1, dtype=f32, device=dev)
        self.b_ids = torch.empty(c.topk, dtype=i32, device=dev)
        self.b_wts = torch.empty(c.topk, dtype=f32, device=dev)
        self.logits = torch.empty(W.vocab_n, dtype=f32, device=dev)
        self.ws_gqa = ops.paged_gqa_workspace(max_ctx, grp, 1, c.head_dim, dev)
        i_loc = W.layers[0]["bank"].intermediate
        self.ws_moe = ops.moe_layer_workspace(c.topk, h, i_loc, dev)
        self.ws_key = torch.empty(N.lib().iq36_tp_argmax_workspace_bytes(), dtype=torch.uint8,
                                  device=dev)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.stream = torch.cuda.Stream(device=dev)
        self.launches_per_step = 0

    # -- state --------------------------------------------------------------
    def reset(self) -> None:
        for kc, vc in self.kv.values():
            kc.zero_()
            vc.zero_()
        for t in self.conv_state.values():
            t.zero_()
        for t in self.rec_state.values():
            t.zero_()
        self.pos.zero_()
        self.ctx.fill_(1)

    def _allreduce(self) -> None:
        N.call("iq36_tp_allreduce_residual", ctypes.byref(self.comm.c), self.hres.data_ptr(),
               self.partial.data_ptr(), ops._stream(self.dev))

    # -- one decode step ----------------------------------------------------
    def enqueue_step(self) -> int:
        c, W = self.cfg, self.w
        D = c.head_dim
        ops.embed(W.embed, self.token, self.hres)
        n = 1
        for l in range(c.layers):
            L = W.layers[l]
            if c.is_attn(l):
                ops.u4_matvec_multi(None, [L["q"], L["k"], L["v"]],
                                    [self.b_qfull, self.b_k, self.b_v], x_f32=self.hres,
                                    norm_weight=L["in_norm"], norm_eps=c.eps)
                kc, vc = self.kv[l]
                ops.attn_prep(self.b_qfull, self.b_k, self.b_v, L["qn"], L["kn"], c.eps, self.pos,
                              self.block_table, kc, vc, self.b_q, self.b_gate,
                              rope_dim=c.rope_dim, rope_base=c.rope_base)
                grp = c.nq // c.nkv
                ops.paged_gqa_decode(self.b_q.view(grp, D), kc, vc, self.block_table,
                                     self.max_ctx, 1.0 / math.sqrt(D), gate=self.b_gate,
                                     ctx_len_dev=self.ctx, workspace=self.ws_gqa,
                                     out=self.b_attn)
                x16 = self.b_attn[W.h_off * D:(W.h_off + W.nh) * D]
                ops.u4_matvec_multi(x16, [L["o"]], [self.partial])
                n += 5
            else:
                ops.u4_matvec_multi(None, [L["qkv"], L["z"], L["a"], L["b"]],
                                    [self.b_qkv, self.b_z, self.b_a, self.b_b], x_f32=self.hres,
                                    norm_weight=L["in_norm"], norm_eps=c.eps)
                ops.delta_prep(self.b_qkv, self.conv_state[l], L["conv_w"], self.b_a, self.b_b,
                               L["a_log"], L["dt_bias"], self.b_act, self.b_g, self.b_beta)
                ops.delta_step(self.b_act, self.b_g, self.b_beta, self.rec_state[l], self.b_z,
                               L["dnorm"], c.eps, W.nk, W.nv, self.b_dout, head_dim=c.dk)
                ops.u4_matvec_multi(self.b_dout, [L["out"]], [self.partial])
                n += 4
            self._allreduce()
            n += 1
            n += self._enqueue_moe(L)
            self._allreduce()
            n += 1
        ops.u4_matvec_multi(None, [W.lm_head], [self.logits], x_f32=self.hres,
                            norm_weight=W.final_norm, norm_eps=c.eps)
        N.call("iq36_tp_argmax", ctypes.byref(self.comm.c), self.logits.data_ptr(), W.vocab_n,
               W.vocab_lo, self.token.data_ptr(), self.ws_key.data_ptr(), ops._stream(self.dev))
        N.call("iq36_decode_positions", self.pos.data_ptr(), self.ctx.data_ptr(), 1,
               ops._stream(self.dev))
        return n + 4

    def _enqueue_moe(self, L: dict) -> int:
        c, W = self.cfg, self.w
        st = ops._stream(self.dev)
        if W.expert_rows:
            rb, sb = L["bank"].c(), L["shared"].c()
            N.call("iq36_moe_layer_decode_partial", self.hres.data_ptr(), c.hidden,
                   L["post_norm"].data_ptr(), c.eps, L["router"].data_ptr(), L["sgate"].data_ptr(),
                   c.topk, ctypes.byref(rb), ctypes.byref(sb), self.b_ids.data_ptr(),
                   self.b_wts.data_ptr(), self.b_logits_r.data_ptr(), self.b_slogit.data_ptr(),
                   self.partial.data_ptr(), self.ws_moe.data_ptr(), self.ws_moe.numel(), st)
            return 1
        # expert-sharded (P = 8): replicated router, this rank's experts
        N.call("iq36_router_logits", None, self.hres.data_ptr(), L["post_norm"].data_ptr(), c.eps,
               1, c.hidden, L["router"].data_ptr(), c.experts, L["sgate"].data_ptr(),
               self.b_logits_r.data_ptr(), self.b_slogit.data_ptr(), st)
        N.call("iq36_router_select", self.b_logits_r.data_ptr(), 1, c.experts, c.topk,
               self.b_ids.data_ptr(), self.b_wts.data_ptr(), st)
        rb = L["bank"].c()
        sb = L["shared"].c() if L["shared"] is not None else None
        N.call("iq36_moe_decode_sharded", None, self.hres.data_ptr(), L["post_norm"].data_ptr(),
               c.eps, self.b_ids.data_ptr(), self.b_wts.data_ptr(), c.topk, ctypes.byref(rb),
               L["expert_lo"], ctypes.byref(sb) if sb is not None else None,
               self.b_slogit.data_ptr() if sb is not None else None, self.partial.data_ptr(),
               N.F32, 0, self.ws_moe.data_ptr(), self.ws_moe.numel(), st)
        return 4

    def capture(self) -> None:
        """Record one decode step as a CUDA graph; as Qwen36Runtime.capture,
        call it before the prompt (it resets the sequence). Every rank must
        call it at the same point (its warm-up step exchanges with peers)."""
        torch.cuda.synchronize(self.dev)
        if int(self.pos.item()) != 0:
            raise RuntimeError("capture() resets the sequence; call it before the prompt")
        tok = self.token.clone()
        with torch.cuda.stream(self.stream):
            self.enqueue_step()
        self.stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self.stream):
            self.launches_per_step = self.enqueue_step()
        self.graph = g
        self.reset()
        self.token.copy_(tok)
        torch.cuda.synchronize(self.dev)

    def step(self) -> None:
        if self.graph is not None:
            self.graph.replay()
        else:
            self.enqueue_step()

    def prefill(self, tokens) -> None:
        """Feed prompt tokens one decode step each (every rank the same tokens)."""
        toks = torch.as_tensor(tokens, dtype=torch.int32).pin_memory()
        for i in range(toks.numel()):
            self.token.copy_(toks[i:i + 1], non_blocking=True)
            self.step()

    def close(self) -> None:
        """Release the graph (it holds no collective) and the exchange mappings."""
        torch.cuda.synchronize(self.dev)
        self.graph = None
        self.comm.close(self.group)
