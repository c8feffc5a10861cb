"""Batch-1 runtime of the synthetic Qwen3.6-35B-A3B-shaped model (config 4).

Mirrors the reference's host loop (engine/service/iq36_server/runtime.py:
461-585: prefill the prompt, then a greedy decode loop feeding each argmax token
back) over the B200 ops of ``engine.ops``. Weights are random-init with the
shared synthetic generator (include/iq36_synth.h), generated directly on the
device. One decode step is a fixed sequence of ~370 kernel launches (per layer:
fused RMSNorm + multi-output u4 GEMV, DeltaNet or attention core, output
projection into the fp32 residual, router + experts into the residual);
``capture()`` records it once as a CUDA graph whose inputs (token, position,
context length) live in device memory, so every later token is one graph
replay with no host work.

Layer order per the reference graph: layer l is full attention when
l % 4 == 3 (tools/intel_qwen36_openvino_fixed_fc.py:17, FULL_ATTENTION_LAYERS
= range(3, 40, 4)), DeltaNet otherwise; every layer ends with the MoE block.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import asdict, dataclass

import torch

from . import _native as N
from . import ops

# slots of include/iq36_synth.h (enum iq36_slot)
T_EMBED, T_LM_HEAD, T_FINAL_NORM = 1, 2, 3
T_IN_NORM, T_POST_NORM = 8, 9
T_Q, T_K, T_V, T_O, T_QNORM, T_KNORM = 10, 11, 12, 13, 14, 15
T_QKV, T_Z, T_A, T_B, T_OUT, T_CONV, T_ALOG, T_DTB, T_DNORM = 16, 17, 18, 19, 20, 21, 22, 23, 24
T_ROUTER, T_SGATE, T_GU, T_DOWN, T_SGU, T_SDOWN = 25, 26, 27, 28, 29, 30


@dataclass
class ModelConfig:
    """BASELINE config 4 (Qwen3.6-35B-A3B shape); smaller values for tests."""

    hidden: int = 2048
    layers: int = 40
    attn_interval: int = 4
    nq: int = 16
    nkv: int = 2
    head_dim: int = 256
    rope_dim: int = 64
    nk: int = 16
    nv: int = 32
    dk: int = 128
    conv: int = 4
    experts: int = 256
    topk: int = 8
    inter: int = 512
    shared_inter: int = 512
    vocab: int = 248320
    group: int = 128      # experts, shared expert, LM head
    rope_base: float = 1e7
    eps: float = 1e-6
    # attention q/k/v/o and DeltaNet in/out projections (the reference's fixed
    # FCs; its checkpoint quantises them at group 64, fixed_fc.py:26); 0 = group
    fc_group: int = 0

    @property
    def proj_group(self) -> int:
        return self.fc_group or self.group

    def as_dict(self) -> dict:
        return asdict(self)

    def is_attn(self, layer: int) -> bool:
        return layer % self.attn_interval == self.attn_interval - 1

    def decode_bytes_per_token(self, ctx: int) -> int:
        """Algorithmic HBM bytes of one decode step at context ctx: every u4
        weight (codes + scales + zero points) read once, fp16 router/shared-gate
        weights, the KV cache of the attention layers, and the DeltaNet state
        read and written once."""
        h = self.hidden

        def u4(rows, k, g=self.group):
            return rows * k // 2 + rows * (k // g) * 2 + rows * (k // g) // 2

        def fc(rows, k):
            return u4(rows, k, self.proj_group)

        n_attn = sum(self.is_attn(l) for l in range(self.layers))
        n_delta = self.layers - n_attn
        attn = fc(2 * self.nq * self.head_dim, h) + 2 * fc(self.nkv * self.head_dim, h) + fc(
            h, self.nq * self.head_dim)
        c = (2 * self.nk + self.nv) * self.dk
        delta = fc(c, h) + fc(self.nv * self.dk, h) + 2 * fc(self.nv, h) + fc(h, self.nv * self.dk)
        moe = (self.experts * h * 2 + h * 2 + (self.topk + 1) * (
            u4(2 * self.inter, h) + u4(h, self.inter)))
        lm = u4(self.vocab, h)
        kv = n_attn * ctx * self.nkv * self.head_dim * 2 * 2
        state = n_delta * self.nv * self.dk * self.dk * 4 * 2
        return n_attn * attn + n_delta * delta + self.layers * moe + lm + kv + state


def _spec(slot: int, sub: int) -> tuple[int, float, float]:
    kind, lo, hi = ctypes.c_int32(), ctypes.c_float(), ctypes.c_float()
    N.lib().iq36_synth_tensor_spec(slot, sub, ctypes.byref(kind), ctypes.byref(lo),
                                   ctypes.byref(hi))
    return kind.value, lo.value, hi.value


def _tid(layer: int, slot: int, sub: int) -> int:
    return N.lib().iq36_synth_tensor_id(layer, slot, sub)


class SyntheticWeights:
    """All device weights of the random-init model, generated on the device."""

    def __init__(self, cfg: ModelConfig, seed: int, device: torch.device):
        self.cfg, self.seed, self.dev = cfg, seed, device
        c, h, g = cfg, cfg.hidden, cfg.group
        fc = cfg.proj_group
        self.layers = []
        for l in range(c.layers):
            L = {"in_norm": self._f32(h, l, T_IN_NORM), "post_norm": self._f32(h, l, T_POST_NORM)}
            if c.is_attn(l):
                L["q"] = self._u4(2 * c.nq * c.head_dim, h, l, T_Q, fc)
                L["k"] = self._u4(c.nkv * c.head_dim, h, l, T_K, fc)
                L["v"] = self._u4(c.nkv * c.head_dim, h, l, T_V, fc)
                L["o"] = self._u4(h, c.nq * c.head_dim, l, T_O, fc)
                L["qn"] = self._f32(c.head_dim, l, T_QNORM)
                L["kn"] = self._f32(c.head_dim, l, T_KNORM)
            else:
                ch = (2 * c.nk + c.nv) * c.dk
                L["qkv"] = self._u4(ch, h, l, T_QKV, fc)
                L["z"] = self._u4(c.nv * c.dk, h, l, T_Z, fc)
                L["a"] = self._u4(c.nv, h, l, T_A, fc)
                L["b"] = self._u4(c.nv, h, l, T_B, fc)
                L["ab"] = self._gate_pair(L["a"], L["b"])
                L["out"] = self._u4(h, c.nv * c.dk, l, T_OUT, fc)
                L["conv_w"] = self._f32(ch * c.conv, l, T_CONV)
                L["a_log"] = self._f32(c.nv, l, T_ALOG)
                L["dt_bias"] = self._f32(c.nv, l, T_DTB)
                L["dnorm"] = self._f32(c.dk, l, T_DNORM)
            L["router"] = self._f16((c.experts, h), l, T_ROUTER)
            L["sgate"] = self._f16((1, h), l, T_SGATE)
            gu = self._u4(c.experts * 2 * c.inter, h, l, T_GU)
            dn = self._u4(c.experts * h, c.inter, l, T_DOWN)
            L["bank"] = ops.ExpertBank(
                gu.weight.view(c.experts, 2 * c.inter, h // 2),
                gu.scale.view(c.experts, 2 * c.inter, h // g), gu.zp.view(c.experts, -1),
                dn.weight.view(c.experts, h, c.inter // 2),
                dn.scale.view(c.experts, h, c.inter // g), dn.zp.view(c.experts, -1), g)
            sgu = self._u4(2 * c.shared_inter, h, l, T_SGU)
            sdn = self._u4(h, c.shared_inter, l, T_SDOWN)
            L["shared"] = ops.ExpertBank(
                sgu.weight.view(1, 2 * c.shared_inter, h // 2),
                sgu.scale.view(1, 2 * c.shared_inter, h // g), sgu.zp.view(1, -1),
                sdn.weight.view(1, h, c.shared_inter // 2),
                sdn.scale.view(1, h, c.shared_inter // g), sdn.zp.view(1, -1), g)
            self.layers.append(L)
        self.embed = self._f16((c.vocab, h), -1, T_EMBED)
        self.final_norm = self._f32(h, -1, T_FINAL_NORM)
        self.lm_head = self._u4(c.vocab, h, -1, T_LM_HEAD)
        torch.cuda.synchronize(device)

    def _fill(self, t: torch.Tensor, layer: int, slot: int, sub: int) -> torch.Tensor:
        kind, lo, hi = _spec(slot, sub)
        return ops.synth_fill(t, kind, self.seed, _tid(layer, slot, sub), lo, hi)

    def _f32(self, n, layer, slot):
        return self._fill(torch.empty(n, dtype=torch.float32, device=self.dev), layer, slot, 0)

    def _f16(self, shape, layer, slot):
        return self._fill(torch.empty(shape, dtype=torch.float16, device=self.dev), layer, slot, 0)

    @staticmethod
    def _gate_pair(a: ops.U4Weight, b: ops.U4Weight) -> ops.U4Weight:
        """[a; b; 0] padded to 256 rows: one batched GEMM (whose row count is a
        multiple of 256) produces both DeltaNet gate projections for the prompt.
        Zero scales make the padding rows exactly 0."""
        n = a.rows + b.rows
        pad = (-n) % 256
        w = torch.cat([a.weight, b.weight, a.weight.new_zeros(pad, a.weight.shape[1])])
        sc = torch.cat([a.scale, b.scale, a.scale.new_zeros(pad, a.scale.shape[1])])
        zp = torch.cat([a.zp.view(-1), b.zp.view(-1),
                        a.zp.new_zeros(pad * a.scale.shape[1] // 2)])
        return ops.U4Weight(w, sc, zp, a.group)

    def _u4(self, rows, k, layer, slot, group: int = 0) -> ops.U4Weight:
        g = group or self.cfg.group
        w = self._fill(torch.empty(rows, k // 2, dtype=torch.uint8, device=self.dev), layer, slot, 0)
        s = self._fill(torch.empty(rows, k // g, dtype=torch.float16, device=self.dev), layer, slot, 1)
        z = self._fill(torch.empty(rows * (k // g) // 2, dtype=torch.uint8, device=self.dev),
                       layer, slot, 2)
        return ops.U4Weight(w, s, z, g)


class Qwen36Runtime:
    """Device state + the decode step of the synthetic model."""

    def __init__(self, cfg: ModelConfig, seed: int = 0, max_ctx: int = 4608,
                 device: str | torch.device = "cuda:0", block_seed: int = 1,
                 weights: SyntheticWeights | None = None, lm_head: str = "full",
                 lm_head_capacity: int = 1024):
        if lm_head not in ("full", "certified"):
            raise ValueError("lm_head must be 'full' or 'certified'")
        self.cfg = cfg
        self.dev = torch.device(device)
        self.w = weights or SyntheticWeights(cfg, seed, self.dev)
        self.max_ctx = max_ctx
        c, dev = cfg, self.dev
        f16, f32, i32 = torch.float16, torch.float32, torch.int32
        nblk = (max_ctx + 15) // 16
        gen = torch.Generator().manual_seed(block_seed)
        # seeded random block table: pages of the cache are deliberately scattered
        self.block_table = torch.randperm(nblk, generator=gen).to(torch.int32).to(dev)
        self.kv = {}
        self.conv_state, self.rec_state = {}, {}
        for l in range(c.layers):
            if c.is_attn(l):
                self.kv[l] = (torch.zeros(nblk, 16, c.nkv, c.head_dim, dtype=f16, device=dev),
                              torch.zeros(nblk, 16, c.nkv, c.head_dim, dtype=f16, device=dev))
            else:
                ch = (2 * c.nk + c.nv) * c.dk
                self.conv_state[l] = torch.zeros(ch, c.conv, dtype=f32, device=dev)
                self.rec_state[l] = torch.zeros(c.nv, c.dk, c.dk, dtype=f32, device=dev)
        h = c.hidden
        self.token = torch.zeros(1, dtype=i32, device=dev)   # input token of the step
        self.pos = torch.zeros(1, dtype=i32, device=dev)     # position of the step
        self.ctx = torch.ones(1, dtype=i32, device=dev)      # pos + 1
        self.hres = torch.zeros(h, dtype=f32, device=dev)    # fp32 residual stream
        ch = (2 * c.nk + c.nv) * c.dk
        self.b_qkv = torch.empty(ch, dtype=f16, device=dev)
        self.b_z = torch.empty(c.nv * c.dk, dtype=f16, device=dev)
        self.b_a = torch.empty(c.nv, dtype=f16, device=dev)
        self.b_b = torch.empty(c.nv, dtype=f16, device=dev)
        self.b_act = torch.empty(ch, dtype=f16, device=dev)
        self.b_g = torch.empty(c.nv, dtype=f32, device=dev)
        self.b_beta = torch.empty(c.nv, dtype=f32, device=dev)
        self.b_dout = torch.empty(c.nv * c.dk, dtype=f16, device=dev)
        self.b_qfull = torch.empty(2 * c.nq * c.head_dim, dtype=f16, device=dev)
        self.b_k = torch.empty(c.nkv * c.head_dim, dtype=f16, device=dev)
        self.b_v = torch.empty(c.nkv * c.head_dim, dtype=f16, device=dev)
        self.b_q = torch.empty(c.nq * c.head_dim, dtype=f16, device=dev)
        self.b_gate = torch.empty(c.nq * c.head_dim, dtype=f16, device=dev)
        self.b_attn = torch.empty(c.nq * c.head_dim, dtype=f16, device=dev)
        self.b_x2 = torch.empty(h, dtype=f16, device=dev)
        self.b_logits_r = torch.empty(c.experts, dtype=f32, device=dev)
        self.b_slogit = torch.empty(1, dtype=f32, device=dev)
        self.b_ids = torch.empty(c.topk, dtype=i32, device=dev)
        self.b_wts = torch.empty(c.topk, dtype=f32, device=dev)
        self.logits = torch.empty(c.vocab, dtype=f32, device=dev)
        self.ws_gqa = ops.paged_gqa_workspace(max_ctx, c.nq, c.nkv, c.head_dim, dev)
        self.ws_moe = ops.moe_layer_workspace(c.topk, h, c.inter, dev)
        self.ws_argmax = torch.empty(N.lib().iq36_argmax_workspace_bytes(), dtype=torch.uint8,
                                     device=dev)
        # LM head: "full" computes every logit; "certified" computes the chunk
        # of the step's input token, bounds every other row and computes only
        # the chunks that can still win (same greedy token; only the evaluated
        # chunks' logits are written, their count lands in lm_evaluated).
        self.lm_mode = lm_head
        self.lm_capacity = lm_head_capacity
        if lm_head == "certified":
            self.lm_table = ops.lm_head_cert_table(self.w.lm_head)
            self.ws_cert = torch.empty(
                N.lib().iq36_lm_head_top1_certified_workspace_bytes(c.vocab, h),
                dtype=torch.uint8, device=dev)
            self.lm_evaluated = torch.zeros(1, dtype=i32, device=dev)
        self._pf: dict | None = None  # batched-prefill buffers (sized on first use)
        # Optional step trace (tests): when set before capture(), every step
        # also copies the residual entering each layer (and leaving the last)
        # into trace [layers + 1, hidden], each layer's routed ids into
        # trace_ids [layers, topk] and its router logits into trace_router
        # [layers, experts].
        self.trace: torch.Tensor | None = None
        self.trace_ids: torch.Tensor | None = None
        self.trace_router: torch.Tensor | None = None
        self.graph: torch.cuda.CUDAGraph | None = None
        self.stream = torch.cuda.Stream(device=dev)
        self.launches_per_step = 0

    # -- state ---------------------------------------------------------------
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

    # -- one decode step (enqueue only) --------------------------------------
    def enqueue_step(self) -> int:
        """Enqueue one decode step on the current stream; returns the number of
        kernel launches."""
        c, W = self.cfg, self.w
        ops.embed(W.embed, self.token, self.hres)
        n = 1
        for l in range(c.layers):
            if self.trace is not None:
                self.trace[l].copy_(self.hres)
            n += self.enqueue_layer(l)
            if self.trace is not None:
                self.trace_ids[l].copy_(self.b_ids)
                self.trace_router[l].copy_(self.b_logits_r)
        if self.trace is not None:
            self.trace[c.layers].copy_(self.hres)
        if self.lm_mode == "certified":
            # the input token seeds the certificate; the token buffer is
            # rewritten only by the last kernel, after the seed was read
            ops.lm_head_top1_certified(W.lm_head, self.lm_table, self.token, self.logits,
                                       self.token, x_f32=self.hres, norm_weight=W.final_norm,
                                       norm_eps=c.eps, capacity_chunks=self.lm_capacity,
                                       evaluated=self.lm_evaluated, workspace=self.ws_cert)
            n += 4
        else:
            ops.u4_matvec_multi(None, [W.lm_head], [self.logits], x_f32=self.hres,
                                norm_weight=W.final_norm, norm_eps=c.eps)
            ops.argmax(self.logits, self.token, self.ws_argmax)
            n += 2
        N.call("iq36_decode_positions", self.pos.data_ptr(), self.ctx.data_ptr(), 1,
               ops._stream(self.dev))
        return n + 1

    def enqueue_layer(self, l: int) -> int:
        """Enqueue decoder layer l of the decode step on the fp32 residual
        ``hres`` at the device position ``pos`` (attention or DeltaNet block,
        then the MoE block); returns the number of launches."""
        c, W = self.cfg, self.w
        n = 0
        L = W.layers[l]
        if c.is_attn(l):
            ops.u4_matvec_multi(None, [L["q"], L["k"], L["v"]],
                                [self.b_qfull, self.b_k, self.b_v], x_f32=self.hres,
                                norm_weight=L["in_norm"], norm_eps=c.eps)
            kc, vc = self.kv[l]
            ops.attn_prep(self.b_qfull, self.b_k, self.b_v, L["qn"], L["kn"], c.eps, self.pos,
                          self.block_table, kc, vc, self.b_q, self.b_gate,
                          rope_dim=c.rope_dim, rope_base=c.rope_base)
            ops.paged_gqa_decode(self.b_q.view(c.nq, c.head_dim), kc, vc, self.block_table,
                                 self.max_ctx, 1.0 / math.sqrt(c.head_dim),
                                 gate=self.b_gate, ctx_len_dev=self.ctx,
                                 workspace=self.ws_gqa, out=self.b_attn)
            ops.u4_matvec_multi(self.b_attn, [L["o"]], [self.hres], accumulate=[True])
            n += 5
        else:
            ops.u4_matvec_multi(None, [L["qkv"], L["z"], L["a"], L["b"]],
                                [self.b_qkv, self.b_z, self.b_a, self.b_b], x_f32=self.hres,
                                norm_weight=L["in_norm"], norm_eps=c.eps)
            ops.delta_prep(self.b_qkv, self.conv_state[l], L["conv_w"], self.b_a, self.b_b,
                           L["a_log"], L["dt_bias"], self.b_act, self.b_g, self.b_beta)
            ops.delta_step(self.b_act, self.b_g, self.b_beta, self.rec_state[l], self.b_z,
                           L["dnorm"], c.eps, c.nk, c.nv, self.b_dout, head_dim=c.dk)
            ops.u4_matvec_multi(self.b_dout, [L["out"]], [self.hres], accumulate=[True])
            n += 4
        # post-attention RMSNorm fused into the router and gate_up prologues
        # (reference run_qwen36_moe_ffn_layer)
        ops.moe_layer_decode(self.hres, L["post_norm"], L["router"], L["sgate"], L["bank"],
                             L["shared"], self.b_ids, self.b_wts, self.b_logits_r,
                             self.b_slogit, workspace=self.ws_moe, k=c.topk, norm_eps=c.eps)
        n += 1
        return n

    def enqueue_gemvs_only(self) -> tuple[int, int]:
        """Enqueue just the multi-output u4 GEMV launches of one decode step
        (same weights and buffers; used to time that kernel alone). Returns
        (algorithmic bytes, launches): u4 codes + scales + zero points, the
        activation read (fp32 residual + norm weight when the RMSNorm is fused,
        else fp16), and the outputs written (fp32 residual updates count a
        read and a write)."""
        c, W = self.cfg, self.w
        nbytes, n = 0, 0

        def u4b(w: ops.U4Weight) -> int:
            return w.weight.numel() + w.scale.numel() * 2 + w.zp.numel()

        for l in range(c.layers):
            L = W.layers[l]
            if c.is_attn(l):
                ins = [L["q"], L["k"], L["v"]]
                outs = [self.b_qfull, self.b_k, self.b_v]
                out_w, x16 = L["o"], self.b_attn
            else:
                ins = [L["qkv"], L["z"], L["a"], L["b"]]
                outs = [self.b_qkv, self.b_z, self.b_a, self.b_b]
                out_w, x16 = L["out"], self.b_dout
            ops.u4_matvec_multi(None, ins, outs, x_f32=self.hres, norm_weight=L["in_norm"],
                                norm_eps=c.eps)
            nbytes += sum(u4b(w) for w in ins) + c.hidden * 8 + sum(o.numel() * 2 for o in outs)
            ops.u4_matvec_multi(x16, [out_w], [self.hres], accumulate=[True])
            nbytes += u4b(out_w) + x16.numel() * 2 + c.hidden * 8
            n += 2
        ops.u4_matvec_multi(None, [W.lm_head], [self.logits], x_f32=self.hres,
                            norm_weight=W.final_norm, norm_eps=c.eps)
        nbytes += u4b(W.lm_head) + c.hidden * 8 + c.vocab * 4
        n += 1
        return nbytes, n

    def capture(self) -> None:
        """Record one decode step as a CUDA graph (state read from device).

        Capturing runs one warm-up step eagerly and then resets the sequence
        (KV cache, conv and recurrent states zeroed, position 0), so it must be
        called before the prompt: a runtime whose position is not 0 raises
        instead of silently dropping its state."""
        torch.cuda.synchronize(self.dev)
        if int(self.pos.item()) != 0:
            raise RuntimeError("capture() resets the sequence; call it before prefill "
                               f"(position is {int(self.pos.item())})")
        saved = (self.pos.clone(), self.token.clone())
        with torch.cuda.stream(self.stream):
            self.enqueue_step()  # warm-up outside capture (also runs lazy init)
        self.stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self.stream):
            self.launches_per_step = self.enqueue_step()
        self.graph = g
        # the warm-up step advanced the state: restore it
        self.reset()
        self.pos.copy_(saved[0])
        self.ctx.copy_(saved[0] + 1)
        self.token.copy_(saved[1])
        torch.cuda.synchronize(self.dev)

    def step(self) -> None:
        """Run one decode step (graph replay if captured)."""
        if self.graph is not None:
            self.graph.replay()
        else:
            self.enqueue_step()

    # -- batched prefill ------------------------------------------------------
    def _prefill_buffers(self, T: int) -> dict:
        if self._pf is not None and self._pf["T"] >= T:
            return self._pf
        c, dev = self.cfg, self.dev
        f16, f32, i32 = torch.float16, torch.float32, torch.int32
        h, hd = c.hidden, c.head_dim
        ch = (2 * c.nk + c.nv) * c.dk
        gemm_k = max(h, c.nq * hd, c.nv * c.dk)
        self._pf = {
            "T": T,
            "tok": torch.empty(T, dtype=i32, device=dev),
            "h": torch.empty(T, h, dtype=f32, device=dev),
            "qfull": torch.empty(T, 2 * c.nq * hd, dtype=f16, device=dev),
            "k": torch.empty(T, c.nkv * hd, dtype=f16, device=dev),
            "v": torch.empty(T, c.nkv * hd, dtype=f16, device=dev),
            "q": torch.empty(T, c.nq * hd, dtype=f16, device=dev),
            "gate": torch.empty(T, c.nq * hd, dtype=f16, device=dev),
            "attn": torch.empty(T, c.nq * hd, dtype=f16, device=dev),
            "qkv": torch.empty(T, ch, dtype=f16, device=dev),
            "z": torch.empty(T, c.nv * c.dk, dtype=f16, device=dev),
            "ab": torch.empty(T, 256 * ((2 * c.nv + 255) // 256), dtype=f16, device=dev),
            "dout": torch.empty(T, c.nv * c.dk, dtype=f16, device=dev),
            "ids": torch.empty(T, c.topk, dtype=i32, device=dev),
            "wts": torch.empty(T, c.topk, dtype=f32, device=dev),
            "logits_r": torch.empty(T, c.experts, dtype=f32, device=dev),
            "gws": torch.empty(N.lib().iq36_u4_gemm_workspace_bytes(T, gemm_k), dtype=torch.uint8,
                               device=dev),
            "dws": ops.delta_prefill_workspace(T, c.nk, c.nv, dev),
            "mws": ops.moe_layer_prefill_workspace(T, c.topk, c.experts, h, c.inter, dev),
        }
        return self._pf

    def enqueue_prefill_chunk(self, T: int) -> int:
        """Enqueue the batched forward of the T prompt tokens already in the
        prefill buffer's ``tok`` rows, at positions pos .. pos+T-1: every
        projection as a tcgen05 u4 GEMM over the T rows, the DeltaNet and
        attention cores over the whole chunk, the MoE block as the grouped
        prefill; then the LM head and argmax of the last row, and pos += T.
        Returns the number of launches."""
        c, W, B = self.cfg, self.w, self._pf
        assert B is not None and B["T"] >= T
        h = B["h"][:T]
        ops.embed_batch(W.embed, B["tok"][:T], h)
        n = 1
        for l in range(c.layers):
            n += self.enqueue_prefill_layer(l, T)
        ops.u4_matvec_multi(None, [W.lm_head], [self.logits], x_f32=h[T - 1],
                            norm_weight=W.final_norm, norm_eps=c.eps)
        ops.argmax(self.logits, self.token, self.ws_argmax)
        N.call("iq36_decode_positions", self.pos.data_ptr(), self.ctx.data_ptr(), T,
               ops._stream(self.dev))
        return n + 4

    def enqueue_prefill_layer(self, l: int, T: int) -> int:
        """Enqueue decoder layer l over the T prompt rows of the prefill
        buffer's fp32 residual ``h`` at positions pos .. pos+T-1 (the batched
        form of ``enqueue_layer``); returns the number of launches."""
        c, W, B = self.cfg, self.w, self._pf
        assert B is not None and B["T"] >= T
        hd = c.head_dim
        sl = lambda name: B[name][:T]
        h = sl("h")
        ws = B["gws"]
        L = W.layers[l]
        if c.is_attn(l):
            ops.u4_gemm_multi(h, [L["q"], L["k"], L["v"]], [sl("qfull"), sl("k"), sl("v")],
                              norm_weight=L["in_norm"], norm_eps=c.eps, workspace=ws)
            kc, vc = self.kv[l]
            ops.attn_prep_batch(sl("qfull"), sl("k"), sl("v"), L["qn"], L["kn"], c.eps,
                                self.pos, self.block_table, kc, vc, sl("q"), sl("gate"),
                                rope_dim=c.rope_dim, rope_base=c.rope_base)
            ops.attn_prefill(sl("q").view(T, c.nq, hd), kc, vc, self.block_table, self.pos,
                             1.0 / math.sqrt(hd), gate=sl("gate").view(T, c.nq, hd),
                             out=sl("attn").view(T, c.nq, hd))
            ops.u4_gemm(sl("attn"), L["o"], out=h, accumulate=True, workspace=ws)
            n = 6
        else:
            ops.u4_gemm_multi(h, [L["qkv"], L["z"], L["ab"]], [sl("qkv"), sl("z"), sl("ab")],
                              norm_weight=L["in_norm"], norm_eps=c.eps, workspace=ws)
            ab = sl("ab")
            ops.delta_prefill(sl("qkv"), self.conv_state[l], L["conv_w"], ab[:, :c.nv],
                              ab[:, c.nv:2 * c.nv], L["a_log"], L["dt_bias"],
                              self.rec_state[l], sl("z"), L["dnorm"], c.eps, c.nk, c.nv,
                              sl("dout"), workspace=B["dws"])
            ops.u4_gemm(sl("dout"), L["out"], out=h, accumulate=True, workspace=ws)
            n = 9
        ops.moe_layer_prefill(h, L["post_norm"], L["router"], L["sgate"], L["bank"],
                              L["shared"], sl("ids"), sl("wts"), sl("logits_r"),
                              workspace=B["mws"], k=c.topk, norm_eps=c.eps)
        return n + 14

    def prefill_batched(self, tokens: list[int] | torch.Tensor, chunk: int = 16384) -> int:
        """Batched prefill of the prompt in chunks of at most ``chunk`` tokens
        (state, KV cache and position carry across chunks); leaves the greedy
        token after the last prompt token in ``self.token``. Returns the number
        of launches enqueued. The reference prefills in tile-aligned chunks of
        8192/4096/2048/32 tokens and finishes the last 0..31 tokens with
        one-token calls (engine/service/iq36_server/runtime.py:25, 334-352,
        501); every kernel here takes any token count, so a chunk is simply up
        to ``chunk`` tokens and the tail needs no special case. 16384-token
        chunks prefill a 32768-token prompt 3.5% faster than 8192 (bigger GEMM
        tiles per launch) for about twice the prefill buffers."""
        toks = torch.as_tensor(tokens, dtype=torch.int32).reshape(-1)
        total = toks.numel()
        if total < 1:
            raise ValueError("empty prompt")
        p0 = int(self.pos.item())
        if p0 + total > self.max_ctx:
            raise ValueError(f"prompt of {total} tokens at position {p0} exceeds the "
                             f"{self.max_ctx}-token cache")
        B = self._prefill_buffers(min(chunk, total))
        src = toks if toks.is_cuda else toks.pin_memory()
        n = 0
        for s0 in range(0, total, chunk):
            T = min(chunk, total - s0)
            B["tok"][:T].copy_(src[s0:s0 + T], non_blocking=True)
            n += self.enqueue_prefill_chunk(T)
        return n

    # -- host loop (reference runtime.py:461-585) ----------------------------
    def prefill(self, tokens: list[int] | torch.Tensor, keep_logits: bool = False):
        """Feed prompt tokens one step each; returns the greedy token after the
        last prompt token (and the per-position logits if asked)."""
        toks = torch.as_tensor(tokens, dtype=torch.int32).pin_memory()
        kept = []
        for i in range(toks.numel()):
            self.token.copy_(toks[i:i + 1], non_blocking=True)
            self.step()
            if keep_logits:
                kept.append(self.logits.clone())
        return (kept if keep_logits else None)

    def generate(self, prompt: list[int], n_new: int, keep_logits: bool = False):
        self.prefill(prompt, keep_logits=False)
        out, logits = [], []
        for _ in range(n_new):
            out.append(int(self.token.item()))
            if keep_logits:
                logits.append(self.logits.clone())
            self.step()
        return out, logits
