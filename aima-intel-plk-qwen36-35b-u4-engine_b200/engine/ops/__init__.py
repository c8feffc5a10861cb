"""engine.ops — the batch-1 hot-path operators behind one call each.

This is the operator boundary the reference reserves as ``engine/ops``
(reference engine/ops/README.md:1-7; the shipped boundary is its OpenVINO
custom-op contract, e.g. tools/intel_qwen36_openvino_fixed_fc.py:31-92 and
engine/openvino/custom/iq36_fixed_fc_multi_output.cl:36-44). Each function
takes and returns torch tensors on a CUDA device and calls the C ABI of
``libiq36_b200.so`` on the current stream. Shapes and dtypes are checked
here, mirroring the reference op classes (ValueError at build time), and the C
ABI checks them again; a failed C call raises ``Iq36Error``.

Operators (north-star names): ``u4_matvec`` / ``u4_matvec_multi`` (u4 GEMV),
``router_topk`` / ``router_select`` (router), ``moe_expert_ffn`` (routed +
shared experts, decode), ``moe_expert_ffn_prefill`` (grouped prefill),
``paged_gqa_decode`` (attention), plus the config-4 support ops.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from .. import _native as N

__all__ = [
    "U4Weight", "ExpertBank", "u4_matvec", "u4_matvec_multi", "router_logits", "router_select",
    "router_topk", "moe_expert_ffn", "moe_block_decode", "moe_expert_ffn_prefill",
    "paged_gqa_decode", "rms_norm", "attn_prep", "delta_prep", "delta_step", "embed", "argmax",
    "synth_fill",
]


def _ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    return t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return N.F32
    if dtype == torch.float16:
        return N.F16
    if dtype == torch.bfloat16:
        return N.BF16
    raise ValueError(f"unsupported output dtype {dtype}")


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _cuda(t: torch.Tensor, name: str, dtype: torch.dtype | None = None) -> None:
    _need(t.is_cuda, f"{name} must be a CUDA tensor")
    _need(t.is_contiguous(), f"{name} must be contiguous")
    if dtype is not None:
        _need(t.dtype == dtype, f"{name} must be {dtype}, got {t.dtype}")


@dataclass
class U4Weight:
    """One u4 group-wise asymmetric matrix [rows, K] (layout in include/iq36_b200.h)."""

    weight: torch.Tensor  # uint8 [rows, K/2]
    scale: torch.Tensor   # float16 [rows, K/G]
    zp: torch.Tensor      # uint8 [rows*K/G/2]
    group: int = 128

    @property
    def rows(self) -> int:
        return self.weight.shape[0]

    @property
    def k(self) -> int:
        return self.weight.shape[1] * 2

    def validate(self) -> None:
        _cuda(self.weight, "weight", torch.uint8)
        _cuda(self.scale, "scale", torch.float16)
        _cuda(self.zp, "zp", torch.uint8)
        ng = self.k // self.group
        _need(self.k % self.group == 0, "K must be a multiple of the group size")
        _need(tuple(self.scale.shape) == (self.rows, ng), "scale must be [rows, K/G]")
        _need(self.zp.numel() == self.rows * ng // 2, "zp must hold rows*K/G nibbles")

    def c(self) -> N.U4Matrix:
        return N.U4Matrix(self.weight.data_ptr(), self.scale.data_ptr(), self.zp.data_ptr(),
                          self.rows)


@dataclass
class ExpertBank:
    """E experts: gate_up [E, 2I, H] and down [E, H, I], u4 group G."""

    gate_up_weight: torch.Tensor  # uint8 [E, 2I, H/2]
    gate_up_scale: torch.Tensor   # float16 [E, 2I, H/G]
    gate_up_zp: torch.Tensor      # uint8 [E, 2I*H/G/2]
    down_weight: torch.Tensor     # uint8 [E, H, I/2]
    down_scale: torch.Tensor      # float16 [E, H, I/G]
    down_zp: torch.Tensor         # uint8 [E, H*I/G/2]
    group: int = 128

    @property
    def num_experts(self) -> int:
        return self.gate_up_weight.shape[0]

    @property
    def hidden(self) -> int:
        return self.gate_up_weight.shape[2] * 2

    @property
    def intermediate(self) -> int:
        return self.gate_up_weight.shape[1] // 2

    def c(self) -> N.ExpertBankC:
        for name in ("gate_up_weight", "gate_up_scale", "gate_up_zp", "down_weight", "down_scale",
                     "down_zp"):
            _cuda(getattr(self, name), name)
        return N.ExpertBankC(self.gate_up_weight.data_ptr(), self.gate_up_scale.data_ptr(),
                             self.gate_up_zp.data_ptr(), self.down_weight.data_ptr(),
                             self.down_scale.data_ptr(), self.down_zp.data_ptr(),
                             self.num_experts, self.hidden, self.intermediate, self.group)


# ---------------------------------------------------------------------------
# (1) u4 GEMV


def u4_matvec(x: torch.Tensor, w: U4Weight, out_dtype: torch.dtype = torch.float32,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """y[n] = sum_k x[k] * (q[n,k] - zp[n,k/G]) * scale[n,k/G] (IQ36FixedFC1)."""
    _cuda(x, "x", torch.float16)
    w.validate()
    _need(x.numel() == w.k, f"x has {x.numel()} elements, weight K is {w.k}")
    if out is None:
        out = torch.empty(w.rows, dtype=out_dtype, device=x.device)
    m = w.c()
    N.call("iq36_u4_gemv", x.data_ptr(), w.k, w.group, ctypes.byref(m), out.data_ptr(),
           _dtype_code(out.dtype), _stream(x.device))
    return out


def u4_matvec_multi(x: torch.Tensor | None, weights: list[U4Weight],
                    outs: list[torch.Tensor], accumulate: list[bool] | None = None,
                    x_f32: torch.Tensor | None = None, norm_weight: torch.Tensor | None = None,
                    norm_eps: float = 1e-6) -> list[torch.Tensor]:
    """Arity 1..4 projections of one activation in one launch (IQ36FixedFC{1,3,4}).

    With ``x_f32`` and ``norm_weight`` the activation is RMS-normalised in the
    kernel prologue; ``x`` must then be None.
    """
    _need(1 <= len(weights) <= 4 and len(outs) == len(weights), "arity must be 1..4")
    acc = accumulate or [False] * len(weights)
    k, g = weights[0].k, weights[0].group
    projs = (N.U4Projection * len(weights))()
    for i, (w, o) in enumerate(zip(weights, outs)):
        w.validate()
        _need(w.k == k and w.group == g, "projections must share K and G")
        _cuda(o, f"out{i}")
        _need(o.numel() == w.rows, f"out{i} must have {w.rows} elements")
        projs[i] = N.U4Projection(w.c(), o.data_ptr(), _dtype_code(o.dtype), int(acc[i]))
    dev = (x if x is not None else x_f32).device
    N.call("iq36_u4_gemv_multi", _ptr(x), _ptr(x_f32), _ptr(norm_weight), norm_eps, k, g,
           len(weights), projs, _stream(dev))
    return outs


# ---------------------------------------------------------------------------
# (4) router


def router_logits(x: torch.Tensor, w_router: torch.Tensor,
                  w_shared_gate: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor | None]:
    """logits [T, E] fp32 (and the shared-expert gate logit [T]) of fp16 x [T, H]."""
    _cuda(x, "x", torch.float16)
    _cuda(w_router, "w_router", torch.float16)
    x2 = x.reshape(-1, x.shape[-1])
    t, h = x2.shape
    e = w_router.shape[0]
    _need(w_router.shape[1] == h, "router weight must be [E, H]")
    logits = torch.empty(t, e, dtype=torch.float32, device=x.device)
    sl = torch.empty(t, dtype=torch.float32, device=x.device) if w_shared_gate is not None else None
    N.call("iq36_router_logits", x2.data_ptr(), None, None, 0.0, t, h, w_router.data_ptr(), e,
           _ptr(w_shared_gate), logits.data_ptr(), _ptr(sl), _stream(x.device))
    return logits, sl


def router_select(logits: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Top-k expert ids (int32) and renormalised weights (fp32) per token,
    bit-exact to select_router_topk (reference gguf_loader.cpp:3733-3743)."""
    _cuda(logits, "logits", torch.float32)
    l2 = logits.reshape(-1, logits.shape[-1])
    t, e = l2.shape
    ids = torch.empty(t, k, dtype=torch.int32, device=logits.device)
    wts = torch.empty(t, k, dtype=torch.float32, device=logits.device)
    N.call("iq36_router_select", l2.data_ptr(), t, e, k, ids.data_ptr(), wts.data_ptr(),
           _stream(logits.device))
    return ids, wts


def router_topk(x: torch.Tensor, w_router: torch.Tensor, k: int = 8):
    """Router logits -> softmax -> top-k -> renormalise. Returns (ids, weights, logits)."""
    logits, _ = router_logits(x, w_router)
    ids, wts = router_select(logits, k)
    return ids, wts, logits


# ---------------------------------------------------------------------------
# (2) experts


def moe_expert_ffn(x: torch.Tensor | None, ids: torch.Tensor, weights: torch.Tensor,
                   routed: ExpertBank, shared: ExpertBank | None = None,
                   shared_logit: torch.Tensor | None = None,
                   out_dtype: torch.dtype = torch.float16, out: torch.Tensor | None = None,
                   accumulate: bool = False, x_f32: torch.Tensor | None = None,
                   norm_weight: torch.Tensor | None = None,
                   norm_eps: float = 1e-6,
                   workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Batch-1 routed (+ shared) expert FFN: sum_r w_r Down(SwiGLU(GateUp(x))).

    With ``x_f32`` and ``norm_weight`` (and ``x`` None) the fp32 residual is
    RMS-normalised in the kernel prologue."""
    if x is not None:
        _cuda(x, "x", torch.float16)
    else:
        _cuda(x_f32, "x_f32", torch.float32)
    dev = (x if x is not None else x_f32).device
    _cuda(ids, "ids", torch.int32)
    _cuda(weights, "weights", torch.float32)
    k = ids.numel()
    h, i = routed.hidden, routed.intermediate
    if out is None:
        out = torch.empty(h, dtype=out_dtype, device=dev)
    if workspace is None:
        workspace = torch.empty(N.lib().iq36_moe_decode_workspace_bytes(k, h, i),
                                dtype=torch.uint8, device=dev)
    rb = routed.c()
    sb = shared.c() if shared is not None else None
    N.call("iq36_moe_decode", _ptr(x), _ptr(x_f32), _ptr(norm_weight), norm_eps,
           ids.data_ptr(), weights.data_ptr(), k, ctypes.byref(rb),
           ctypes.byref(sb) if sb is not None else None, _ptr(shared_logit), out.data_ptr(),
           _dtype_code(out.dtype), int(accumulate), workspace.data_ptr(), workspace.numel(),
           _stream(dev))
    return out


def moe_block_decode(x: torch.Tensor, w_router: torch.Tensor, w_shared_gate: torch.Tensor | None,
                     routed: ExpertBank, shared: ExpertBank | None, k: int = 8,
                     out_dtype: torch.dtype = torch.float16):
    """Config-1 MoE block: router + select + routed/shared experts in one call.
    Returns (out, ids, weights, logits)."""
    _cuda(x, "x", torch.float16)
    dev = x.device
    e, h, i = routed.num_experts, routed.hidden, routed.intermediate
    ids = torch.empty(k, dtype=torch.int32, device=dev)
    wts = torch.empty(k, dtype=torch.float32, device=dev)
    logits = torch.empty(e, dtype=torch.float32, device=dev)
    out = torch.empty(h, dtype=out_dtype, device=dev)
    ws = torch.empty(N.lib().iq36_moe_block_decode_workspace_bytes(k, h, i), dtype=torch.uint8,
                     device=dev)
    rb = routed.c()
    sb = shared.c() if shared is not None else None
    N.call("iq36_moe_block_decode", x.data_ptr(), w_router.data_ptr(), _ptr(w_shared_gate), k,
           ctypes.byref(rb), ctypes.byref(sb) if sb is not None else None, ids.data_ptr(),
           wts.data_ptr(), logits.data_ptr(), out.data_ptr(), _dtype_code(out_dtype),
           ws.data_ptr(), ws.numel(), _stream(dev))
    return out, ids, wts, logits


def moe_layer_workspace(k: int, hidden: int, intermediate: int, device) -> torch.Tensor:
    """Workspace of iq36_moe_layer_decode (reusable across calls on one stream).
    Zero-filled: its grid-barrier words must start at zero."""
    n = N.lib().iq36_moe_layer_decode_workspace_bytes(k, hidden, intermediate)
    return torch.zeros(n, dtype=torch.uint8, device=device)


def moe_layer_decode(residual: torch.Tensor, norm_weight: torch.Tensor, w_router: torch.Tensor,
                     w_shared_gate: torch.Tensor | None, routed: ExpertBank,
                     shared: ExpertBank | None, ids: torch.Tensor, weights: torch.Tensor,
                     logits: torch.Tensor, shared_logit: torch.Tensor | None,
                     workspace: torch.Tensor | None = None, k: int = 8,
                     norm_eps: float = 1e-6) -> None:
    """One decode MoE FFN layer on the fp32 residual (in place): RMSNorm ->
    router logits -> top-k -> routed + shared experts -> residual += f16(out).
    ids / weights / logits / shared_logit receive the router outputs."""
    _cuda(residual, "residual", torch.float32)
    dev = residual.device
    _cuda(ids, "ids", torch.int32)
    _cuda(weights, "weights", torch.float32)
    _cuda(logits, "logits", torch.float32)
    h, i = routed.hidden, routed.intermediate
    if workspace is None:
        workspace = moe_layer_workspace(k, h, i, dev)
    rb = routed.c()
    sb = shared.c() if shared is not None else None
    N.call("iq36_moe_layer_decode", residual.data_ptr(), h, norm_weight.data_ptr(), norm_eps,
           w_router.data_ptr(), _ptr(w_shared_gate), k, ctypes.byref(rb),
           ctypes.byref(sb) if sb is not None else None, ids.data_ptr(), weights.data_ptr(),
           logits.data_ptr(), _ptr(shared_logit), workspace.data_ptr(), workspace.numel(),
           _stream(dev))


def moe_layer_prefill_workspace(T: int, k: int, num_experts: int, hidden: int,
                                intermediate: int, device) -> torch.Tensor:
    n = N.lib().iq36_moe_layer_prefill_workspace_bytes(T, k, num_experts, hidden, intermediate)
    return torch.empty(n, dtype=torch.uint8, device=device)


def moe_layer_prefill(residual: torch.Tensor, norm_weight: torch.Tensor, w_router: torch.Tensor,
                      w_shared_gate: torch.Tensor | None, routed: ExpertBank,
                      shared: ExpertBank | None, ids: torch.Tensor, weights: torch.Tensor,
                      logits: torch.Tensor, workspace: torch.Tensor | None = None, k: int = 8,
                      norm_eps: float = 1e-6) -> None:
    """The MoE FFN block over T prompt tokens on the fp32 residual [T, H] (in
    place): RMSNorm -> router -> top-k -> grouped routed experts + shared
    expert, added to the residual. ids / weights [T, k] and logits [T, E]
    receive the router outputs."""
    _cuda(residual, "residual", torch.float32)
    _cuda(ids, "ids", torch.int32)
    _cuda(weights, "weights", torch.float32)
    _cuda(logits, "logits", torch.float32)
    dev = residual.device
    T, h = residual.shape
    if workspace is None:
        workspace = moe_layer_prefill_workspace(T, k, routed.num_experts, h, routed.intermediate,
                                                dev)
    rb = routed.c()
    sb = shared.c() if shared is not None else None
    N.call("iq36_moe_layer_prefill", residual.data_ptr(), T, h, norm_weight.data_ptr(), norm_eps,
           w_router.data_ptr(), _ptr(w_shared_gate), k, ctypes.byref(rb),
           ctypes.byref(sb) if sb is not None else None, ids.data_ptr(), weights.data_ptr(),
           logits.data_ptr(), workspace.data_ptr(), workspace.numel(), _stream(dev))


def moe_expert_ffn_prefill(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                           routed: ExpertBank, out_dtype: torch.dtype = torch.float32,
                           out: torch.Tensor | None = None) -> torch.Tensor:
    """Grouped MoE prefill over T tokens (bf16 x [T, H], ids/weights [T, k])."""
    _cuda(x, "x", torch.bfloat16)
    _cuda(ids, "ids", torch.int32)
    _cuda(weights, "weights", torch.float32)
    t, h = x.shape
    k = ids.shape[1]
    _need(ids.shape[0] == t and weights.shape == ids.shape, "ids/weights must be [T, k]")
    if out is None:
        out = torch.empty(t, h, dtype=out_dtype, device=x.device)
    nbytes = N.lib().iq36_moe_prefill_workspace_bytes(t, k, routed.num_experts, h,
                                                      routed.intermediate)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    rb = routed.c()
    N.call("iq36_moe_prefill", x.data_ptr(), t, ids.data_ptr(), weights.data_ptr(), k,
           ctypes.byref(rb), out.data_ptr(), _dtype_code(out.dtype), ws.data_ptr(), ws.numel(),
           _stream(x.device))
    return out


def u4_gemm(x: torch.Tensor, w: U4Weight, out: torch.Tensor | None = None,
            out_dtype: torch.dtype = torch.float16, accumulate: bool = False,
            norm_weight: torch.Tensor | None = None, norm_eps: float = 1e-6,
            workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Batched u4 projection out[T, N] = x W^T (x fp16, or fp32 with an optional
    fused RMSNorm); out fp16, or fp32 (accumulate: out += f16(x W^T))."""
    _cuda(x, "x")
    _need(x.dim() == 2 and x.dtype in (torch.float16, torch.float32), "x must be [T, K] fp16/fp32")
    t, k = x.shape
    n = w.rows
    if out is None:
        out = torch.empty(t, n, dtype=out_dtype, device=x.device)
    if workspace is None:
        workspace = torch.empty(N.lib().iq36_u4_gemm_workspace_bytes(t, k), dtype=torch.uint8,
                                device=x.device)
    m = w.c()
    N.call("iq36_u4_gemm", x.data_ptr(), _dtype_code(x.dtype), _ptr(norm_weight), norm_eps, t, k,
           w.group, ctypes.byref(m), out.data_ptr(), _dtype_code(out.dtype), int(accumulate),
           workspace.data_ptr(), workspace.numel(), _stream(x.device))
    return out


def u4_gemm_multi(x: torch.Tensor, ws: list[U4Weight], outs: list[torch.Tensor],
                  accumulate: list[bool] | None = None,
                  norm_weight: torch.Tensor | None = None, norm_eps: float = 1e-6,
                  workspace: torch.Tensor | None = None) -> None:
    """Up to 4 batched u4 projections of one input x [T, K] in one launch:
    outs[p] [T, rows_p] = x W_p^T (fp16, or fp32 with accumulate)."""
    _cuda(x, "x")
    _need(x.dim() == 2 and x.dtype in (torch.float16, torch.float32), "x must be [T, K] fp16/fp32")
    _need(1 <= len(ws) == len(outs) <= 4, "1..4 projections with one output each")
    t, k = x.shape
    accumulate = accumulate or [False] * len(ws)
    arr = (N.U4Projection * len(ws))()
    for i, (w, o, acc) in enumerate(zip(ws, outs, accumulate)):
        _cuda(o, f"out[{i}]")
        _need(o.shape == (t, w.rows), f"out[{i}] must be [{t}, {w.rows}]")
        arr[i] = N.U4Projection(w.c(), o.data_ptr(), _dtype_code(o.dtype), int(acc))
    if workspace is None:
        workspace = torch.empty(N.lib().iq36_u4_gemm_workspace_bytes(t, k), dtype=torch.uint8,
                                device=x.device)
    N.call("iq36_u4_gemm_multi", x.data_ptr(), _dtype_code(x.dtype), _ptr(norm_weight), norm_eps,
           t, k, ws[0].group, len(ws), arr, workspace.data_ptr(), workspace.numel(),
           _stream(x.device))


def moe_prefill_rows(x_rows: torch.Tensor, row_of: torch.Tensor, ids: torch.Tensor,
                     weights: torch.Tensor, routed: ExpertBank,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """Per-assignment fp16 contributions over deduplicated rows: out[a] =
    fp16(weights[a] * Expert_{ids[a]}(x_rows[row_of[a]])), out [n_assign, H]."""
    _cuda(x_rows, "x_rows", torch.bfloat16)
    for t, name in ((row_of, "row_of"), (ids, "ids")):
        _cuda(t, name, torch.int32)
    _cuda(weights, "weights", torch.float32)
    n_rows, h = x_rows.shape
    n = ids.numel()
    _need(row_of.numel() == n and weights.numel() == n, "row_of/ids/weights must match")
    if out is None:
        out = torch.empty(n, h, dtype=torch.float16, device=x_rows.device)
    if n == 0:
        return out
    nbytes = N.lib().iq36_moe_prefill_rows_workspace_bytes(n, routed.num_experts, h,
                                                           routed.intermediate)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=x_rows.device)
    rb = routed.c()
    N.call("iq36_moe_prefill_rows", x_rows.data_ptr(), n_rows, n, row_of.data_ptr(),
           ids.data_ptr(), weights.data_ptr(), ctypes.byref(rb), out.data_ptr(), ws.data_ptr(),
           ws.numel(), _stream(x_rows.device))
    return out


def moe_combine(contrib: torch.Tensor, inv: torch.Tensor, k: int,
                out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """out[t] = sum_r float(contrib[inv[t*k + r]]) in rank order (fp16 rows)."""
    _cuda(contrib, "contrib", torch.float16)
    _cuda(inv, "inv", torch.int32)
    _need(inv.numel() % k == 0, "inv must hold T*k rows")
    t, h = inv.numel() // k, contrib.shape[1]
    out = torch.empty(t, h, dtype=out_dtype, device=contrib.device)
    N.call("iq36_moe_combine", contrib.data_ptr(), inv.data_ptr(), t, h, k, out.data_ptr(),
           _dtype_code(out_dtype), _stream(contrib.device))
    return out


# ---------------------------------------------------------------------------
# (3) attention


def paged_gqa_workspace(max_ctx: int, n_q: int = 16, n_kv: int = 2, head_dim: int = 256,
                        device: torch.device | str = "cuda") -> torch.Tensor:
    n = N.lib().iq36_paged_gqa_workspace_bytes(max_ctx, n_q, n_kv, head_dim)
    return torch.empty(n, dtype=torch.uint8, device=device)


def paged_gqa_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     block_table: torch.Tensor, ctx_len: int, scale: float,
                     gate: torch.Tensor | None = None, out_dtype: torch.dtype = torch.float32,
                     ctx_len_dev: torch.Tensor | None = None,
                     workspace: torch.Tensor | None = None,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """Split-K flash decode over an fp16 paged KV cache [blocks, 16, n_kv, 256]."""
    _cuda(q, "q", torch.float16)
    _cuda(k_cache, "k_cache", torch.float16)
    _cuda(v_cache, "v_cache", torch.float16)
    _cuda(block_table, "block_table", torch.int32)
    nq, d = q.shape[-2], q.shape[-1]
    _need(k_cache.dim() == 4, "k_cache must be [blocks, block_size, n_kv, head_dim]")
    bs, nkv = k_cache.shape[1], k_cache.shape[2]
    if out is None:
        out = torch.empty(nq, d, dtype=out_dtype, device=q.device)
    if workspace is None:
        workspace = paged_gqa_workspace(ctx_len, nq, nkv, d, q.device)
    N.call("iq36_paged_gqa_decode", q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
           block_table.data_ptr(), ctx_len, _ptr(ctx_len_dev), nq, nkv, d, bs, scale,
           _ptr(gate), out.data_ptr(), _dtype_code(out.dtype), workspace.data_ptr(),
           workspace.numel(), _stream(q.device))
    return out


# ---------------------------------------------------------------------------
# config-4 support ops


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
             out_dtype: torch.dtype = torch.float16, out: torch.Tensor | None = None):
    _cuda(x, "x", torch.float32)
    _cuda(weight, "weight", torch.float32)
    x2 = x.reshape(-1, x.shape[-1])
    if out is None:
        out = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    N.call("iq36_rms_norm", x2.data_ptr(), x2.shape[0], x2.shape[1], weight.data_ptr(),
           weight.numel(), eps, out.data_ptr(), _dtype_code(out.dtype), _stream(x.device))
    return out


def attn_prep(q_full, k, v, q_norm_w, k_norm_w, eps, pos_dev, block_table, k_cache, v_cache,
              q_out, gate_out, rope_dim: int = 64, rope_base: float = 1e7):
    nq = q_full.numel() // (2 * 256)
    nkv = k.numel() // 256
    N.call("iq36_attn_prep", q_full.data_ptr(), k.data_ptr(), v.data_ptr(), q_norm_w.data_ptr(),
           k_norm_w.data_ptr(), eps, pos_dev.data_ptr(), nq, nkv, 256, rope_dim, rope_base,
           block_table.data_ptr(), k_cache.shape[1], k_cache.data_ptr(), v_cache.data_ptr(),
           q_out.data_ptr(), gate_out.data_ptr(), _stream(q_full.device))


def attn_prep_batch(q_full, k, v, q_norm_w, k_norm_w, eps, pos_dev, block_table, k_cache,
                    v_cache, q_out, gate_out, rope_dim: int = 64, rope_base: float = 1e7):
    """attn_prep for T tokens at positions pos_dev + t: q_full [T, n_q*2*256],
    k, v [T, n_kv*256], q_out, gate_out [T, n_q*256] (fp16, contiguous)."""
    T = q_full.shape[0]
    for t_, nm in ((q_full, "q_full"), (k, "k"), (v, "v"), (q_out, "q_out"),
                   (gate_out, "gate_out")):
        _cuda(t_, nm, torch.float16)
        _need(t_.shape[0] == T, f"{nm} must have {T} rows")
    nq = q_full[0].numel() // (2 * 256)
    nkv = k[0].numel() // 256
    N.call("iq36_attn_prep_batch", q_full.data_ptr(), k.data_ptr(), v.data_ptr(),
           q_norm_w.data_ptr(), k_norm_w.data_ptr(), eps, pos_dev.data_ptr(), T, nq, nkv, 256,
           rope_dim, rope_base, block_table.data_ptr(), k_cache.shape[1], k_cache.data_ptr(),
           v_cache.data_ptr(), q_out.data_ptr(), gate_out.data_ptr(), _stream(q_full.device))


def attn_prefill(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                 block_table: torch.Tensor, pos_dev: torch.Tensor, scale: float,
                 gate: torch.Tensor | None = None, out_dtype: torch.dtype = torch.float16,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """Causal attention of T prompt queries q [T, n_q, 256] (positions
    pos_dev + t) over the fp16 paged cache; out [T, n_q, 256]."""
    _cuda(q, "q", torch.float16)
    _cuda(k_cache, "k_cache", torch.float16)
    _cuda(v_cache, "v_cache", torch.float16)
    _cuda(block_table, "block_table", torch.int32)
    _cuda(pos_dev, "pos_dev", torch.int32)
    _need(q.dim() == 3, "q must be [T, n_q, head_dim]")
    T, nq, d = q.shape
    bs, nkv = k_cache.shape[1], k_cache.shape[2]
    if gate is not None:
        _cuda(gate, "gate", torch.float16)
    if out is None:
        out = torch.empty(T, nq, d, dtype=out_dtype, device=q.device)
    N.call("iq36_attn_prefill", q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
           block_table.data_ptr(), bs, k_cache.shape[0], pos_dev.data_ptr(), T, nq, nkv, d,
           scale, _ptr(gate), out.data_ptr(), _dtype_code(out.dtype), _stream(q.device))
    return out


def delta_prep(qkv, conv_state, conv_w, a, b, a_log, dt_bias, act_out, g_out, beta_out):
    N.call("iq36_delta_prep", qkv.data_ptr(), qkv.numel(), conv_state.data_ptr(),
           conv_w.data_ptr(), a.data_ptr(), b.data_ptr(), a_log.data_ptr(), dt_bias.data_ptr(),
           a_log.numel(), act_out.data_ptr(), g_out.data_ptr(), beta_out.data_ptr(),
           _stream(qkv.device))


def delta_step(act, g, beta, state, z, norm_w, eps, n_k_heads, n_v_heads, out,
               head_dim: int = 128):
    N.call("iq36_delta_step", act.data_ptr(), g.data_ptr(), beta.data_ptr(), state.data_ptr(),
           z.data_ptr(), norm_w.data_ptr(), eps, n_k_heads, n_v_heads, head_dim, out.data_ptr(),
           _stream(act.device))


def delta_prefill_workspace(tokens: int, n_k_heads: int, n_v_heads: int,
                            device) -> torch.Tensor:
    n = N.lib().iq36_delta_prefill_workspace_bytes(tokens, n_k_heads, n_v_heads)
    return torch.empty(n, dtype=torch.uint8, device=device)


def delta_prefill(qkv, conv_state, conv_w, a, b, a_log, dt_bias, state, z, norm_w, eps,
                  n_k_heads, n_v_heads, out, workspace=None, head_dim: int = 128):
    """DeltaNet block over T tokens (qkv [T, C] fp16; a, b [T, >=nv] fp16 views
    sharing one row stride; z, out [T, nv*D] fp16); conv_state and state are
    updated in place as if the T tokens were decoded one by one."""
    T = qkv.shape[0]
    for t_, nm in ((qkv, "qkv"), (z, "z"), (out, "out")):
        _cuda(t_, nm, torch.float16)
    _need(a.stride(0) == b.stride(0) and a.stride(1) == 1 and b.stride(1) == 1,
          "a and b must be row views with one common row stride")
    if workspace is None:
        workspace = delta_prefill_workspace(T, n_k_heads, n_v_heads, qkv.device)
    N.call("iq36_delta_prefill", qkv.data_ptr(), T, n_k_heads, n_v_heads, head_dim,
           conv_state.data_ptr(), conv_w.data_ptr(), a.data_ptr(), b.data_ptr(), a.stride(0),
           a_log.data_ptr(), dt_bias.data_ptr(), state.data_ptr(), z.data_ptr(),
           norm_w.data_ptr(), eps, out.data_ptr(), workspace.data_ptr(), workspace.numel(),
           _stream(qkv.device))
    return out


def embed(table: torch.Tensor, token_dev: torch.Tensor, h: torch.Tensor):
    N.call("iq36_embed", table.data_ptr(), table.shape[0], table.shape[1], token_dev.data_ptr(),
           h.data_ptr(), _stream(table.device))


def embed_batch(table: torch.Tensor, tokens_dev: torch.Tensor, h: torch.Tensor):
    """h [T, H] fp32 = embedding rows of tokens_dev [T] int32."""
    _cuda(tokens_dev, "tokens", torch.int32)
    _cuda(h, "h", torch.float32)
    N.call("iq36_embed_batch", table.data_ptr(), table.shape[0], table.shape[1],
           tokens_dev.data_ptr(), tokens_dev.numel(), h.data_ptr(), _stream(table.device))


def argmax(logits: torch.Tensor, token_out: torch.Tensor, workspace: torch.Tensor | None = None):
    if workspace is None:
        workspace = torch.empty(N.lib().iq36_argmax_workspace_bytes(), dtype=torch.uint8,
                                device=logits.device)
    N.call("iq36_argmax", logits.data_ptr(), logits.numel(), token_out.data_ptr(),
           workspace.data_ptr(), workspace.numel(), _stream(logits.device))
    return token_out


def lm_head_cert_table(w: U4Weight) -> torch.Tensor:
    """Per-row, per-group fp16 bound table of the certified LM-head top-1
    (|s| times the group's ||q - zp||, rounded up); built once per head."""
    w.validate()
    n = N.lib().iq36_lm_head_cert_table_bytes(w.rows, w.k, w.group)
    _need(n > 0, "the certified top-1 needs a group-128 head")
    table = torch.empty(n // 2, dtype=torch.float16, device=w.weight.device)
    m = w.c()
    N.call("iq36_lm_head_cert_table", ctypes.byref(m), w.k, w.group, table.data_ptr(),
           _stream(w.weight.device))
    return table


def lm_head_top1_certified(w: U4Weight, table: torch.Tensor, seed_token: torch.Tensor,
                           logits: torch.Tensor, token_out: torch.Tensor,
                           x: torch.Tensor | None = None, x_f32: torch.Tensor | None = None,
                           norm_weight: torch.Tensor | None = None, norm_eps: float = 1e-6,
                           capacity_chunks: int = 1024, evaluated: torch.Tensor | None = None,
                           workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Greedy top-1 of the LM head by the bound certificate: the same token as
    the full head's argmax; only the evaluated 16-row chunks' logits are
    written (their count into ``evaluated``)."""
    w.validate()
    dev = w.weight.device
    _cuda(logits, "logits", torch.float32)
    _need(logits.numel() == w.rows, f"logits must have {w.rows} elements")
    _cuda(token_out, "token_out", torch.int32)
    _cuda(seed_token, "seed_token", torch.int32)
    _need(table.numel() * 2 == N.lib().iq36_lm_head_cert_table_bytes(w.rows, w.k, w.group),
          "table does not match the head")
    if workspace is None:
        workspace = torch.empty(N.lib().iq36_lm_head_top1_certified_workspace_bytes(w.rows, w.k),
                                dtype=torch.uint8, device=dev)
    m = w.c()
    N.call("iq36_lm_head_top1_certified", _ptr(x), _ptr(x_f32), _ptr(norm_weight), norm_eps, w.k,
           w.group, ctypes.byref(m), table.data_ptr(), seed_token.data_ptr(), capacity_chunks,
           logits.data_ptr(), token_out.data_ptr(), _ptr(evaluated), workspace.data_ptr(),
           workspace.numel(), _stream(dev))
    return token_out


def synth_fill(dst: torch.Tensor, kind: int, seed: int, tensor_id: int, lo: float,
               hi: float = 0.0) -> torch.Tensor:
    _cuda(dst, "dst")
    N.call("iq36_synth_fill", dst.data_ptr(), dst.numel(), kind, seed, tensor_id, lo, hi,
           _stream(dst.device))
    return dst


# the same operators registered as torch.ops.iq36.* custom ops (schemas and
# fake kernels over these functions)
from . import library  # noqa: E402,F401
