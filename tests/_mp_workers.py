"""Rank entry points for the multi-process tests (spawned children import
this module by name, so it sets up sys.path itself)."""

from __future__ import annotations

import os
import sys
import traceback
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
for _p in (str(ROOT), str(ROOT / "aima-intel-plk-qwen36-35b-u4-engine_b200"), str(ROOT / "tests")):
    if _p not in sys.path:
        sys.path.insert(0, _p)


def _init(rank: int, world: int, port: int, backend: str):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    kw = {}
    if backend == "nccl":
        import torch
        torch.cuda.set_device(rank)
        kw["device_id"] = torch.device(f"cuda:{rank}")
    dist.init_process_group(backend, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), **kw)


def _finish(q, rank, fn, *args):
    import torch.distributed as dist
    try:
        fn(*args)
        q.put((rank, "ok"))
    except Exception:  # report to the parent instead of hanging it
        q.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


# ---------------------------------------------------------------------------
# CPU (gloo): expert-parallel exchange with the CPU reference as the expert fn

def ep_prefill_cpu(rank, world, port, q):
    _init(rank, world, port, "gloo")
    _finish(q, rank, _ep_prefill_cpu_body, rank, world)


def _ep_prefill_cpu_body(rank, world):
    import numpy as np
    import torch
    from engine.parallel_ep import ep_moe_prefill
    from helpers import make_bank
    from oracle import oracle

    H, I, E, k, T = 256, 128, 4 * world, 4, 24
    bank = make_bank(np.random.default_rng(7), E, H, I)      # same on every rank
    rng = np.random.default_rng(100 + rank)                  # rank's own tokens
    x = rng.standard_normal((T, H)).astype(np.float32)
    xb = oracle.bf16_bits(x)
    xf = oracle.bf16_to_f32(xb)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    e_local = E // world
    for t in range(0, T, 5):  # tokens whose experts all live on one rank (no row to the other)
        ids[t] = (t // 5) % world * e_local + rng.permutation(e_local)[:k]
    w = rng.uniform(0.05, 0.5, (T, k)).astype(np.float32)
    local = {key: v[rank * e_local:(rank + 1) * e_local] for key, v in bank.items()}

    def expert_fn(x_rows, row_of, local_ids, weights):
        n = local_ids.shape[0]
        if n == 0:
            return torch.zeros(0, H)
        xr = oracle.bf16_bits(x_rows.numpy()[row_of.numpy()])
        y = oracle.moe_prefill(xr, np.arange(n), local_ids.numpy().reshape(n, 1),
                               weights.numpy().reshape(n, 1), local, 128)
        return torch.from_numpy(y)

    out = ep_moe_prefill(torch.from_numpy(xf), torch.from_numpy(ids), torch.from_numpy(w), E,
                         expert_fn)
    ref = oracle.moe_prefill(xb, np.arange(T), ids, w, bank, 128)
    np.testing.assert_array_equal(out.numpy(), ref)  # same fp32 sums in slot order


# CPU (gloo): row-/K-sharded u4 GEMV composed with all_reduce / all_gather

def tp_gemv_cpu(rank, world, port, q):
    _init(rank, world, port, "gloo")
    _finish(q, rank, _tp_gemv_cpu_body, rank, world)


def _tp_gemv_cpu_body(rank, world):
    import numpy as np
    import torch
    import torch.distributed as dist
    from engine.ops import U4Weight
    from engine.parallel_tp import shard_u4_k, shard_u4_rows
    from helpers import make_u4
    from oracle import oracle

    rng = np.random.default_rng(3)
    wn, sn, zn = make_u4(rng, 256, 1024, 128)
    x = rng.standard_normal(1024).astype(np.float16)
    full = oracle.u4_gemv(x, wn, sn, zn, 128)
    W = U4Weight(torch.from_numpy(wn), torch.from_numpy(sn), torch.from_numpy(zn), 128)
    # row-parallel: K slices, partial sums, all-reduce
    ks = shard_u4_k(W, rank, world)
    k0 = rank * (1024 // world)
    part = oracle.u4_gemv(x[k0:k0 + 1024 // world], ks.weight.numpy(), ks.scale.numpy(),
                          ks.zp.numpy(), 128)
    t = torch.from_numpy(part.copy())
    dist.all_reduce(t)
    np.testing.assert_allclose(t.numpy(), full, rtol=1e-5, atol=1e-4)
    # column-parallel: row blocks, all-gather
    rs = shard_u4_rows(W, rank, world)
    y = torch.from_numpy(oracle.u4_gemv(x, rs.weight.numpy(), rs.scale.numpy(), rs.zp.numpy(),
                                        128).copy())
    parts = [torch.empty_like(y) for _ in range(world)]
    dist.all_gather(parts, y)
    np.testing.assert_array_equal(torch.cat(parts).numpy(), full)


# ---------------------------------------------------------------------------
# GPU (NCCL), one rank per GPU

def ep_prefill_gpu(rank, world, port, q):
    _init(rank, world, port, "nccl")
    _finish(q, rank, _ep_prefill_gpu_body, rank, world)


def _ep_prefill_gpu_body(rank, world):
    import numpy as np
    import torch
    from engine.ops import moe_expert_ffn_prefill, router_select
    from engine.parallel_ep import ep_moe_prefill, gpu_expert_fn
    from engine.parallel_tp import shard_expert_bank
    from helpers import bank_to_torch, make_bank, zipf_router_logits

    dev = torch.device(f"cuda:{rank}")
    E, T = 32, 512
    bank = bank_to_torch(make_bank(np.random.default_rng(5), E, 2048, 512), dev)
    rng = np.random.default_rng(50 + rank)
    logits = torch.from_numpy(zipf_router_logits(rng, T, E)).to(dev)
    ids, w = router_select(logits, 8)
    x = torch.from_numpy(rng.standard_normal((T, 2048)).astype(np.float32)).to(dev).to(
        torch.bfloat16)
    local, e0 = shard_expert_bank(bank, rank, world)
    out = ep_moe_prefill(x, ids, w, E, gpu_expert_fn(local))
    ref = moe_expert_ffn_prefill(x, ids, w, bank)
    torch.cuda.synchronize(dev)
    assert torch.equal(out, ref), float((out - ref).abs().max())


def ep_decode_gpu(rank, world, port, q):
    _init(rank, world, port, "nccl")
    _finish(q, rank, _ep_decode_gpu_body, rank, world)


def _ep_decode_gpu_body(rank, world):
    import numpy as np
    import torch
    from engine.ops import moe_expert_ffn
    from engine.parallel_tp import ep_moe_decode, shard_expert_bank
    from helpers import bank_to_torch, make_bank

    dev = torch.device(f"cuda:{rank}")
    rng = np.random.default_rng(11)
    bank = bank_to_torch(make_bank(rng, 64, 2048, 512), dev)
    shared = bank_to_torch(make_bank(rng, 1, 2048, 512), dev)
    x = torch.from_numpy(rng.standard_normal(2048).astype(np.float16)).to(dev)
    ids = torch.tensor([3, 60, 17, 33, 8, 41, 25, 50], dtype=torch.int32, device=dev)
    w = torch.tensor([0.3, 0.2, 0.15, 0.1, 0.1, 0.06, 0.05, 0.04], device=dev)
    sl = torch.tensor([0.3], device=dev)
    local, e0 = shard_expert_bank(bank, rank, world)
    out = ep_moe_decode(x, ids, w, local, e0, shared if rank == 0 else None, sl)
    ref = moe_expert_ffn(x, ids, w, bank, shared, sl, out_dtype=torch.float32)
    torch.cuda.synchronize(dev)
    err = float(((out - ref).abs().max() / ref.abs().max()).item())
    assert err < 1e-5, err


def tp_decode_gpu(rank, world, port, q):
    _init(rank, world, port, "nccl")
    _finish(q, rank, _tp_decode_gpu_body, rank, world)


def _tp_decode_gpu_body(rank, world):
    import numpy as np
    import torch
    from engine.ops import moe_expert_ffn
    from engine.parallel_tp import shard_expert_bank_rows, tp_moe_decode
    from helpers import bank_to_torch, make_bank

    dev = torch.device(f"cuda:{rank}")
    rng = np.random.default_rng(12)
    bank = bank_to_torch(make_bank(rng, 64, 2048, 512), dev)
    shared = bank_to_torch(make_bank(rng, 1, 2048, 512), dev)
    x = torch.from_numpy(rng.standard_normal(2048).astype(np.float16)).to(dev)
    ids = torch.tensor([3, 60, 17, 33, 8, 41, 25, 50], dtype=torch.int32, device=dev)
    w = torch.tensor([0.3, 0.2, 0.15, 0.1, 0.1, 0.06, 0.05, 0.04], device=dev)
    sl = torch.tensor([0.3], device=dev)
    out = tp_moe_decode(x, ids, w, shard_expert_bank_rows(bank, rank, world),
                        shard_expert_bank_rows(shared, rank, world), sl)
    ref = moe_expert_ffn(x, ids, w, bank, shared, sl, out_dtype=torch.float32)
    torch.cuda.synchronize(dev)
    err = float(((out - ref).abs().max() / ref.abs().max()).item())
    assert err < 1e-5, err


# ---------------------------------------------------------------------------
# GPU (NCCL + CUDA IPC exchange): the tensor-parallel decode runtime against
# the single-GPU runtime on the same weights

def tp_runtime_gpu(rank, world, port, q):
    _init(rank, world, port, "nccl")
    _finish(q, rank, _tp_runtime_gpu_body, rank, world)


def _kld(p_logits, q_logits) -> float:
    import numpy as np
    p = np.exp(p_logits - p_logits.max())
    p /= p.sum()
    q = np.exp(q_logits - q_logits.max())
    q /= q.sum()
    return float(np.sum(p * (np.log(p + 1e-30) - np.log(q + 1e-30))))


def _tp_runtime_gpu_body(rank, world):
    import numpy as np
    import torch
    import torch.distributed as dist
    from engine import _native
    from engine.runtime import ModelConfig, Qwen36Runtime, SyntheticWeights
    from engine.tp_decode import TPRuntime

    dev = torch.device(f"cuda:{rank}")
    cfg = ModelConfig(layers=4, experts=16, vocab=4096)
    full = SyntheticWeights(cfg, 4242, dev)
    prompt = np.random.default_rng(7).integers(0, cfg.vocab, 20).tolist()
    steps = 8
    # single GPU on every rank (identical): reference tokens and logits
    ref = Qwen36Runtime(cfg, max_ctx=64, device=dev, weights=full)
    ref.capture()
    ref.prefill(prompt)
    ref_tok, ref_logits = [int(ref.token.item())], [ref.logits.cpu().numpy()]
    for _ in range(steps):
        ref.step()
        ref_tok.append(int(ref.token.item()))
        ref_logits.append(ref.logits.cpu().numpy())
    del ref
    # tensor parallel
    tp = TPRuntime(cfg, rank, world, dev, max_ctx=64, full=full)
    tp.capture()
    tp.prefill(prompt)
    got_tok, got_logits = [], []
    for i in range(steps + 1):
        if i:
            tp.step()
        torch.cuda.synchronize(dev)
        parts = [torch.empty_like(tp.logits) for _ in range(world)]
        dist.all_gather(parts, tp.logits)
        got_tok.append(int(tp.token.item()))
        got_logits.append(torch.cat(parts).cpu().numpy())
    assert _native.wait_timeouts(reset=True) == 0
    tp.close()
    assert got_tok == ref_tok, (got_tok, ref_tok)
    worst = max(_kld(r, g) for r, g in zip(ref_logits, got_logits))
    assert worst <= 1e-3, worst
