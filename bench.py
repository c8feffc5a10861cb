#!/usr/bin/env python
"""Benchmark: batch-1 decode of the synthetic Qwen3.6-35B-A3B-shaped model on B200.

Workload: random-init 40-layer model (10 x (3 DeltaNet +
1 gated GQA), each followed by the 256-expert top-8 MoE, u4 g128 weights,
vocab 248320). A seeded uniform-random prompt of --ctx tokens (default 4096)
is fed through the decode step, then --warmup untimed and --steps timed greedy
decode steps run as CUDA-graph replays. One step reads ~1.77 GB (> L2), so no
L2 flush is needed between steps.

JSON line (rank 0): value = decode tok/s over all ranks (device time, CUDA
events, max over ranks); e2e = the same through the public API with the input
token copied from pinned host memory and the greedy token read back every
step; roofline = the dominant kernel (multi-output u4 GEMV) measured live;
cpu_baseline = the CPU restatement (oracle/) on a bounded sample.

--impl reference: the reference path's CPU implementation (the oracle port;
OpenVINO is not installable here) on the host cores, same metric.
Multi-GPU: replicas only (each rank decodes its own sequence; no collective on
the data path), value summed over ranks.

Other workloads: --workload prefill (BASELINE config 4 prefill tok/s: the batched
prefill of a --ctx-token prompt, 4096 or 32768; a step is one whole prompt),
--workload attn_prefill / delta_prefill (one prompt-path op alone over --tokens),
--workload moe_prefill (grouped MoE
prefill; replicas at --gpus > 1, expert-parallel over NCCL with --ep), --workload gemv
(one u4 GEMV per step, --rows / --k for other shapes), --workload
moe_decode (the batch-1 MoE block, HBM GB/s) and --workload gqa_decode
(paged GQA decode at --ctx, HBM GB/s).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "aima-intel-plk-qwen36-35b-u4-engine_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

BASELINE = json.loads((ROOT / "BASELINE.json").read_text())
METRIC = BASELINE["metric"]
PREFILL_CHUNK = 16384  # tokens per batched-prefill launch sequence (Qwen36Runtime default)
DECODE_GEMV_TRAFFIC = 11551662  # B per launch, ncu dram__bytes_read+write over one step's 81
# B per launch, ncu dram__bytes_read + dram__bytes_write of moe_layer_kernel at the config-1 /
# config-4 layer shape (profiles/moe_layer_decode_config1.md): 15,857,152 read, 0 written
DECODE_MOE_TRAFFIC = 15857152
PUBLISHED_DECODE_4K = 50.57  # reference's published figure: Arc B390, 4k prompt, batch-1 decode tok/s
PUBLISHED_PREFILL = {4096: 2367.89, 32768: 2065.28}  # reference prefill tok/s, Arc B390


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------------------
class ClockSampler:
    """SM clock and clock-event reasons sampled DURING the timed region.

    An NVML thread polls every ~1 ms (a decode timed region can last only tens
    of milliseconds; nvidia-smi's loop mode samples every 100 ms at best), on
    the GPU that holds this process's CUDA device (matched by PCI bus id);
    falls back to an `nvidia-smi -lms 100` subprocess when NVML is missing."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None
        self.thread = None
        self.rows: list[tuple[int, int]] = []
        self.max_mhz = None

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        try:
            p = torch.cuda.get_device_properties(self.index)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def start(self):
        import threading
        try:
            import pynvml
            h = self._nvml_handle()
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception:
            return self._start_smi()
        self.stop_flag = threading.Event()

        def poll():
            while not self.stop_flag.is_set():
                try:
                    self.rows.append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
                                      pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)))
                except Exception:
                    pass
                time.sleep(0.001)

        self.thread = threading.Thread(target=poll, daemon=True)
        self.thread.start()
        t0 = time.time()
        while not self.rows and time.time() - t0 < 2.0:
            time.sleep(0.001)

    def _start_smi(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.index)], stdout=open(self.path, "w"),
                stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return
        t0 = time.time()
        while time.time() - t0 < 5.0 and os.path.getsize(self.path) == 0:
            time.sleep(0.02)

    def stop(self) -> dict:
        if self.thread is not None:
            import pynvml
            self.stop_flag.set()
            self.thread.join()
            bits = {"hw_slowdown": pynvml.nvmlClocksEventReasonHwSlowdown,
                    "hw_thermal_slowdown": pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                    "sw_thermal_slowdown": pynvml.nvmlClocksEventReasonSwThermalSlowdown,
                    "sw_power_cap": pynvml.nvmlClocksEventReasonSwPowerCap}
            sm = sorted(r[0] for r in self.rows)
            reasons = sorted(n for n, b in bits.items() if any(r[1] & b for r in self.rows))
            return {"sm_mhz": float(sm[len(sm) // 2]) if sm else None,
                    "sm_max_mhz": float(self.max_mhz) if self.max_mhz else None,
                    "reasons": reasons, "samples": len(self.rows), "source": "nvml 1 ms"}
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait()
        rows = [ln.split(",") for ln in open(self.path).read().strip().splitlines() if ln.strip()]
        os.unlink(self.path)
        sm = sorted(float(r[1]) for r in rows if len(r) >= 9 and r[1].strip().isdigit())
        mx = [float(r[2]) for r in rows if len(r) >= 9 and r[2].strip().isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in rows:
            if len(r) >= 9:
                for n, v in zip(names, r[5:9]):
                    if v.strip() == "Active":
                        reasons.add(n)
        return {"sm_mhz": sm[len(sm) // 2] if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(rows), "source": "nvidia-smi 100 ms"}


# ---------------------------------------------------------------------------
def dist_setup():
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device(f"cuda:{local}"))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
def _oracle_timing_model(layers: int):
    """The CPU restatement (oracle/) of a `layers`-layer slice of the config-4
    model with every expert held in host memory, as the reference's CPU model
    holds its weights (the checker's lazy mode, which regenerates the selected
    experts each step, is off: that cost is not the reference's). The banks
    are timing banks: one generated expert copied to all 256, so each step
    still reads 8 + 1 distinct experts' bytes per layer."""
    from engine.runtime import ModelConfig
    from oracle import oracle
    env = {"IQ36_ORACLE_LAZY": "0", "IQ36_ORACLE_REPLICATED": "1"}
    prev = {k: os.environ.get(k) for k in env}
    os.environ.update(env)
    try:
        return oracle.OracleModel(ModelConfig(layers=layers).as_dict(), 1234, 64)
    finally:
        for k, v in prev.items():
            if v is None:
                del os.environ[k]
            else:
                os.environ[k] = v


def cpu_sample(ctx: int, threads: int, steps: int, warm: int) -> dict:
    """Time the CPU restatement on a bounded sample of the decode step: the
    median of `steps` timed decode steps (after `warm` untimed ones) of a
    4-layer slice (3 DeltaNet + 1 GQA layer, 256 experts, full vocab) and of a
    0-layer model (embedding + LM head), plus one config-2 paged attention at
    ctx; per token t0 + 10 (t4 - t0) + 10 t_attn(ctx). Medians over 12 steps
    keep the sample within a few percent run to run (the 10x extrapolation
    of a 3-step mean varied by 30%)."""
    import numpy as np
    from engine.runtime import ModelConfig
    from oracle import oracle
    full = ModelConfig()
    rng = np.random.default_rng(0)
    toks = rng.integers(0, full.vocab, steps + warm + 1).tolist()

    def timed(layers):
        m = _oracle_timing_model(layers)
        for i in range(warm):
            m.step(toks[i], i, want_logits=False, threads=threads)
        ts = []
        for i in range(warm, warm + steps):
            t = time.perf_counter()
            m.step(toks[i], i, want_logits=False, threads=threads)
            ts.append(time.perf_counter() - t)
        m.close()
        return float(np.median(ts))

    t4, t0 = timed(4), timed(0)
    q = rng.standard_normal((16, 256)).astype(np.float16)
    nblk = (ctx + 15) // 16
    kc = rng.standard_normal((nblk, 16, 2, 256)).astype(np.float16)
    vc = rng.standard_normal((nblk, 16, 2, 256)).astype(np.float16)
    bt = np.arange(nblk, dtype=np.int32)
    oracle.paged_gqa(q, kc, vc, bt, ctx, 1 / 16, threads=threads)  # warm
    t = time.perf_counter()
    oracle.paged_gqa(q, kc, vc, bt, ctx, 1 / 16, threads=threads)
    ta = time.perf_counter() - t
    n_attn = sum(full.is_attn(l) for l in range(full.layers))
    per_tok = t0 + (full.layers / 4) * (t4 - t0) + n_attn * ta
    return {"value": round(1.0 / per_tok, 3), "unit": "tok/s", "cores": threads,
            "kind": "port",
            "sample": (f"median of {steps} decode steps (after {warm} warm-up) of a 4-layer slice "
                       f"(3 DeltaNet + 1 GQA, 256 experts) and of a 0-layer model (LM head), plus "
                       f"one {ctx}-token paged attention, extrapolated to 40 layers: "
                       f"{t0 * 1e3:.1f} + 10 x {(t4 - t0) * 1e3:.1f} + {n_attn} x "
                       f"{ta * 1e3:.2f} = {per_tok * 1e3:.1f} ms/token")}


def cpu_baseline(ctx: int, threads: int) -> dict:
    return cpu_sample(ctx, threads, steps=12, warm=1)


# ---------------------------------------------------------------------------
def run_reference(args, world, rank) -> None:
    """The reference path's CPU implementation (the oracle port; OpenVINO is not
    installable here) on all host threads: the same bounded sample as the
    cpu_baseline of the default line (cpu_sample), with --warmup untimed and
    --steps timed steps per slice, bounded to 2 and 12 so the run stays within
    a few minutes."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    warm = max(1, min(args.warmup, 2))
    steps = max(3, min(args.steps, 12))
    t = time.perf_counter()
    v = cpu_sample(args.ctx, threads, steps=steps, warm=warm)
    elapsed = time.perf_counter() - t
    line = {
        "impl": "reference", "metric": METRIC, "value": v["value"], "unit": "tok/s",
        "n_gpus": args.gpus, "steps": steps, "warmup": warm,
        "ms_per_step": round(1e3 / v["value"], 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": round(v["value"] / PUBLISHED_DECODE_4K, 4), "dtype": "u4xf16",
        "data": "synthetic",
        "config": {"workload": f"config4 batch-1 greedy decode after a {args.ctx}-token prompt "
                               "(Qwen3.6-35B-A3B-shaped, random-init u4 g128)",
                   "note": "OpenVINO CPU u4 path unavailable here (not installable); the "
                           "reference arm is the CPU restatement in oracle/",
                   "wall_s": round(elapsed, 2)},
        "cpu_baseline": {**v},
        "e2e": {"value": v["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# The rest of BASELINE's metric, measured after the decode timed region of the
# default line (rank 0 at N = 1): each on its own small budget.

def _device_time(fn, reps, dev, flush=None) -> float:
    """Mean seconds per call of fn() over reps calls (CUDA events on the
    current stream; L2 flushed before each call when flush is given)."""
    import torch
    tot = 0.0
    for _ in range(reps):
        if flush is not None:
            flush()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize(dev)
        tot += s.elapsed_time(e) / 1e3
    return tot / reps


def part_gemv_config0(dev) -> dict:
    """1024 x 2048 u4 g128 GEMV, 512 weight copies rotated
    in one CUDA graph of 512 launches (as --workload gemv)."""
    import ctypes
    import torch
    from engine import _native as N
    from engine import ops
    rows, K, G, copies = 1024, 2048, 128, 512
    one = rows * K // 2 + rows * (K // G) * 2 + rows * (K // G) // 2
    step_bytes = one + K * 2 + rows * 4
    w = torch.empty(copies, rows, K // 2, dtype=torch.uint8, device=dev)
    sc = torch.empty(copies, rows, K // G, dtype=torch.float16, device=dev)
    z = torch.empty(copies, rows * (K // G) // 2, dtype=torch.uint8, device=dev)
    ops.synth_fill(w, 0, 11, 1, 0, 0)
    ops.synth_fill(sc, 1, 11, 2, 0.005, 0.02)
    ops.synth_fill(z, 0, 11, 3, 0, 0)
    x = torch.randn(K, device=dev).to(torch.float16)
    out = torch.empty(rows, dtype=torch.float32, device=dev)
    mats = [N.U4Matrix(w[c].data_ptr(), sc[c].data_ptr(), z[c].data_ptr(), rows)
            for c in range(copies)]
    cap = torch.cuda.Stream(dev)
    cap.wait_stream(torch.cuda.current_stream(dev))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=cap):
        for c in range(copies):
            N.call("iq36_u4_gemv", x.data_ptr(), K, G, ctypes.byref(mats[c]), out.data_ptr(), 0,
                   cap.cuda_stream)
    graph.replay()
    t = _device_time(graph.replay, 3, dev) / copies
    hbm, src = peaks()
    gbs = step_bytes / t / 1e9
    del graph
    return {"gemv_config0_gbs": round(gbs, 1), "gemv_config0_frac": round(gbs / hbm, 4),
            "gemv_config0_us": round(t * 1e6, 3)}


def part_moe_prefill_config3(dev, T: int = 4096) -> dict:
    """BASELINE config 3 at T tokens: grouped MoE prefill, L2 flushed before
    each call; tensor roofline against the measured bf16 peak."""
    import ctypes
    import numpy as np
    import torch
    from engine import _native as N
    from engine import ops
    E, H, I, k = 256, 2048, 512, 8
    t = [torch.empty(E, 2 * I, H // 2, dtype=torch.uint8, device=dev),
         torch.empty(E, 2 * I, H // 128, dtype=torch.float16, device=dev),
         torch.empty(E, 2 * I * H // 256, dtype=torch.uint8, device=dev),
         torch.empty(E, H, I // 2, dtype=torch.uint8, device=dev),
         torch.empty(E, H, I // 128, dtype=torch.float16, device=dev),
         torch.empty(E, H * I // 256, dtype=torch.uint8, device=dev)]
    for j, v in enumerate(t):
        ops.synth_fill(v, 1 if v.dtype == torch.float16 else 0, 77, 1000 + j, 0.005, 0.02)
    bank = ops.ExpertBank(*t, 128)
    rng = np.random.default_rng(T)
    zw = (rng.permutation(E) + 1).astype(np.float64) ** -1.1
    bias = -2 + 4 * (zw - zw.min()) / (zw.max() - zw.min())
    logits = torch.from_numpy((rng.standard_normal((T, E)) + bias).astype(np.float32)).to(dev)
    ids, wts = ops.router_select(logits, k)
    x = torch.randn(T, H, device=dev).to(torch.bfloat16)
    out = torch.empty(T, H, dtype=torch.float32, device=dev)
    ws = torch.empty(N.lib().iq36_moe_prefill_workspace_bytes(T, k, E, H, I), dtype=torch.uint8,
                     device=dev)
    rb = bank.c()
    stream = torch.cuda.current_stream(dev)

    def call():
        N.call("iq36_moe_prefill", x.data_ptr(), T, ids.data_ptr(), wts.data_ptr(), k,
               ctypes.byref(rb), out.data_ptr(), 0, ws.data_ptr(), ws.numel(),
               stream.cuda_stream)

    for _ in range(3):
        call()
    per = _device_time(call, 5, dev, flush=L2Flush(dev))
    peak = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"] \
        if (ROOT / "MEASURED_PEAKS.json").exists() else 1590.0
    tf = T * 50331648 / per / 1e12
    return {f"moe_prefill_config3_T{T}_tok_s": round(T / per, 1),
            f"moe_prefill_config3_T{T}_tflops": round(tf, 1),
            f"moe_prefill_config3_T{T}_frac": round(tf / peak, 4)}


def part_long_context(weights, dev, ctx: int = 32768, steps: int = 32) -> dict:
    """BASELINE config 4 at a 32768-token prompt: batched prefill tok/s, then
    greedy decode tok/s at that context (CUDA-graph replays)."""
    import torch
    from engine.runtime import ModelConfig, Qwen36Runtime
    cfg = ModelConfig()
    rt = Qwen36Runtime(cfg, max_ctx=ctx + steps + 40, device=dev, weights=weights)
    rt.capture()
    gen = torch.Generator().manual_seed(32768)
    prompt = torch.randint(0, cfg.vocab, (ctx,), generator=gen, dtype=torch.int32)
    rt.prefill_batched(prompt, chunk=PREFILL_CHUNK)  # sizes the buffers
    rt.reset()
    torch.cuda.synchronize(dev)
    t_pf = _device_time(lambda: rt.prefill_batched(prompt, chunk=PREFILL_CHUNK), 1, dev)
    for _ in range(4):
        rt.step()
    t_dec = _device_time(lambda: [rt.step() for _ in range(steps)], 1, dev) / steps
    out = {f"prefill_{ctx}_tok_s": round(ctx / t_pf, 1),
           f"decode_ctx{ctx}_tok_s": round(1.0 / t_dec, 2),
           f"decode_ctx{ctx}_ms_per_step": round(t_dec * 1e3, 4),
           f"decode_ctx{ctx}_step_hbm_frac": round(
               cfg.decode_bytes_per_token(ctx + 20) / t_dec / 1e9 / peaks()[0], 4)}
    del rt
    torch.cuda.empty_cache()
    return out


def tp_decode_part(args, cfg, weights, world: int, rank: int, dev) -> dict:
    """Tensor-parallel decode of ONE sequence over all ranks (the north star's
    decode split, engine/tp_decode.py), timed like the replicas: --warmup
    untimed and --steps timed graph replays, max over ranks. The context is
    set to --ctx over a zero-filled cache: a decode step reads the same cache
    bytes and weights whatever the cache holds."""
    import torch
    from engine.tp_decode import TPRuntime
    tp = TPRuntime(cfg, rank, world, dev, max_ctx=args.ctx + args.warmup + args.steps + 32,
                   full=weights)
    tp.capture()
    tp.pos.fill_(args.ctx)
    tp.ctx.fill_(args.ctx + 1)
    for _ in range(args.warmup):
        tp.step()
    barrier(world)
    torch.cuda.synchronize(dev)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        tp.step()
    e.record()
    torch.cuda.synchronize(dev)
    barrier(world)
    t = max_over_ranks(s.elapsed_time(e) / 1e3, world)
    from engine import _native
    timeouts = _native.wait_timeouts(reset=True)
    launches = tp.launches_per_step
    tp.close()
    del tp
    torch.cuda.empty_cache()
    return {"tok_s": round(args.steps / t, 3), "ms_per_step": round(t / args.steps * 1e3, 4),
            "ctx": args.ctx, "ranks": world, "launches_per_step": launches,
            "exchanges_per_step": 2 * cfg.layers + 1, "wait_timeouts": timeouts,
            "partition": ("q/k/v by KV head, DeltaNet in-proj by head, LM head by vocab "
                          "(column-parallel); o/out proj and experts row-parallel "
                          + ("(I/P rows of every expert)" if cfg.inter % (world * cfg.group) == 0
                             else "(experts sharded, 256/P per rank)")
                          + "; one-shot CUDA-IPC allreduce per sub-block")}


# ---------------------------------------------------------------------------
def run_ours(args, world, rank, local) -> None:
    import torch
    from engine import ops
    from engine.runtime import ModelConfig, Qwen36Runtime

    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    cfg = ModelConfig()
    max_ctx = args.ctx + args.warmup + 2 * args.steps + 32
    rt = Qwen36Runtime(cfg, seed=1234, max_ctx=max_ctx, device=dev)
    rt.capture()
    gen = torch.Generator().manual_seed(4096 + rank)
    prompt = torch.randint(0, cfg.vocab, (args.ctx,), generator=gen, dtype=torch.int32)

    # batched prefill of the prompt (one untimed pass sizes the buffers)
    rt.prefill_batched(prompt, chunk=PREFILL_CHUNK)
    rt.reset()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    rt.prefill_batched(prompt, chunk=PREFILL_CHUNK)
    e1.record()
    torch.cuda.synchronize(dev)
    prefill_s = e0.elapsed_time(e1) / 1e3

    for _ in range(args.warmup):
        rt.step()
    torch.cuda.synchronize(dev)

    if args.profile_step:
        # One decode step between cudaProfilerStart/Stop, for
        # `ncu --profile-from-start off` (launch lists and kernel captures).
        torch.cuda.profiler.start()
        rt.step()
        torch.cuda.synchronize(dev)
        torch.cuda.profiler.stop()
        if rank == 0:
            print(json.dumps({"profile_step": "done", "launches": rt.launches_per_step}))
        return

    # timed region: device-resident decode steps (graph replays)
    sampler = ClockSampler(local)
    barrier(world)
    torch.cuda.synchronize(dev)
    sampler.start()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        rt.step()
    e.record()
    torch.cuda.synchronize(dev)
    barrier(world)
    clocks = sampler.stop()
    t_dev = max_over_ranks(s.elapsed_time(e) / 1e3, world)
    value = world * args.steps / t_dev
    ms_per_step = t_dev / args.steps * 1e3

    # e2e: host-resident token in, greedy token out, every step
    pin_in = torch.empty(1, dtype=torch.int32).pin_memory()
    pin_out = torch.empty(1, dtype=torch.int32).pin_memory()
    pin_in.copy_(rt.token.cpu())
    cur = torch.cuda.current_stream(dev)
    barrier(world)
    torch.cuda.synchronize(dev)
    s.record()
    for _ in range(args.steps):
        rt.token.copy_(pin_in, non_blocking=True)
        rt.step()
        pin_out.copy_(rt.token, non_blocking=True)
        cur.synchronize()
        pin_in.copy_(pin_out)
    e.record()
    torch.cuda.synchronize(dev)
    barrier(world)
    t_e2e = max_over_ranks(s.elapsed_time(e) / 1e3, world)
    e2e = {"value": round(world * args.steps / t_e2e, 3), "unit": "tok/s",
           "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4}

    # dominant kernel by time: the one-launch MoE layer, its 40 launches of one
    # step replayed alone (algorithmic bytes: BASELINE config 1 per layer)
    moe_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(moe_graph, stream=rt.stream):
        for l in range(cfg.layers):
            L = rt.w.layers[l]
            ops.moe_layer_decode(rt.hres, L["post_norm"], L["router"], L["sgate"], L["bank"],
                                 L["shared"], rt.b_ids, rt.b_wts, rt.b_logits_r, rt.b_slogit,
                                 workspace=rt.ws_moe, k=cfg.topk, norm_eps=cfg.eps)
    for _ in range(3):
        moe_graph.replay()
    torch.cuda.synchronize(dev)
    s.record()
    for _ in range(10):
        moe_graph.replay()
    e.record()
    torch.cuda.synchronize(dev)
    moe_launch_s = s.elapsed_time(e) / 1e3 / (10 * cfg.layers)
    del moe_graph
    h2 = cfg.hidden

    def u4b(rows, kk):
        return rows * kk // 2 + rows * (kk // cfg.group) * 5 // 2
    moe_bytes = (cfg.experts * h2 * 2 + h2 * 2 + (cfg.topk + 1) *
                 (u4b(2 * cfg.inter, h2) + u4b(h2, cfg.inter)))

    # every multi-output u4 GEMV of one step, replayed alone
    gemv_bytes, gemv_launches = 0, 0
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2, stream=rt.stream):
        gemv_bytes, gemv_launches = rt.enqueue_gemvs_only()
    for _ in range(3):
        g2.replay()
    torch.cuda.synchronize(dev)
    reps = 20
    s.record()
    for _ in range(reps):
        g2.replay()
    e.record()
    torch.cuda.synchronize(dev)
    per_launch_s = s.elapsed_time(e) / 1e3 / (reps * gemv_launches)
    hbm, src = peaks()
    achieved = gemv_bytes / gemv_launches / per_launch_s / 1e9
    ctx_mid = args.ctx + args.warmup + args.steps // 2
    step_bytes = cfg.decode_bytes_per_token(ctx_mid)
    step_gbs = step_bytes / (ms_per_step / 1e3) / 1e9

    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "weak",
        "vs_baseline": round(value / PUBLISHED_DECODE_4K, 3), "dtype": "u4xf16",
        "data": "synthetic",
        "config": {"workload": f"config4 batch-1 greedy decode after a {args.ctx}-token prompt "
                               "(Qwen3.6-35B-A3B-shaped, random-init u4 g128)",
                   "ctx": args.ctx, "decode_steps": args.steps, "parallelism": "replicas",
                   "l2": "inputs larger than L2 (~1.77 GB of weights per step)",
                   "prefill_tok_s": round(world * args.ctx / max_over_ranks(prefill_s, world), 1),
                   "prefill_mode": "batched: tcgen05 u4 GEMMs, DeltaNet scan, causal "
                                   "flash attention, grouped MoE; one pass, device-timed",
                   "step_bytes": step_bytes,
                   "step_hbm_gbs": round(step_gbs, 1),
                   "step_hbm_frac": round(step_gbs / hbm, 4)},
        "e2e": e2e,
        "gpu_launches": rt.launches_per_step * args.steps,
        "roofline": {"bound": "hbm",
                     "kernel": "moe_layer_kernel (one-launch MoE decode layer: router, top-8, "
                               "8 routed + 1 shared expert), its 40 launches of one step",
                     "achieved": round(moe_bytes / moe_launch_s / 1e9, 1), "peak": hbm,
                     "unit": "GB/s", "frac": round(moe_bytes / moe_launch_s / 1e9 / hbm, 4),
                     # DRAM bytes per launch from one ncu capture of this kernel at the
                     # config-1 layer shape (profiles/moe_layer_decode_config1.md)
                     "traffic": DECODE_MOE_TRAFFIC if cfg.layers == 40 else None,
                     "peak_source": src, "bytes_per_launch": moe_bytes,
                     "us_per_launch": round(moe_launch_s * 1e6, 3), "launches": cfg.layers},
        "roofline_gemv": {"bound": "hbm",
                          "kernel": "u4 multi-output GEMV (u4_stream_proj_kernel; ragged shapes "
                                    "u4_gemv_multi_kernel), all launches of one step",
                          "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                          "frac": round(achieved / hbm, 4),
                          # DRAM bytes per launch of these 81 launches from one ncu capture
                          # (profiles/decode_gemv_traffic_ctx256.md)
                          "traffic": DECODE_GEMV_TRAFFIC if cfg.layers == 40 else None,
                          "bytes_per_launch": gemv_bytes // gemv_launches,
                          "launches": gemv_launches},
        "clocks": clocks,
    }
    if world > 1 and not args.no_tp:
        line["tp_decode"] = tp_decode_part(args, cfg, rt.w, world, rank, dev)
    if rank == 0 and world == 1 and not args.no_parts:
        # the rest of BASELINE's metric ("decode & prefill tok/s (4k/32k ctx); u4
        # GEMV HBM GB/s vs peak"), measured after the timed region
        parts = {"decode_ctx4096_tok_s": round(value, 3),
                 "prefill_4096_tok_s": line["config"]["prefill_tok_s"]}
        parts.update(part_long_context(rt.w, dev))
        parts.update(part_gemv_config0(dev))
        parts.update(part_moe_prefill_config3(dev))
        line["metric_parts"] = parts
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.ctx, os.cpu_count() or 1)
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_prefill(args, world, rank, local) -> None:
    """BASELINE config 4 prefill: the batched prefill of a seeded uniform-random
    prompt of --ctx tokens (4096 or 32768) through the full 40-layer model,
    from an empty state. A step is one whole prompt; the state is reset
    between steps outside the timed region. value: prompt tokens/s (token ids
    already on the device); e2e: token ids from pinned host memory and the
    greedy next token read back, every step."""
    import torch
    from engine.runtime import ModelConfig, Qwen36Runtime

    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    cfg = ModelConfig()
    rt = Qwen36Runtime(cfg, seed=1234, max_ctx=args.ctx + 32, device=dev)
    gen = torch.Generator().manual_seed(4096 + rank)
    prompt = torch.randint(0, cfg.vocab, (args.ctx,), generator=gen, dtype=torch.int32)
    dprompt = prompt.to(dev)
    launches = 0
    for _ in range(args.warmup):
        rt.reset()
        launches = rt.prefill_batched(dprompt, chunk=PREFILL_CHUNK)
    torch.cuda.synchronize(dev)
    if args.profile_step:
        rt.reset()
        torch.cuda.synchronize(dev)
        torch.cuda.profiler.start()
        rt.prefill_batched(dprompt, chunk=PREFILL_CHUNK)
        torch.cuda.synchronize(dev)
        torch.cuda.profiler.stop()
        if rank == 0:
            print(json.dumps({"profile_step": "done", "workload": "prefill", "ctx": args.ctx}))
        return
    sampler = ClockSampler(local)
    barrier(world)
    torch.cuda.synchronize(dev)
    sampler.start()
    total = 0.0
    for _ in range(args.steps):
        rt.reset()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        rt.prefill_batched(dprompt, chunk=PREFILL_CHUNK)
        e.record()
        e.synchronize()
        total += s.elapsed_time(e) / 1e3
    barrier(world)
    clocks = sampler.stop()
    per_step = max_over_ranks(total / args.steps, world)
    # e2e through the public API: host token ids in, greedy next token out
    pin_out = torch.empty(1, dtype=torch.int32).pin_memory()
    t_e2e = 0.0
    for _ in range(args.steps):
        rt.reset()
        torch.cuda.synchronize(dev)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        rt.prefill_batched(prompt, chunk=PREFILL_CHUNK)
        pin_out.copy_(rt.token, non_blocking=True)
        e.record()
        e.synchronize()
        t_e2e += s.elapsed_time(e) / 1e3
    t_e2e = max_over_ranks(t_e2e / args.steps, world)
    # dominant kernel group: the MoE block of one layer over one prefill chunk
    # (router + grouped routed experts + shared expert), timed alone
    T = min(args.ctx, PREFILL_CHUNK)
    h = torch.randn(T, cfg.hidden, device=dev, generator=torch.Generator(dev).manual_seed(3))
    L = rt.w.layers[0]
    from engine import ops
    B = rt._prefill_buffers(T)
    ids, wts, lg = B["ids"][:T], B["wts"][:T], B["logits_r"][:T]

    def moe():
        ops.moe_layer_prefill(h, L["post_norm"], L["router"], L["sgate"], L["bank"],
                              L["shared"], ids, wts, lg, workspace=B["mws"], k=cfg.topk)
    for _ in range(3):
        moe()
    reps = 10
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        moe()
    e.record()
    torch.cuda.synchronize(dev)
    moe_s = s.elapsed_time(e) / 1e3 / reps
    flops = T * (cfg.topk * 2 * (2 * cfg.inter * cfg.hidden + cfg.hidden * cfg.inter)
                 + 2 * (2 * cfg.shared_inter * cfg.hidden + cfg.hidden * cfg.shared_inter))
    peak = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"] \
        if (ROOT / "MEASURED_PEAKS.json").exists() else 1590.0
    tflops = flops / moe_s / 1e12
    line = {
        "metric": METRIC, "value": round(world * args.ctx / per_step, 1), "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(per_step * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": round(args.ctx / per_step / PUBLISHED_PREFILL.get(args.ctx, float("nan")),
                             2) if args.ctx in PUBLISHED_PREFILL else None,
        "dtype": "u4xf16", "data": "synthetic",
        "config": {"workload": f"config4 batch-1 prefill of a {args.ctx}-token prompt "
                               "(Qwen3.6-35B-A3B-shaped, random-init u4 g128), batched",
                   "ctx": args.ctx, "parallelism": "replicas" if world > 1 else "single GPU",
                   "l2": "inputs larger than L2 (17.6 GB of weights per pass)",
                   "chunk_tokens": PREFILL_CHUNK},
        "e2e": {"value": round(world * args.ctx / t_e2e, 1), "unit": "tok/s",
                "h2d_bytes_per_step": args.ctx * 4, "d2h_bytes_per_step": 4},
        "gpu_launches": launches * args.steps,
        "roofline": {"bound": "tensor",
                     "kernel": "MoE block of one layer over the prompt (router, grouped "
                               "experts, shared expert; 14 launches), timed alone",
                     "achieved": round(tflops, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(tflops / peak, 4), "traffic": None,
                     "tokens": T, "ms": round(moe_s * 1e3, 3)},
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.ctx // 2, os.cpu_count() or 1)
        line["cpu_baseline"]["sample"] += " (prefill: the same per-token work at the mean context)"
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_op_prefill(args, world, rank, local) -> None:
    """One prompt-path op alone over --tokens T tokens (BASELINE config 4 shapes):
    --workload attn_prefill: causal GQA attention (16 q / 2 kv heads, D 256,
    16-token paged cache, random block table, p0 = 0; tensor roofline);
    --workload delta_prefill: the DeltaNet block (32 v / 16 k heads, D 128;
    reported as tokens/s, the recurrence is sequential over 32-token chunks).
    --profile-step runs one call between cudaProfilerStart/Stop."""
    import torch
    from engine import ops

    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    T = args.tokens
    g = torch.Generator(dev).manual_seed(11 + rank)
    if args.workload == "attn_prefill":
        nblk = (T + 15) // 16 + 2
        q = torch.randn(T, 16, 256, device=dev, generator=g).half()
        kc = torch.randn(nblk, 16, 2, 256, device=dev, generator=g).half()
        vc = torch.randn(nblk, 16, 2, 256, device=dev, generator=g).half()
        bt = torch.randperm(nblk, device=dev, generator=g).int()
        gate = torch.randn(T, 16, 256, device=dev, generator=g).half()
        pos = torch.zeros(1, dtype=torch.int32, device=dev)
        out = torch.empty(T, 16, 256, dtype=torch.float16, device=dev)

        def call():
            ops.attn_prefill(q, kc, vc, bt, pos, 1 / 16, gate=gate, out=out)
        flops = 2 * 2 * T * (T + 16) / 2 * 256 * 16
        metric, launches = "prompt attention tok/s (config 4 shapes)", 1
    else:
        nk, nv, d = 16, 32, 128
        c = (2 * nk + nv) * d
        qkv = (torch.randn(T, c, device=dev, generator=g) * 2).half()
        st = torch.randn(c, 4, device=dev, generator=g).half().float()
        cw = torch.rand(c, 4, device=dev, generator=g) - 0.5
        ab = torch.randn(T, 256, device=dev, generator=g).half()
        alog = torch.rand(nv, device=dev, generator=g) * 3 - 2
        dtb = torch.rand(nv, device=dev, generator=g) * 2 - 1
        state = torch.randn(nv, d, d, device=dev, generator=g) * 0.05
        z = torch.randn(T, nv * d, device=dev, generator=g).half()
        nw = torch.rand(d, device=dev, generator=g) * 0.2 + 0.9
        out = torch.empty(T, nv * d, dtype=torch.float16, device=dev)
        ws = ops.delta_prefill_workspace(T, nk, nv, dev)

        def call():
            ops.delta_prefill(qkv, st, cw, ab[:, :nv], ab[:, nv:2 * nv], alog, dtb, state, z, nw,
                              1e-6, nk, nv, out, workspace=ws)
        flops = None
        metric, launches = "DeltaNet prefill tok/s (config 4 shapes)", 5
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize(dev)
    if args.profile_step:
        torch.cuda.profiler.start()
        call()
        torch.cuda.synchronize(dev)
        torch.cuda.profiler.stop()
        if rank == 0:
            print(json.dumps({"profile_step": "done", "workload": args.workload, "T": T}))
        return
    sampler = ClockSampler(local)
    barrier(world)
    torch.cuda.synchronize(dev)
    sampler.start()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        call()
    e.record()
    torch.cuda.synchronize(dev)
    barrier(world)
    clocks = sampler.stop()
    per = max_over_ranks(s.elapsed_time(e) / 1e3 / args.steps, world)
    line = {"metric": metric, "value": round(world * T / per, 1), "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(per * 1e3, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16" if flops else "f32 state, 3xTF32 products",
            "data": "synthetic",
            "config": {"workload": f"{args.workload} T={T}", "T": T,
                       "l2": "inputs resident; the op's working set is what a layer sees"},
            "gpu_launches": launches * args.steps, "clocks": clocks}
    if flops:
        peak = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"] \
            if (ROOT / "MEASURED_PEAKS.json").exists() else 1590.0
        tf = flops / per / 1e12
        line["roofline"] = {"bound": "tensor", "kernel": "attn_prefill_kernel",
                            "achieved": round(tf, 1), "peak": peak, "unit": "TFLOP/s",
                            "frac": round(tf / peak, 4), "traffic": None}
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_moe_prefill(args, world, rank, local) -> None:
    """grouped MoE prefill of T tokens (bf16 ~N(0,1)) over
    256 u4 g128 experts, router logits N(0,1) + Zipf(1.1)-ranked bias (+-2),
    top-8. Value: tokens/s; roofline: tensor (T * 50,331,648 FLOP per call)."""
    import ctypes

    import numpy as np
    import torch
    from engine import _native as N
    from engine import ops

    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    E, H, I, k, T = 256, 2048, 512, 8, args.tokens
    t = {}
    t["gu_w"] = torch.empty(E, 2 * I, H // 2, dtype=torch.uint8, device=dev)
    t["gu_s"] = torch.empty(E, 2 * I, H // 128, dtype=torch.float16, device=dev)
    t["gu_z"] = torch.empty(E, 2 * I * H // 256, dtype=torch.uint8, device=dev)
    t["d_w"] = torch.empty(E, H, I // 2, dtype=torch.uint8, device=dev)
    t["d_s"] = torch.empty(E, H, I // 128, dtype=torch.float16, device=dev)
    t["d_z"] = torch.empty(E, H * I // 256, dtype=torch.uint8, device=dev)
    for j, v in enumerate(t.values()):
        ops.synth_fill(v, 1 if v.dtype == torch.float16 else 0, 77, 1000 + j, 0.005, 0.02)
    bank = ops.ExpertBank(*t.values(), 128)
    rng = np.random.default_rng(T + rank)
    ranks = rng.permutation(E) + 1
    zw = ranks.astype(np.float64) ** -1.1
    bias = -2 + 4 * (zw - zw.min()) / (zw.max() - zw.min())
    logits = torch.from_numpy((rng.standard_normal((T, E)) + bias).astype(np.float32)).to(dev)
    ids, wts = ops.router_select(logits, k)
    x = torch.randn(T, H, device=dev, generator=torch.Generator(dev).manual_seed(5)).to(
        torch.bfloat16)
    out = torch.empty(T, H, dtype=torch.float32, device=dev)
    ws = torch.empty(N.lib().iq36_moe_prefill_workspace_bytes(T, k, E, H, I), dtype=torch.uint8,
                     device=dev)
    rb = bank.c()
    stream = torch.cuda.current_stream(dev)

    if world > 1 and args.ep:
        # expert parallel: this rank owns E/world experts and its own T tokens
        from engine.parallel_ep import ep_moe_prefill, gpu_expert_fn
        from engine.parallel_tp import shard_expert_bank
        local, _ = shard_expert_bank(bank, rank, world)
        efn = gpu_expert_fn(local)

        def call():
            out.copy_(ep_moe_prefill(x, ids, wts, E, efn))
    else:
        def call():
            N.call("iq36_moe_prefill", x.data_ptr(), T, ids.data_ptr(), wts.data_ptr(), k,
                   ctypes.byref(rb), out.data_ptr(), 0, ws.data_ptr(), ws.numel(),
                   stream.cuda_stream)

    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize(dev)
    if args.profile_step:
        torch.cuda.profiler.start()
        call()
        torch.cuda.synchronize(dev)
        torch.cuda.profiler.stop()
        if rank == 0:
            print(json.dumps({"profile_step": "done", "workload": "moe_prefill", "T": T}))
        return
    # the expert weights (418 MB) exceed L2; flush L2 between calls anyway
    flush = L2Flush(dev)
    sampler = ClockSampler(local)
    barrier(world)
    torch.cuda.synchronize(dev)
    sampler.start()
    # one more untimed call once the clock sampler runs: the expert-parallel
    # path reads split sizes on the host every call, and its first call after
    # the sampler starts was measured 3-20 ms slower than the steady ~1.9 ms
    call()
    barrier(world)
    torch.cuda.synchronize(dev)
    evs = []
    for _ in range(args.steps):
        flush()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        call()
        e.record()
        evs.append((s, e))
    torch.cuda.synchronize(dev)
    barrier(world)
    clocks = sampler.stop()
    per_call = max_over_ranks(sum(s.elapsed_time(e) for s, e in evs) / len(evs) / 1e3, world)
    flops = T * 50331648
    tflops = flops / per_call / 1e12
    peak = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"] \
        if (ROOT / "MEASURED_PEAKS.json").exists() else 1590.0
    # e2e: activations and routing from pinned host memory, output back to host
    hx = x.cpu().pin_memory()
    hids, hw = ids.cpu().pin_memory(), wts.cpu().pin_memory()
    hout = torch.empty(T, H, dtype=torch.float32).pin_memory()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        x.copy_(hx, non_blocking=True)
        ids.copy_(hids, non_blocking=True)
        wts.copy_(hw, non_blocking=True)
        call()
        hout.copy_(out, non_blocking=True)
    e.record()
    torch.cuda.synchronize(dev)
    t_e2e = max_over_ranks(s.elapsed_time(e) / 1e3 / args.steps, world)
    line = {
        "metric": "grouped MoE prefill tok/s (BASELINE config 3)", "value": round(
            world * T / per_call, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(per_call * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u4xbf16->fp16 mma, fp32 accumulate",
        "data": "synthetic",
        "config": {"workload": f"config3 grouped MoE prefill T={T}, 256 experts, top-8, "
                               "Zipf(1.1)-skewed routing", "T": T, "l2": "flushed between calls",
                   "parallelism": (f"ep{world} (NCCL all-to-all dispatch/combine)" if args.ep
                                   else "replicas (every GPU holds all 256 experts, 17 GB)")
                   if world > 1 else "single GPU"},
        "e2e": {"value": round(world * T / t_e2e, 1), "unit": "tok/s",
                "h2d_bytes_per_step": T * H * 2 + T * k * 8, "d2h_bytes_per_step": T * H * 4},
        "gpu_launches": 7 * args.steps,
        "roofline": {"bound": "tensor", "kernel": "iq36_moe_prefill (all 7 launches)",
                     "achieved": round(tflops, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(tflops / peak, 4), "traffic": None},
        "clocks": clocks,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)


class L2Flush:
    """Flush L2 between timed calls: write a buffer larger than L2 (126 MB),
    then read another one, so the dirty lines of the write are written back
    before the timed call instead of during it."""

    def __init__(self, dev):
        import torch
        self.w = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        self.r = torch.zeros(64 << 20, dtype=torch.int32, device=dev)

    def __call__(self):
        self.w.zero_()
        self.r.sum()


def _flushed_call_times(call, steps, flush, dev):
    """Device time of each call, L2 flushed before it (L2Flush)."""
    import torch
    evs = []
    for i in range(steps):
        flush()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        call(i)
        e.record()
        evs.append((s, e))
    torch.cuda.synchronize(dev)
    return [s.elapsed_time(e) / 1e3 for s, e in evs]


def run_moe_decode(args, world, rank, local) -> None:
    """the batch-1 MoE block (router 2048 -> 256 fp16
    ~N(0, 0.02), top-8, 8 routed + 1 shared u4 g128 experts, shared gate) in
    one iq36_moe_block_decode call per step on a fresh x ~N(0,1) from a pool of
    64 (so the routed experts change step to step). L2 flushed before every
    step; value = algorithmic bytes (15,761,408 + 8 KB in/out) / device time."""
    import ctypes

    import numpy as np
    import torch
    from engine import _native as N
    from engine import ops

    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    E, H, I, k, G = 256, 2048, 512, 8, 128

    def make_bank(n, seed):
        t = [torch.empty(n, 2 * I, H // 2, dtype=torch.uint8, device=dev),
             torch.empty(n, 2 * I, H // G, dtype=torch.float16, device=dev),
             torch.empty(n, 2 * I * H // G // 2, dtype=torch.uint8, device=dev),
             torch.empty(n, H, I // 2, dtype=torch.uint8, device=dev),
             torch.empty(n, H, I // G, dtype=torch.float16, device=dev),
             torch.empty(n, H * I // G // 2, dtype=torch.uint8, device=dev)]
        for j, v in enumerate(t):
            ops.synth_fill(v, 1 if v.dtype == torch.float16 else 0, seed, 100 + j, 0.005, 0.02)
        return ops.ExpertBank(*t, G)

    bank, shared = make_bank(E, 21), make_bank(1, 22)
    g = torch.Generator(dev).manual_seed(23 + rank)
    w_router = (torch.randn(E, H, device=dev, generator=g) * 0.02).to(torch.float16)
    w_sg = (torch.randn(1, H, device=dev, generator=g) * 0.02).to(torch.float16)
    xs = torch.randn(64, H, device=dev, generator=g).to(torch.float16)
    ids = torch.empty(k, dtype=torch.int32, device=dev)
    wts = torch.empty(k, dtype=torch.float32, device=dev)
    logits = torch.empty(E, dtype=torch.float32, device=dev)
    out = torch.empty(H, dtype=torch.float16, device=dev)
    ws = torch.empty(N.lib().iq36_moe_block_decode_workspace_bytes(k, H, I), dtype=torch.uint8,
                     device=dev)
    rb, sb = bank.c(), shared.c()
    stream = torch.cuda.current_stream(dev)

    sharded = world > 1 and (args.ep or args.tp)
    if sharded:
        # one block split over the ranks: router replicated, experts sharded
        # (--ep: E/P experts per rank; --tp: I/P intermediate rows of every
        # expert), one NCCL all-reduce of the [H] fp32 partial sums
        from engine import parallel_tp as PT
        if args.ep:
            local, e0 = PT.shard_expert_bank(bank, rank, world)
            sh_local = shared if rank == 0 else None
        else:
            local = PT.shard_expert_bank_rows(bank, rank, world)
            sh_local = PT.shard_expert_bank_rows(shared, rank, world)
        slog = torch.empty(1, dtype=torch.float32, device=dev)
        ws_l = torch.empty(N.lib().iq36_moe_decode_workspace_bytes(k, H, local.intermediate),
                           dtype=torch.uint8, device=dev)

        def call(i):
            x = xs[i % 64]
            N.call("iq36_router_logits", x.data_ptr(), None, None, 0.0, 1, H, w_router.data_ptr(),
                   E, w_sg.data_ptr(), logits.data_ptr(), slog.data_ptr(), stream.cuda_stream)
            N.call("iq36_router_select", logits.data_ptr(), 1, E, k, ids.data_ptr(),
                   wts.data_ptr(), stream.cuda_stream)
            if args.ep:
                part = PT.ep_moe_decode(x, ids, wts, local, e0, sh_local, slog, workspace=ws_l)
            else:
                part = PT.tp_moe_decode(x, ids, wts, local, sh_local, slog, workspace=ws_l)
            out.copy_(part)
    else:
        def call(i):
            N.call("iq36_moe_block_decode", xs[i % 64].data_ptr(), w_router.data_ptr(),
                   w_sg.data_ptr(), k, ctypes.byref(rb), ctypes.byref(sb), ids.data_ptr(),
                   wts.data_ptr(), logits.data_ptr(), out.data_ptr(), 1, ws.data_ptr(),
                   ws.numel(), stream.cuda_stream)

    for i in range(args.warmup):
        call(i)
    torch.cuda.synchronize(dev)
    flush = L2Flush(dev)
    sampler = ClockSampler(local)
    barrier(world)
    torch.cuda.synchronize(dev)
    sampler.start()
    times = _flushed_call_times(call, args.steps, flush, dev)
    clocks = sampler.stop()
    barrier(world)
    per_call = max_over_ranks(sum(times) / len(times), world)
    step_bytes = 15761408 + 2 * H * 2
    hbm, src = peaks()
    gbs = step_bytes / per_call / 1e9
    # end to end: x from pinned host memory, the block output read back, every step
    x_host = xs.cpu().pin_memory()
    out_host = torch.empty(H, dtype=torch.float16).pin_memory()
    barrier(world)
    torch.cuda.synchronize(dev)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(args.steps):
        xs[i % 64].copy_(x_host[i % 64], non_blocking=True)
        call(i)
        out_host.copy_(out, non_blocking=True)
    e.record()
    torch.cuda.synchronize(dev)
    t_e2e = max_over_ranks(s.elapsed_time(e) / 1e3 / args.steps, world)
    agg = 1 if sharded else world
    line = {
        "metric": "MoE decode block HBM GB/s (BASELINE config 1)",
        "value": round(agg * gbs, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(per_call * 1e3, 5),
        "higher_is_better": True, "scaling": "strong" if sharded else "weak",
        "vs_baseline": None, "dtype": "u4xf16", "data": "synthetic",
        "config": {"workload": "config1 MoE decode block: router 2048->256 + top-8 + 8 routed "
                               "and 1 shared u4 g128 experts (I=512) + shared gate, fp16 out",
                   "bytes_per_step": step_bytes, "l2": "flushed before every step",
                   "parallelism": (f"ep{world} (experts sharded, NCCL all-reduce)" if args.ep
                                   else f"tp{world} (expert rows sharded, NCCL all-reduce)")
                   if sharded else ("replicas" if world > 1 else "single GPU")},
        "e2e": {"value": round(agg * step_bytes / t_e2e / 1e9, 1), "unit": "GB/s",
                "h2d_bytes_per_step": H * 2, "d2h_bytes_per_step": H * 2},
        "gpu_launches": 4 * args.steps,
        "roofline": {"bound": "hbm", "kernel": "iq36_moe_block_decode (router, select, gate_up, "
                     "down: 4 launches)", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(gbs / hbm, 4), "traffic": None, "peak_source": src},
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle
        torch.cuda.synchronize(dev)
        sel = ids.cpu().numpy()
        keys = ("gu_w", "gu_s", "gu_z", "d_w", "d_s", "d_z")

        def parts(b):
            return (b.gate_up_weight, b.gate_up_scale, b.gate_up_zp, b.down_weight,
                    b.down_scale, b.down_zp)
        b8 = {key: t[torch.from_numpy(sel.astype(np.int64)).to(dev)].cpu().numpy()
              for key, t in zip(keys, parts(bank))}
        sh = {key: t[0].cpu().numpy() for key, t in zip(keys, parts(shared))}
        wr, wg = w_router.cpu().numpy(), w_sg.cpu().numpy()
        x0 = xs[(args.steps - 1) % 64].cpu().numpy()
        reps, t0 = 0, time.time()
        while time.time() - t0 < 10.0 and reps < 500:
            lg = oracle.f16_linear(x0, wr)
            oid, ow = oracle.router_select(lg[None], k)
            sl = oracle.f16_linear(x0, wg)[0]
            oracle.moe_decode(x0, np.arange(k, dtype=np.int32), ow[0], b8, sh, sl, G,
                              threads=os.cpu_count() or 1)
            reps += 1
        dt = (time.time() - t0) / reps
        line["cpu_baseline"] = {"value": round(step_bytes / dt / 1e9, 3), "unit": "GB/s",
                                "cores": os.cpu_count() or 1, "kind": "port",
                                "sample": f"{reps} oracle MoE blocks (router, top-8, 8 routed + "
                                          "1 shared expert) on one x"}
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_gqa_decode(args, world, rank, local) -> None:
    """paged GQA decode, 16 q heads over 2 KV heads, head
    dim 256, fp16 KV cache in 16-token blocks behind a seeded permuted block
    table, output gate, scale 1/16, at --ctx tokens. L2 flushed before every
    call; value = algorithmic bytes (ctx * 2048 + block table + q/gate/out) /
    device time."""
    import numpy as np
    import torch
    from engine import ops

    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    ctx, nq, nkv, d, bs = args.ctx, 16, 2, 256, 16
    nb = ctx // bs
    g = torch.Generator(dev).manual_seed(31 + rank)
    kc = torch.randn(nb, bs, nkv, d, device=dev, generator=g).to(torch.float16)
    vc = torch.randn(nb, bs, nkv, d, device=dev, generator=g).to(torch.float16)
    bt = torch.from_numpy(np.random.default_rng(ctx + rank).permutation(nb).astype(np.int32)).to(dev)
    q = torch.randn(nq, d, device=dev, generator=g).to(torch.float16)
    gate = torch.randn(nq, d, device=dev, generator=g).to(torch.float16)
    ws = ops.paged_gqa_workspace(ctx, nq, nkv, d, dev)
    out = torch.empty(nq, d, dtype=torch.float32, device=dev)

    def call(i):
        ops.paged_gqa_decode(q, kc, vc, bt, ctx, 1.0 / 16, gate=gate, workspace=ws, out=out)

    for i in range(args.warmup):
        call(i)
    torch.cuda.synchronize(dev)
    flush = L2Flush(dev)
    sampler = ClockSampler(local)
    barrier(world)
    torch.cuda.synchronize(dev)
    sampler.start()
    times = _flushed_call_times(call, args.steps, flush, dev)
    clocks = sampler.stop()
    barrier(world)
    per_call = max_over_ranks(sum(times) / len(times), world)
    step_bytes = ctx * 2048 + nb * 4 + 2 * nq * d * 2 + nq * d * 4
    hbm, src = peaks()
    gbs = step_bytes / per_call / 1e9
    q_host, out_host = q.cpu().pin_memory(), torch.empty(nq, d).pin_memory()
    barrier(world)
    torch.cuda.synchronize(dev)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(args.steps):
        q.copy_(q_host, non_blocking=True)
        call(i)
        out_host.copy_(out, non_blocking=True)
    e.record()
    torch.cuda.synchronize(dev)
    t_e2e = max_over_ranks(s.elapsed_time(e) / 1e3 / args.steps, world)
    line = {
        "metric": "paged GQA decode HBM GB/s (BASELINE config 2)",
        "value": round(world * gbs, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(per_call * 1e3, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic",
        "config": {"workload": f"config2 paged GQA decode, ctx {ctx}, 16 q / 2 KV heads, D 256, "
                               "16-token blocks, permuted block table, output gate",
                   "ctx": ctx, "bytes_per_step": step_bytes, "l2": "flushed before every call",
                   "parallelism": "replicas" if world > 1 else "single GPU"},
        "e2e": {"value": round(world * step_bytes / t_e2e / 1e9, 1), "unit": "GB/s",
                "h2d_bytes_per_step": nq * d * 2, "d2h_bytes_per_step": nq * d * 4},
        "gpu_launches": 2 * args.steps,
        "roofline": {"bound": "hbm", "kernel": "gqa_split_kernel + gqa_combine_kernel",
                     "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(gbs / hbm, 4), "traffic": None, "peak_source": src},
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle
        qn, kn, vn = q.cpu().numpy(), kc.cpu().numpy(), vc.cpu().numpy()
        btn, gn = bt.cpu().numpy(), gate.cpu().numpy()
        reps, t0 = 0, time.time()
        while time.time() - t0 < 10.0 and reps < 200:
            oracle.paged_gqa(qn, kn, vn, btn, ctx, 1.0 / 16, gn, threads=os.cpu_count() or 1)
            reps += 1
        dt = (time.time() - t0) / reps
        line["cpu_baseline"] = {"value": round(step_bytes / dt / 1e9, 3), "unit": "GB/s",
                                "cores": os.cpu_count() or 1, "kind": "port",
                                "sample": f"{reps} oracle paged-GQA decodes at ctx {ctx}"}
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_gemv(args, world, rank, local) -> None:
    """BASELINE config 0 (default 1024 x 2048) or any --rows x --k shape: one
    u4 g128 GEMV per step (fp16 x ~N(0,1), fp32 out) through iq36_u4_gemv.
    Weights rotate through a pool of copies larger than twice the L2, so every
    step reads its weights from HBM. Value: algorithmic GB/s (codes + scales +
    zero points + x + out) over all ranks; roofline: the same per GPU against
    the measured HBM copy bandwidth."""
    import ctypes

    import numpy as np
    import torch
    from engine import _native as N
    from engine import ops

    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    rows, K, G = args.rows, args.k, 128
    one = rows * K // 2 + rows * (K // G) * 2 + rows * (K // G) // 2
    step_bytes = one + K * 2 + rows * 4
    # at least 512 distinct weight copies and twice L2, rotated inside a CUDA graph
    copies = min(max(512, math.ceil(2 * 126e6 / one)), max(2, math.ceil(4e9 / one)))
    pool = []
    for c in range(copies):
        w = torch.empty(rows, K // 2, dtype=torch.uint8, device=dev)
        sc = torch.empty(rows, K // G, dtype=torch.float16, device=dev)
        z = torch.empty(rows * (K // G) // 2, dtype=torch.uint8, device=dev)
        ops.synth_fill(w, 0, 11, 3 * c + 1, 0, 0)
        ops.synth_fill(sc, 1, 11, 3 * c + 2, 0.005, 0.02)
        ops.synth_fill(z, 0, 11, 3 * c + 3, 0, 0)
        pool.append(ops.U4Weight(w, sc, z, G))
    gen = torch.Generator().manual_seed(rank)
    x_host = torch.randn(K, generator=gen).to(torch.float16).pin_memory()
    x = x_host.to(dev)
    out = torch.empty(rows, dtype=torch.float32, device=dev)
    out_host = torch.empty(rows, dtype=torch.float32).pin_memory()
    mats = [N.U4Matrix(wt.weight.data_ptr(), wt.scale.data_ptr(), wt.zp.data_ptr(), rows)
            for wt in pool]
    stream = torch.cuda.current_stream(dev)

    def call(i):
        N.call("iq36_u4_gemv", x.data_ptr(), K, G, ctypes.byref(mats[i % copies]),
               out.data_ptr(), 0, stream.cuda_stream)

    for i in range(args.warmup):
        call(i)
    torch.cuda.synchronize(dev)
    if args.profile_step:
        torch.cuda.profiler.start()
        call(args.warmup)
        torch.cuda.synchronize(dev)
        torch.cuda.profiler.stop()
        if rank == 0:
            print(json.dumps({"profile_step": "done", "workload": "gemv", "rows": rows, "k": K}))
        return
    # the K timed GEMVs (copy i % copies each) captured in one CUDA graph, so the
    # device time is not bounded by per-call host launch cost
    cap = torch.cuda.Stream(dev)
    cap.wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=cap):
        for i in range(args.steps):
            N.call("iq36_u4_gemv", x.data_ptr(), K, G, ctypes.byref(mats[i % copies]),
                   out.data_ptr(), 0, cap.cuda_stream)
    graph.replay()
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(local)
    barrier(world)
    torch.cuda.synchronize(dev)
    sampler.start()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    graph.replay()
    e.record()
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    barrier(world)
    per_call = max_over_ranks(s.elapsed_time(e) / 1e3 / args.steps, world)
    del graph
    # end to end: x from pinned host memory, out read back, every step
    barrier(world)
    torch.cuda.synchronize(dev)
    s.record()
    for i in range(args.steps):
        x.copy_(x_host, non_blocking=True)
        call(i)
        out_host.copy_(out, non_blocking=True)
    e.record()
    torch.cuda.synchronize(dev)
    t_e2e = max_over_ranks(s.elapsed_time(e) / 1e3 / args.steps, world)
    hbm, src = peaks()
    gbs = step_bytes / per_call / 1e9
    line = {
        "metric": "u4 GEMV HBM GB/s (BASELINE config 0 shape unless --rows/--k)",
        "value": round(world * gbs, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(per_call * 1e3, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u4xf16",
        "data": "synthetic",
        "config": {"workload": f"u4 g128 GEMV {rows} x {K}, fp16 x, fp32 out",
                   "rows": rows, "k": K, "bytes_per_step": step_bytes,
                   "l2": f"weights rotate over {copies} copies (> 2x L2) inside a CUDA graph",
                   "parallelism": "replicas" if world > 1 else "single GPU"},
        "e2e": {"value": round(world * step_bytes / t_e2e / 1e9, 1), "unit": "GB/s",
                "h2d_bytes_per_step": K * 2, "d2h_bytes_per_step": rows * 4},
        "gpu_launches": args.steps,
        "roofline": {"bound": "hbm", "kernel": "u4_stream_proj_kernel" if rows % 16 == 0 and
                     K % 512 == 0 and K <= 4096 else "u4_gemv_multi_kernel",
                     "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(gbs / hbm, 4), "traffic": None, "peak_source": src},
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle
        w0 = pool[0]
        wn, sn, zn = (w0.weight.cpu().numpy(), w0.scale.cpu().numpy(), w0.zp.cpu().numpy())
        xn = x_host.numpy()
        reps, t0 = 0, time.time()
        while time.time() - t0 < 10.0 and reps < 200:
            oracle.u4_gemv(xn, wn, sn, zn, G, precise=True)
            reps += 1
        dt = (time.time() - t0) / reps
        line["cpu_baseline"] = {"value": round(step_bytes / dt / 1e9, 3), "unit": "GB/s",
                                "cores": os.cpu_count() or 1, "kind": "port",
                                "sample": f"{reps} oracle GEMVs of the same shape"}
    if rank == 0:
        print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--workload", choices=["decode", "prefill", "moe_prefill", "gemv",
                                           "attn_prefill", "delta_prefill", "moe_decode",
                                           "gqa_decode"],
                    default="decode")
    ap.add_argument("--rows", type=int, default=1024, help="output rows for --workload gemv")
    ap.add_argument("--k", type=int, default=2048, help="input length for --workload gemv")
    ap.add_argument("--tokens", type=int, default=4096,
                    help="T for --workload moe_prefill / attn_prefill / delta_prefill")
    ap.add_argument("--ep", action="store_true",
                    help="--workload moe_prefill / moe_decode at --gpus > 1: expert parallel "
                         "instead of replicas")
    ap.add_argument("--tp", action="store_true",
                    help="--workload moe_decode at --gpus > 1: every expert's rows sharded")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-tp", action="store_true",
                    help="N > 1: skip the tensor-parallel decode of one sequence")
    ap.add_argument("--no-parts", action="store_true",
                    help="decode line only: skip the 32k / config-0 / config-3 parts")
    ap.add_argument("--profile-step", action="store_true",
                    help="run one decode step inside cudaProfilerStart/Stop and exit")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_setup()
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        elif args.workload == "prefill":
            run_prefill(args, world, rank, local)
        elif args.workload == "moe_prefill":
            run_moe_prefill(args, world, rank, local)
        elif args.workload in ("attn_prefill", "delta_prefill"):
            run_op_prefill(args, world, rank, local)
        elif args.workload == "gemv":
            run_gemv(args, world, rank, local)
        elif args.workload == "moe_decode":
            run_moe_decode(args, world, rank, local)
        elif args.workload == "gqa_decode":
            run_gqa_decode(args, world, rank, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
