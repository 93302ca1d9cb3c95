"""Benchmark of the B200 MoE block (BASELINE.json metric: MoE-layer tokens/s
and HBM GB/s or tensor-pipe % of peak).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload decode|prefill] [--impl ours|reference]

Workloads (synthetic, seeded, GPT-OSS-120B MoE layout: E=128, H=I=2880, top-4):
  decode   config 1: T=256 tokens per GPU (headline), plus a sweep over T=1,8,64,256
  prefill  config 2: T=4096 tokens, router biased to a Zipf(1.1) expert popularity

A step is one MoE-layer forward (router -> dispatch -> MXFP4 SwiGLU experts ->
combine) over the step's tokens with the weights resident in HBM.  With N>1
(one process per GPU under torchrun) every rank runs the same per-GPU
workload on its own layer replica (weak scaling; the layer needs no
collective when tokens are split by rank).  Timing: W untimed warm-up steps,
then K steps bracketed by a barrier and cuda synchronize, CUDA events on the
launching stream, max over ranks.  The weights (1.7 GB per layer) exceed the
126 MB L2, so each step streams them from HBM; for T <= 8 (52-380 MB of
weights touched) a 256 MB buffer is written between timed steps to flush L2.

``--impl reference`` times the reference algorithm on the host CPU (the numpy
restatement in oracle/, used only here and in tests) on the same layer,
rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

import torch  # noqa: E402

GPT_OSS_E, GPT_OSS_H, GPT_OSS_I, TOP_K = 128, 2880, 2880, 4
BYTES_PER_EXPERT = (2 * GPT_OSS_I * GPT_OSS_H // 2 + 2 * GPT_OSS_I * GPT_OSS_H // 32 + 2 * GPT_OSS_I * 2) + (
    GPT_OSS_H * GPT_OSS_I // 2 + GPT_OSS_H * GPT_OSS_I // 32 + GPT_OSS_H * 2
)  # 13,236,480
GATE_UP_BYTES_PER_EXPERT = 2 * GPT_OSS_I * GPT_OSS_H // 2 + 2 * GPT_OSS_I * GPT_OSS_H // 32 + 2 * GPT_OSS_I * 2  # 8,824,320
FLOPS_PER_TOKEN = 2 * TOP_K * (GPT_OSS_H * 2 * GPT_OSS_I + GPT_OSS_I * GPT_OSS_H)  # 199,065,600
# dram__bytes_read.sum + dram__bytes_write.sum of one gate_up launch from an ncu capture of
# this workload at T=256 (decode) and T=4096 (prefill) (ncu --set full, one launch); None where
# no capture was taken
PROFILED_GATE_UP_TRAFFIC = {"decode": 1_145_114_000 + 8_942_592, "prefill": 1_024_244_000 + 95_751_424}


def peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """SM clock and clock-event reasons polled through NVML (read-only queries) every
    millisecond between start() and stop(), i.e. while the timed steps run on the GPU."""

    REASONS = {"hw_slowdown": "nvmlClocksEventReasonHwSlowdown", "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
               "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown", "sw_power_cap": "nvmlClocksEventReasonSwPowerCap"}

    def __init__(self, cuda_index: int):
        self.samples: list[int] = []
        self.reasons: set[str] = set()
        self.max_mhz = None
        self.h = None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml as nv

            nv.nvmlInit()
            self.nv = nv
            self.h = self._handle(cuda_index)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
        except Exception:  # no NVML: the line says so through samples == 0
            self.h = None

    def _handle(self, i: int):
        nv = self.nv
        p = torch.cuda.get_device_properties(i)
        if all(hasattr(p, a) for a in ("pci_domain_id", "pci_bus_id", "pci_device_id")):
            try:
                return nv.nvmlDeviceGetHandleByPciBusId(f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0")
            except Exception:
                pass
        return nv.nvmlDeviceGetHandleByIndex(i)

    def _poll(self):
        nv = self.nv
        bits = {n: getattr(nv, a) for n, a in self.REASONS.items()}
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.reasons.update(n for n, b in bits.items() if r & b)
            except Exception:
                return
            time.sleep(0.001)

    def start(self):
        if self.h is not None:
            self._stop.clear()
            self._t = threading.Thread(target=self._poll, daemon=True)
            self._t.start()

    def stop(self):
        if self._t is not None:
            self._stop.set()
            self._t.join(timeout=5)
            self._t = None

    def summary(self) -> dict:
        sm = self.samples
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(sm), "source": "nvml" if self.h is not None else "unavailable"}


def dist_setup(use_gpu: bool = True, force_group: bool = False):
    """One process per GPU under torchrun (RANK/LOCAL_RANK/WORLD_SIZE); NCCL for the GPU arm, gloo for the CPU arm."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if use_gpu:
        torch.cuda.set_device(local)
    if world > 1 or force_group:
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if "MASTER_PORT" not in os.environ:
            import socket

            with socket.socket() as sk:
                sk.bind(("127.0.0.1", 0))
                os.environ["MASTER_PORT"] = str(sk.getsockname()[1])
        os.environ.setdefault("RANK", str(rank))
        os.environ.setdefault("WORLD_SIZE", str(world))
        if use_gpu:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    return world, rank, local


def barrier(world):
    import torch.distributed as dist

    if world > 1 or (dist.is_available() and dist.is_initialized()):
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def make_layer(workload: str, seed: int, device):
    from kcapw_klcquant_b200 import MoeLayer
    from kcapw_klcquant_b200 import synthetic as syn

    zipf = 1.1 if workload == "prefill" else None
    layer = syn.make_layer(syn.GPT_OSS_120B, seed=seed, zipf=zipf, device=device)
    return MoeLayer.from_tensors(0, layer, device, top_k=TOP_K)


def time_steps(fn, steps: int, warmup: int, flush: torch.Tensor | None, world: int, clk: ClockSampler | None = None):
    """Per-step device times (ms) of ``fn`` with CUDA events on the current stream; ``clk``
    samples clocks from the first timed launch to the end of the last timed step."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    if clk is not None:
        clk.start()
    for i in range(steps):
        if flush is not None:
            flush.add_(1)
        ev[i][0].record(stream)
        fn()
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    if clk is not None:
        clk.stop()
    barrier(world)
    return [a.elapsed_time(b) for a, b in ev]


def time_e2e(forward, x_host: torch.Tensor, steps: int, warmup: int, world: int) -> float:
    """Milliseconds per step through the public API with host buffers, as a serving loop
    runs it: every step uploads its input from pinned host memory and reads its result
    back, on their own streams and double-buffered, so step i+1's upload and step i-1's
    read-back overlap step i's kernels.  The timed window starts before the first upload
    and ends after the last read-back (CUDA events; max over ranks by the caller).

    ``forward(x_dev, y_dev)`` runs one step on the current stream and returns its output
    tensor (``y_dev`` when it writes there)."""
    comp = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    T, H = x_host.shape
    xb = [torch.empty((T, H), dtype=x_host.dtype, device=comp.device) for _ in range(2)]
    yb = [torch.empty((T, GPT_OSS_H), dtype=torch.bfloat16, device=comp.device) for _ in range(2)]
    yh = [torch.empty((T, GPT_OSS_H), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    up_done = [torch.cuda.Event() for _ in range(2)]
    comp_done = [torch.cuda.Event() for _ in range(2)]
    down_done = [torch.cuda.Event() for _ in range(2)]

    def run(n: int):
        with torch.cuda.stream(up):
            xb[0].copy_(x_host, non_blocking=True)
            up_done[0].record(up)
        for i in range(n):
            b = i & 1
            if i + 1 < n:
                with torch.cuda.stream(up):
                    if i >= 1:
                        up.wait_event(comp_done[b ^ 1])  # step i-1 has read that input buffer
                    xb[b ^ 1].copy_(x_host, non_blocking=True)
                    up_done[b ^ 1].record(up)
            comp.wait_event(up_done[b])
            if i >= 2:
                comp.wait_event(down_done[b])  # step i-2's result has left that output buffer
            y = forward(xb[b], yb[b])
            comp_done[b].record(comp)
            with torch.cuda.stream(down):
                down.wait_event(comp_done[b])
                if y is not yb[b]:
                    y.record_stream(down)
                yh[b].copy_(y, non_blocking=True)
                down_done[b].record(down)
        comp.wait_stream(down)

    run(warmup)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(comp)
    run(steps)
    t1.record(comp)
    torch.cuda.synchronize()
    barrier(world)
    return t0.elapsed_time(t1) / steps


def unique_experts(ml, x) -> int:
    _, rb = ml.forward(x, precision="bf16")
    return int(torch.unique(rb.indices).numel())


def cpu_baseline_sample(layer: dict[str, torch.Tensor], x_host: torch.Tensor, n_tokens: int) -> dict:
    """Time the CPU restatement of the reference (oracle/) on the first tokens, dense experts cached.

    ``layer`` holds the checkpoint-named tensors on the CPU.  Mirrors the
    reference's warm decode path: one route() per token (bf16 logits, top-k,
    softmax, per-expert GEMVs with the dequantized experts already cached,
    bf16 combine).
    """
    import numpy as np

    from oracle import moe_oracle as orc

    p = "model.layers.0.mlp"
    bits = lambda t: t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    xs = bits(x_host[:n_tokens])
    rw, rbias = bits(layer[f"{p}.router.weight"]), bits(layer[f"{p}.router.bias"])
    lg = orc.router_logits_bits(xs, rw, rbias)
    idx, _ = orc.select_topk(orc.bf16_bits_to_f32(lg), TOP_K)
    ex = orc.DenseExperts(*(layer[f"{p}.experts.{n}"].cpu().numpy() for n in ("gate_up_proj_blocks", "gate_up_proj_scales", "down_proj_blocks", "down_proj_scales")))
    for e in np.unique(idx):  # warm the dequantized-expert cache (the reference's warm path)
        ex.get(int(e))
    gub, dnb = bits(layer[f"{p}.experts.gate_up_proj_bias"]), bits(layer[f"{p}.experts.down_proj_bias"])
    t0 = time.perf_counter()
    for t in range(n_tokens):  # one token at a time, as route() does
        lgt = orc.router_logits_bits(xs[t : t + 1], rw, rbias)
        it, st = orc.select_topk(orc.bf16_bits_to_f32(lgt), TOP_K)
        orc.moe_layer(xs[t : t + 1], it, orc.softmax_weights_bits(st), ex, gub, dnb, "bf16")
    dt = time.perf_counter() - t0
    return {"value": n_tokens / dt, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{n_tokens} tokens of the same layer, one token per route() call, experts pre-dequantized (warm cache), numpy with all host threads"}


def run_reference(args, world, rank):
    """Reference arm: the reference algorithm (CPU restatement) on the host cores, rank 0 only."""
    if rank != 0:
        return
    from kcapw_klcquant_b200 import synthetic as syn

    T = args.tokens
    zipf = 1.1 if args.workload == "prefill" else None
    layer = syn.make_layer(syn.GPT_OSS_120B, seed=args.seed, zipf=zipf, device="cpu")
    x = syn.make_hidden(T, GPT_OSS_H, seed=args.seed, device="cpu")
    n = 4
    vals, r = [], {}
    for i in range(args.warmup + args.steps):
        r = cpu_baseline_sample(layer, x, n)
        if i >= args.warmup:
            vals.append(r["value"])
    v = statistics.median(vals)
    out = {
        "impl": "reference", "metric": "moe_layer_tokens_per_s", "value": v, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": n / v * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"config {'1' if args.workload == 'decode' else '2'}: {args.workload} MoE layer, T={T}, E=128, H=I=2880, top-4",
                   "cpu_sample_tokens": n},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port", "sample": r["sample"]},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out))


def run_ours(args, world, rank, local):
    from kcapw_klcquant_b200 import _lib
    from kcapw_klcquant_b200 import synthetic as syn

    device = torch.device("cuda", local)
    T = args.tokens
    ml = make_layer(args.workload, args.seed, device)
    x = syn.make_hidden(T, GPT_OSS_H, seed=args.seed + rank, device=device)
    pk = peaks()
    flush = torch.empty(256 * 2**20 // 4, dtype=torch.float32, device=device) if T <= 8 else None
    out = torch.empty((T, GPT_OSS_H), dtype=torch.bfloat16, device=device)
    fwd = lambda: ml.forward(x, precision=args.precision, out=out, path=args.path)  # noqa: E731

    U = unique_experts(ml, x)
    clk = ClockSampler(local)
    times = time_steps(fwd, args.steps, args.warmup, flush, world, clk)
    ms = max_over_ranks(sum(times) / len(times), world)
    tokens_per_s = world * T / (ms / 1e3)

    # stage breakdown (same workload, separate pass)
    _lib.stage_timing(True)
    stage = {}
    for _ in range(3):
        for _ in range(2):  # the first call keeps the GPU busy while the second's launches are issued
            if flush is not None:
                flush.add_(1)
            fwd()
        stage = _lib.stage_times()
    _lib.stage_timing(False)
    # end-to-end through the public API with host buffers
    x_host = x.cpu().pin_memory()
    e2e_ms = max_over_ranks(time_e2e(lambda xd, yd: ml.forward(xd, precision=args.precision, out=yd, path=args.path)[0],
                                     x_host, args.steps, args.warmup, world), world)
    ml.check_device_status()  # a kernel that gave up on a bounded wait would make every number above invalid

    # roofline of the dominant kernel (gate_up GEMM for decode)
    decode = args.workload == "decode"
    if decode:
        gu_ms = stage.get("gate_up", float("nan"))
        bytes_gu = U * GATE_UP_BYTES_PER_EXPERT + T * TOP_K * GPT_OSS_H * 2
        achieved = bytes_gu / (gu_ms / 1e3) / 1e9
        roof = {"bound": "hbm", "kernel": "gate_up GEMM (MXFP4 dequant + SwiGLU epilogue)", "achieved": achieved, "peak": pk["hbm_gbs"],
                "unit": "GB/s", "frac": achieved / pk["hbm_gbs"], "peak_source": pk["source"],
                "traffic": PROFILED_GATE_UP_TRAFFIC.get("decode") if T == 256 else None,
                "algorithmic_bytes": bytes_gu, "unique_experts": U}
        layer_bytes = U * BYTES_PER_EXPERT + GPT_OSS_E * GPT_OSS_H * 2 + GPT_OSS_E * 2 + T * GPT_OSS_H * 4
        layer_roof = {"bytes": layer_bytes, "achieved_gbs": layer_bytes / (ms / 1e3) / 1e9, "frac": layer_bytes / (ms / 1e3) / 1e9 / pk["hbm_gbs"]}
    else:
        gu_ms = stage.get("gate_up", float("nan"))
        flops_gu = 2 * T * TOP_K * GPT_OSS_H * 2 * GPT_OSS_I
        achieved = flops_gu / (gu_ms / 1e3) / 1e12
        roof = {"bound": "tensor", "kernel": "gate_up GEMM", "achieved": achieved, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": achieved / pk["bf16_tflops"], "peak_source": pk["source"], "algorithmic_flops": flops_gu,
                "traffic": PROFILED_GATE_UP_TRAFFIC.get("prefill") if args.workload == "prefill" and T == 4096 else None}
        layer_roof = {"flops": T * FLOPS_PER_TOKEN, "achieved_tflops": T * FLOPS_PER_TOKEN / (ms / 1e3) / 1e12}

    result = {
        "metric": "moe_layer_tokens_per_s",
        "value": tokens_per_s,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded GPT-OSS-120B MXFP4 MoE layer, bf16 N(0,1) activations)",
        "config": {
            "workload": f"config {'1' if decode else '2'}: {args.workload} MoE layer, T={T} tokens per GPU, E=128, H=I=2880, top-4"
                        + (", Zipf(1.1) router bias" if not decode else ""),
            "precision": args.precision, "expert_path": args.path, "l2": "L2 flushed between steps" if flush is not None else "weights (>=1.4 GB) exceed L2",
            "parallelism": f"replicas x{world}" if world > 1 else "1 GPU",
        },
        "roofline": roof,
        "layer_roofline": layer_roof,
        "stages_ms": stage,
        "e2e": {"value": world * T / (e2e_ms / 1e3), "unit": "tokens/s", "mode": "serving loop: per-step upload and read-back on copy streams, double-buffered", "h2d_bytes_per_step": T * GPT_OSS_H * 2, "d2h_bytes_per_step": T * GPT_OSS_H * 2},
        "gpu_launches": 7 * args.steps,
        "clocks": clk.summary(),
    }
    if decode and args.sweep and world == 1:
        sweep = {}
        for t in (1, 8, 64, 256):
            xs = syn.make_hidden(t, GPT_OSS_H, seed=args.seed + t, device=device)
            ob = torch.empty((t, GPT_OSS_H), dtype=torch.bfloat16, device=device)
            u = unique_experts(ml, xs)
            tt = time_steps(lambda: ml.forward(xs, precision=args.precision, out=ob, path=args.path), max(args.steps, 5), args.warmup, flush if t <= 8 else None, 1)
            m = sum(tt) / len(tt)
            b = u * BYTES_PER_EXPERT + GPT_OSS_E * GPT_OSS_H * 2 + GPT_OSS_E * 2 + t * GPT_OSS_H * 4
            sweep[str(t)] = {"tokens_per_s": t / (m / 1e3), "ms": m, "unique_experts": u, "layer_gbs": b / (m / 1e3) / 1e9,
                             "layer_frac_hbm": b / (m / 1e3) / 1e9 / pk["hbm_gbs"]}
        result["decode_sweep"] = sweep
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        p = ml.packed
        layer_cpu = {
            "model.layers.0.mlp.router.weight": ml.router_weight.cpu(), "model.layers.0.mlp.router.bias": ml.router_bias.cpu(),
            "model.layers.0.mlp.experts.gate_up_proj_bias": ml.gate_up_bias.cpu(), "model.layers.0.mlp.experts.down_proj_bias": ml.down_bias.cpu(),
            "model.layers.0.mlp.experts.gate_up_proj_blocks": p.gu_blocks.cpu(), "model.layers.0.mlp.experts.gate_up_proj_scales": p.gu_scales.cpu(),
            "model.layers.0.mlp.experts.down_proj_blocks": p.dn_blocks.cpu(), "model.layers.0.mlp.experts.down_proj_scales": p.dn_scales.cpu(),
        }
        result["cpu_baseline"] = cpu_baseline_sample(layer_cpu, x.cpu(), 4)
    if rank == 0:
        print(json.dumps(result))


def run_ep(args, world, rank, local):
    """N > 1: experts sharded over the ranks (EP), NCCL all-to-all dispatch and combine."""
    from kcapw_klcquant_b200 import synthetic as syn
    from kcapw_klcquant_b200.ep import ExpertParallelMoe

    device = torch.device("cuda", local)
    strong = args.workload == "ep-prefill"
    T = (args.tokens // world) if strong else args.tokens
    zipf = 1.1 if (args.workload == "prefill" or args.zipf) else None
    layer = syn.make_layer(syn.GPT_OSS_120B, seed=args.seed, zipf=zipf, device=device)  # same seed: same layer on every rank
    moe = ExpertParallelMoe(0, layer, device, top_k=TOP_K, path=args.path)
    del layer
    torch.cuda.empty_cache()
    x = syn.make_hidden(T, GPT_OSS_H, seed=args.seed + rank, device=device)
    pk = peaks()
    fwd = lambda: moe.forward(x, precision=args.precision)  # noqa: E731
    clk = ClockSampler(local)
    times = time_steps(fwd, args.steps, args.warmup, None, world, clk)
    ms = max_over_ranks(sum(times) / len(times), world)
    x_host = x.cpu().pin_memory()
    e2e_ms = max_over_ranks(time_e2e(lambda xd, yd: moe.forward(xd, precision=args.precision)[0], x_host, args.steps,
                                     args.warmup, world), world)
    moe.check_device_status()
    epr = GPT_OSS_E // world
    layer_bytes = epr * BYTES_PER_EXPERT  # per rank: its experts' weights (all are routed to at these sizes)
    result = {
        "metric": "moe_layer_tokens_per_s",
        "value": world * T / (ms / 1e3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "strong" if strong else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded GPT-OSS-120B MXFP4 MoE layer, bf16 N(0,1) activations)",
        "config": {
            "workload": (f"config 3: expert-parallel MoE layer, {args.tokens} tokens split over {world} ranks" if strong
                         else f"config 1 layout, expert-parallel decode: T={T} tokens per GPU") + f", E=128 ({epr} per GPU), H=I=2880, top-4"
                        + (", Zipf(1.1) router bias" if zipf else ", uniform routing"),
            "precision": args.precision, "expert_path": args.path, "l2": "weights (>=210 MB per GPU) exceed L2",
            "parallelism": f"ep{world} (NCCL all-to-all dispatch + combine)",
        },
        "roofline": {"bound": "hbm" if not strong else "tensor", "kernel": "whole EP layer step (per rank)",
                     "achieved": layer_bytes / (ms / 1e3) / 1e9, "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": layer_bytes / (ms / 1e3) / 1e9 / pk["hbm_gbs"], "traffic": None, "peak_source": pk["source"]},
        "e2e": {"value": world * T / (e2e_ms / 1e3), "unit": "tokens/s", "mode": "serving loop: per-step upload and read-back on copy streams, double-buffered", "h2d_bytes_per_step": T * GPT_OSS_H * 2,
                "d2h_bytes_per_step": T * GPT_OSS_H * 2},
        "gpu_launches": 11 * args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0:
        print(json.dumps(result))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["decode", "prefill", "ep-prefill"], default="decode")
    ap.add_argument("--zipf", action="store_true", help="Zipf(1.1)-skewed router for the EP workloads")
    ap.add_argument("--tokens", type=int, default=None)
    ap.add_argument("--precision", choices=["bf16", "fp32"], default="bf16")
    ap.add_argument("--path", choices=["auto", "simt", "tc"], default="auto")
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--sweep", action="store_true", default=True)
    ap.add_argument("--no-sweep", dest="sweep", action="store_false")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.tokens is None:
        args.tokens = {"decode": 256, "prefill": 4096, "ep-prefill": 16384}[args.workload]
    world, rank, local = dist_setup(use_gpu=args.impl != "reference",
                                    force_group=(args.impl != "reference" and args.workload == "ep-prefill"))
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        elif world > 1 or args.workload == "ep-prefill":
            run_ep(args, world, rank, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        import torch.distributed as dist

        if dist.is_available() and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
