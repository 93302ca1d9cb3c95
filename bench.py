"""Benchmark of the B200 MoE block (BASELINE.json metric: MoE-layer tokens/s
and HBM GB/s or tensor-pipe % of peak at 1/2/4/8 B200).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload ep|decode|prefill|stack]
                    [--impl ours|reference] [--exchange p2p|nccl] [--layers L] [--decode-steps S]
                    [--no-extras] [--no-cpu-baseline] [--no-oracle]

Workloads (synthetic, seeded, GPT-OSS-120B MoE layout: E=128, H=I=2880, top-4):
  ep       (default) config 3: one MoE layer over 16 384 tokens shared evenly by
           the N ranks (strong scaling).  N=1 runs the whole layer on one GPU;
           N>1 shards the experts (rank r holds experts [r*E/N, (r+1)*E/N)) and
           exchanges token rows and expert outputs between the ranks.  Routing
           uniform (headline) and Zipf(1.1)-skewed (the ``zipf`` key).
  decode   config 1: T=256 decode tokens per GPU, plus a sweep over T=1,8,64,256
  prefill  config 2: T=4096 tokens, router biased to a Zipf(1.1) expert popularity
  stack    config 4: a 36-layer MoE-only stack (RMSNorm + residual between the
           blocks), 32
           sequences x 128 decode steps, experts sharded over the ranks

A step is one MoE-layer forward (router -> dispatch -> MXFP4 SwiGLU experts ->
combine) over the step's tokens with the weights resident in HBM.  Timing: W
untimed warm-up steps, then K steps inside one pair of CUDA events on the
launching stream, bracketed by a barrier and a device synchronize on both
sides; the value is the maximum over ranks.  The layer's weights (1.7 GB, or
1.7/N GB per rank) exceed the 126 MB L2; where the touched weights would fit
(decode T <= 8), a 256 MB buffer is written between timed steps to flush L2.

On N=1 the line also carries the config-1 decode figures with the HBM
roofline of the gate_up kernel (``decode``), the config-2 prefill figures with
its tensor-pipe fraction (``prefill_c2``), the oracle parity of a token
subsample (``parity``) and the CPU baseline (``cpu_baseline``).  On N>1 every
rank compares its expert-parallel output with the single-GPU layer on the same
tokens (``parity``).

``--impl reference`` times the reference algorithm on the host cores (the
numpy restatement in oracle/, used only here and in tests) on the same
workload's layer, one token per call as the reference's route() runs, with
every host thread; rank 0 only.
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
GATE_UP_BYTES_PER_EXPERT = 2 * GPT_OSS_I * GPT_OSS_H // 2 + 2 * GPT_OSS_I * GPT_OSS_H // 32 + 2 * GPT_OSS_I * 2  # 8,824,320
DOWN_BYTES_PER_EXPERT = GPT_OSS_H * GPT_OSS_I // 2 + GPT_OSS_H * GPT_OSS_I // 32 + GPT_OSS_H * 2  # 4,412,160
BYTES_PER_EXPERT = GATE_UP_BYTES_PER_EXPERT + DOWN_BYTES_PER_EXPERT  # 13,236,480
FLOPS_PER_TOKEN = 2 * TOP_K * (GPT_OSS_H * 2 * GPT_OSS_I + GPT_OSS_I * GPT_OSS_H)  # 199,065,600
GATE_UP_FLOPS_PER_PAIR = 2 * GPT_OSS_H * 2 * GPT_OSS_I  # 33,177,600
# dram__bytes_read.sum + dram__bytes_write.sum of one gate_up launch from ncu captures
# (profiles/): decode T=256, prefill T=4096 Zipf.  None where no capture was taken.
PROFILED_GATE_UP_TRAFFIC = {"decode": 1_191_247_000 + 8_817_664, "prefill": 1_068_494_336 + 100_976_128,
                           "config3": 1_583_132_416 + 379_182_848}


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


# ---------------------------------------------------------------------------
# process group and timing helpers
# ---------------------------------------------------------------------------


def dist_setup(use_gpu: bool = True):
    """One process per GPU under torchrun (RANK/LOCAL_RANK/WORLD_SIZE); NCCL for the GPU arm, gloo for the CPU arm."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if use_gpu:
        torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if use_gpu:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def reduce_over_ranks(v: float, world: int, op: str = "max") -> float:
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op={"max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN, "sum": dist.ReduceOp.SUM}[op])
    return float(t.item())


def launch_count() -> int:
    from kcapw_klcquant_b200 import _lib

    return _lib.launch_count()


def time_window(fn, steps: int, warmup: int, world: int, clk: ClockSampler | None = None) -> tuple[float, float]:
    """(ms per step, library kernel launches per step) of ``fn``: W warm-up calls, then K
    calls inside one pair of CUDA events on the current stream, with a barrier and a
    device synchronize on both sides.  ``clk`` samples clocks over the timed calls."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if clk is not None:
        clk.start()
    n0 = launch_count()
    a.record(stream)
    for _ in range(steps):
        fn()
    b.record(stream)
    n1 = launch_count()
    torch.cuda.synchronize()
    if clk is not None:
        clk.stop()
    barrier(world)
    return a.elapsed_time(b) / steps, (n1 - n0) / steps


def time_steps_flushed(fn, steps: int, warmup: int, flush: torch.Tensor | None) -> float:
    """Mean ms of ``fn`` over K calls, each timed alone with CUDA events; when ``flush``
    is given, a buffer larger than L2 is written before every call (outside the events)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        if flush is not None:
            flush.add_(1)
        ev[i][0].record(stream)
        fn()
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    return sum(x.elapsed_time(y) for x, y in ev) / steps


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


def stage_pass(fn, reps: int = 3, flush: torch.Tensor | None = None) -> dict[str, float]:
    """Per-stage milliseconds of ``fn`` (klc_stage_timing), last of ``reps`` passes."""
    from kcapw_klcquant_b200 import _lib

    _lib.stage_timing(True)
    stage = {}
    try:
        for _ in range(reps):
            for _ in range(2):  # the first call keeps the GPU busy while the second's launches are issued
                if flush is not None:
                    flush.add_(1)
                fn()
            stage = _lib.stage_times()
    finally:
        _lib.stage_timing(False)
    return stage


# ---------------------------------------------------------------------------
# layers and parity
# ---------------------------------------------------------------------------


def make_tensors(seed: int, device, zipf: float | None = None) -> dict[str, torch.Tensor]:
    from kcapw_klcquant_b200 import synthetic as syn

    return syn.make_layer(syn.GPT_OSS_120B, seed=seed, zipf=zipf, device=device)


def with_router_bias(tensors: dict[str, torch.Tensor], zipf: float, seed: int) -> dict[str, torch.Tensor]:
    """The same layer with the Zipf(s) router bias (configs 2 and 3-skewed): only the bias differs."""
    from kcapw_klcquant_b200 import synthetic as syn

    t = dict(tensors)
    key = "model.layers.0.mlp.router.bias"
    t[key] = syn.zipf_router_bias(GPT_OSS_E, seed, s=zipf).to(tensors[key].device)
    return t


def layer_from(tensors, device, packed=None):
    """A single-GPU MoeLayer over checkpoint-named tensors (``packed``: reuse resident expert weights)."""
    from kcapw_klcquant_b200 import MoeLayer
    from kcapw_klcquant_b200.mxfp4_expert import PackedLayer

    p = "model.layers.0.mlp"
    if packed is None:
        packed = PackedLayer.from_checkpoint_tensors(tensors[f"{p}.experts.gate_up_proj_blocks"], tensors[f"{p}.experts.gate_up_proj_scales"],
                                                     tensors[f"{p}.experts.down_proj_blocks"], tensors[f"{p}.experts.down_proj_scales"], device)
    return MoeLayer(packed, tensors[f"{p}.router.weight"], tensors[f"{p}.router.bias"], tensors[f"{p}.experts.gate_up_proj_bias"],
                    tensors[f"{p}.experts.down_proj_bias"], top_k=TOP_K)


def compare(y: torch.Tensor, ref: torch.Tensor) -> dict:
    """cosine, max-abs / max|ref| and the fraction of bit-identical bf16 outputs."""
    a, b = y.float().flatten(), ref.float().flatten()
    cos = float((a @ b) / (a.norm() * b.norm()).clamp_min(1e-30))
    nmax = float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))
    beq = float((y.view(torch.int16) == ref.view(torch.int16)).float().mean())
    return {"cosine": cos, "norm_max_abs": nmax, "bit_equal_frac": beq}


def oracle_parity(tensors: dict[str, torch.Tensor], x: torch.Tensor, y: torch.Tensor, idx: torch.Tensor, w: torch.Tensor,
                  n_tokens: int) -> dict:
    """The first ``n_tokens`` outputs against the CPU oracle (the reference's bf16 expert
    path restated) on the device's own routing, one dense expert in host memory at a time."""
    import numpy as np

    from oracle import moe_oracle as orc

    p = "model.layers.0.mlp"

    def bits(t):
        return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)

    sel = idx[:n_tokens].cpu().numpy()
    used = np.unique(sel)
    # only the experts the sample routes to cross to the host
    blocks = {n: tensors[f"{p}.experts.{n}"] for n in ("gate_up_proj_blocks", "gate_up_proj_scales", "down_proj_blocks", "down_proj_scales")}
    sub = {n: t[torch.from_numpy(used).to(t.device).long()].cpu().numpy() for n, t in blocks.items()}
    remap = {int(e): i for i, e in enumerate(used)}
    ex = orc.DenseExperts(sub["gate_up_proj_blocks"], sub["gate_up_proj_scales"], sub["down_proj_blocks"], sub["down_proj_scales"], max_cached=1)
    local_idx = np.vectorize(remap.get)(sel)
    gub = bits(tensors[f"{p}.experts.gate_up_proj_bias"])[used]
    dnb = bits(tensors[f"{p}.experts.down_proj_bias"])[used]
    want = orc.moe_layer(bits(x[:n_tokens]), local_idx, bits(w[:n_tokens]), ex, gub, dnb, "bf16")
    got = bits(y[:n_tokens])
    a = orc.bf16_bits_to_f32(got).astype(np.float64).ravel()
    b = orc.bf16_bits_to_f32(want).astype(np.float64).ravel()
    return {"tokens": n_tokens, "experts": int(used.size), "cosine": float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b))),
            "norm_max_abs": float(np.abs(a - b).max() / np.abs(b).max()), "bit_equal_frac": float(np.mean(got == want))}


# ---------------------------------------------------------------------------
# CPU baseline (the reference algorithm on the host cores)
# ---------------------------------------------------------------------------


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def use_all_host_threads() -> int:
    """Every host thread for torch and numpy's BLAS (torchrun sets OMP_NUM_THREADS=1)."""
    n = host_threads()
    torch.set_num_threads(n)
    try:
        import threadpoolctl

        threadpoolctl.threadpool_limits(n)
    except Exception:
        pass
    return n


def cpu_reference_sample(tensors_cpu: dict[str, torch.Tensor], x_host: torch.Tensor, n_tokens: int, precision: str = "bf16",
                         cold: bool = False) -> float:
    """Tokens/s of the CPU restatement of the reference's route() on the first tokens,
    one token per call (router logits, top-k, softmax, one expert at a time, bf16
    combine).  Warm: the dense experts those tokens use are dequantized before the
    clock starts (the reference's warm cache); cold: the dequantization of each
    expert on first use is timed too (the reference's cache misses)."""
    import numpy as np

    from oracle import moe_oracle as orc

    p = "model.layers.0.mlp"
    bits = lambda t: t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    xs = bits(x_host[:n_tokens])
    rw, rbias = bits(tensors_cpu[f"{p}.router.weight"]), bits(tensors_cpu[f"{p}.router.bias"])
    ex = orc.DenseExperts(*(tensors_cpu[f"{p}.experts.{n}"].numpy() for n in ("gate_up_proj_blocks", "gate_up_proj_scales", "down_proj_blocks", "down_proj_scales")))
    if not cold:
        lg = orc.router_logits_bits(xs, rw, rbias)
        idx, _ = orc.select_topk(orc.bf16_bits_to_f32(lg), TOP_K)
        for e in np.unique(idx):
            ex.get(int(e))
    gub, dnb = bits(tensors_cpu[f"{p}.experts.gate_up_proj_bias"]), bits(tensors_cpu[f"{p}.experts.down_proj_bias"])
    t0 = time.perf_counter()
    for t in range(n_tokens):  # one token at a time, as route() does
        lgt = orc.router_logits_bits(xs[t : t + 1], rw, rbias)
        it, st = orc.select_topk(orc.bf16_bits_to_f32(lgt), TOP_K)
        orc.moe_layer(xs[t : t + 1], it, orc.softmax_weights_bits(st), ex, gub, dnb, precision)
    return n_tokens / (time.perf_counter() - t0)


def cpu_baseline(tensors_cpu: dict[str, torch.Tensor], x_host: torch.Tensor) -> dict:
    """The reported CPU baseline: warm bf16 (value), warm fp32 and cold bf16, all host threads."""
    n = use_all_host_threads()
    warm_bf16 = cpu_reference_sample(tensors_cpu, x_host, 16, "bf16")
    warm_fp32 = cpu_reference_sample(tensors_cpu, x_host, 8, "fp32")
    cold_bf16 = cpu_reference_sample(tensors_cpu, x_host[16:], 2, "bf16", cold=True)
    return {"value": warm_bf16, "unit": "tokens/s", "cores": n, "cpu_model": cpu_model(), "kind": "port",
            "sample": "route() restated in numpy (oracle/), one token per call on the same layer: 16 tokens warm "
                      "(their experts dequantized beforehand), matmul_precision bf16; value = that rate",
            "warm_fp32_tokens_per_s": warm_fp32, "cold_bf16_tokens_per_s": cold_bf16,
            "cold_sample": "2 tokens with every expert dequantized on first use inside the timed region"}


# ---------------------------------------------------------------------------
# arms
# ---------------------------------------------------------------------------


def base_line(args, world: int, value: float, ms: float, launches: float, workload: str, scaling: str, parallelism: str,
              extra_config: dict | None = None) -> dict:
    cfg = {"workload": workload, "precision": args.precision, "expert_path": args.path, "parallelism": parallelism}
    cfg.update(extra_config or {})
    return {"metric": "moe_layer_tokens_per_s", "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded GPT-OSS-120B MXFP4 MoE layer, bf16 N(0,1) activations)",
            "config": cfg, "gpu_launches": launches * args.steps, "gpu_launches_per_step": launches}


def decode_extras(args, ml, device, pk) -> dict:
    """Config 1 on the same layer: T=256 with the gate_up HBM roofline, plus the T sweep."""
    from kcapw_klcquant_b200 import synthetic as syn

    out = {"workload": "config 1: decode MoE layer, E=128, H=I=2880, top-4, uniform routing"}
    flush = torch.empty(256 * 2**20 // 4, dtype=torch.float32, device=device)
    sweep = {}
    for t in (1, 8, 64, 256):
        xs = syn.make_hidden(t, GPT_OSS_H, seed=args.seed + t, device=device)
        ob = torch.empty((t, GPT_OSS_H), dtype=torch.bfloat16, device=device)
        _, rb = ml.forward(xs, precision=args.precision)
        u = int(torch.unique(rb.indices).numel())
        fl = flush if t <= 8 else None
        fn = lambda: ml.forward(xs, precision=args.precision, out=ob, path=args.path)  # noqa: E731
        m = time_steps_flushed(fn, max(args.steps, 10), args.warmup, fl)
        b = u * BYTES_PER_EXPERT + GPT_OSS_E * GPT_OSS_H * 2 + GPT_OSS_E * 2 + t * GPT_OSS_H * 4
        sweep[str(t)] = {"tokens_per_s": t / (m / 1e3), "ms": m, "unique_experts": u, "layer_bytes": b,
                         "layer_gbs": b / (m / 1e3) / 1e9, "layer_frac_hbm": b / (m / 1e3) / 1e9 / pk["hbm_gbs"],
                         "l2": "flushed between steps" if fl is not None else "weights exceed L2"}
        if t == 256:
            stage = stage_pass(fn)
            gu_ms = stage.get("gate_up", float("nan"))
            bytes_gu = u * GATE_UP_BYTES_PER_EXPERT + t * TOP_K * GPT_OSS_H * 2
            ach = bytes_gu / (gu_ms / 1e3) / 1e9
            out.update({"tokens": t, "tokens_per_s": t / (m / 1e3), "ms_per_step": m, "stages_ms": stage,
                        "roofline": {"bound": "hbm", "kernel": "gate_up (block-scaled tcgen05 MMA on packed E2M1, SwiGLU epilogue)",
                                     "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": ach / pk["hbm_gbs"],
                                     "peak_source": pk["source"], "algorithmic_bytes": bytes_gu, "unique_experts": u,
                                     "traffic": PROFILED_GATE_UP_TRAFFIC.get("decode")},
                        "layer_roofline": {"bytes": b, "achieved_gbs": b / (m / 1e3) / 1e9, "frac": b / (m / 1e3) / 1e9 / pk["hbm_gbs"]}})
    out["sweep"] = sweep
    return out


def prefill_extras(args, ml_zipf, device, pk) -> dict:
    """Config 2: T=4096 with the Zipf router bias, gate_up tensor-pipe fraction."""
    from kcapw_klcquant_b200 import synthetic as syn

    T = 4096
    x = syn.make_hidden(T, GPT_OSS_H, seed=args.seed + 2, device=device)
    ob = torch.empty((T, GPT_OSS_H), dtype=torch.bfloat16, device=device)
    fn = lambda: ml_zipf.forward(x, precision=args.precision, out=ob, path=args.path)  # noqa: E731
    ms, launches = time_window(fn, args.steps, args.warmup, 1)
    stage = stage_pass(fn)
    _, rb = ml_zipf.forward(x, precision=args.precision)
    counts = torch.bincount(rb.indices.flatten().long(), minlength=GPT_OSS_E)
    gu_ms = stage.get("gate_up", float("nan"))
    flops_gu = T * TOP_K * GATE_UP_FLOPS_PER_PAIR
    ach = flops_gu / (gu_ms / 1e3) / 1e12
    return {"workload": "config 2: prefill MoE layer, T=4096, E=128, H=I=2880, top-4, Zipf(1.1) router bias",
            "tokens_per_s": T / (ms / 1e3), "ms_per_step": ms, "gpu_launches_per_step": launches, "stages_ms": stage,
            "expert_rows": {"max": int(counts.max()), "min": int(counts.min()), "mean": float(counts.float().mean())},
            "roofline": {"bound": "tensor", "kernel": "gate_up", "achieved": ach, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": ach / pk["bf16_tflops"], "frac_of_sustained": ach / pk["bf16_tflops_sustained"],
                         "peak_source": pk["source"], "algorithmic_flops": flops_gu, "traffic": PROFILED_GATE_UP_TRAFFIC.get("prefill")},
            "layer_tflops": T * FLOPS_PER_TOKEN / (ms / 1e3) / 1e12,
            "layer_frac": T * FLOPS_PER_TOKEN / (ms / 1e3) / 1e12 / pk["bf16_tflops"]}


def run_ep(args, world, rank, local):
    """Config 3: 16 384 tokens shared evenly by the ranks (strong scaling); N=1 is the
    whole layer on one GPU, N>1 shards the experts (expert parallelism)."""
    from kcapw_klcquant_b200 import synthetic as syn

    device = torch.device("cuda", local)
    pk = peaks()
    T_total = args.tokens
    if T_total % world:
        raise SystemExit(f"--tokens {T_total} is not divisible by {world} ranks")
    T = T_total // world
    tensors = make_tensors(args.seed, device)  # same seed and generator: the same layer on every rank
    x_all = syn.make_hidden(T_total, GPT_OSS_H, seed=args.seed, device=device)
    x = x_all[rank * T : (rank + 1) * T].contiguous()
    del x_all
    zipf_tensors = with_router_bias(tensors, 1.1, args.seed)

    if world == 1:
        ml = layer_from(tensors, device)
        ml_zipf = layer_from(zipf_tensors, device, packed=ml.packed)
        out = torch.empty((T, GPT_OSS_H), dtype=torch.bfloat16, device=device)
        fwd = lambda: ml.forward(x, precision=args.precision, out=out, path=args.path)  # noqa: E731
        fwd_zipf = lambda: ml_zipf.forward(x, precision=args.precision, out=out, path=args.path)  # noqa: E731
        e2e_fwd = lambda xd, yd: ml.forward(xd, precision=args.precision, out=yd, path=args.path)[0]  # noqa: E731
        parallelism = "1 GPU"
    else:
        from kcapw_klcquant_b200.ep import ExpertParallelMoe

        moe = ExpertParallelMoe(0, tensors, device, top_k=TOP_K, path=args.path, exchange=args.exchange, max_tokens=T)
        moe_zipf = ExpertParallelMoe(0, zipf_tensors, device, top_k=TOP_K, path=args.path, share_local=moe, exchange=args.exchange,
                                     max_tokens=T)
        if args.fused_return != "auto" and moe._ep is not None:
            for m in (moe, moe_zipf):
                m._ep.set_fused_return(args.fused_return == "on")
        fwd = lambda: moe.forward(x, precision=args.precision)  # noqa: E731
        fwd_zipf = lambda: moe_zipf.forward(x, precision=args.precision)  # noqa: E731
        e2e_fwd = lambda xd, yd: moe.forward(xd, precision=args.precision)[0]  # noqa: E731
        ret = {"auto": "fused into the down epilogue" if world <= 2 else "copy kernel", "on": "fused into the down epilogue",
               "off": "copy kernel"}[args.fused_return] if args.exchange == "p2p" else "all_to_all"
        parallelism = f"ep{world}: experts sharded {GPT_OSS_E // world} per GPU, {moe.exchange_name}; expert outputs returned by {ret}"

    # clocks sampled over the timed legs (headline, Zipf and end-to-end), all of them under load
    clk = ClockSampler(local)
    clk.start()
    ms_local, launches = time_window(fwd, args.steps, args.warmup, world)
    ms = reduce_over_ranks(ms_local, world, "max")
    ms_zipf = reduce_over_ranks(time_window(fwd_zipf, args.steps, args.warmup, world)[0], world, "max")
    e2e_ms = reduce_over_ranks(time_e2e(e2e_fwd, x.cpu().pin_memory(), args.steps, args.warmup, world), world, "max")
    clk.stop()

    # roofline of the dominant kernel: the gate_up grouped GEMM (tensor-bound at these sizes)
    stage = stage_pass(fwd)
    if world == 1:
        pairs = T * TOP_K
        ml.check_device_status()
    else:
        pairs = moe.last_received_rows()
        moe.check_device_status()
    gu_ms = stage.get("gate_up", float("nan"))
    flops_gu = pairs * GATE_UP_FLOPS_PER_PAIR
    ach = flops_gu / (gu_ms / 1e3) / 1e12
    roof = {"bound": "tensor", "kernel": "gate_up grouped GEMM (block-scaled tcgen05 MMA, SwiGLU epilogue)" + (" of rank 0" if world > 1 else ""),
            "achieved": ach, "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": ach / pk["bf16_tflops"],
            "frac_of_sustained": ach / pk["bf16_tflops_sustained"], "peak_source": pk["source"], "algorithmic_flops": flops_gu,
            "rows": pairs, "traffic": PROFILED_GATE_UP_TRAFFIC["config3"] if world == 1 and T == 16384 else None}

    # parity: N=1 against the CPU oracle on a token subsample; N>1 every rank's EP
    # output against the single-GPU layer on the same tokens
    if world == 1:
        y, rb = ml.forward(x, precision=args.precision, path=args.path)
        ys, _ = ml.forward(x[:1024], precision=args.precision, path="simt")  # the CUDA-core path on the first 1024 tokens
        parity = {"vs_oracle": oracle_parity(tensors, x, y, rb.indices, rb.weights, 6) if not args.no_oracle else None,
                  "vs_cuda_core_path_1024_tokens": compare(y[:1024], ys)}
    else:
        y, _ = moe.forward(x, precision=args.precision)
        full = layer_from(tensors, device)
        yref, _ = full.forward(x, precision=args.precision, path=args.path)
        m = compare(y, yref)
        parity = {"vs_single_gpu_layer": {"cosine_min": reduce_over_ranks(m["cosine"], world, "min"),
                                          "norm_max_abs_max": reduce_over_ranks(m["norm_max_abs"], world, "max"),
                                          "bit_equal_frac_min": reduce_over_ranks(m["bit_equal_frac"], world, "min")}}
        del full
        moe_zipf.close()
        moe.close()

    line = base_line(args, world, T_total / (ms / 1e3), ms, launches,
                     f"config 3: MoE layer over {T_total} tokens shared by {world} rank(s) ({T} each), E=128, H=I=2880, top-4, uniform routing",
                     "strong", parallelism, {"l2": "layer weights (1.7 GB, 1.7/N GB per rank) exceed L2", "tokens_total": T_total})
    line.update({
        "roofline": roof,
        "stages_ms": stage,
        "layer_tflops": T_total * FLOPS_PER_TOKEN / (ms / 1e3) / 1e12,
        "zipf": {"routing": "Zipf(1.1) router bias", "value": T_total / (ms_zipf / 1e3), "ms_per_step": ms_zipf},
        "e2e": {"value": T_total / (e2e_ms / 1e3), "unit": "tokens/s",
                "mode": "serving loop: per-step upload and read-back on copy streams, double-buffered",
                "h2d_bytes_per_step": T_total * GPT_OSS_H * 2, "d2h_bytes_per_step": T_total * GPT_OSS_H * 2},
        "parity": parity,
        "clocks": clk.summary(),
    })
    if world == 1 and not args.no_extras:
        line["decode"] = decode_extras(args, ml, device, pk)
        line["prefill_c2"] = prefill_extras(args, ml_zipf, device, pk)
    if world == 1 and not args.no_cpu_baseline:
        cpu = {k: v.cpu() for k, v in tensors.items()}
        line["cpu_baseline"] = cpu_baseline(cpu, x.cpu())
    if rank == 0:
        print(json.dumps(line))


def run_layer(args, world, rank, local):
    """Configs 1 and 2 as single-GPU workloads (N>1: one independent replica per GPU)."""
    from kcapw_klcquant_b200 import synthetic as syn

    device = torch.device("cuda", local)
    pk = peaks()
    decode = args.workload == "decode"
    T = args.tokens
    tensors = make_tensors(args.seed, device, zipf=None if decode else 1.1)
    ml = layer_from(tensors, device)
    x = syn.make_hidden(T, GPT_OSS_H, seed=args.seed + rank, device=device)
    out = torch.empty((T, GPT_OSS_H), dtype=torch.bfloat16, device=device)
    fwd = lambda: ml.forward(x, precision=args.precision, out=out, path=args.path)  # noqa: E731
    clk = ClockSampler(local)
    ms_local, launches = time_window(fwd, args.steps, args.warmup, world, clk)
    ms = reduce_over_ranks(ms_local, world, "max")
    e2e_ms = reduce_over_ranks(time_e2e(lambda xd, yd: ml.forward(xd, precision=args.precision, out=yd, path=args.path)[0],
                                        x.cpu().pin_memory(), args.steps, args.warmup, world), world, "max")
    stage = stage_pass(fwd)
    ml.check_device_status()
    wl = (f"config 1: decode MoE layer, T={T} tokens per GPU" if decode else f"config 2: prefill MoE layer, T={T}, Zipf(1.1) router bias") + ", E=128, H=I=2880, top-4"
    line = base_line(args, world, world * T / (ms / 1e3), ms, launches, wl, "weak", f"replicas x{world}" if world > 1 else "1 GPU",
                     {"l2": "weights (>=1.4 GB) exceed L2"})
    gu_ms = stage.get("gate_up", float("nan"))
    if decode:
        _, rb = ml.forward(x, precision=args.precision)
        u = int(torch.unique(rb.indices).numel())
        b = u * GATE_UP_BYTES_PER_EXPERT + T * TOP_K * GPT_OSS_H * 2
        ach = b / (gu_ms / 1e3) / 1e9
        line["roofline"] = {"bound": "hbm", "kernel": "gate_up", "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s",
                            "frac": ach / pk["hbm_gbs"], "peak_source": pk["source"], "algorithmic_bytes": b, "unique_experts": u,
                            "traffic": PROFILED_GATE_UP_TRAFFIC.get("decode") if T == 256 else None}
    else:
        f = T * TOP_K * GATE_UP_FLOPS_PER_PAIR
        ach = f / (gu_ms / 1e3) / 1e12
        line["roofline"] = {"bound": "tensor", "kernel": "gate_up", "achieved": ach, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                            "frac": ach / pk["bf16_tflops"], "peak_source": pk["source"], "algorithmic_flops": f,
                            "traffic": PROFILED_GATE_UP_TRAFFIC.get("prefill") if T == 4096 else None}
    line.update({"stages_ms": stage, "clocks": clk.summary(),
                 "e2e": {"value": world * T / (e2e_ms / 1e3), "unit": "tokens/s", "mode": "serving loop, double-buffered copies",
                         "h2d_bytes_per_step": T * GPT_OSS_H * 2, "d2h_bytes_per_step": T * GPT_OSS_H * 2}})
    if rank == 0:
        print(json.dumps(line))


def run_stack(args, world, rank, local):
    """Config 4: a 36-layer MoE-only stack (RMSNorm + residual between the blocks), 32
    sequences x 128 decode steps, experts sharded over the ranks (N=1: one GPU).  One
    decode step of all layers is captured as a CUDA graph and replayed per step."""
    from kcapw_klcquant_b200 import synthetic as syn
    from kcapw_klcquant_b200.ep import ExpertParallelMoe
    from kcapw_klcquant_b200.stack import MoeStack

    device = torch.device("cuda", local)
    n_layers, seqs, steps = args.layers, args.tokens, args.decode_steps
    if seqs % world:
        raise SystemExit(f"{seqs} sequences cannot be split over {world} ranks")
    T = seqs // world
    layers, norms = [], []
    for li in range(n_layers):  # independent seeded weights per layer (seed 1000 + layer)
        t = make_tensors(1000 + li, device)
        if world == 1:
            layers.append(layer_from(t, device))
        else:
            layers.append(ExpertParallelMoe(0, t, device, top_k=TOP_K, path=args.path, exchange="p2p", max_tokens=T))
        norms.append(syn.make_rms_weight(GPT_OSS_H, seed=1000 + li, device=device))
        del t
        torch.cuda.empty_cache()
    stack = MoeStack(layers, norms)
    inputs = syn.make_hidden(steps * seqs, GPT_OSS_H, seed=args.seed, device=device).view(steps, seqs, GPT_OSS_H)
    inputs = inputs[:, rank * T : (rank + 1) * T].contiguous()
    n0 = launch_count()
    eager = stack.step(inputs[0]).clone()  # also sizes every workspace before the capture
    launches = launch_count() - n0
    stack.capture(inputs[0])
    replayed = stack.replay(inputs[0]).clone()
    graph_equal = bool(torch.equal(replayed, eager))
    for s in range(args.warmup):
        stack.replay(inputs[s % steps])
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    clk = ClockSampler(local)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk.start()
    a.record()
    for s in range(steps):
        stack.replay(inputs[s])
    b.record()
    torch.cuda.synchronize()
    clk.stop()
    barrier(world)
    ms = reduce_over_ranks(a.elapsed_time(b), world, "max")
    # end to end: every step's input uploaded from pinned host memory, its output read back
    host_in = inputs.cpu().pin_memory()
    host_out = torch.empty((T, GPT_OSS_H), dtype=torch.bfloat16).pin_memory()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for s in range(steps):
        y = stack.replay(host_in[s].to(device, non_blocking=True))
        host_out.copy_(y, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = reduce_over_ranks(e0.elapsed_time(e1), world, "max")
    for layer in layers:
        if hasattr(layer, "check_device_status"):
            layer.check_device_status()
    # parity: N>1, the first two layers of the stack against the single-GPU layers on this rank's tokens
    parity = {"graph_replay_equals_eager": bool(reduce_over_ranks(1.0 if graph_equal else 0.0, world, "min") == 1.0)}
    if world > 1:
        sub = MoeStack(layers[:2], norms[:2])
        y_ep = sub.step(inputs[1])
        full = [layer_from(make_tensors(1000 + li, device), device) for li in range(2)]
        y_ref = MoeStack(full, norms[:2]).step(inputs[1])
        m = compare(y_ep, y_ref)
        parity["two_layers_vs_single_gpu"] = {"cosine_min": reduce_over_ranks(m["cosine"], world, "min"),
                                              "bit_equal_frac_min": reduce_over_ranks(m["bit_equal_frac"], world, "min")}
        del full
    stack.release()
    for layer in layers:
        if hasattr(layer, "close"):
            layer.close()
    tok = seqs * steps
    line = base_line(args, world, tok / (ms / 1e3), ms / steps, launches,
                     f"config 4: {n_layers}-layer MoE stack (RMSNorm + residual between blocks), {seqs} sequences x {steps} decode steps, "
                     f"E=128 ({GPT_OSS_E // world} per GPU), H=I=2880, top-4, independent seeded weights per layer",
                     "weak", f"ep{world}: NVLink peer-memory exchange, one CUDA graph per decode step" if world > 1 else "1 GPU, one CUDA graph per decode step",
                     {"l2": "each layer's weights exceed L2", "sequences": seqs, "decode_steps": steps, "layers": n_layers})
    line.update({"steps": steps, "gpu_launches": launches * steps, "gpu_launches_per_step": launches,
                 "ms_per_step_note": "ms_per_step is one decode step of all layers (one graph replay)",
                 "e2e": {"value": tok / (e2e_ms / 1e3), "unit": "tokens/s", "mode": "per step: input uploaded from pinned host memory, output read back",
                         "h2d_bytes_per_step": seqs * GPT_OSS_H * 2, "d2h_bytes_per_step": seqs * GPT_OSS_H * 2},
                 "parity": parity, "clocks": clk.summary()})
    if rank == 0:
        print(json.dumps(line))


def run_reference(args, world, rank):
    """Reference arm: the reference algorithm (CPU restatement) on the host cores, rank 0
    only, on the same workload's layer; each step a bounded sample of tokens."""
    if rank != 0:
        return
    from kcapw_klcquant_b200 import synthetic as syn

    n_threads = use_all_host_threads()
    zipf = 1.1 if args.workload == "prefill" else None
    tensors = make_tensors(args.seed, "cpu", zipf=zipf)
    x = syn.make_hidden(64, GPT_OSS_H, seed=args.seed, device="cpu")
    n = 4
    vals = []
    for i in range(args.warmup + args.steps):
        v = cpu_reference_sample(tensors, x[(i % 8) * n :], n, args.precision)
        if i >= args.warmup:
            vals.append(v)
    v = statistics.median(vals)
    if args.workload == "stack":
        v /= args.layers  # a stack token passes every layer: the per-layer rate over the layer count
    wl = {"ep": f"config 3: MoE layer over {args.tokens} tokens, E=128, H=I=2880, top-4, uniform routing",
          "decode": f"config 1: decode MoE layer, T={args.tokens}, E=128, H=I=2880, top-4",
          "prefill": f"config 2: prefill MoE layer, T={args.tokens}, Zipf(1.1), E=128, H=I=2880, top-4",
          "stack": "config 4: 36-layer MoE stack, 32 sequences x 128 steps"}[args.workload]
    out = {
        "impl": "reference", "metric": "moe_layer_tokens_per_s", "value": v, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": n / v * 1e3, "higher_is_better": True, "scaling": "strong" if args.workload == "ep" else "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": wl, "precision": args.precision, "cpu_sample_tokens_per_step": n},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": n_threads, "cpu_model": cpu_model(), "kind": "port",
                         "sample": f"{n} tokens per step, one route() call per token restated in numpy (oracle/), experts dequantized beforehand (warm), "
                                   f"matmul_precision {args.precision}, {n_threads} host threads"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["ep", "decode", "prefill", "stack"], default="ep")
    ap.add_argument("--layers", type=int, default=36, help="stack: MoE layers")
    ap.add_argument("--decode-steps", type=int, default=128, help="stack: decode steps (the timed steps)")
    ap.add_argument("--tokens", type=int, default=None)
    ap.add_argument("--precision", choices=["bf16", "fp32"], default="bf16")
    ap.add_argument("--path", choices=["auto", "simt", "tc"], default="auto")
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--no-extras", action="store_true", help="N=1: skip the decode and config-2 figures")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-oracle", action="store_true", help="skip the CPU oracle parity subsample")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p", help="N>1: the expert-parallel exchange")
    ap.add_argument("--fused-return", choices=["auto", "on", "off"], default="auto",
                    help="N>1 p2p: expert outputs stored to the source ranks by the down epilogue (auto: 2 ranks)")
    ap.add_argument("--pair-tiles", type=int, choices=[0, 1, 2], default=1,
                    help="two-SM expert tiles: 0 never, 1 from 192 rows per expert (default), 2 always")
    ap.add_argument("--fused-quantize", type=int, choices=[0, 1], default=1,
                    help="1: the gate_up epilogue writes the down GEMM's E4M3 operand (default); 0: a separate pass")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.tokens is None:
        args.tokens = {"decode": 256, "prefill": 4096, "ep": 16384, "stack": 32}[args.workload]
    world, rank, local = dist_setup(use_gpu=args.impl != "reference")
    if args.impl != "reference":
        from kcapw_klcquant_b200 import _lib

        _lib.check(_lib.lib().klc_set_pair_tiles(args.pair_tiles))
        _lib.check(_lib.lib().klc_set_fused_quantize(args.fused_quantize))
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        elif args.workload == "ep":
            run_ep(args, world, rank, local)
        elif args.workload == "stack":
            run_stack(args, world, rank, local)
        else:
            run_layer(args, world, rank, local)
    finally:
        import torch.distributed as dist

        if dist.is_available() and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
