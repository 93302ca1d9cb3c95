"""Generate the golden fixtures in this directory by running the reference itself.

The reference (KLCquant, a pure Python/PyTorch package) is imported from its
source tree on the CPU; nothing here runs on a GPU.  Usage::

    python tests/golden/make_golden.py --reference <path to the klcquant source tree>

The script links the source tree as a package named ``klcquant`` in a temporary
directory, writes seeded synthetic checkpoints in the GPT-OSS MXFP4 layout (see
``kcapw_klcquant_b200/synthetic.py``), and records what these reference
functions return:

* ``dequantize_mxfp4_matrix``        (klcquant mxfp4_expert.py:357-379)
* ``StreamedMoERouter.route``        (klcquant streamed_moe_router.py:257-329), per token, both
  ``matmul_precision`` values, through ``Mxfp4ExpertStore`` (mxfp4_expert.py:382-525)
* ``StreamedMoERouter.route`` with ``RoutingLocalityConfig`` enabled (streamed_moe_router.py:12-35,
  331-476) on correlated token sequences: per-token routing dicts and the final
  ``RouterStats.to_json()`` (:38-235)
* ``rms_norm``                       (klcquant streamed_attention.py:27-28)
* ``RuntimeDequantizer.dequantize``  (klcquant runtime_dequantizer.py:30-52) on artefacts made by
  ``quantize_for_storage`` / ``prune_for_storage`` (adaptive_quantizer.py:123-143, tensor_pruner.py:46-59)

Inputs are regenerated from their seeds by the tests, so only outputs (and the
small runtime-dequantizer artefacts) are stored.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from kcapw_klcquant_b200 import synthetic as syn  # noqa: E402
from tests.golden.cases import LOCALITY_CASES, ROUTE_CASES, correlated_hidden, resident_set, tie_layer  # noqa: E402

def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def f16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.float16).contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def f32_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.float32).contiguous().numpy().view(np.uint32).copy()


def import_reference(reference: Path):
    tmp = Path(tempfile.mkdtemp(prefix="klcref_"))
    (tmp / "klcquant").symlink_to(reference.resolve(), target_is_directory=True)
    sys.path.insert(0, str(tmp))
    import klcquant.mxfp4_expert as mx
    import klcquant.streamed_moe_router as rt
    import klcquant.streamed_attention as at
    import klcquant.runtime_dequantizer as rd
    import klcquant.adaptive_quantizer as aq
    import klcquant.tensor_pruner as tp

    return mx, rt, at, rd, aq, tp


def make_dequant_fixtures(mx) -> None:
    blocks = torch.zeros(256, 1, 16, dtype=torch.uint8)
    for i in range(16):
        blocks[:, 0, i] = i | (((i + 5) % 16) << 4)
    scales = torch.arange(256, dtype=torch.uint8).reshape(256, 1)
    g = torch.Generator().manual_seed(5)
    rb = torch.randint(0, 256, (40, 3, 16), generator=g, dtype=torch.uint8)
    rs = torch.randint(0, 256, (40, 3), generator=g, dtype=torch.uint8)
    out = {"table_blocks": blocks.numpy(), "table_scales": scales.numpy(), "rand_blocks": rb.numpy(), "rand_scales": rs.numpy()}
    for tag, (b, s) in {"table": (blocks, scales), "rand": (rb, rs)}.items():
        out[f"{tag}_bf16"] = bf16_bits(mx.dequantize_mxfp4_matrix(b, s, torch.bfloat16))
        out[f"{tag}_f16"] = f16_bits(mx.dequantize_mxfp4_matrix(b, s, torch.float16))
        out[f"{tag}_f32"] = f32_bits(mx.dequantize_mxfp4_matrix(b, s, torch.float32))
    np.savez_compressed(HERE / "dequant.npz", **out)


def write_checkpoint(layer: dict[str, torch.Tensor], root: Path) -> None:
    from safetensors.torch import save_file

    experts = {k: v.contiguous() for k, v in layer.items() if ".experts." in k and (k.endswith("_blocks") or k.endswith("_scales"))}
    save_file(experts, str(root / "model-00000.safetensors"))
    (root / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {k: "model-00000.safetensors" for k in experts}}))


def run_route_case(mx, rt, name: str, spec) -> None:
    E, H, I, k, T, seed, zipf, tie_rows, capture = spec
    dims = syn.LayerDims(E, H, I, k)
    layer = syn.make_layer(dims, seed, zipf=zipf)
    tie_layer(layer, tie_rows, seed)
    x = syn.make_hidden(T, H, seed)
    tensors = syn.dense_tensors(layer)
    out: dict[str, np.ndarray] = {"meta": np.array([E, H, I, k, T, seed, -1 if zipf is None else int(zipf * 1000), tie_rows], dtype=np.int64)}
    with tempfile.TemporaryDirectory() as d:
        root = Path(d)
        write_checkpoint(layer, root)
        # router weights alone (bf16 logits exactly as route() computes them, :269)
        logits = torch.nn.functional.linear(x, tensors["model.layers.0.mlp.router.weight"], tensors["model.layers.0.mlp.router.bias"])
        out["logits"] = bf16_bits(logits)
        if tie_rows:
            out["router_weight"] = bf16_bits(tensors["model.layers.0.mlp.router.weight"])
        for precision in ("fp32", "bf16"):
            store = mx.Mxfp4ExpertStore(root, root, torch.device("cpu"), dtype=torch.bfloat16, cache_bytes=1 << 40)
            router = rt.StreamedMoERouter(experts_per_token=k, swiglu_limit=7.0, matmul_precision=precision)
            captured_gu: list[torch.Tensor] = []
            captured_gated: list[torch.Tensor] = []
            if capture:
                orig = router._apply_gate

                def gate_hook(gu, _orig=orig):
                    captured_gu.append(gu.detach().clone())
                    r = _orig(gu)
                    captured_gated.append(r.detach().clone())
                    return r

                router._apply_gate = gate_hook
            ys, experts, weights, norms = [], [], [], []
            for t in range(T):
                y, route = router.route(0, x[t], tensors, store, True, t)
                ys.append(y)
                experts.append(route["experts"])
                weights.append(route["weights"])
                norms.append([[e["gate_up_norm"], e["output_norm"]] for e in route["expert_logs"]])
            out[f"out_{precision}"] = bf16_bits(torch.stack(ys))
            out[f"experts_{precision}"] = np.array(experts, dtype=np.int32)
            out[f"weights_{precision}"] = bf16_bits(torch.tensor(weights, dtype=torch.float32))
            out[f"norms_{precision}"] = np.array(norms, dtype=np.float64)
            if capture:
                # the first tokens only, to keep the fixture small
                nt = min(T, 6)
                out[f"gu_{precision}"] = torch.stack(captured_gu).reshape(T, k, 2 * I)[:nt].numpy()
                out[f"gated_{precision}"] = torch.stack(captured_gated).reshape(T, k, I)[:nt].numpy()
            # bias-only path (execute_experts=False, :317-329)
            if precision == "fp32":
                r2 = rt.StreamedMoERouter(experts_per_token=k, swiglu_limit=7.0, matmul_precision=precision)
                yb = torch.stack([r2.route(0, x[t], tensors, None, False, t)[0] for t in range(T)])
                out["out_bias_only"] = bf16_bits(yb)
    np.savez_compressed(HERE / f"route_{name}.npz", **out)


def run_locality_case(mx, rt, name: str, spec) -> None:
    E, H, I, k, T, seed, execute, cfg_kw = spec
    dims = syn.LayerDims(E, H, I, k)
    layer = syn.make_layer(dims, seed)
    x = correlated_hidden(T, H, seed)
    tensors = syn.dense_tensors(layer)
    cfg = rt.RoutingLocalityConfig(**cfg_kw) if cfg_kw is not None else None
    out: dict[str, np.ndarray] = {"meta": np.array([E, H, I, k, T, seed, int(execute)], dtype=np.int64)}
    logits = torch.nn.functional.linear(x, tensors["model.layers.0.mlp.router.weight"], tensors["model.layers.0.mlp.router.bias"])
    out["logits"] = bf16_bits(logits)
    with tempfile.TemporaryDirectory() as d:
        root = Path(d)
        write_checkpoint(layer, root)
        store = mx.Mxfp4ExpertStore(root, root, torch.device("cpu"), dtype=torch.bfloat16, cache_bytes=1 << 40) if execute else None
        router = rt.StreamedMoERouter(experts_per_token=k, swiglu_limit=7.0, locality_config=cfg, matmul_precision="bf16")
        routes, ys = [], []
        prev: list[int] = []
        for t in range(T):
            resident = resident_set(t, prev) if cfg is not None else None
            y, route = router.route(0, x[t], tensors, store, execute, t, resident_experts=resident)
            prev = [int(e) for e in route["experts"]]
            ys.append(y)
            routes.append({key: route.get(key) for key in ("experts", "raw_experts", "weights", "sticky_adjusted", "predicted_experts",
                                                          "resident_experts", "active_expert_cap", "mode")})
        out["out"] = bf16_bits(torch.stack(ys))
        out["routes_json"] = np.array(json.dumps(routes))
        out["stats_json"] = np.array(json.dumps(router.stats.to_json()))
        out["dynamic_caps_json"] = np.array(json.dumps({str(a): b for a, b in router.dynamic_caps.items()}))
    np.savez_compressed(HERE / f"locality_{name}.npz", **out)


def make_rmsnorm_fixture(at) -> None:
    out = {}
    for H, T, seed in ((2880, 4, 21), (128, 7, 22)):
        x = syn.make_hidden(T, H, seed) * 3.0
        x = x.to(torch.bfloat16)
        w = syn.make_rms_weight(H, seed)
        y = at.rms_norm(x, w, 1e-5)
        out[f"h{H}_x"] = bf16_bits(x)
        out[f"h{H}_w"] = bf16_bits(w)
        out[f"h{H}_y"] = bf16_bits(y)
    np.savez_compressed(HERE / "rmsnorm.npz", **out)


def make_runtime_dequant_fixture(rd, aq, tp) -> None:
    g = torch.Generator().manual_seed(31)
    shape = (37, 29)
    src = torch.randn(shape, generator=g, dtype=torch.float32).to(torch.bfloat16)
    out: dict[str, np.ndarray] = {"shape": np.array(shape, dtype=np.int64)}
    deq = rd.RuntimeDequantizer()
    for mode in ("q1", "q2", "q3", "q4", "q8", "q16", "fp16"):
        qt = aq.quantize_for_storage("t", src, mode)
        meta = rd.QuantizedTensorMeta("t", mode, shape, "torch.bfloat16", qt.bits or 16, qt.packed, "g", "f")
        for dtype, tag in ((torch.float16, "f16"), (torch.bfloat16, "bf16"), (torch.float32, "f32")):
            y = deq.dequantize(meta, qt.qvalues, qt.scale, torch.device("cpu"), dtype)
            bits = {"f16": f16_bits, "bf16": bf16_bits, "f32": f32_bits}[tag](y)
            out[f"{mode}_{tag}"] = bits
        qv = qt.qvalues
        out[f"{mode}_data"] = (qv.view(torch.int16).numpy().view(np.uint16) if qv.dtype == torch.float16 else qv.numpy()).copy()
        out[f"{mode}_data_dtype"] = np.array(str(qv.dtype))
        out[f"{mode}_scale"] = (qt.scale.float().numpy() if qt.scale is not None else np.zeros(0, np.float32))
        out[f"{mode}_meta"] = np.array([qt.bits or 16, int(qt.packed)], dtype=np.int64)
    qt, _stats = tp.prune_for_storage("t", src, magnitude_fraction=0.9)
    for dtype, tag in ((torch.float16, "f16"), (torch.bfloat16, "bf16"), (torch.float32, "f32")):
        meta = rd.QuantizedTensorMeta("t", "pruned", shape, "torch.bfloat16", 16, False, "g", "f")
        y = deq.dequantize(meta, qt.qvalues, qt.zero_point, torch.device("cpu"), dtype)
        out[f"pruned_{tag}"] = {"f16": f16_bits, "bf16": bf16_bits, "f32": f32_bits}[tag](y)
    out["pruned_values"] = bf16_bits(qt.qvalues)
    out["pruned_indices"] = qt.zero_point.numpy().astype(np.int64)
    np.savez_compressed(HERE / "runtime_dequant.npz", **out)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    ap.add_argument("--only", default=None, help="comma-separated fixture names")
    args = ap.parse_args()
    torch.set_num_threads(max(os.cpu_count() or 1, 1))
    mx, rt, at, rd, aq, tp = import_reference(args.reference)
    only = set(args.only.split(",")) if args.only else None
    if only is None or "dequant" in only:
        make_dequant_fixtures(mx)
    if only is None or "rmsnorm" in only:
        make_rmsnorm_fixture(at)
    if only is None or "runtime_dequant" in only:
        make_runtime_dequant_fixture(rd, aq, tp)
    for name, spec in ROUTE_CASES.items():
        if only is None or name in only:
            run_route_case(mx, rt, name, spec)
            print("wrote", name, flush=True)
    for name, spec in LOCALITY_CASES.items():
        if only is None or name in only:
            run_locality_case(mx, rt, name, spec)
            print("wrote", name, flush=True)


if __name__ == "__main__":
    main()
