"""Checkpoint reading of the expert store on the CPU: a rank's expert shard is
read as safetensors slices [lo, hi) of the reference's tensors (the reference
reads one expert at a time the same way, mxfp4_expert.py:515-525), equal to
the matching slice of the whole tensor."""
from __future__ import annotations

import json

import torch

from kcapw_klcquant_b200 import synthetic as syn


def _write(layer, root):
    from safetensors.torch import save_file

    experts = {k: v.contiguous() for k, v in layer.items() if ".experts." in k and (k.endswith("_blocks") or k.endswith("_scales"))}
    save_file(experts, str(root / "model-00000.safetensors"))
    (root / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {k: "model-00000.safetensors" for k in experts}}))


def test_expert_shard_read_equals_slice(tmp_path):
    from kcapw_klcquant_b200.mxfp4_expert import Mxfp4ExpertStore

    layer = syn.make_layer(syn.LayerDims(8, 64, 64, 2), seed=5, layer_idx=3)
    _write(layer, tmp_path)
    # host-side reading only: the store object is built without touching a GPU
    store = Mxfp4ExpertStore.__new__(Mxfp4ExpertStore)
    store.model_dir, store.support_dir, store.quant_loader, store.dtype = tmp_path, tmp_path, None, torch.bfloat16
    store.weight_map = json.loads((tmp_path / "model.safetensors.index.json").read_text())["weight_map"]
    for kind in ("gate_up_proj_blocks", "gate_up_proj_scales", "down_proj_blocks", "down_proj_scales"):
        name = f"model.layers.3.mlp.experts.{kind}"
        full = store._load_tensor(name)
        assert torch.equal(full, layer[name])
        for lo, hi in ((0, 4), (4, 8), (2, 3)):
            assert torch.equal(store._load_tensor(name, (lo, hi)), layer[name][lo:hi])
