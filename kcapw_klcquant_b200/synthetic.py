"""Seeded synthetic MoE layers in the GPT-OSS MXFP4 checkpoint layout.

The reference runs on a real GPT-OSS checkpoint that is not available here, so
every test, fixture and benchmark uses seeded synthetic tensors with the same
names, shapes and dtypes:

* ``model.layers.{L}.mlp.experts.gate_up_proj_blocks``  uint8 [E, 2I, H/32, 16]
* ``model.layers.{L}.mlp.experts.gate_up_proj_scales``  uint8 [E, 2I, H/32]
* ``model.layers.{L}.mlp.experts.down_proj_blocks``     uint8 [E, H, I/32, 16]
* ``model.layers.{L}.mlp.experts.down_proj_scales``     uint8 [E, H, I/32]
* ``model.layers.{L}.mlp.experts.gate_up_proj_bias``    bf16 [E, 2I]
* ``model.layers.{L}.mlp.experts.down_proj_bias``       bf16 [E, H]
* ``model.layers.{L}.mlp.router.weight``                bf16 [E, H]
* ``model.layers.{L}.mlp.router.bias``                  bf16 [E]

Gate/up rows are interleaved (even rows gate, odd rows up), as the reference's
``_apply_gate`` expects (klcquant streamed_moe_router.py:524-529).  Nibbles are
uniform over 0..15, E8M0 scales uniform in [118, 126], biases and the router
weight N(0, 0.02), activations N(0, 1).  ``zipf`` adds a router bias
``beta * log(p_e)`` with ``p_e`` proportional to ``rank_e ** -s`` over a seeded
rank permutation, which skews top-k selection toward a Zipf popularity.

The CPU generator (``torch.Generator``) is used for anything the reference or
the oracle consumes, so the same seed gives the same bytes on every machine
with this torch version.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class LayerDims:
    experts: int
    hidden: int
    intermediate: int
    top_k: int = 4

    def __post_init__(self) -> None:
        if self.hidden % 32 or self.intermediate % 32:
            raise ValueError("hidden and intermediate sizes must be multiples of the MXFP4 block (32)")


GPT_OSS_20B = LayerDims(experts=32, hidden=2880, intermediate=2880, top_k=4)
GPT_OSS_120B = LayerDims(experts=128, hidden=2880, intermediate=2880, top_k=4)


def prefix(layer_idx: int) -> str:
    return f"model.layers.{layer_idx}.mlp"


def zipf_router_bias(experts: int, seed: int, s: float = 1.1, beta: float = 1.0) -> torch.Tensor:
    """Router bias that skews selection toward a Zipf(s) popularity over experts."""
    g = torch.Generator().manual_seed(seed + 7919)
    ranks = torch.randperm(experts, generator=g).to(torch.float64) + 1.0
    p = ranks.pow(-s)
    p = p / p.sum()
    bias = beta * (p.log() - math.log(1.0 / experts))
    return bias.to(torch.bfloat16)


def make_layer(
    dims: LayerDims,
    seed: int,
    layer_idx: int = 0,
    zipf: float | None = None,
    scale_lo: int = 118,
    scale_hi: int = 126,
    device: str | torch.device = "cpu",
) -> dict[str, torch.Tensor]:
    """Return the tensors of one MoE layer, keyed by checkpoint name.

    With ``device='cpu'`` the bytes depend only on ``seed`` (CPU generator).  A
    CUDA ``device`` generates on the GPU (fast, for the large benchmark
    layouts) and gives different bytes for the same seed.
    """
    E, H, I = dims.experts, dims.hidden, dims.intermediate
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    p = prefix(layer_idx)

    def randint(lo: int, hi: int, shape: tuple[int, ...]) -> torch.Tensor:
        return torch.randint(lo, hi, shape, generator=g, dtype=torch.uint8, device=dev)

    def normal(shape: tuple[int, ...], std: float) -> torch.Tensor:
        return (torch.randn(shape, generator=g, dtype=torch.float32, device=dev) * std).to(torch.bfloat16)

    t: dict[str, torch.Tensor] = {}
    t[f"{p}.experts.gate_up_proj_blocks"] = randint(0, 256, (E, 2 * I, H // 32, 16))
    t[f"{p}.experts.gate_up_proj_scales"] = randint(scale_lo, scale_hi + 1, (E, 2 * I, H // 32))
    t[f"{p}.experts.down_proj_blocks"] = randint(0, 256, (E, H, I // 32, 16))
    t[f"{p}.experts.down_proj_scales"] = randint(scale_lo, scale_hi + 1, (E, H, I // 32))
    t[f"{p}.experts.gate_up_proj_bias"] = normal((E, 2 * I), 0.02)
    t[f"{p}.experts.down_proj_bias"] = normal((E, H), 0.02)
    t[f"{p}.router.weight"] = normal((E, H), 0.02)
    if zipf is None:
        t[f"{p}.router.bias"] = torch.zeros(E, dtype=torch.bfloat16, device=dev)
    else:
        t[f"{p}.router.bias"] = zipf_router_bias(E, seed, s=zipf).to(dev)
    return t


def make_hidden(tokens: int, hidden: int, seed: int, device: str | torch.device = "cpu") -> torch.Tensor:
    """bf16 N(0, 1) activations [tokens, hidden]."""
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed + 104729)
    return torch.randn((tokens, hidden), generator=g, dtype=torch.float32, device=dev).to(torch.bfloat16)


def make_rms_weight(hidden: int, seed: int, device: str | torch.device = "cpu") -> torch.Tensor:
    """bf16 N(1, 0.02) RMSNorm weight [hidden]."""
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed + 15485863)
    return (1.0 + 0.02 * torch.randn((hidden,), generator=g, dtype=torch.float32, device=dev)).to(torch.bfloat16)


def dense_tensors(layer: dict[str, torch.Tensor], layer_idx: int = 0) -> dict[str, torch.Tensor]:
    """The non-expert tensors the executor passes to ``route()`` in its ``tensors`` dict."""
    p = prefix(layer_idx)
    keys = (f"{p}.router.weight", f"{p}.router.bias", f"{p}.experts.gate_up_proj_bias", f"{p}.experts.down_proj_bias")
    return {k: layer[k] for k in keys}
