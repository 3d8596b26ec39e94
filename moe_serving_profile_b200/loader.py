"""Load-time expert preparation straight from a safetensors checkpoint.

Reads only the expert tensors of one layer and one expert-parallel rank
(the tensor names and slicing of moe_serving/qwen3_parallel.py:180-242 and
gpt_oss_parallel.py:394-452), opens only the shards that hold them, moves
them to the device and packs them into the grouped GEMM's blobs
(``layout``) — the reference's load followed by ``prepare_fp8`` /
``prepare_mxfp4`` (efficient_kernels.py:136-154, 217-240) without the
per-expert module tensors in between.
"""

from __future__ import annotations

import json
from contextlib import ExitStack
from pathlib import Path

import torch

from moe_serving_profile_b200 import layout
from moe_serving_profile_b200.layout import ExpertWeights


def _weight_map(checkpoint: Path) -> dict[str, str]:
    from safetensors import safe_open

    index = checkpoint / "model.safetensors.index.json"
    if index.exists():
        return json.loads(index.read_text())["weight_map"]
    with safe_open(checkpoint / "model.safetensors", framework="pt") as handle:
        return dict.fromkeys(handle.keys(), "model.safetensors")


class _Reader:
    """Lazily opened shards of one checkpoint."""

    def __init__(self, checkpoint: Path, stack: ExitStack):
        self.checkpoint, self.stack = checkpoint, stack
        self.weight_map = _weight_map(checkpoint)
        self.handles = {}

    def slice(self, name: str):
        from safetensors import safe_open

        if name not in self.weight_map:
            raise ValueError(f"Missing checkpoint tensor: {name}")
        file = self.weight_map[name]
        if file not in self.handles:
            self.handles[file] = self.stack.enter_context(
                safe_open(self.checkpoint / file, framework="pt"))
        return self.handles[file].get_slice(name)


def qwen3_fp8_experts(checkpoint, layer: int, start: int, count: int,
                      block: tuple[int, int] = (128, 128), device="cuda") -> ExpertWeights:
    """Experts start .. start + count - 1 of layer ``layer``: e4m3
    ``{gate,up,down}_proj.weight`` with fp32 ``weight_scale_inv`` block scales
    under ``model.layers.{layer}.mlp.experts.{e}``, packed on ``device``."""
    checkpoint = Path(checkpoint)
    prefix = f"model.layers.{layer}.mlp.experts"
    with ExitStack() as stack:
        rd = _Reader(checkpoint, stack)
        parts = {}
        for proj in ("gate_proj", "up_proj", "down_proj"):
            ws, ss = [], []
            for e in range(start, start + count):
                name = f"{prefix}.{e}.{proj}.weight"
                w = rd.slice(name)[:]
                if w.dtype != torch.float8_e4m3fn:
                    raise ValueError(f"{name}: expected float8_e4m3fn, got {w.dtype}")
                s = rd.slice(name.removesuffix(".weight") + ".weight_scale_inv")[:]
                br, bc = block
                if list(s.shape) != [-(-w.shape[0] // br), -(-w.shape[1] // bc)]:
                    raise ValueError(f"Invalid FP8 scale shape for {name}")
                ws.append(w.to(device))
                ss.append(s.to(device=device, dtype=torch.float32))
            parts[proj] = (torch.stack(ws), torch.stack(ss))
    return layout.fp8_experts(*parts["gate_proj"], *parts["up_proj"], *parts["down_proj"], block)


def gpt_oss_mxfp4_experts(checkpoint, layer: int, start: int, count: int, alpha: float = 1.702,
                          limit: float = 7.0, device="cuda") -> ExpertWeights:
    """Experts start .. start + count - 1 of layer ``layer``: the stacked
    ``{gate_up,down}_proj_{blocks,scales,bias}`` tensors under
    ``model.layers.{layer}.mlp.experts``, sliced along the expert axis and
    packed on ``device``."""
    checkpoint = Path(checkpoint)
    prefix = f"model.layers.{layer}.mlp.experts"
    with ExitStack() as stack:
        rd = _Reader(checkpoint, stack)
        t = {}
        for attr in ("gate_up_proj_blocks", "gate_up_proj_scales", "gate_up_proj_bias",
                     "down_proj_blocks", "down_proj_scales", "down_proj_bias"):
            t[attr] = rd.slice(f"{prefix}.{attr}")[start:start + count].to(device)
    return layout.gpt_oss_mxfp4_experts(t["gate_up_proj_blocks"], t["gate_up_proj_scales"],
                                        t["gate_up_proj_bias"], t["down_proj_blocks"],
                                        t["down_proj_scales"], t["down_proj_bias"], alpha, limit)
