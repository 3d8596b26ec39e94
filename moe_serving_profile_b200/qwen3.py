"""Qwen3-MoE expert layer with the reference module API.

``ParallelExperts(config, parallel, numerics)`` mirrors
moe_serving/qwen3_parallel.py:73-118: ``num_experts`` local experts starting
at global id ``start``, a ``local`` list of ``ModuleDict``s that a loader
fills with ``ExpertProjection(weight, scales, block_size)`` for ``gate_proj``,
``up_proj`` and ``down_proj`` (FP8 E4M3 with fp32 block scales, or bf16 with
no scales), and ``forward(hidden [T,H] bf16, indices [T,K] int64 global ids,
weights [T,K] fp32) -> [T,H] bf16`` already reduced over the EP group.
``numerics="efficient"`` runs the W8A8 experts of the reference's
grouped_fp8 (moe_serving/efficient_kernels.py:243-274).

On the first forward (or an explicit ``prepare()``) the per-expert modules
are packed into the device layout of :mod:`layout` and released, as the
reference's ``prepare_fp8`` does (moe_serving/efficient_kernels.py:217-240).
"""

from __future__ import annotations

import torch
from torch import nn

from moe_serving_profile_b200 import experts as _experts
from moe_serving_profile_b200 import layout
from moe_serving_profile_b200.parallel import ParallelGroup

NUMERICS = ("reference", "fast", "efficient")


class ExpertProjection(nn.Module):
    """One projection's storage: weight [out, in] (e4m3 or bf16), optional fp32
    block scales [ceil(out/br), ceil(in/bc)] (moe_serving/qwen3_parallel.py:56-70)."""

    def __init__(self, weight, scales=None, block_size=(128, 128)):
        super().__init__()
        self.register_buffer("weight", weight)
        self.register_buffer("scales", scales)
        self.block_size = tuple(block_size)


class ParallelExperts(nn.Module):
    def __init__(self, config, parallel: ParallelGroup, numerics: str = "reference"):
        super().__init__()
        if numerics not in NUMERICS:
            raise ValueError(f"numerics must be one of {NUMERICS}, got {numerics!r}")
        if config.num_experts % parallel.size:
            raise ValueError("Expert count must be divisible by EP size")
        act = getattr(config, "hidden_act", "silu")
        if act != "silu":
            raise NotImplementedError(f"b200 Qwen experts implement SiLU gating, not {act!r}")
        self.parallel, self.numerics = parallel, numerics
        self.global_experts = config.num_experts
        self.num_experts = config.num_experts // parallel.size
        self.start = self.num_experts * parallel.rank
        self.local = nn.ModuleList([nn.ModuleDict() for _ in range(self.num_experts)])
        self.packed: layout.ExpertWeights | None = None

    def prepare(self) -> layout.ExpertWeights:
        if self.packed is not None:
            return self.packed
        projs = [[m[name] for m in self.local] for name in ("gate_proj", "up_proj", "down_proj")]
        g, u, d = projs
        if any(len(p) != self.num_experts for p in projs):
            raise ValueError("every local expert needs gate_proj, up_proj and down_proj")
        # checked before anything is packed or released, so every forward of
        # a misconfigured module raises (prepare_fp8 refuses the same case,
        # moe_serving/efficient_kernels.py:228-231)
        if self.numerics == "efficient" and any(p.scales is None for p in g + u + d):
            raise ValueError("efficient Qwen mode requires block FP8 expert weights")
        gw = torch.stack([p.weight for p in g])
        uw = torch.stack([p.weight for p in u])
        dw = torch.stack([p.weight for p in d])
        if g[0].scales is not None:
            blocks = {p.block_size for p in g + u + d}
            if len(blocks) != 1 or any(p.scales is None for p in g + u + d):
                raise ValueError("all FP8 projections need scales with one block size")
            self.packed = layout.fp8_experts(
                gw, torch.stack([p.scales for p in g]), uw, torch.stack([p.scales for p in u]),
                dw, torch.stack([p.scales for p in d]), blocks.pop())
        else:
            self.packed = layout.bf16_experts(gw.to(torch.bfloat16), uw.to(torch.bfloat16),
                                              dw.to(torch.bfloat16))
        self.local = None
        return self.packed

    def forward(self, hidden, indices, weights):
        w = self.prepare()
        return _experts.layer_forward(w, hidden, indices, weights,
                                      num_experts=self.global_experts, expert_begin=self.start,
                                      parallel=self.parallel, numerics=self.numerics)
