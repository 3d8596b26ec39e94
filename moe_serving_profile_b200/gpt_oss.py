"""GPT-OSS expert layer with the reference module API.

``ParallelExperts(config, parallel, storage, numerics)`` mirrors
moe_serving/gpt_oss_parallel.py:173-244. A loader registers, per local
expert stack, either the packed MXFP4 buffers ``gate_up_proj_blocks``
[E_loc, 2I, H/32, 16] u8, ``gate_up_proj_scales`` [E_loc, 2I, H/32] u8,
``down_proj_blocks`` / ``down_proj_scales``, or the bf16 ``gate_up_proj``
[E_loc, H, 2I] / ``down_proj`` [E_loc, I, H]; plus ``gate_up_proj_bias``
[E_loc, 2I] and ``down_proj_bias`` [E_loc, H]. ``forward(hidden [T,H] bf16,
router_indices [T,K] int64 global ids, routing_weights [T,K] bf16)`` returns
the [T,H] bf16 output reduced over the EP group.

The experts compute interleaved gate/up, +bias, clamped SwiGLU (limit,
alpha, up + 1) and the down projection + bias with bf16 rounding after each
op, as the reference's ``project`` does (gpt_oss_parallel.py:195-204), with
MXFP4 decoded exactly in shared memory.
"""

from __future__ import annotations

from torch import nn

from moe_serving_profile_b200 import experts as _experts
from moe_serving_profile_b200 import layout
from moe_serving_profile_b200.parallel import ParallelGroup

NUMERICS = ("reference", "fast", "efficient")


class ParallelExperts(nn.Module):
    def __init__(self, config, parallel: ParallelGroup, storage: str = "mxfp4",
                 numerics: str = "reference"):
        super().__init__()
        if numerics not in NUMERICS:
            raise ValueError(f"numerics must be one of {NUMERICS}, got {numerics!r}")
        if storage not in ("mxfp4", "bf16"):
            raise ValueError("expert_storage must be mxfp4 or bf16")
        if numerics == "efficient" and storage != "mxfp4":
            raise ValueError("efficient gpt_oss requires mxfp4 checkpoint storage")
        if config.num_local_experts % parallel.size:
            raise ValueError("Number of experts must be divisible by EP size")
        self.parallel, self.storage, self.numerics = parallel, storage, numerics
        self.global_experts = config.num_local_experts
        self.num_experts = config.num_local_experts // parallel.size
        self.start = self.num_experts * parallel.rank
        self.alpha, self.limit = config.swiglu_alpha, config.swiglu_limit
        self.packed: layout.ExpertWeights | None = None

    def prepare(self) -> layout.ExpertWeights:
        if self.packed is not None:
            return self.packed
        if hasattr(self, "gate_up_proj_blocks"):
            self.packed = layout.gpt_oss_mxfp4_experts(
                self.gate_up_proj_blocks, self.gate_up_proj_scales, self.gate_up_proj_bias,
                self.down_proj_blocks, self.down_proj_scales, self.down_proj_bias,
                self.alpha, self.limit)
            names = ("gate_up_proj_blocks", "gate_up_proj_scales", "down_proj_blocks",
                     "down_proj_scales")
        elif hasattr(self, "gate_up_proj"):
            self.packed = layout.gpt_oss_bf16_experts(
                self.gate_up_proj, self.gate_up_proj_bias, self.down_proj, self.down_proj_bias,
                self.alpha, self.limit)
            names = ("gate_up_proj", "down_proj")
        else:
            raise ValueError("no expert weights registered")
        for name in names:
            delattr(self, name)
        return self.packed

    def forward(self, hidden_states, router_indices, routing_weights):
        w = self.prepare()
        return _experts.layer_forward(w, hidden_states, router_indices, routing_weights,
                                      num_experts=self.global_experts, expert_begin=self.start,
                                      parallel=self.parallel, numerics=self.numerics)
