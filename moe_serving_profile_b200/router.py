"""Router modules that drop in at ``block.mlp.gate`` / ``block.mlp.router``.

They keep the Transformers router interface — attributes ``top_k``,
``num_experts``, ``weight`` (and ``bias``), ``forward(h) -> (logits, scores,
indices)`` — so forward hooks such as the reference's ``RoutingRecorder``
(moe_serving/gpt_oss_parallel.py:273-288) keep working, but run the fused
router kernel. Each forward also leaves the per-expert token counts of the
batch in ``last_counts`` (int32, on the device) for load statistics.
"""

from __future__ import annotations

import torch
from torch import nn

from moe_serving_profile_b200 import _lib, ops


class Qwen3Router(nn.Module):
    """Qwen3MoeTopKRouter (transformers qwen3_moe/modeling_qwen3_moe.py:254-272):
    fp32 softmax over bf16 logits, top-k, optional renormalisation.
    Returns (probs fp32 [T,E], scores fp32 [T,K], indices int64 [T,K])."""

    def __init__(self, config):
        super().__init__()
        self.top_k = config.num_experts_per_tok
        self.num_experts = config.num_experts
        self.norm_topk_prob = bool(getattr(config, "norm_topk_prob", False))
        self.hidden_dim = config.hidden_size
        self.weight = nn.Parameter(torch.zeros(self.num_experts, self.hidden_dim), requires_grad=False)
        # Optional per-expert logit bias (not part of Qwen3; used by synthetic
        # load-skew workloads). None keeps the exact Qwen3 router.
        self.bias: torch.Tensor | None = None
        self.last_counts: torch.Tensor | None = None

    def forward(self, hidden_states: torch.Tensor):
        h = hidden_states.reshape(-1, self.hidden_dim)
        out = ops.router(_lib.ROUTER_QWEN3, h, self.weight, self.bias, self.top_k,
                         self.norm_topk_prob)
        self.last_counts = out.counts
        return out.probs, out.scores, out.indices


class GptOssRouter(nn.Module):
    """GptOssTopKRouter (transformers gpt_oss/modeling_gpt_oss.py:117-131):
    bf16 logits with bias, top-k on the logits, bf16 softmax over the k values.
    Returns (logits bf16 [T,E], scores bf16 [T,K], indices int64 [T,K])."""

    def __init__(self, config):
        super().__init__()
        self.top_k = config.num_experts_per_tok
        self.num_experts = config.num_local_experts
        self.hidden_dim = config.hidden_size
        self.weight = nn.Parameter(torch.zeros(self.num_experts, self.hidden_dim), requires_grad=False)
        self.bias = nn.Parameter(torch.zeros(self.num_experts), requires_grad=False)
        self.last_counts: torch.Tensor | None = None

    def forward(self, hidden_states: torch.Tensor):
        h = hidden_states.reshape(-1, self.hidden_dim)
        out = ops.router(_lib.ROUTER_GPT_OSS, h, self.weight, self.bias, self.top_k, False)
        self.last_counts = out.counts
        return out.logits, out.scores, out.indices


def native_route(hidden: torch.Tensor, gate_weight: torch.Tensor, top_k: int,
                 renormalize: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """moe_serving/moe.py:97-107 (route): fp32 logits and softmax, top-k,
    renormalise with clamp 1e-20; returns (index int64, weight in bf16)."""
    out = ops.router(_lib.ROUTER_NATIVE, hidden, gate_weight, None, top_k, renormalize)
    return out.indices, out.scores
