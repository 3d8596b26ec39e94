"""Router modules that drop in at ``block.mlp.gate`` / ``block.mlp.router``.

They keep the Transformers router interface — attributes ``top_k``,
``num_experts``, ``weight`` (and ``bias``), ``forward(h) -> (logits, scores,
indices)`` — so forward hooks such as the reference's ``RoutingRecorder``
(moe_serving/gpt_oss_parallel.py:273-288) keep working. Each forward also
leaves the per-expert token counts of the batch in ``last_counts`` (int32, on
the device) for load statistics.

Two ways to get the logits (``logits=`` at construction):

* ``"exact"`` (default): the logits come from ``F.linear`` — the very GEMM
  the reference's routers call on the same device — and the library's
  selection kernel does softmax / top-k / renormalisation / counts in one
  launch, reproducing torch's CUDA softmax, ``topk`` (including the slot
  order of equal values) and ``sum`` bit for bit. Probabilities, scores and
  indices are then identical to the reference's router on the same inputs.
* ``"fused"``: one more kernel of the library computes the logits on CUDA
  cores in a fixed fp32 order (row-independent, identical in every batch and
  on every rank), within one bf16 ulp of ``F.linear``; top-k can then differ
  from the reference's on near-ties.

Under replicated-token expert parallelism every rank needs every token's
routing. In ``"fused"`` mode, ``shard_over(parallel)`` routes a batch of at
least ``SHARD_MIN_TOKENS`` tokens (a multiple of the group size) in slices,
one per rank, and all-gathers them (bit-identical to routing the whole batch,
the order being row-independent). In ``"exact"`` mode every rank routes the
whole batch, as the reference's ranks do, because a GEMM library may choose a
different kernel, and summation order, for a slice.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn

from moe_serving_profile_b200 import _lib, ops

SHARD_MIN_TOKENS = 1024


LOGITS_MODES = ("exact", "fused")


def _check_logits_mode(mode: str) -> str:
    if mode not in LOGITS_MODES:
        raise ValueError(f"logits must be one of {LOGITS_MODES}, got {mode!r}")
    return mode


def _route(mode: int, h: torch.Tensor, weight, bias, top_k: int, normalize: bool, parallel,
           logits_mode: str = "fused"):
    """(first output, scores, indices, counts) of ops.router, routed in
    per-rank slices and all-gathered when sharding applies. The first output
    is the fp32 probabilities (Qwen3) or the bf16 logits (others)."""
    if logits_mode == "exact":
        if not h.is_cuda:
            raise ValueError(f"hidden states must be a CUDA tensor (b200moe has no CPU path), got {h.device}")
        logits = F.linear(h, weight, bias)   # the reference router's own GEMM
        out = ops.router(mode, None, weight, bias, top_k, normalize, logits=logits.contiguous())
        return (out.probs if mode == _lib.ROUTER_QWEN3 else out.logits), out.scores, out.indices, out.counts
    T = h.shape[0]
    n = 1 if parallel is None else parallel.size
    if n == 1 or T < SHARD_MIN_TOKENS or T % n or not h.is_cuda:
        out = ops.router(mode, h, weight, bias, top_k, normalize)
        return (out.probs if mode == _lib.ROUTER_QWEN3 else out.logits), out.scores, out.indices, out.counts
    ts = T // n
    out = ops.router(mode, h[parallel.rank * ts:(parallel.rank + 1) * ts], weight, bias, top_k, normalize)
    parts = [out.probs if mode == _lib.ROUTER_QWEN3 else out.logits, out.scores, out.indices, out.counts]
    flat = torch.cat([p.reshape(-1).view(torch.uint8) for p in parts])   # one collective
    gathered = torch.empty(n, flat.numel(), dtype=torch.uint8, device=h.device)
    dist.all_gather_into_tensor(gathered, flat, group=parallel.group)
    res, o = [], 0
    for p in parts:
        nb = p.numel() * p.element_size()
        chunk = gathered[:, o:o + nb].contiguous().view(p.dtype)
        res.append(chunk.reshape(n * p.shape[0], *p.shape[1:]) if p is not parts[3] else
                   chunk.reshape(n, -1).sum(0, dtype=torch.int32))
        o += nb
    return tuple(res)


class Qwen3Router(nn.Module):
    """Qwen3MoeTopKRouter (transformers qwen3_moe/modeling_qwen3_moe.py:254-272):
    fp32 softmax over bf16 logits, top-k, optional renormalisation.
    Returns (probs fp32 [T,E], scores fp32 [T,K], indices int64 [T,K])."""

    def __init__(self, config, logits: str = "exact"):
        super().__init__()
        self.logits_mode = _check_logits_mode(logits)
        self.top_k = config.num_experts_per_tok
        self.num_experts = config.num_experts
        self.norm_topk_prob = bool(getattr(config, "norm_topk_prob", False))
        self.hidden_dim = config.hidden_size
        self.weight = nn.Parameter(torch.zeros(self.num_experts, self.hidden_dim), requires_grad=False)
        # Optional per-expert logit bias (not part of Qwen3; used by synthetic
        # load-skew workloads). None keeps the exact Qwen3 router.
        self.bias: torch.Tensor | None = None
        self.last_counts: torch.Tensor | None = None
        self.parallel = None

    def shard_over(self, parallel) -> "Qwen3Router":
        """Route large batches in per-rank slices of ``parallel`` (a
        ParallelGroup whose ranks all call forward on the same tokens);
        "fused" logits only (an "exact" router always routes the whole batch)."""
        self.parallel = parallel
        return self

    def forward(self, hidden_states: torch.Tensor):
        h = hidden_states.reshape(-1, self.hidden_dim)
        probs, scores, indices, counts = _route(_lib.ROUTER_QWEN3, h, self.weight, self.bias,
                                                self.top_k, self.norm_topk_prob, self.parallel,
                                                self.logits_mode)
        self.last_counts = counts
        return probs, scores, indices


class GptOssRouter(nn.Module):
    """GptOssTopKRouter (transformers gpt_oss/modeling_gpt_oss.py:117-131):
    bf16 logits with bias, top-k on the logits, bf16 softmax over the k values.
    Returns (logits bf16 [T,E], scores bf16 [T,K], indices int64 [T,K])."""

    def __init__(self, config, logits: str = "exact"):
        super().__init__()
        self.logits_mode = _check_logits_mode(logits)
        self.top_k = config.num_experts_per_tok
        self.num_experts = config.num_local_experts
        self.hidden_dim = config.hidden_size
        self.weight = nn.Parameter(torch.zeros(self.num_experts, self.hidden_dim), requires_grad=False)
        self.bias = nn.Parameter(torch.zeros(self.num_experts), requires_grad=False)
        self.last_counts: torch.Tensor | None = None
        self.parallel = None

    def shard_over(self, parallel) -> "GptOssRouter":
        """Route large batches in per-rank slices of ``parallel`` (see Qwen3Router)."""
        self.parallel = parallel
        return self

    def forward(self, hidden_states: torch.Tensor):
        h = hidden_states.reshape(-1, self.hidden_dim)
        logits, scores, indices, counts = _route(_lib.ROUTER_GPT_OSS, h, self.weight, self.bias,
                                                 self.top_k, False, self.parallel, self.logits_mode)
        self.last_counts = counts
        return logits, scores, indices


def native_route(hidden: torch.Tensor, gate_weight: torch.Tensor, top_k: int,
                 renormalize: bool, logits: str = "exact") -> tuple[torch.Tensor, torch.Tensor]:
    """moe_serving/moe.py:97-107 (route): fp32 logits and softmax, top-k,
    renormalise with clamp 1e-20; returns (index int64, weight in bf16).
    "exact" takes the fp32 logits from ``F.linear`` as the reference does."""
    if _check_logits_mode(logits) == "exact":
        if not hidden.is_cuda:
            raise ValueError(f"hidden must be a CUDA tensor (b200moe has no CPU path), got {hidden.device}")
        lg = F.linear(hidden.float(), gate_weight.float()).contiguous()
        out = ops.router(_lib.ROUTER_NATIVE, None, gate_weight, None, top_k, renormalize, logits=lg)
    else:
        out = ops.router(_lib.ROUTER_NATIVE, hidden, gate_weight, None, top_k, renormalize)
    return out.indices, out.scores
