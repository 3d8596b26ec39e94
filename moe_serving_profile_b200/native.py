"""Token all-to-all expert parallelism: the native runtime's MoE block.

Same names, arguments and results as moe_serving/moe.py (ExpertPlan,
RoutingStats, LocalSwiGLUExperts, route, routed_forward, MoELayer,
simulate_ranks) and moe_serving/distributed.py (Collective, SingleRank,
ProcessGroupCollective, exchange_inplace, collective_for), computed by the
b200moe kernels:

* dispatch: one expert-major permutation of the T*K assignments. A rank's
  experts are a contiguous id range, so expert-major order is already grouped
  by destination rank; one row gather packs the send buffer
  (hidden[token_index[order]] of moe.py:127).
* one count exchange of the [ep][experts_per_rank] per-expert counts and a
  single host read of the split sizes (the reference reads counts on the host
  once per exchange, three times per layer, distributed.py:37-45);
* receive side: ``a2a_recv_plan`` transposes the [source][expert] segments
  into expert-major order and the grouped GEMMs read the rows through that
  map, then one gather restores the arrival order for the return exchange;
* combine: ``index_add_`` of moe.py:134-136 — per token, contributions
  bf16(y * w) added in (destination rank, slot) order starting from bf16 zero.

Expert arithmetic is LocalSwiGLUExperts.forward (moe.py:73-81): bf16 gate/up
projection, bf16(bf16(silu(gate)) * up), bf16 down projection.
"""

from __future__ import annotations

import dataclasses
from dataclasses import dataclass

import torch
import torch.distributed as dist

from moe_serving_profile_b200 import _lib, ops
from moe_serving_profile_b200.experts import _max_tile, check_inputs, run_experts, tile_policy
from moe_serving_profile_b200.layout import ExpertWeights, bf16_experts
from moe_serving_profile_b200.router import native_route


# --------------------------------------------------------------------------- collectives
class Collective:
    """Moves a row tensor that is grouped by destination rank
    (moe_serving/distributed.py:14-18)."""

    world_size: int

    def exchange(self, rows: torch.Tensor, send_counts, recv_counts=None):
        raise NotImplementedError


class SingleRank(Collective):
    world_size = 1

    def exchange(self, rows: torch.Tensor, send_counts, recv_counts=None):
        return rows, send_counts


class ProcessGroupCollective(Collective):
    """NCCL (or gloo) all_to_all_single over ``group``. ``exchange(rows,
    send_counts)`` matches moe_serving/distributed.py:27-46; given the receive
    split sizes as a host list it skips the count exchange."""

    def __init__(self, group=None):
        self.group = group
        self.world_size = dist.get_world_size(group)

    def exchange(self, rows: torch.Tensor, send_counts, recv_counts=None):
        device = rows.device
        if recv_counts is None:
            send = torch.as_tensor(send_counts).to(device=device, dtype=torch.int64)
            recv = torch.empty(self.world_size, device=device, dtype=torch.int64)
            dist.all_to_all_single(recv, send, group=self.group)
            both = torch.cat([send, recv]).tolist()
            send_list, recv_list = both[: self.world_size], both[self.world_size:]
            recv_out = recv
        else:
            send_list = [int(c) for c in send_counts]
            recv_list = [int(c) for c in recv_counts]
            recv_out = recv_list
        out = rows.new_empty(sum(recv_list), *rows.shape[1:])
        dist.all_to_all_single(out, rows.contiguous(), output_split_sizes=recv_list,
                               input_split_sizes=send_list, group=self.group)
        return out, recv_out


class PeerCollective(ProcessGroupCollective):
    """ProcessGroupCollective whose ``routed_forward`` exchange runs over
    NVLink peer memory (b200moe_a2a_counts / dispatch / return): counts, rows
    out and rows back each move in one kernel with no host read, the rows
    landing in the receiver's expert-major order. ``max_tokens`` bounds the
    tokens any rank routes in one call (the buffers hold world x max_tokens x
    top-k received rows per rank). ``exchange`` is inherited (NCCL)."""

    def __init__(self, group=None, max_tokens: int = 8192, timeout_ns: int = 0):
        super().__init__(group)
        self.max_tokens = max_tokens
        self.timeout_ns = timeout_ns
        self.rank = dist.get_rank(group)
        self._rows = None

    def peer_rows(self, device: torch.device, hidden: int, top_k: int):
        """The exchange buffers for (hidden, top_k), created collectively by
        the first eager call (not under CUDA graph capture)."""
        from moe_serving_profile_b200.parallel import PeerRows
        b = self._rows
        if b is None or b.hidden != hidden or b.top_k != top_k or b.device != device:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("the NVLink exchange buffers are created by an eager call "
                                   "before CUDA graph capture")
            if b is not None:
                b.close()
            cap_b = self.max_tokens * top_k
            b = PeerRows(self.group, self.rank, self.world_size, device, hidden,
                         self.world_size * cap_b, cap_b, self.timeout_ns)
            b.top_k = top_k
            self._rows = b
        return b

    def close(self) -> None:
        """Release the exchange buffers (collective)."""
        if self._rows is not None:
            self._rows.close()
            self._rows = None


def exchange_inplace(payloads: list[torch.Tensor], splits: list) -> list[tuple[torch.Tensor, torch.Tensor]]:
    """One-process stand-in for the all-to-all (moe_serving/distributed.py:49-67):
    ``payloads[r]`` is grouped by destination; each result is grouped by source."""
    world = len(payloads)
    starts = [[0] * (world + 1) for _ in range(world)]
    for s in range(world):
        for d in range(world):
            starts[s][d + 1] = starts[s][d] + int(splits[s][d])
    received = []
    for d in range(world):
        chunks = [payloads[s][starts[s][d]:starts[s][d + 1]] for s in range(world)]
        counts = torch.tensor([int(splits[s][d]) for s in range(world)], dtype=torch.int64)
        received.append((torch.cat(chunks, dim=0), counts))
    return received


def collective_for(world_size: int) -> Collective:
    if world_size == 1 or not dist.is_initialized():
        return SingleRank()
    return ProcessGroupCollective()


# --------------------------------------------------------------------------- plan / stats
@dataclass
class ExpertPlan:
    """Contiguous expert ranges per rank (moe_serving/moe.py:19-37)."""

    num_experts: int
    ep_size: int
    rank: int

    def __post_init__(self) -> None:
        if self.num_experts % self.ep_size:
            raise ValueError(f"{self.num_experts} experts do not divide across {self.ep_size} ranks")
        self.experts_per_rank = self.num_experts // self.ep_size
        self.expert_start = self.rank * self.experts_per_rank
        self.expert_end = self.expert_start + self.experts_per_rank

    def owner(self, expert_ids: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        dest = torch.div(expert_ids, self.experts_per_rank, rounding_mode="floor")
        return dest, expert_ids - dest * self.experts_per_rank


@dataclass
class RoutingStats:
    """Per-layer routing counts (moe_serving/moe.py:40-55)."""

    counts: torch.Tensor
    layer: int = 0
    moe_seconds: float = 0.0
    engram_seconds: float = 0.0

    @property
    def expert_load_cv(self) -> float:
        mean = self.counts.float().mean()
        if float(mean) == 0:
            return 0.0
        return float(self.counts.float().std(unbiased=False) / mean)

    @property
    def expert_dead_fraction(self) -> float:
        return float((self.counts == 0).float().mean())


# --------------------------------------------------------------------------- experts
class LocalSwiGLUExperts(torch.nn.Module):
    """The experts one rank owns (moe_serving/moe.py:58-81): ``gate_up``
    [local_experts, 2 * intermediate, hidden] bf16 with the gate half first,
    ``down`` [local_experts, hidden, intermediate]. The weights are packed
    once into the grouped GEMM's K-major layout."""

    def __init__(self, gate_up: torch.Tensor, down: torch.Tensor):
        super().__init__()
        if gate_up.dtype != torch.bfloat16 or down.dtype != torch.bfloat16:
            raise ValueError("LocalSwiGLUExperts weights must be bfloat16")
        self.hidden = down.shape[1]
        self.intermediate = down.shape[2]
        self.num_experts = gate_up.shape[0]
        inter = self.intermediate
        self.weights = bf16_experts(gate_up[:, :inter], gate_up[:, inter:], down)

    def forward(self, hidden: torch.Tensor, local_expert_ids: torch.Tensor) -> torch.Tensor:
        """Row i of the result is expert local_expert_ids[i] applied to row i."""
        if hidden.shape[0] == 0:
            return hidden.new_empty(0, self.hidden)
        ids = local_expert_ids.reshape(-1, 1).to(torch.int64).contiguous()
        hidden = hidden.contiguous()
        perm = ops.permute(ids, self.num_experts)
        y = run_experts(self.weights, hidden, perm, None, K=1, num_experts=self.num_experts,
                        expert_begin=0)
        return ops.gather_rows(y, perm.inverse, 1)


class SharedSwiGLU(torch.nn.Module):
    """The shared expert every token passes through (moe_serving/moe.py:84-95):
    sigmoid(hidden . score) * down(silu(hidden . gate) * (hidden . up)), all
    bf16. gate / up [I_s, H], down [H, I_s], score [1, H]. The two
    projections run as a one-expert launch of the grouped GEMM over all T rows
    (SwiGLU epilogue, then the down epilogue); the [T, 1] score projection and
    the final scaling are a GEMV and one elementwise multiply."""

    def __init__(self, gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor,
                 score: torch.Tensor):
        super().__init__()
        for t in (gate, up, down, score):
            if t.dtype != torch.bfloat16:
                raise ValueError("SharedSwiGLU weights must be bfloat16")
        self.hidden = down.shape[0]
        self.intermediate = down.shape[1]
        self.weights = bf16_experts(gate[None], up[None], down[None])
        self.score = torch.nn.Parameter(score, requires_grad=False)

    def forward(self, hidden: torch.Tensor) -> torch.Tensor:
        T = hidden.shape[0]
        if T == 0:
            return hidden.new_empty(0, self.hidden)
        w = self.weights
        hidden = hidden.contiguous()
        offsets = torch.zeros(2, dtype=torch.int32, device=hidden.device)
        offsets[1] = T
        bn = tile_policy(T, 1, 1)
        act = torch.empty(T, w.i_pad, device=hidden.device, dtype=torch.bfloat16)
        ops.expert_gemm(offsets=offsets, expert_begin=0, n_experts=1, max_rows=T, wfmt=_lib.W_BF16,
                        planes=2, feat_pad=w.i_pad, n_feat=w.inter, k_pad=w.h_k, weight=w.w1,
                        b_src=hidden, k_valid=self.hidden, epilogue=_lib.EPI_SWIGLU, out=act,
                        token_tile=bn)
        y = torch.empty(T, self.hidden, device=hidden.device, dtype=torch.bfloat16)
        ops.expert_gemm(offsets=offsets, expert_begin=0, n_experts=1, max_rows=T, wfmt=_lib.W_BF16,
                        planes=1, feat_pad=w.h_f, n_feat=self.hidden, k_pad=w.i_pad, weight=w.w2,
                        b_src=act, k_valid=self.intermediate, epilogue=_lib.EPI_DOWN, out=y,
                        token_tile=bn)
        return torch.sigmoid(torch.nn.functional.linear(hidden, self.score)) * y


def route(hidden: torch.Tensor, gate_weight: torch.Tensor, top_k: int,
          renormalize: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """moe_serving/moe.py:97-107: (index int64 [T,K], weight [T,K] in hidden's dtype)."""
    return native_route(hidden, gate_weight, top_k, renormalize)


# --------------------------------------------------------------------------- dispatch / combine
@dataclass
class _Send:
    hidden: torch.Tensor
    index: torch.Tensor
    weight: torch.Tensor       # bf16 [T, K]
    perm: ops.Permutation
    rows: torch.Tensor | None  # [T*K, H] grouped by destination rank (None: no exchange)


def _prepare(hidden, expert_index, expert_weight, num_experts, exchange: bool = True) -> _Send:
    hidden, index, weight = check_inputs(hidden, expert_index, expert_weight)
    perm = ops.permute(index, num_experts)
    # the packed send rows only when they travel (one rank reads the tokens
    # through the permutation instead)
    rows = ops.gather_rows(hidden, perm.perm_src, index.shape[1]) if exchange else None
    # the reference scales by weight.to(rows.dtype) (moe.py:136)
    return _Send(hidden, index, weight.to(hidden.dtype).contiguous(), perm, rows)


def _compute(experts: LocalSwiGLUExperts, recv_rows: torch.Tensor, recv_counts: torch.Tensor,
             ep: int) -> torch.Tensor:
    """Expert outputs for the received rows, in arrival order."""
    R = recv_rows.shape[0]
    if R == 0:
        return recv_rows.new_empty(0, experts.hidden)
    el = experts.num_experts
    plan = ops.a2a_recv_plan(recv_counts.to(torch.int32).contiguous(), ep, el, R)
    rperm = ops.Permutation(None, plan.offsets, plan.map_in, plan.map_back)
    y = run_experts(experts.weights, recv_rows, rperm, None, K=1, num_experts=el, expert_begin=0,
                    b_map_div=1)
    return ops.gather_rows(y, plan.map_back, 1)


def _combine(send: _Send, returned: torch.Tensor, experts_per_rank: int) -> torch.Tensor:
    return ops.combine(returned, send.perm.inverse, send.index, order=_lib.ORDER_RANK_SLOT,
                       experts_per_rank=experts_per_rank, weights=send.weight)


def run_experts_received(w, rows: torch.Tensor, offsets: torch.Tensor, *, tile_tokens: int, K: int,
                         num_experts: int) -> torch.Tensor:
    """Expert outputs y = down(SwiGLU(gate/up(row))) (no routing weight) of
    rows already in expert-major order, ``offsets`` (device, int32 [local
    experts + 1]) their segments; every row of ``rows`` is an upper bound.
    The token tile follows the global batch (``tile_tokens`` tokens routed
    to ``num_experts`` experts, ``K`` each), as on one GPU."""
    R = rows.shape[0]
    bn = tile_policy(tile_tokens, K, num_experts, _max_tile(w))
    act = torch.empty(R, w.i_pad, device=rows.device, dtype=torch.bfloat16)
    ops.expert_gemm(offsets=offsets, expert_begin=0, n_experts=w.n_experts, max_rows=R, wfmt=w.fmt,
                    planes=2, feat_pad=w.i_pad, n_feat=w.inter, k_pad=w.h_k, weight=w.w1,
                    fp8_block=w.block, b_src=rows, k_valid=rows.shape[1], epilogue=w.gated_epilogue,
                    bias=w.b1, alpha=w.alpha, limit=w.limit, out=act, token_tile=bn)
    y = torch.empty(R, w.hidden, device=rows.device, dtype=torch.bfloat16)
    ops.expert_gemm(offsets=offsets, expert_begin=0, n_experts=w.n_experts, max_rows=R, wfmt=w.fmt,
                    planes=1, feat_pad=w.h_f, n_feat=w.hidden, k_pad=w.i_pad, weight=w.w2,
                    fp8_block=w.block, b_src=act, k_valid=w.inter, epilogue=_lib.EPI_DOWN, bias=w.b2,
                    out=y, token_tile=bn)
    return y


def _routed_forward_peer(hidden, index, weight, w, plan: ExpertPlan, collective: PeerCollective):
    """routed_forward over NVLink peer memory: count exchange, dispatch into
    the owners' receive areas, grouped GEMMs in place, return into the
    sources' areas, combine in (rank, slot) order."""
    T, K = index.shape
    if T > collective.max_tokens:
        raise ValueError(f"{T} tokens exceed the exchange buffers' {collective.max_tokens}")
    E, el = plan.num_experts, plan.experts_per_rank
    buf = collective.peer_rows(hidden.device, hidden.shape[1], K)
    perm = ops.permute(index, E)
    recv_offsets = torch.empty(el + 1, device=hidden.device, dtype=torch.int32)
    ops.a2a_counts(buf, perm.counts, recv_offsets, E)
    ops.a2a_dispatch(buf, hidden, index, perm, E)
    y = run_experts_received(w, buf.area_a, recv_offsets, tile_tokens=T * plan.ep_size, K=K,
                             num_experts=E)
    ops.a2a_return(buf, y, E)
    return ops.combine(buf.area_b[:T * K], perm.inverse, index, order=_lib.ORDER_RANK_SLOT,
                       experts_per_rank=el, weights=weight.to(hidden.dtype).contiguous())


def routed_forward(hidden: torch.Tensor, expert_index: torch.Tensor, expert_weight: torch.Tensor,
                   experts: LocalSwiGLUExperts, plan: ExpertPlan, collective: Collective) -> torch.Tensor:
    """Dispatch local tokens, run the owned experts, combine (moe_serving/moe.py:110-137)."""
    if plan.ep_size > 1 and isinstance(collective, SingleRank):
        raise RuntimeError("expert parallel needs a process group; launch with torchrun")
    if experts.num_experts != plan.experts_per_rank:
        raise ValueError(f"rank holds {experts.num_experts} experts, plan expects {plan.experts_per_rank}")
    ep, el = plan.ep_size, plan.experts_per_rank
    if ep > 1 and isinstance(collective, PeerCollective) and hidden.is_cuda:
        # every rank takes part in each exchange, also with no tokens
        h, idx, wt = check_inputs(hidden, expert_index, expert_weight)
        return _routed_forward_peer(h, idx, wt, experts.weights, plan, collective)
    send = _prepare(hidden, expert_index, expert_weight, plan.num_experts, exchange=ep > 1)
    if ep == 1:
        # no exchange: the experts read the tokens through the permutation
        returned = run_experts(experts.weights, send.hidden, send.perm, None, K=send.index.shape[1],
                               num_experts=el, expert_begin=0)
        return _combine(send, returned, el)
    ours = isinstance(collective, ProcessGroupCollective)
    # per-expert counts, experts_per_rank of them to every destination
    count_rows = send.perm.counts.view(-1, 1)
    if ours:
        recv_counts, _ = collective.exchange(count_rows, [el] * ep, [el] * ep)
    else:
        recv_counts, _ = collective.exchange(
            count_rows, torch.full((ep,), el, dtype=torch.int64, device=hidden.device))
    recv_counts = recv_counts.reshape(-1)
    splits = torch.stack([send.perm.counts.view(ep, el).sum(1),
                          recv_counts.view(ep, el).sum(1).to(torch.int32)]).tolist()
    send_list, recv_list = splits
    if ours:
        recv_rows, _ = collective.exchange(send.rows, send_list, recv_list)
    else:
        recv_rows, _ = collective.exchange(send.rows, torch.tensor(send_list, device=hidden.device))
    computed = _compute(experts, recv_rows, recv_counts, ep)
    if ours:
        returned, _ = collective.exchange(computed, recv_list, send_list)
    else:
        returned, _ = collective.exchange(computed, torch.tensor(recv_list, device=hidden.device))
    return _combine(send, returned, el)


def _joint_weights(experts: LocalSwiGLUExperts, shared: SharedSwiGLU) -> ExpertWeights | None:
    """The shared expert packed as expert E after the E routed experts, so
    that one grouped launch runs both; None when its intermediate does not fit
    the routed experts' padded intermediate (then it runs as its own launch).
    The shared expert's extra features are zero rows of gate / up and zero
    columns of down: SwiGLU(0, 0) = 0 and adding zero products leaves every
    sum unchanged, so the result is exact. The routed experts' pack becomes a
    view of the joint one (no second copy of their weights)."""
    w, sw = experts.weights, shared.weights
    # both packs are bf16 [E][2][I_p][H_k] / [E][H_f][I_p] (LocalSwiGLUExperts
    # and SharedSwiGLU take bf16 weights only), so the intermediate is axis 2
    # of both; quantised blobs would need another slicing
    if w.fmt != _lib.W_BF16 or sw.fmt != _lib.W_BF16 or sw.hidden != w.hidden or sw.inter > w.i_pad:
        return None
    E = w.n_experts
    ips = sw.i_pad
    w1 = torch.zeros((E + 1,) + tuple(w.w1.shape[1:]), device=w.w1.device, dtype=w.w1.dtype)
    w1[:E] = w.w1
    w1[E, :, :ips] = sw.w1[0]
    w2 = torch.zeros((E + 1,) + tuple(w.w2.shape[1:]), device=w.w2.device, dtype=w.w2.dtype)
    w2[:E] = w.w2
    w2[E, :, :ips] = sw.w2[0]
    experts.weights = dataclasses.replace(w, w1=w1[:E], w2=w2[:E])
    return dataclasses.replace(w, n_experts=E + 1, inter=max(w.inter, sw.inter), w1=w1, w2=w2)


class MoELayer(torch.nn.Module):
    """Router + token all-to-all experts + optional shared expert
    (moe_serving/moe.py:140-168). On one rank a shared expert whose
    intermediate fits the routed experts' padded intermediate runs inside the
    routed launch: every token gets one more slot routed to it (expert E,
    weight sigmoid(hidden . score)), and the ordered combine adds that slot
    last, which is the reference's ``output + shared(hidden)`` bit for bit.
    """

    def __init__(self, gate_weight: torch.Tensor, experts: LocalSwiGLUExperts, plan: ExpertPlan,
                 top_k: int, renormalize: bool = True, shared: SharedSwiGLU | None = None,
                 collective: Collective | None = None, layer_id: int = 0, logits: str = "exact"):
        super().__init__()
        if logits not in ("exact", "fused"):
            raise ValueError(f"logits must be 'exact' or 'fused', got {logits!r}")
        self.logits_mode = logits   # "exact": fp32 F.linear as moe.route does; "fused": fixed-order kernel
        self.gate_weight = torch.nn.Parameter(gate_weight, requires_grad=False)
        self.experts = experts
        self.shared = shared
        self.plan = plan
        self.top_k = top_k
        self.renormalize = renormalize
        self.collective = collective or SingleRank()
        self.layer_id = layer_id
        self.joint = _joint_weights(experts, shared) if shared is not None and plan.ep_size == 1 else None

    def _joint_forward(self, hidden: torch.Tensor, indices: torch.Tensor,
                       scores: torch.Tensor) -> torch.Tensor:
        h, idx, wt = check_inputs(hidden, indices, scores)
        T, K = idx.shape
        if T == 0:
            return h.new_zeros(h.shape)
        E = self.plan.num_experts
        # the score projection is the reference's own F.linear (moe.py:95)
        logit = torch.nn.functional.linear(h, self.shared.score)
        idx1, w1 = ops.append_shared_slot(idx, wt, logit, E)
        perm = ops.permute(idx1, E + 1)
        y = run_experts(self.joint, h, perm, None, K=K + 1, num_experts=E + 1, expert_begin=0)
        return ops.combine(y, perm.inverse, idx1, order=_lib.ORDER_RANK_SLOT, experts_per_rank=E + 1,
                           weights=w1)

    def forward(self, hidden: torch.Tensor) -> tuple[torch.Tensor, RoutingStats]:
        if self.logits_mode == "exact":
            lg = torch.nn.functional.linear(hidden.float(), self.gate_weight.float()).contiguous()
            out = ops.router(_lib.ROUTER_NATIVE, None, self.gate_weight, None, self.top_k,
                             self.renormalize, logits=lg)
        else:
            out = ops.router(_lib.ROUTER_NATIVE, hidden, self.gate_weight, None, self.top_k,
                             self.renormalize)
        if self.joint is not None:
            output = self._joint_forward(hidden, out.indices, out.scores)
        else:
            output = routed_forward(hidden, out.indices, out.scores, self.experts, self.plan,
                                    self.collective)
            if self.shared is not None:
                output = output + self.shared(hidden)
        return output, RoutingStats(counts=out.counts.to(torch.int64).cpu(), layer=self.layer_id)


def simulate_routed(hiddens: list[torch.Tensor], indices: list[torch.Tensor],
                    weights: list[torch.Tensor], expert_banks: list[LocalSwiGLUExperts],
                    num_experts: int) -> list[torch.Tensor]:
    """The lockstep all-to-all of ``simulate_ranks`` for given per-rank routing."""
    ep = len(hiddens)
    el = ExpertPlan(num_experts, ep, 0).experts_per_rank
    sends = [_prepare(h, i, w, num_experts) for h, i, w in zip(hiddens, indices, weights)]
    counts = exchange_inplace([s.perm.counts.view(-1, 1) for s in sends], [[el] * ep] * ep)
    recv_counts = [c.reshape(-1) for c, _ in counts]
    send_splits = [s.perm.counts.view(ep, el).sum(1).tolist() for s in sends]
    recv = exchange_inplace([s.rows for s in sends], send_splits)
    computed = [_compute(expert_banks[r], recv[r][0], recv_counts[r], ep) for r in range(ep)]
    returned = exchange_inplace(computed, [recv[r][1].tolist() for r in range(ep)])
    return [_combine(sends[r], returned[r][0], el) for r in range(ep)]


def simulate_ranks(hiddens: list[torch.Tensor], gates: torch.Tensor,
                   expert_banks: list[LocalSwiGLUExperts], top_k: int, renormalize: bool = True,
                   shared: list[SharedSwiGLU] | None = None) -> list[torch.Tensor]:
    """Every rank inside one process (moe_serving/moe.py:171-224): the same
    kernels as ``routed_forward`` with ``exchange_inplace`` standing in for
    the all-to-all, plus each rank's shared expert. Used to check the
    all-to-all math on one GPU."""
    routes = [route(h, gates, top_k, renormalize) for h in hiddens]
    outs = simulate_routed(hiddens, [r[0] for r in routes], [r[1] for r in routes], expert_banks,
                           gates.shape[0])
    if shared is not None:
        outs = [o + shared[r](h) for r, (o, h) in enumerate(zip(outs, hiddens))]
    return outs
