"""Token all-to-all expert parallelism (moe_serving/moe.py) on the GPU.

The ranks run in one process (``simulate_ranks`` / ``simulate_routed``, the
reference's own one-process stand-in for the all-to-all), so every kernel of
the a2a path — permutation, dispatch gather, receive plan, grouped GEMMs
through the receive map, return gather, (rank, slot)-ordered combine — runs
on one GPU. Routing must match the reference bit for bit where its top-k has
no tie; outputs are compared with the oracle on identical routing within the
BF16 layer tolerance (relative L2 <= 1e-2, max |error| <= 2^-5 max |ref|).
"""

import pytest
import torch

from moe_serving_profile_b200 import _lib, native, ops
from moe_serving_profile_b200 import synthetic as S
from oracle import oracle
from tests.conftest import load_golden, max_abs, rel_l2, tie_free_rows

pytestmark = pytest.mark.gpu

REL_L2 = 1e-2
MAX_ABS_FRAC = 2 ** -5


def _close(out, ref, what=""):
    r, m = rel_l2(out, ref), max_abs(out, ref)
    bound = MAX_ABS_FRAC * float(ref.float().abs().max())
    assert r <= REL_L2 and m <= bound, f"{what}: rel_l2 {r:.2e} max_abs {m:.3e} (bound {bound:.3e})"


def _banks(gate_up, down, ep, dev):
    el = gate_up.shape[0] // ep
    return [native.LocalSwiGLUExperts(gate_up[r * el:(r + 1) * el].to(dev),
                                      down[r * el:(r + 1) * el].to(dev)) for r in range(ep)]


def test_native_golden_two_ranks(cuda):
    g = load_golden("native_a2a")
    tokens = g["tokens"].to(cuda)
    idx, w = native.route(tokens, g["gate"].to(cuda), g["top_k"], True)
    assert torch.equal(idx.cpu(), g["index"])
    outs = native.simulate_ranks([tokens[:3], tokens[3:]], g["gate"].to(cuda),
                                 _banks(g["gate_up"], g["down"], 2, cuda), g["top_k"])
    for o, ref in zip(outs, g["rank_outputs"]):
        _close(o, ref, "golden rank")
    assert _lib.device_status(cuda.index) == 0


def _case(E, H, I, K, tokens_per_rank, seed):
    g = torch.Generator().manual_seed(seed)
    gate_up = (torch.randn(E, 2 * I, H, generator=g) * 0.02).bfloat16()
    down = (torch.randn(E, H, I, generator=g) * 0.02).bfloat16()
    gate = (torch.randn(E, H, generator=g) * 0.02).bfloat16()
    hiddens = [torch.randn(t, H, generator=g).bfloat16() for t in tokens_per_rank]
    return gate_up, down, gate, hiddens


@pytest.mark.parametrize("ep,tokens", [(1, [64]), (2, [64, 48]), (4, [16, 0, 64, 33]),
                                       (8, [8] * 8)])
def test_a2a_matches_oracle(cuda, ep, tokens):
    E, H, I, K = 128, 2048, 768, 8
    gate_up, down, gate, hiddens = _case(E, H, I, K, tokens, seed=ep)
    banks = _banks(gate_up, down, ep, cuda)
    hd = [h.to(cuda) for h in hiddens]
    routes = [native.route(h, gate.to(cuda), K, True) if h.shape[0] else
              (torch.empty(0, K, dtype=torch.int64, device=cuda),
               torch.empty(0, K, dtype=torch.bfloat16, device=cuda)) for h in hd]
    outs = native.simulate_routed(hd, [r[0] for r in routes], [r[1] for r in routes], banks, E)
    refs = oracle.routed_forward_ranks(hiddens, gate, gate_up, down, K,
                                       routes=[(r[0].cpu(), r[1].cpu()) for r in routes])
    for rank, (o, ref) in enumerate(zip(outs, refs)):
        assert o.shape == ref.shape
        if ref.numel():
            _close(o, ref, f"rank {rank}")
    # routing agrees with the reference's router wherever its top-k has no tie
    for h, (idx, _) in zip(hiddens, routes):
        if h.shape[0] == 0:
            continue
        ridx, _, scores = oracle.native_route(h, gate, K, True)
        ok = tie_free_rows(scores, K)
        assert torch.equal(idx.cpu()[ok], ridx[ok])
    assert _lib.device_status(cuda.index) == 0


def test_routed_forward_single_rank(cuda):
    E, H, I, K = 32, 512, 256, 4
    gate_up, down, gate, (h,) = _case(E, H, I, K, [100], seed=7)
    experts = native.LocalSwiGLUExperts(gate_up.to(cuda), down.to(cuda))
    plan = native.ExpertPlan(E, 1, 0)
    idx, w = native.route(h.to(cuda), gate.to(cuda), K, True)
    out = native.routed_forward(h.to(cuda), idx, w, experts, plan, native.SingleRank())
    (ref,) = oracle.routed_forward_ranks([h], gate, gate_up, down, K, routes=[(idx.cpu(), w.cpu())])
    _close(out, ref, "ep1")
    layer = native.MoELayer(gate.to(cuda), experts, plan, K)
    out2, stats = layer(h.to(cuda))
    assert torch.equal(out2, out)
    assert int(stats.counts.sum()) == 100 * K and stats.counts.shape == (E,)


def test_local_experts_forward(cuda):
    E, H, I = 8, 256, 128
    gate_up, down, _, (h,) = _case(E, H, I, 1, [77], seed=3)
    ids = torch.randint(0, E, (77,), generator=torch.Generator().manual_seed(1))
    experts = native.LocalSwiGLUExperts(gate_up.to(cuda), down.to(cuda))
    out = experts(h.to(cuda), ids.to(cuda))
    ref = torch.empty(77, H, dtype=torch.bfloat16)
    for e in ids.unique().tolist():
        m = ids == e
        gg, uu = torch.nn.functional.linear(h[m], gate_up[e]).chunk(2, dim=-1)
        ref[m] = torch.nn.functional.linear(torch.nn.functional.silu(gg) * uu, down[e])
    _close(out, ref, "LocalSwiGLUExperts")


def test_recv_plan_transposes_segments(cuda):
    ep, el = 3, 4
    counts = torch.tensor([[2, 0, 1, 3], [0, 0, 2, 1], [1, 4, 0, 0]], dtype=torch.int32)
    rows = int(counts.sum())
    plan = ops.a2a_recv_plan(counts.flatten().to(cuda), ep, el, rows)
    # arrival row j -> (source, expert); expert-major order sorts by (expert, source, arrival)
    src_e = [(s, e) for s in range(ep) for e in range(el) for _ in range(int(counts[s, e]))]
    order = sorted(range(rows), key=lambda j: (src_e[j][1], src_e[j][0], j))
    assert plan.map_in.cpu().tolist() == order
    back = [0] * rows
    for p, j in enumerate(order):
        back[j] = p
    assert plan.map_back.cpu().tolist() == back
    assert plan.offsets.cpu().tolist() == [0] + torch.cumsum(counts.sum(0), 0).tolist()
    assert _lib.device_status(cuda.index) == 0


def test_routing_records_match_the_reference_capture(cuda):
    """Per step, every router call's ids as int16 and weights as fp16 (the
    capture of moe_serving/record_routing.py:71-77), read back in one copy:
    equal to converting each router output on the host."""
    from types import SimpleNamespace

    from torch import nn

    from moe_serving_profile_b200.recording import RoutingRecords
    from moe_serving_profile_b200.router import GptOssRouter, Qwen3Router

    g = torch.Generator().manual_seed(3)
    q = Qwen3Router(SimpleNamespace(num_experts_per_tok=8, num_experts=128, norm_topk_prob=True,
                                    hidden_size=256)).to(cuda)
    q.weight.data = (torch.randn(128, 256, generator=g) * 0.05).bfloat16().to(cuda)
    o = GptOssRouter(SimpleNamespace(num_experts_per_tok=4, num_local_experts=32,
                                     hidden_size=256)).to(cuda)
    o.weight.data = (torch.randn(32, 256, generator=g) * 0.05).bfloat16().to(cuda)
    o.bias.data = (torch.randn(32, generator=g) * 0.1).bfloat16().to(cuda)
    model = nn.ModuleDict({"layer0": q, "layer1": o})
    rec = RoutingRecords.attach(model)
    try:
        for T in (5, 300):
            x = torch.randn(T, 256, generator=g).bfloat16().to(cuda)
            rec.begin()
            outs = {"layer0": q(x), "layer1": o(x)}
            step = rec.end()
            assert set(step) == {"layer0", "layer1"}
            for name, (_, scores, idx) in outs.items():
                assert torch.equal(step[name]["indices"], idx.to(torch.int16).cpu())
                assert torch.equal(step[name]["scores"], scores.to(torch.float16).cpu())
    finally:
        rec.close()


@pytest.mark.parametrize("T", [1, 37, 300])
def test_shared_expert_and_layer(cuda, T):
    """SharedSwiGLU (moe_serving/moe.py:84-95) against the same op in fp32
    PyTorch, and MoELayer with a shared expert = routed part + shared part
    (moe.py:161-162), also through simulate_ranks."""
    H, I_s, E, I, K = 512, 384, 16, 256, 4
    g = torch.Generator().manual_seed(T)
    sg = (torch.randn(I_s, H, generator=g) * 0.05).bfloat16()
    su = (torch.randn(I_s, H, generator=g) * 0.05).bfloat16()
    sd = (torch.randn(H, I_s, generator=g) * 0.05).bfloat16()
    sc = (torch.randn(1, H, generator=g) * 0.05).bfloat16()
    h = torch.randn(T, H, generator=g).bfloat16()
    shared = native.SharedSwiGLU(sg.to(cuda), su.to(cuda), sd.to(cuda), sc.to(cuda))
    out = shared(h.to(cuda))
    hf = h.float()
    act = torch.nn.functional.silu(hf @ sg.float().T) * (hf @ su.float().T)
    ref = torch.sigmoid(hf @ sc.float().T) * (act @ sd.float().T)
    _close(out.cpu(), ref.bfloat16(), "shared expert")

    gate_up, down, gate, (hh,) = _case(E, H, I, K, [T], seed=T + 1)
    experts = native.LocalSwiGLUExperts(gate_up.to(cuda), down.to(cuda))
    plan = native.ExpertPlan(E, 1, 0)
    layer = native.MoELayer(gate.to(cuda), experts, plan, K, shared=shared)
    y, stats = layer(hh.to(cuda))
    idx, wts = native.route(hh.to(cuda), gate.to(cuda), K, True)
    routed = native.routed_forward(hh.to(cuda), idx, wts, experts, plan, native.SingleRank())
    assert torch.equal(y, routed + shared(hh.to(cuda)))
    sim = native.simulate_ranks([hh.to(cuda)], gate.to(cuda), [experts], K, shared=[shared])
    assert torch.equal(sim[0], y)


@pytest.mark.parametrize("T,I_s", [(1, 256), (37, 192), (300, 128)])
def test_shared_expert_inside_the_routed_launch(cuda, T, I_s):
    """On one rank a shared expert whose intermediate fits the routed
    experts' padded intermediate runs as expert E of the routed launch
    (one more slot per token, weight sigmoid(hidden . score), combined last):
    bit for bit the routed output plus the separately computed shared
    expert (moe.py:161-162), and within the layer tolerance of fp32 PyTorch."""
    H, E, I, K = 512, 16, 256, 4
    g = torch.Generator().manual_seed(T + I_s)
    sg = (torch.randn(I_s, H, generator=g) * 0.05).bfloat16()
    su = (torch.randn(I_s, H, generator=g) * 0.05).bfloat16()
    sd = (torch.randn(H, I_s, generator=g) * 0.05).bfloat16()
    sc = (torch.randn(1, H, generator=g) * 0.05).bfloat16()
    gate_up, down, gate, (hh,) = _case(E, H, I, K, [T], seed=T + 7)
    shared = native.SharedSwiGLU(sg.to(cuda), su.to(cuda), sd.to(cuda), sc.to(cuda))
    experts = native.LocalSwiGLUExperts(gate_up.to(cuda), down.to(cuda))
    plan = native.ExpertPlan(E, 1, 0)
    layer = native.MoELayer(gate.to(cuda), experts, plan, K, shared=shared)
    assert layer.joint is not None and layer.joint.n_experts == E + 1
    x = hh.to(cuda)
    y, stats = layer(x)
    idx, wts = native.route(x, gate.to(cuda), K, True)
    routed = native.routed_forward(x, idx, wts, experts, plan, native.SingleRank())
    assert torch.equal(y, routed + shared(x))
    assert torch.equal(stats.counts, torch.bincount(idx.reshape(-1).cpu(), minlength=E))
    # the appended slot itself: routed ids and bf16 weights, then (E, torch.sigmoid)
    logit = torch.nn.functional.linear(x, sc.to(cuda))
    idx1, w1 = ops.append_shared_slot(idx, wts, logit, E)
    assert torch.equal(idx1[:, :K], idx) and bool((idx1[:, K] == E).all())
    assert torch.equal(w1[:, :K], wts.to(torch.bfloat16)) and torch.equal(w1[:, K], torch.sigmoid(logit)[:, 0])
    # fp32 PyTorch of the whole layer on the same routing
    hf = x.float().cpu()
    ref = torch.zeros(T, H)
    for t in range(T):
        for k in range(K):
            e = int(idx[t, k])
            gu = gate_up[e].float() @ hf[t]
            ref[t] += float(wts[t, k]) * (down[e].float() @ (torch.nn.functional.silu(gu[:I]) * gu[I:]))
    act = torch.nn.functional.silu(hf @ sg.float().T) * (hf @ su.float().T)
    ref += torch.sigmoid(hf @ sc.float().T) * (act @ sd.float().T)
    _close(y.cpu(), ref.bfloat16(), "layer with the shared expert inside the routed launch")
    assert _lib.device_status(cuda.index) == 0


def test_shared_expert_too_wide_runs_as_its_own_launch(cuda):
    """A shared intermediate beyond the routed experts' padded one keeps the
    separate launch (the routed pack is left as it was)."""
    H, E, I, K = 512, 8, 128, 2
    gate_up, down, gate, (hh,) = _case(E, H, I, K, [24], seed=5)
    g = torch.Generator().manual_seed(6)
    w = lambda *s: (torch.randn(*s, generator=g) * 0.05).bfloat16().to(cuda)
    shared = native.SharedSwiGLU(w(256, H), w(256, H), w(H, 256), w(1, H))
    experts = native.LocalSwiGLUExperts(gate_up.to(cuda), down.to(cuda))
    layer = native.MoELayer(gate.to(cuda), experts, native.ExpertPlan(E, 1, 0), K, shared=shared)
    assert layer.joint is None
    x = hh.to(cuda)
    y, _ = layer(x)
    idx, wts = native.route(x, gate.to(cuda), K, True)
    assert torch.equal(y, native.routed_forward(x, idx, wts, experts, native.ExpertPlan(E, 1, 0),
                                                native.SingleRank()) + shared(x))
