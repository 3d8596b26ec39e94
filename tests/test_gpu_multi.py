"""Expert parallelism over NCCL on two GPUs (skipped with fewer than two).

* replicated-token EP (qwen3.ParallelExperts with ParallelGroup(2), the
  reference's --ep-size layout): with numerics="reference" the output on
  every rank equals the one-GPU layer bit for bit; numerics="fast" stays
  within the BF16 layer tolerance;
* replicated-token EP with numerics="reference" runs the exact NVLink gather
  of contribution rows (b200moe_ep_gather) and must equal the one-GPU layer
  on two calls in a row;
* token all-to-all (native.routed_forward with ProcessGroupCollective, NCCL,
  and with PeerCollective, NVLink peer memory, eager and in CUDA graph
  replays): each rank's output equals native.simulate_routed (all ranks in
  one process, the same kernels) bit for bit;
* the fused NVLink combine + all-reduce (ParallelGroup.combine_reduce) equals
  its definition, bf16(fp32(partial_0) + fp32(partial_1)), bit for bit, in
  eager calls and in CUDA graph replays, for the one-shot exchange (T = 200)
  and the two-shot one (T = 4200); the NCCL path
  (B200MOE_P2P=0) agrees within bf16 rounding;
* a router sharded over the group (each rank routes a slice, one
  all-gather) returns what the whole-batch router returns, bit for bit.

Ranks are spawned processes, one per GPU, with a 60 s process-group timeout;
the parent gives them a bounded time to report.
"""

import os
import socket
from types import SimpleNamespace

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _qwen_module(cfg, w, dev, parallel, numerics):
    from moe_serving_profile_b200 import qwen3

    conf = SimpleNamespace(num_experts=cfg.experts, hidden_act="silu")
    m = qwen3.ParallelExperts(conf, parallel, numerics)
    for i, mods in enumerate(m.local):
        e = m.start + i
        mods["gate_proj"] = qwen3.ExpertProjection(w.gate[e].to(dev), w.gate_scale[e].to(dev), cfg.block)
        mods["up_proj"] = qwen3.ExpertProjection(w.up[e].to(dev), w.up_scale[e].to(dev), cfg.block)
        mods["down_proj"] = qwen3.ExpertProjection(w.down[e].to(dev), w.down_scale[e].to(dev), cfg.block)
    return m


def _worker(rank: int, port: int, q):
    try:
        from datetime import timedelta

        import torch.distributed as dist

        from moe_serving_profile_b200 import native
        from moe_serving_profile_b200 import synthetic as S
        from moe_serving_profile_b200.parallel import ParallelGroup
        from oracle import oracle

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=WORLD, device_id=dev,
                                timeout=timedelta(seconds=60))
        res = {}
        # ---- replicated-token EP
        cfg = S.CONFIGS["qwen3-30b-a3b"]
        w = S.make_qwen(cfg, seed=4, device=dev)   # same seed, same values on every GPU
        T = 64
        x = S.make_hidden(T, cfg.hidden, seed=5, device=dev)
        _, scores, idx, _ = oracle.qwen_router(x.cpu(), w.router.cpu(), cfg.top_k, True)
        scores, idx = scores.to(dev), idx.to(dev)
        one = _qwen_module(cfg, w, dev, ParallelGroup(1), "reference")(x, idx, scores)
        pg = ParallelGroup(WORLD)
        ref_mod = _qwen_module(cfg, w, dev, pg, "reference")
        ref_ep = [ref_mod(x, idx, scores) for _ in range(2)]   # the exact NVLink gather, twice
        fast_ep = _qwen_module(cfg, w, dev, pg, "fast")(x, idx, scores)
        res["gather_used"] = pg._gather is not None
        res["reference_equal"] = all(bool(torch.equal(o, one)) for o in ref_ep)
        diff = (fast_ep.float() - one.float())
        res["fast_rel_l2"] = float(diff.norm() / one.float().norm())
        # ---- token all-to-all
        E, H, I, K = 128, 2048, 768, 8
        g = torch.Generator().manual_seed(7)
        gate_up = (torch.randn(E, 2 * I, H, generator=g) * 0.02).bfloat16()
        down = (torch.randn(E, H, I, generator=g) * 0.02).bfloat16()
        gate = (torch.randn(E, H, generator=g) * 0.02).bfloat16()
        tokens = [48, 33]
        hiddens = [torch.randn(t, H, generator=g).bfloat16().to(dev) for t in tokens]
        el = E // WORLD
        banks = [native.LocalSwiGLUExperts(gate_up[r * el:(r + 1) * el].to(dev),
                                           down[r * el:(r + 1) * el].to(dev)) for r in range(WORLD)]
        routes = [native.route(h, gate.to(dev), K, True) for h in hiddens]
        sim = native.simulate_routed(hiddens, [r_[0] for r_ in routes], [r_[1] for r_ in routes], banks, E)
        plan = native.ExpertPlan(E, WORLD, rank)
        out = native.routed_forward(hiddens[rank], routes[rank][0], routes[rank][1], banks[rank], plan,
                                    native.ProcessGroupCollective())
        res["a2a_equal"] = bool(torch.equal(out, sim[rank]))
        # ---- token all-to-all over NVLink peer memory: two eager calls, then
        # CUDA graph replays
        pc = native.PeerCollective(max_tokens=64)
        outs = [native.routed_forward(hiddens[rank], routes[rank][0], routes[rank][1], banks[rank],
                                      plan, pc) for _ in range(2)]
        res["a2a_peer_equal"] = all(bool(torch.equal(o, sim[rank])) for o in outs)
        stream = torch.cuda.Stream(dev)
        stream.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            gout = native.routed_forward(hiddens[rank], routes[rank][0], routes[rank][1], banks[rank],
                                         plan, pc)
        ok = True
        for _ in range(2):
            graph.replay()
            torch.cuda.synchronize(dev)
            ok = ok and bool(torch.equal(gout, sim[rank]))
        del graph
        res["a2a_peer_graph_equal"] = ok
        pc.close()
        # ---- fused NVLink combine + all-reduce
        from moe_serving_profile_b200 import _lib, ops
        T2, K2, E2, H2 = 200, 8, 128, 2048
        g2 = torch.Generator().manual_seed(21)
        idx2 = torch.stack([torch.randperm(E2, generator=g2)[:K2] for _ in range(T2)]).long()
        rows2 = torch.randn(T2 * K2, H2, generator=g2).bfloat16().to(dev)
        _, _, _, inv2 = oracle.permute(idx2, E2)
        inv2, idx2 = inv2.to(dev), idx2.to(dev)
        half = E2 // WORLD
        parts = [ops.combine(rows2, inv2, idx2, order=_lib.ORDER_EXPERT, expert_lo=q * half,
                             expert_hi=(q + 1) * half).float() for q in range(WORLD)]
        exact = (parts[0] + parts[1]).bfloat16()
        lo, hi = rank * half, (rank + 1) * half
        eager = [pg.combine_reduce(rows2, inv2, idx2, lo, hi) for _ in range(3)]
        res["p2p_used"] = pg._exchange is not None
        res["p2p_equal"] = all(bool(torch.equal(o, exact)) for o in eager)
        stream = torch.cuda.Stream(dev)
        stream.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            gout = pg.combine_reduce(rows2, inv2, idx2, lo, hi)
        ok = True
        for _ in range(2):
            graph.replay()
            torch.cuda.synchronize(dev)
            ok = ok and bool(torch.equal(gout, exact))
        del graph
        res["p2p_graph_equal"] = ok
        os.environ["B200MOE_P2P"] = "0"
        nccl = pg.combine_reduce(rows2, inv2, idx2, lo, hi)
        os.environ["B200MOE_P2P"] = "1"
        res["nccl_close"] = float((nccl.float() - exact.float()).abs().max()) <= \
            float(exact.float().abs().max()) * 2 ** -7
        # two-shot exchange (T * H * 2 > 16 MiB at two ranks): same definition
        T3 = 4200
        idx3 = torch.stack([torch.randperm(E2, generator=g2)[:K2] for _ in range(T3)]).long()
        rows3 = torch.randn(T3 * K2, H2, generator=g2).bfloat16().to(dev)
        _, _, _, inv3 = oracle.permute(idx3, E2)
        inv3, idx3 = inv3.to(dev), idx3.to(dev)
        parts3 = [ops.combine(rows3, inv3, idx3, order=_lib.ORDER_EXPERT, expert_lo=q * half,
                              expert_hi=(q + 1) * half).float() for q in range(WORLD)]
        exact3 = (parts3[0] + parts3[1]).bfloat16()
        res["p2p_two_shot_equal"] = all(bool(torch.equal(pg.combine_reduce(rows3, inv3, idx3, lo, hi),
                                                        exact3)) for _ in range(2))
        del rows3
        # ---- router sharded over the group == routed whole, bit for bit
        from moe_serving_profile_b200.router import Qwen3Router
        rconf = SimpleNamespace(num_experts_per_tok=8, num_experts=128, norm_topk_prob=True,
                                hidden_size=2048)
        whole = Qwen3Router(rconf, logits="fused").to(dev)
        whole.weight.data = w.router
        shard = Qwen3Router(rconf, logits="fused").to(dev).shard_over(pg)
        shard.weight.data = w.router
        xr = S.make_hidden(2048, 2048, seed=9, device=dev)
        a, b = whole(xr), shard(xr)
        res["router_shard_equal"] = all(bool(torch.equal(u, v)) for u, v in zip(a, b)) and \
            bool(torch.equal(whole.last_counts, shard.last_counts))
        res["status"] = _lib.device_status(rank)
        torch.cuda.synchronize(dev)
        pg.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, res))
    except Exception as exc:  # report instead of leaving the parent waiting
        q.put((rank, repr(exc)))


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs two GPUs")
def test_expert_parallel_over_nccl():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=600) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=120)
    for r in range(WORLD):
        res = results[r]
        assert isinstance(res, dict), res
        assert res["reference_equal"], f"rank {r}: replicated-token EP differs from one GPU"
        assert res["fast_rel_l2"] < 1e-2, res
        assert res["a2a_equal"], f"rank {r}: all-to-all differs from the one-process run"
        assert res["a2a_peer_equal"] and res["a2a_peer_graph_equal"], res
        assert res["gather_used"], res
        assert res["p2p_used"] and res["p2p_equal"] and res["p2p_graph_equal"], res
        assert res["nccl_close"] and res["status"] == 0, res
        assert res["router_shard_equal"], res
        assert res["p2p_two_shot_equal"], res
