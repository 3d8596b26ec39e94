"""MoE expert-layer benchmark (router -> permute -> grouped GEMMs -> combine).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload qwen3-30b-a3b|gpt-oss-20b|gpt-oss-120b|qwen3-235b-a22b]

One step runs the layer once for every batch size of the workload (decode and
prefill batches of one layer shape) on seeded synthetic weights and tokens
with the workload's shapes (random-init, quantised as the checkpoints are).
``value`` is tokens/s over the step: sum of batch tokens / sum of device
time, each batch replayed from a CUDA graph with L2 flushed (a 256 MiB write)
before it, timed with CUDA events. ``e2e`` is the same metric through the
public modules (router + ParallelExperts forward, eager) with the tokens
copied from pinned host memory and the outputs copied back every batch; the
copies run on their own streams and overlap other batches' compute.

N > 1 (torchrun, one rank per GPU): replicated-token expert parallelism, the
reference's record_* layout: every rank routes all tokens and runs its E/N
experts, combines its own experts' contributions and the [T, H] partial sums
are summed over the group ("fast" numerics, the reference's efficient EP
exchange, through the fused NVLink combine). Work per step is fixed (strong
scaling). Before timing, every rank checks the EP layer against the
single-GPU layer on one decode and one prefill batch ("parity").

``--impl reference`` times the reference algorithm on the host CPU (the
oracle's torch restatement of the reference numerics), rank 0 only, with no
library code loaded: step i runs batch i mod (number of batches), each batch
timed whole.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path
from types import SimpleNamespace

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

# plain torch: loads no library (the reference arm imports nothing else of the package)
from moe_serving_profile_b200 import synthetic as S  # noqa: E402

PEAKS = ROOT / "MEASURED_PEAKS.json"
L2_FLUSH_BYTES = 256 << 20
METRIC = "MoE-layer tokens/s at 1/2/4/8 B200 (decode & prefill), % HBM/tensor roofline"


def peaks():
    if PEAKS.exists():
        p = json.loads(PEAKS.read_text())
        return p["hbm_gbs"], p["bf16_tflops"], p["bf16_tflops_sustained"], "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, index: int):
        self.index, self.proc, self.lines = index, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def wait_first(self, limit_s: float) -> None:
        """Wait (at most limit_s) until nvidia-smi has printed its first sample:
        it takes a moment to start, and a short timed region could pass first."""
        t0 = time.perf_counter()
        while self.proc is not None and not self.lines and time.perf_counter() - t0 < limit_s:
            time.sleep(0.05)

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) != 6:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for name, flag in zip(self.NAMES, parts[2:]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------------- workload
def workload_config(cfg, world: int) -> dict:
    """The workload's shape, identical in the line of both arms."""
    return {"workload": cfg.name, "batches": list(cfg.batches), "hidden": cfg.hidden,
            "experts": cfg.experts, "top_k": cfg.top_k, "intermediate": cfg.inter,
            "weights": cfg.storage, "parallelism": f"ep{world} replicated-token"}


def build_layer(cfg, dev, ep: int, rank: int, seed: int = 1):
    """Router module + rank-local packed experts for one synthetic layer."""
    from moe_serving_profile_b200 import layout
    from moe_serving_profile_b200.router import GptOssRouter, Qwen3Router
    epr = cfg.experts // ep
    sl = slice(rank * epr, (rank + 1) * epr)
    if cfg.family == "qwen3":
        w = S.make_qwen(cfg, seed, dev)
        router = Qwen3Router(SimpleNamespace(num_experts_per_tok=cfg.top_k, num_experts=cfg.experts,
                                             norm_topk_prob=cfg.norm_topk, hidden_size=cfg.hidden)).to(dev)
        router.weight.data = w.router
        if w.router_bias is not None:
            router.bias = w.router_bias
        packed = layout.fp8_experts(w.gate[sl], w.gate_scale[sl], w.up[sl], w.up_scale[sl],
                                    w.down[sl], w.down_scale[sl], cfg.block)
    else:
        w = S.make_gpt_oss(cfg, seed, dev)
        router = GptOssRouter(SimpleNamespace(num_experts_per_tok=cfg.top_k,
                                              num_local_experts=cfg.experts,
                                              hidden_size=cfg.hidden)).to(dev)
        router.weight.data = w.router
        router.bias.data = w.router_bias
        packed = layout.gpt_oss_mxfp4_experts(w.gu_blocks[sl], w.gu_scales[sl], w.gu_bias[sl],
                                              w.dn_blocks[sl], w.dn_scales[sl], w.dn_bias[sl],
                                              cfg.alpha, cfg.limit)
    del w
    torch.cuda.empty_cache()
    return router, packed


def numerics_for(ep: int) -> str:
    """One GPU: the reference's ordered combine. Several: each rank combines
    its own experts and the [T, H] partial sums are all-reduced (the
    reference's fast / efficient EP exchange; the exact ordered combine would
    move every [T*K, H] contribution row to every rank)."""
    return "reference" if ep == 1 else "fast"


def layer_call(cfg, router, packed, x, parallel, rank, ep, numerics=None):
    from moe_serving_profile_b200 import experts as X
    _, scores, idx = router(x)
    return X.layer_forward(packed, x, idx, scores, num_experts=cfg.experts,
                           expert_begin=rank * (cfg.experts // ep), parallel=parallel,
                           numerics=numerics or numerics_for(ep))


def w8a8_leg(args, cfg, router, packed, xs, flush, stream, dev, hbm, tf_burst):
    """The same layer in the reference's efficient FP8 numerics (W8A8,
    ``numerics="efficient"``), reported beside the weight-only headline:
    per-batch CUDA-graph replays after an L2 flush, and the W8A8 gate/up GEMM
    of the largest batch timed alone."""
    from moe_serving_profile_b200 import _lib, ops
    from moe_serving_profile_b200 import experts as X
    def call(x):
        _, scores, idx = router(x)
        return X.layer_forward(packed, x, idx, scores, num_experts=cfg.experts, expert_begin=0,
                               numerics="efficient")

    batches = list(xs)
    graphs = {}
    with torch.cuda.stream(stream):
        for T in batches:
            for _ in range(2):
                call(xs[T])
    torch.cuda.synchronize(dev)
    for T in batches:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            call(xs[T])
        graphs[T] = g
    warm = max(3, args.warmup)
    recs = []
    with torch.cuda.stream(stream):
        for it in range(warm + args.steps):
            for T in batches:
                flush.fill_(T & 0xff)
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record(stream)
                graphs[T].replay()
                e.record(stream)
                if it >= warm:
                    recs.append((T, s, e))
    torch.cuda.synchronize(dev)
    ms = {T: 0.0 for T in batches}
    for T, s, e in recs:
        ms[T] += s.elapsed_time(e) / args.steps
    per_batch = []
    for T in batches:
        with torch.cuda.stream(stream):
            _, _, idx = router(xs[T])
            counts = torch.bincount(idx.flatten(), minlength=cfg.experts).cpu()
        gbs = S.algorithmic_bytes(cfg, T, counts) / (ms[T] / 1e3) / 1e9
        tfs = S.algorithmic_flops(cfg, T) / (ms[T] / 1e3) / 1e12
        per_batch.append({"tokens": T, "ms": round(ms[T], 4), "tokens_per_s": round(T / (ms[T] / 1e3), 1),
                          "hbm_frac": round(gbs / hbm, 4), "tflops": round(tfs, 2)})
    # the W8A8 gate/up GEMM of the largest batch, timed alone
    Tm = max(batches)
    with torch.cuda.stream(stream):
        x = xs[Tm]
        _, scores, idx = router(x)
        perm = ops.permute(idx, cfg.experts)
        R = Tm * cfg.top_k
        q, qs = ops.act_quant_fp8(x, k_pad=packed.h_k, rows_src=perm.perm_src, src_div=cfg.top_k)
        act = torch.empty(R, packed.i_pad, device=dev, dtype=torch.bfloat16)
        kw = dict(offsets=perm.offsets, expert_begin=0, n_experts=packed.n_experts, max_rows=R, planes=2,
                  feat_pad=packed.i_pad, n_feat=packed.inter, k_pad=packed.h_k, weight=packed.w1,
                  fp8_block=packed.block, q=q, q_scale=qs, epilogue=_lib.EPI_SWIGLU, out=act,
                  token_tile=X.tile_policy(Tm, cfg.top_k, cfg.experts, 128))
        for _ in range(3):
            ops.w8a8_gemm(**kw)
        kms = 0.0
        for _ in range(10):
            flush.fill_(2)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            ops.w8a8_gemm(**kw)
            e.record(stream)
            e.synchronize()
            kms += s.elapsed_time(e) / 10
    gemm_tf = 2 * R * cfg.hidden * 2 * cfg.inter / (kms / 1e3) / 1e12
    for g in graphs.values():
        del g
    total_ms = sum(ms.values())
    return {"value": round(sum(batches) / (total_ms / 1e3), 1), "unit": "tokens/s",
            "ms_per_step": round(total_ms, 4), "numerics": "efficient (W8A8: e4m3 activations per "
            "row and 128 columns, e4m3 block-128 weights, kind::f8f6f4 MMAs)", "per_batch": per_batch,
            "gate_up": {"tokens": Tm, "ms": round(kms, 4), "tflops": round(gemm_tf, 2),
                        "frac_of_bf16_burst": round(gemm_tf / tf_burst, 4),
                        "frac_of_fp8_nominal_2x_bf16": round(gemm_tf / (2 * tf_burst), 4)}}


def kernel_launches(T: int, K: int, E: int) -> int:
    """Our kernels per layer call: router selection (1; the logits are the
    reference's own F.linear) + permute (1 or 3) + row gather (large token
    tiles only) + 2 GEMMs + combine."""
    from moe_serving_profile_b200 import experts as X
    gather = 1 if X.tile_policy(T, K, E) >= 64 else 0
    return 1 + (1 if T * K <= 8192 else 3) + gather + 2 + 1


# --------------------------------------------------------------------------- CPU leg
_CPU_WEIGHTS = {}


def cpu_layer_time(cfg, T: int, seed: int = 1) -> float:
    """Seconds for one reference-numerics layer call (router + experts) on the host CPU."""
    from oracle import oracle
    if cfg.name not in _CPU_WEIGHTS:
        _CPU_WEIGHTS[cfg.name] = (S.make_qwen(cfg, seed, "cpu") if cfg.family == "qwen3"
                                  else S.make_gpt_oss(cfg, seed, "cpu"))
    w = _CPU_WEIGHTS[cfg.name]
    x = S.make_hidden(T, cfg.hidden, T, "cpu")
    with torch.inference_mode():
        t0 = time.perf_counter()
        if cfg.family == "qwen3":
            probs, scores, idx, _ = oracle.qwen_router(x, w.router, cfg.top_k, cfg.norm_topk)
            oracle.qwen_layer(x, idx, scores, w.gate, w.gate_scale, w.up, w.up_scale, w.down,
                              w.down_scale, cfg.block)
        else:
            logits, scores, idx = oracle.gpt_oss_router(x, w.router, w.router_bias, cfg.top_k)
            oracle.gpt_oss_layer(x, idx, scores, w.gu_blocks, w.gu_scales, w.gu_bias, w.dn_blocks,
                                 w.dn_scales, w.dn_bias, cfg.alpha, cfg.limit)
        return time.perf_counter() - t0


def cpu_batches(cfg, budget_s: float):
    """The reference path on the host over the workload's batches, each batch
    timed whole (no extrapolation), in increasing size until ``budget_s`` of
    CPU time is spent. Returns (tokens/s over the measured batches, {T: s},
    sample text)."""
    torch.set_num_threads(os.cpu_count() or 1)
    secs, spent = {}, 0.0
    for T in sorted(cfg.batches):
        if secs and spent > budget_s:
            break
        secs[T] = cpu_layer_time(cfg, T)
        spent += secs[T]
    value = sum(secs) / sum(secs.values())
    skipped = [T for T in cfg.batches if T not in secs]
    sample = ("reference numerics on host CPU, each batch timed whole: "
              + ", ".join(f"T={T} {secs[T]:.2f} s" for T in sorted(secs))
              + (f"; not measured (budget): {skipped}" if skipped else ""))
    return value, secs, sample


def reference_arm(args, cfg):
    """The reference's CPU path, timed on the host cores (rank 0 only). With
    at least as many steps as batches, step i runs batch i mod n_batches
    (every batch timed whole at least once); with fewer, every step runs all
    of them. value = sum of batch tokens / sum of the batches' mean times, the
    GPU arm's metric."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    batches = list(cfg.batches)
    rotate = args.steps >= len(batches)

    def step(i):
        return [batches[i % len(batches)]] if rotate else batches

    for i in range(args.warmup):
        for T in step(i):
            cpu_layer_time(cfg, T)
    times = {T: [] for T in batches}
    t0 = time.perf_counter()
    for i in range(args.steps):
        for T in step(args.warmup + i):
            times[T].append(cpu_layer_time(cfg, T))
    wall = time.perf_counter() - t0
    mean = {T: statistics.mean(v) for T, v in times.items() if v}
    value = sum(mean) / sum(mean.values())
    cores = torch.get_num_threads()
    sample = (("step i runs batch i mod %d" % len(batches)) if rotate else "every step runs all batches") + \
        ", each batch timed whole: " + ", ".join(f"T={T} {mean[T] * 1e3:.1f} ms (x{len(times[T])})"
                                                 for T in batches if T in mean)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(wall / max(1, args.steps) * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded random-init weights, quantised like the checkpoints)",
        "config": workload_config(cfg, args.gpus),
        "reference_path": "the reference numerics (dequantise-then-BF16 per expert, ordered bf16 merge; "
                          "the oracle's torch restatement) on the host CPU, one process",
        "per_batch_ms": {str(T): round(mean[T] * 1e3, 3) for T in batches if T in mean},
        "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- GPU arm
def ep_parity(cfg, router, packed, parallel, rank, world, dev):
    """EP layer against the single-GPU layer on every rank, on the smallest
    and the largest batch: "reference" numerics must be bitwise equal (the
    ordered global-expert combine is EP-invariant), "fast" numerics within
    the layer tolerance (rel. L2 <= 1e-2). Every rank builds the whole layer
    for the comparison; the result is reduced over the group (max error,
    AND of bitwise)."""
    from moe_serving_profile_b200 import experts as X
    _, packed1 = build_layer(cfg, dev, 1, 0)
    res = {}
    for T in (min(cfg.batches), max(cfg.batches)):
        x = S.make_hidden(T, cfg.hidden, seed=7000 + T, device=dev)
        _, scores, idx = router(x)
        one = X.layer_forward(packed1, x, idx, scores, num_experts=cfg.experts, expert_begin=0)
        for num in ("reference", "fast"):
            out = X.layer_forward(packed, x, idx, scores, num_experts=cfg.experts,
                                  expert_begin=rank * (cfg.experts // world), parallel=parallel,
                                  numerics=num)
            d = (out.float() - one.float())
            stats = torch.tensor([float(d.abs().max()), float(d.norm() / one.float().norm().clamp_min(1e-30)),
                                  0.0 if torch.equal(out, one) else 1.0], device=dev, dtype=torch.float64)
            dist.all_reduce(stats, op=dist.ReduceOp.MAX)
            res[f"{num}_T{T}"] = {"max_abs": float(stats[0]), "rel_l2": float(stats[1]),
                                  "bitwise": bool(stats[2] == 0.0)}
    del packed1
    torch.cuda.empty_cache()
    res["ok"] = all(v["bitwise"] for k, v in res.items() if k.startswith("reference")) and \
        all(v["rel_l2"] <= 1e-2 for k, v in res.items() if k.startswith("fast"))
    return res


def stage_breakdown(cfg, router, packed, xs, parallel, rank, world, stream, reps=5):
    """Per-stage device time (ms, warm L2, eager) of one layer call per batch:
    router, permute, row gather + gate/up GEMM, down GEMM, combine (+ the EP
    exchange at N > 1). Every rank runs the same sequence, so the collective
    steps line up."""
    from moe_serving_profile_b200 import _lib, ops
    from moe_serving_profile_b200 import experts as X
    lo = rank * (cfg.experts // world)
    out = {}
    for T, x in xs.items():
        acc = [0.0] * 5
        for it in range(reps + 2):
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
            with torch.cuda.stream(stream):
                ev[0].record(stream)
                _, scores, idx = router(x)
                ev[1].record(stream)
                perm = ops.permute(idx, cfg.experts)
                ev[2].record(stream)
                act = X.gate_up(packed, x, perm, K=cfg.top_k, num_experts=cfg.experts, expert_begin=lo,
                                tokens=T)
                ev[3].record(stream)
                contrib = X.down(packed, act, perm, scores, K=cfg.top_k, num_experts=cfg.experts,
                                 expert_begin=lo, tokens=T)
                ev[4].record(stream)
                if parallel is None:
                    ops.combine(contrib, perm.inverse, idx, order=_lib.ORDER_EXPERT)
                else:
                    parallel.combine_reduce(contrib, perm.inverse, idx, lo, lo + packed.n_experts)
                ev[5].record(stream)
            ev[5].synchronize()
            if it >= 2:
                for j in range(5):
                    acc[j] += ev[j].elapsed_time(ev[j + 1]) / reps
        t = torch.tensor(acc, device=x.device, dtype=torch.float64)
        if parallel is not None:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        names = ("router", "permute", "gather+gate_up", "down", "combine" if parallel is None else "exchange")
        out[str(T)] = {n: round(float(v), 4) for n, v in zip(names, t.tolist())}
    return out


# --------------------------------------------------------------------------- EP workloads
# Expert-parallel legs reported beside the headline: (workload, mode). "a2a":
# token all-to-all (moe.py:110-137), each rank routes its 1/N of the tokens
# and the rows move over NVLink peer memory (native.PeerCollective);
# "replicated": every rank routes all tokens, runs its experts and the
# contribution rows are gathered over NVLink for the ordered global-expert
# combine (reference numerics, parallel_numerics.py:13-36).
EP_LEGS = (("qwen3-30b-a3b", "a2a"), ("qwen3-235b-a22b", "a2a"), ("gpt-oss-120b", "a2a"),
           ("gpt-oss-120b", "replicated"))


def ep_leg(args, name, mode, world, rank, dev, stream, flush, pg):
    """Tokens/s of one expert-parallel workload over its batches (CUDA-graph
    replays, L2 flushed before each batch, max over ranks), with each batch
    checked on every rank against the single-GPU computation of the same
    tokens (bitwise: the same combine order, expert outputs independent of
    where they run)."""
    from moe_serving_profile_b200 import _lib, native, ops
    from moe_serving_profile_b200 import experts as X
    cfg = S.CONFIGS[name]
    E, K, el = cfg.experts, cfg.top_k, cfg.experts // world
    router, packed = build_layer(cfg, dev, world, rank)
    _, full = build_layer(cfg, dev, 1, 0) if world > 1 else (None, packed)
    local = SimpleNamespace(num_experts=el, weights=packed)
    plan = native.ExpertPlan(E, world, rank)
    a2a = mode == "a2a"
    # all-to-all: rank r routes tokens [r T / N, (r + 1) T / N) of each batch
    # (a batch smaller than N leaves some ranks without tokens)
    span = {T: ((rank * T) // world, ((rank + 1) * T) // world) if a2a else (0, T) for T in cfg.batches}
    cap = max(-(-T // world) for T in cfg.batches)
    coll = native.PeerCollective(max_tokens=cap) if (a2a and world > 1) else native.SingleRank()
    xs = {}
    for T in cfg.batches:
        x = S.make_hidden(T, cfg.hidden, seed=2000 + T, device=dev)
        xs[T] = x[span[T][0]:span[T][1]].contiguous()

    def call(T):
        _, scores, idx = router(xs[T])
        if a2a:
            return native.routed_forward(xs[T], idx, scores, local, plan, coll)
        return X.layer_forward(packed, xs[T], idx, scores, num_experts=E, expert_begin=rank * el,
                               parallel=pg, numerics="reference")

    # parity against one GPU (full layer) on every batch, and the global load cv
    parity, cvs = {}, {}
    with torch.cuda.stream(stream):
        for T in cfg.batches:
            out = call(T)
            _, scores, idx = router(xs[T])
            if a2a:
                perm = ops.permute(idx, E)
                # the token tile of the all-to-all's GEMMs: the global batch,
                # estimated as this rank's share times the group size
                y = X.run_experts(full, xs[T], perm, None, K=K, num_experts=E, expert_begin=0,
                                  tile_tokens=xs[T].shape[0] * world)
                ref = ops.combine(y, perm.inverse, idx, order=_lib.ORDER_RANK_SLOT, experts_per_rank=el,
                                  weights=scores.to(torch.bfloat16).contiguous())
            else:
                ref = X.layer_forward(full, xs[T], idx, scores, num_experts=E, expert_begin=0)
            d = (out.float() - ref.float())
            st = torch.tensor([float(d.abs().max()) if d.numel() else 0.0,
                               float(d.norm() / ref.float().norm().clamp_min(1e-30)) if d.numel() else 0.0,
                               0.0 if torch.equal(out, ref) else 1.0], device=dev, dtype=torch.float64)
            counts = torch.bincount(idx.flatten(), minlength=E).to(dev)
            if world > 1:
                dist.all_reduce(st, op=dist.ReduceOp.MAX)
                dist.all_reduce(counts)
            parity[str(T)] = {"max_abs": float(st[0]), "rel_l2": float(st[1]), "bitwise": bool(st[2] == 0)}
            cvs[T] = S.expert_load_cv(counts.cpu())
    del full
    torch.cuda.synchronize(dev)
    graphs = {}
    with torch.cuda.stream(stream):
        for T in cfg.batches:
            call(T)
    torch.cuda.synchronize(dev)
    for T in cfg.batches:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            call(T)
        graphs[T] = g
    if world > 1:
        dist.barrier()
    recs = []
    with torch.cuda.stream(stream):
        for it in range(max(3, args.warmup) + args.steps):
            for T in cfg.batches:
                flush.fill_(T & 0xff)
                s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s_.record(stream)
                graphs[T].replay()
                e_.record(stream)
                if it >= max(3, args.warmup):
                    recs.append((T, s_, e_))
    torch.cuda.synchronize(dev)
    ms = {T: 0.0 for T in cfg.batches}
    for T, s_, e_ in recs:
        ms[T] += s_.elapsed_time(e_) / args.steps
    t = torch.tensor([ms[T] for T in cfg.batches], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = dict(zip(cfg.batches, t.tolist()))
    for g in graphs.values():
        del g
    graphs.clear()
    torch.cuda.synchronize(dev)
    if world > 1 and a2a:
        coll.close()
    total = sum(ms.values())
    per_batch = [{"tokens": T, "ms": round(ms[T], 4), "tokens_per_s": round(T / (ms[T] / 1e3), 1),
                  "expert_load_cv": round(cvs[T], 3),
                  "tflops": round(S.algorithmic_flops(cfg, T) / (ms[T] / 1e3) / 1e12, 2)}
                 for T in cfg.batches]
    return {"workload": name, "mode": mode + (" (NVLink peer memory)" if world > 1 else ""),
            "value": round(sum(cfg.batches) / (total / 1e3), 1), "unit": "tokens/s",
            "ms_per_step": round(total, 4), "per_batch": per_batch, "parity": parity,
            "parity_ok": all(v["bitwise"] for v in parity.values())}


def profile_calls(args, cfg):
    """Three eager layer calls per batch size, nothing timed (an ncu target)."""
    from moe_serving_profile_b200 import _lib
    from moe_serving_profile_b200 import experts as X
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    router, packed = build_layer(cfg, dev, 1, 0)
    for T in (args.tokens or cfg.batches):
        x = S.make_hidden(T, cfg.hidden, seed=1000 + T, device=dev)
        for _ in range(3):
            if args.w8a8_profile:
                _, scores, idx = router(x)
                X.layer_forward(packed, x, idx, scores, num_experts=cfg.experts, expert_begin=0,
                                numerics="efficient")
            else:
                layer_call(cfg, router, packed, x, None, 0, 1)
        torch.cuda.synchronize(dev)
    assert _lib.device_status(0) == 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=("b200", "reference"))
    ap.add_argument("--workload", default="qwen3-30b-a3b")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-w8a8", action="store_true", help="skip the W8A8 (efficient FP8) report")
    ap.add_argument("--no-ep-legs", action="store_true",
                    help="skip the expert-parallel workloads (qwen3-235b-a22b all-to-all, gpt-oss-120b "
                         "all-to-all and replicated-token)")
    ap.add_argument("--profile", action="store_true",
                    help="eager layer calls only (for ncu): 3 calls per --tokens batch")
    ap.add_argument("--tokens", type=int, nargs="*", default=None)
    ap.add_argument("--w8a8-profile", action="store_true",
                    help="with --profile: the W8A8 (efficient FP8) layer instead of weight-only")
    args = ap.parse_args()
    cfg = S.CONFIGS[args.workload]
    if args.impl == "reference":
        return reference_arm(args, cfg)
    if args.profile:
        return profile_calls(args, cfg)

    from moe_serving_profile_b200 import _lib, ops  # noqa: F401  (loads the library)
    from moe_serving_profile_b200 import experts as X
    from moe_serving_profile_b200.parallel import ParallelGroup

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    parallel = ParallelGroup(world) if world > 1 else None
    hbm, tf_burst, tf_sust, peak_kind = peaks()

    router, packed = build_layer(cfg, dev, world, rank)
    batches = list(cfg.batches)
    parity = ep_parity(cfg, router, packed, parallel, rank, world, dev) if world > 1 else None
    xs = {T: S.make_hidden(T, cfg.hidden, seed=1000 + T, device=dev) for T in batches}
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(device=dev)

    # ---- CUDA graphs, one per batch size
    graphs, outs = {}, {}
    with torch.cuda.stream(stream):
        for T in batches:
            for _ in range(2):
                layer_call(cfg, router, packed, xs[T], parallel, rank, world)
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    for T in batches:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            outs[T] = layer_call(cfg, router, packed, xs[T], parallel, rank, world)
        graphs[T] = g
    torch.cuda.synchronize(dev)

    def step(record):
        times = {}
        with torch.cuda.stream(stream):
            for T in batches:
                flush.fill_(T & 0xff)
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record(stream)
                graphs[T].replay()
                e.record(stream)
                times[T] = (s, e)
        return times

    per_batch_ms = {T: 0.0 for T in batches}
    with ClockSampler(local) as clocks:
        clocks.wait_first(5.0)
        # warm-up: at least W steps and ~0.5 s, so the clock sampler sees load.
        # Every rank must replay the same collectives, so the count is agreed
        # over the group (max) from the time of the first W steps.
        t0 = time.perf_counter()
        for _ in range(max(3, args.warmup)):
            step(False)
        torch.cuda.synchronize(dev)
        per = (time.perf_counter() - t0) / max(3, args.warmup)
        extra = torch.tensor([max(0, math.ceil((0.5 - (time.perf_counter() - t0)) / max(per, 1e-6)))],
                             device=dev, dtype=torch.int64)
        if world > 1:
            dist.all_reduce(extra, op=dist.ReduceOp.MAX)
        for _ in range(int(extra)):
            step(False)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        # NVTX range "timed": lets a profiler's launch list select the timed steps
        torch.cuda.nvtx.range_push("timed")
        recs = [step(True) for _ in range(args.steps)]
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    for rec in recs:
        for T, (s, e) in rec.items():
            per_batch_ms[T] += s.elapsed_time(e) / args.steps
    step_ms = sum(per_batch_ms.values())
    if world > 1:
        t = torch.tensor([step_ms] + [per_batch_ms[T] for T in batches], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_ms, per = float(t[0]), t[1:].tolist()
        per_batch_ms = dict(zip(batches, per))
    tokens = sum(batches)
    value = tokens / (step_ms / 1e3)

    # ---- per-batch roofline (algorithmic bytes from the actual routing)
    per_batch = []
    for T in batches:
        with torch.cuda.stream(stream):
            _, _, idx = router(xs[T])
            counts = torch.bincount(idx.flatten(), minlength=cfg.experts).cpu()
        ms = per_batch_ms[T]
        byts = S.algorithmic_bytes(cfg, T, counts)
        flops = S.algorithmic_flops(cfg, T)
        gbs = byts / (ms / 1e3) / 1e9
        tfs = flops / (ms / 1e3) / 1e12
        per_batch.append({"tokens": T, "ms": round(ms, 4), "tokens_per_s": round(T / (ms / 1e3), 1),
                          "hbm_gbs": round(gbs, 1), "hbm_frac": round(gbs / hbm, 4),
                          "hbm_frac_per_gpu": round(gbs / (hbm * world), 4),
                          "tflops": round(tfs, 2), "tensor_frac": round(tfs / tf_burst, 4),
                          "tensor_frac_per_gpu": round(tfs / (tf_burst * world), 4),
                          "used_experts": int((counts > 0).sum()),
                          "expert_load_cv": round(S.expert_load_cv(counts), 3)})

    # ---- dominant kernel: the gate/up grouped GEMM launch of the largest
    # batch, timed alone (its input rows gathered beforehand, as the layer's
    # row gather does in its own launch)
    Tm = max(batches)
    lo = rank * (cfg.experts // world)
    with torch.cuda.stream(stream):
        x = xs[Tm]
        _, scores, idx = router(x)
        perm = ops.permute(idx, cfg.experts)
        R = Tm * cfg.top_k
        bn = X.tile_policy(Tm, cfg.top_k, cfg.experts, X._max_tile(packed))
        act = torch.empty(R, packed.i_pad, device=dev, dtype=torch.bfloat16)
        if bn >= 64:
            rows_src = dict(b_src=ops.gather_rows(x, perm.perm_src, cfg.top_k, offsets=perm.offsets,
                                                  expert_lo=lo, expert_hi=lo + packed.n_experts))
        else:
            rows_src = dict(b_src=x, b_map=perm.perm_src, b_div=cfg.top_k)

        def gemm():
            ops.expert_gemm(offsets=perm.offsets, expert_begin=lo, n_experts=packed.n_experts, max_rows=R,
                            wfmt=packed.fmt, planes=2, feat_pad=packed.i_pad, n_feat=packed.inter,
                            k_pad=packed.h_k, weight=packed.w1, fp8_block=packed.block,
                            k_valid=cfg.hidden, epilogue=packed.gated_epilogue, bias=packed.b1,
                            alpha=packed.alpha, limit=packed.limit, out=act, token_tile=bn, **rows_src)

        for _ in range(3):
            gemm()
        n_rep, kms = 10, 0.0
        for _ in range(n_rep):
            flush.fill_(1)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            gemm()
            e.record(stream)
            e.synchronize()
            kms += s.elapsed_time(e) / n_rep
    local_rows = int(perm.offsets[rank * (cfg.experts // world) + packed.n_experts]
                     - perm.offsets[rank * (cfg.experts // world)])
    gemm_flops = 2 * local_rows * cfg.hidden * 2 * cfg.inter
    achieved = gemm_flops / (kms / 1e3) / 1e12
    traffic = None
    tfile = ROOT / "profiles" / "traffic.json"
    if tfile.exists():
        traffic = json.loads(tfile.read_text()).get(f"{cfg.name}:gate_up:T{Tm}")
    roofline = {"bound": "tensor", "achieved": round(achieved, 2), "peak": tf_burst,
                "unit": "TFLOP/s", "frac": round(achieved / tf_burst, 4), "traffic": traffic,
                "kernel": f"gate/up grouped GEMM, T={Tm}", "peak_kind": f"{peak_kind} bf16 burst",
                "kernel_ms": round(kms, 4)}

    # ---- end to end through the public modules with host buffers
    # On N GPUs every token crosses the host link once per step: rank r
    # uploads rows [r c, (r + 1) c) of each batch (c = ceil(T / N), the last
    # slice padded), an all-gather over NVLink replicates the tokens the
    # replicated-token layer needs on every rank, and rank r reads back the
    # same rows of the (replicated) output. (Every rank copying whole batches
    # made host memory traffic, not the layer, set the pace from 4 GPUs.)
    chunk = {T: -(-T // world) for T in batches}
    lo_hi = {T: (min(T, rank * chunk[T]), min(T, (rank + 1) * chunk[T])) for T in batches}
    host_x = {T: xs[T][lo_hi[T][0]:lo_hi[T][1]].cpu().pin_memory() for T in batches}
    host_o = {T: torch.empty(lo_hi[T][1] - lo_hi[T][0], cfg.hidden, dtype=torch.bfloat16).pin_memory()
              for T in batches}
    h2d = sum((lo_hi[T][1] - lo_hi[T][0]) * cfg.hidden * 2 for T in batches)
    d2h = h2d

    # Copies run on their own streams: every batch's tokens go host -> device
    # on copy_in up front, each output goes device -> host on copy_out as soon
    # as its layer call ends, so transfers overlap other batches' compute.
    # Device token buffers alternate between two sets, so the next step's
    # uploads overlap this step's compute. Batches run with the largest in
    # the middle: its upload hides behind the batches before it and its
    # download behind those after it; the smallest runs last.
    copy_in, copy_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    # (N GPUs: the all-gather's padded buffer, chunk rows per rank)
    dev_x = [{T: torch.empty(chunk[T] * world, cfg.hidden, dtype=torch.bfloat16, device=dev) for T in batches}
             for _ in range(2)]
    rest = sorted(batches)
    big = rest.pop()
    smallest = rest.pop(0) if rest else None
    second = rest.pop() if rest else None
    order = rest + [big] + ([second] if second is not None else []) + \
        ([smallest] if smallest is not None else [])
    read_done = [None, None]

    def e2e_step(i):
        xs_dev = dev_x[i % 2]
        if read_done[i % 2] is not None:
            copy_in.wait_event(read_done[i % 2])   # the layer calls of step i - 2 have read it
        landed = {}
        with torch.cuda.stream(copy_in):
            for T in order:
                r0, r1 = lo_hi[T]
                if world > 1:
                    mine = xs_dev[T][rank * chunk[T]:(rank + 1) * chunk[T]]
                    if r1 > r0:
                        mine[:r1 - r0].copy_(host_x[T], non_blocking=True)
                else:
                    xs_dev[T].copy_(host_x[T], non_blocking=True)
                landed[T] = torch.cuda.Event()
                landed[T].record(copy_in)
        for T in order:
            stream.wait_event(landed[T])
            with torch.cuda.stream(stream):
                if world > 1:
                    full = xs_dev[T]
                    dist.all_gather_into_tensor(full, full[rank * chunk[T]:(rank + 1) * chunk[T]].clone())
                o = layer_call(cfg, router, packed, xs_dev[T][:T], parallel, rank, world)
            copy_out.wait_stream(stream)
            with torch.cuda.stream(copy_out):
                r0, r1 = lo_hi[T]
                if r1 > r0:
                    host_o[T].copy_(o[r0:r1], non_blocking=True)
                o.record_stream(copy_out)
        done = torch.cuda.Event()
        done.record(stream)
        read_done[i % 2] = done

    for i in range(2):
        e2e_step(i)
    stream.wait_stream(copy_out)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    copy_in.wait_stream(stream)   # the timed region starts before the first copy
    for i in range(args.steps):
        e2e_step(2 + i)
    stream.wait_stream(copy_out)
    e.record(stream)   # after every copy of the last step
    torch.cuda.synchronize(dev)
    e2e_ms = s.elapsed_time(e) / args.steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t[0])
    e2e_value = tokens / (e2e_ms / 1e3)

    w8a8 = None
    if world == 1 and cfg.storage == "fp8" and not args.no_w8a8:
        w8a8 = w8a8_leg(args, cfg, router, packed, xs, flush, stream, dev, hbm, tf_burst)

    stages = stage_breakdown(cfg, router, packed, xs, parallel, rank, world, stream)

    legs = []
    if not args.no_ep_legs:
        for name, mode in EP_LEGS:
            pg = ParallelGroup(world) if (world > 1 and mode == "replicated") else None
            legs.append(ep_leg(args, name, mode, world, rank, dev, stream, flush, pg))
            if pg is not None:
                pg.close()   # its NVLink gather buffers (collective)
            torch.cuda.empty_cache()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, _, sample = cpu_batches(cfg, budget_s=25.0)
        cpu = {"value": round(v, 3), "unit": "tokens/s", "cores": torch.get_num_threads(),
               "kind": "port", "sample": sample}

    launches = args.steps * sum(kernel_launches(T, cfg.top_k, cfg.experts) for T in batches)
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": round(step_ms, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random-init weights, quantised like the checkpoints)",
            "config": workload_config(cfg, world),
            "numerics": numerics_for(world), "routing": "exact (F.linear logits, fused selection)",
            "l2": "flushed (256 MiB write) before every batch",
            "timing": "CUDA graph replay per batch, CUDA events",
            "per_batch": per_batch, "roofline": roofline, "stages_ms": stages,
            "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": launches, "clocks": clocks.summary(), "cpu_baseline": cpu,
        }
        if w8a8 is not None:
            line["w8a8"] = w8a8
        if parity is not None:
            line["parity"] = parity
        if legs:
            line["ep_workloads"] = legs
        print(json.dumps(line), flush=True)
    for g in graphs.values():
        del g
    graphs.clear()
    if world > 1:
        parallel.close()   # NVLink exchange buffers (collective)
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
