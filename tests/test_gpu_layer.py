"""Whole expert layer on the GPU through the reference-compatible modules.

Tolerance (BF16 expert outputs; the reference's torch GEMMs and our tcgen05
GEMMs differ only in fp32 summation order, so intermediate bf16 roundings
may differ by one ulp): relative L2 error <= 1e-2 and max |error| <=
2^-5 * max |reference|. Routing (indices) must be identical wherever the
reference's own top-k has no tie.
"""

from types import SimpleNamespace

import pytest
import torch

from moe_serving_profile_b200 import _lib, gpt_oss, qwen3
from moe_serving_profile_b200 import synthetic as S
from moe_serving_profile_b200.parallel import ParallelGroup
from moe_serving_profile_b200.router import GptOssRouter, Qwen3Router
from oracle import oracle
from tests.conftest import load_golden, max_abs, rel_l2, tie_free_rows
from tests.golden.make_golden import GPT_CASES, QWEN_CASES, gpt_inputs, qwen_inputs

pytestmark = pytest.mark.gpu

REL_L2 = 1e-2
MAX_ABS_FRAC = 2 ** -5


def assert_close_bf16(out, ref, what=""):
    r, m = rel_l2(out, ref), max_abs(out, ref)
    bound = MAX_ABS_FRAC * float(ref.float().abs().max())
    print(f"\n{what}: rel_l2={r:.2e} max_abs={m:.2e} (bound {bound:.2e})")
    assert out.isfinite().all()
    assert r <= REL_L2 and m <= bound, (what, r, m)


def qwen_module(cfg, w, dev, numerics="reference"):
    conf = SimpleNamespace(num_experts=cfg.experts, hidden_act="silu")
    m = qwen3.ParallelExperts(conf, ParallelGroup(1), numerics)
    for e, mods in enumerate(m.local):
        mods["gate_proj"] = qwen3.ExpertProjection(w.gate[e].to(dev), w.gate_scale[e].to(dev), cfg.block)
        mods["up_proj"] = qwen3.ExpertProjection(w.up[e].to(dev), w.up_scale[e].to(dev), cfg.block)
        mods["down_proj"] = qwen3.ExpertProjection(w.down[e].to(dev), w.down_scale[e].to(dev), cfg.block)
    return m


def gpt_module(cfg, w, dev, numerics="reference"):
    conf = SimpleNamespace(num_local_experts=cfg.experts, swiglu_alpha=cfg.alpha, swiglu_limit=cfg.limit)
    m = gpt_oss.ParallelExperts(conf, ParallelGroup(1), "mxfp4", numerics)
    for name, t in (("gate_up_proj_blocks", w.gu_blocks), ("gate_up_proj_scales", w.gu_scales),
                    ("gate_up_proj_bias", w.gu_bias), ("down_proj_blocks", w.dn_blocks),
                    ("down_proj_scales", w.dn_scales), ("down_proj_bias", w.dn_bias)):
        m.register_buffer(name, t.to(dev))
    return m


@pytest.mark.parametrize("name", list(QWEN_CASES))
def test_qwen_golden(cuda, name):
    cfg, T, seed = QWEN_CASES[name]
    g = load_golden(name)
    w, x = qwen_inputs(cfg, T, seed)
    router = Qwen3Router(SimpleNamespace(num_experts_per_tok=cfg.top_k, num_experts=cfg.experts,
                                         norm_topk_prob=cfg.norm_topk, hidden_size=cfg.hidden)).to(cuda)
    router.weight.data = w.router.to(cuda)
    probs, scores, idx = router(x.to(cuda))
    free = tie_free_rows(g["probs"], cfg.top_k)
    assert torch.equal(idx.cpu()[free], g["indices"][free])
    assert torch.allclose(scores.cpu(), g["scores"], rtol=1e-5, atol=1e-6)
    m = qwen_module(cfg, w, cuda)
    out = m(x.to(cuda), g["indices"].to(cuda), g["scores"].to(cuda))
    assert_close_bf16(out, g["out_reference"], name)
    assert _lib.device_status(cuda.index) == 0


@pytest.mark.parametrize("name", list(GPT_CASES))
def test_gpt_oss_golden(cuda, name):
    cfg, T, seed = GPT_CASES[name]
    g = load_golden(name)
    w, x = gpt_inputs(cfg, T, seed)
    router = GptOssRouter(SimpleNamespace(num_experts_per_tok=cfg.top_k, num_local_experts=cfg.experts,
                                          hidden_size=cfg.hidden)).to(cuda)
    router.weight.data = w.router.to(cuda)
    router.bias.data = w.router_bias.to(cuda)
    logits, scores, idx = router(x.to(cuda))
    free = tie_free_rows(g["logits"], cfg.top_k)
    assert torch.equal(idx.cpu()[free], g["indices"][free])
    m = gpt_module(cfg, w, cuda)
    out = m(x.to(cuda), g["indices"].to(cuda), g["scores"].to(cuda))
    assert_close_bf16(out, g["out_reference"], name)
    assert _lib.device_status(cuda.index) == 0


def _qwen_ref(w, x, idx, scores, cfg, device):
    mv = lambda t: t.to(device)
    return oracle.qwen_layer(x.to(device), idx.to(device), scores.to(device), mv(w.gate), mv(w.gate_scale),
                             mv(w.up), mv(w.up_scale), mv(w.down), mv(w.down_scale), cfg.block)


@pytest.mark.parametrize("T", [1, 8, 64, 512, 4096])
def test_qwen3_30b_layer(cuda, T):
    cfg = S.CONFIGS["qwen3-30b-a3b"]
    w = S.make_qwen(cfg, seed=1, device=cuda)
    x = S.make_hidden(T, cfg.hidden, seed=T, device=cuda)
    router = Qwen3Router(SimpleNamespace(num_experts_per_tok=cfg.top_k, num_experts=cfg.experts,
                                         norm_topk_prob=True, hidden_size=cfg.hidden)).to(cuda)
    router.weight.data = w.router
    _, scores, idx = router(x)
    m = qwen_module(cfg, w, cuda)
    out = m(x, idx, scores)
    # small batches against the CPU oracle, large ones against the same torch
    # restatement executed on the GPU
    dev = "cpu" if T <= 64 else cuda
    ref = _qwen_ref(w, x, idx, scores, cfg, dev)
    assert_close_bf16(out, ref, f"qwen3-30b T={T}")
    again = m(x, idx, scores)
    assert torch.equal(out, again)                       # deterministic
    assert _lib.device_status(cuda.index) == 0


@pytest.mark.parametrize("T", [1, 16, 64, 2048])
def test_gpt_oss_20b_layer(cuda, T):
    cfg = S.CONFIGS["gpt-oss-20b"]
    w = S.make_gpt_oss(cfg, seed=2, device=cuda)
    x = S.make_hidden(T, cfg.hidden, seed=T, device=cuda)
    router = GptOssRouter(SimpleNamespace(num_experts_per_tok=cfg.top_k, num_local_experts=cfg.experts,
                                          hidden_size=cfg.hidden)).to(cuda)
    router.weight.data = w.router
    router.bias.data = w.router_bias
    _, scores, idx = router(x)
    m = gpt_module(cfg, w, cuda)
    out = m(x, idx, scores)
    dev = "cpu" if T <= 16 else cuda
    ref = oracle.gpt_oss_layer(x.to(dev), idx.to(dev), scores.to(dev), w.gu_blocks.to(dev),
                               w.gu_scales.to(dev), w.gu_bias.to(dev), w.dn_blocks.to(dev),
                               w.dn_scales.to(dev), w.dn_bias.to(dev), cfg.alpha, cfg.limit)
    assert_close_bf16(out, ref, f"gpt-oss-20b T={T}")
    assert _lib.device_status(cuda.index) == 0


def test_qwen3_235b_skewed_layer(cuda):
    cfg = S.CONFIGS["qwen3-235b-a22b"]
    T = 256
    w = S.make_qwen(cfg, seed=3, device=cuda)
    x = S.make_hidden(T, cfg.hidden, seed=9, device=cuda)
    router = Qwen3Router(SimpleNamespace(num_experts_per_tok=cfg.top_k, num_experts=cfg.experts,
                                         norm_topk_prob=True, hidden_size=cfg.hidden)).to(cuda)
    router.weight.data = w.router
    router.bias = w.router_bias
    _, scores, idx = router(x)
    cv = S.expert_load_cv(router.last_counts)
    print(f"\nqwen3-235b T={T}: expert_load_cv={cv:.3f}")
    # the skew the workload names: expert_load_cv ~ 0.5 (seeded CPU draws of
    # this shape give 0.49-0.57; the band leaves room for sampling noise)
    assert 0.35 < cv < 0.75
    m = qwen_module(cfg, w, cuda)
    out = m(x, idx, scores)
    ref = _qwen_ref(w, x, idx, scores, cfg, cuda)
    assert_close_bf16(out, ref, "qwen3-235b T=256")


def test_expert_parallel_split_is_bitwise_invariant(cuda):
    """Running the experts as 4 rank-local ranges (zero-filled contribution
    rows, summed) and combining equals the single-range result bit for bit:
    the replicated-token EP contract of parallel_numerics.ordered_expert_merge."""
    from moe_serving_profile_b200 import experts as X
    from moe_serving_profile_b200 import layout, ops
    cfg = S.CONFIGS["qwen3-30b-a3b"]
    T = 64
    w = S.make_qwen(cfg, seed=4, device=cuda)
    x = S.make_hidden(T, cfg.hidden, seed=5, device=cuda)
    probs, scores, idx, _ = oracle.qwen_router(x, w.router, cfg.top_k, True)
    full = layout.fp8_experts(w.gate, w.gate_scale, w.up, w.up_scale, w.down, w.down_scale, cfg.block)
    base = X.layer_forward(full, x, idx, scores, num_experts=cfg.experts, expert_begin=0)
    perm = ops.permute(idx, cfg.experts)
    contrib = torch.zeros(T * cfg.top_k, cfg.hidden, dtype=torch.bfloat16, device=cuda)
    ep, epr = 4, cfg.experts // 4
    for r in range(ep):
        sl = slice(r * epr, (r + 1) * epr)
        part = layout.fp8_experts(w.gate[sl], w.gate_scale[sl], w.up[sl], w.up_scale[sl], w.down[sl],
                                  w.down_scale[sl], cfg.block)
        c = torch.zeros_like(contrib)
        X.run_experts(part, x, perm, scores, K=cfg.top_k, num_experts=cfg.experts, expert_begin=r * epr,
                      contrib=c)
        contrib += c
    out = ops.combine(contrib, perm.inverse, idx, order=_lib.ORDER_EXPERT)
    assert torch.equal(out, base)


@pytest.mark.parametrize("name,T", [("qwen3-30b-a3b", 1), ("qwen3-30b-a3b", 64), ("qwen3-30b-a3b", 512),
                                    ("qwen3-30b-a3b", 4096), ("gpt-oss-20b", 16), ("gpt-oss-20b", 2048),
                                    ("qwen3-30b-a3b-bf16", 512)])
def test_expert_layer_one_call_equals_separate_calls(cuda, name, T):
    """b200moe_expert_layer (one C-ABI call: permutation, gather, both
    GEMMs, ordered combine) against the same kernels called one by one:
    bit for bit."""
    from moe_serving_profile_b200 import experts as X
    from moe_serving_profile_b200 import layout, ops
    bf16 = name.endswith("-bf16")
    cfg = S.CONFIGS[name.removesuffix("-bf16")]
    if cfg.family == "qwen3":
        w = S.make_qwen(cfg, seed=3, device=cuda)
        if bf16:
            def dq(q, s):
                E = q.shape[0]
                return torch.stack([oracle.dequant_fp8(q[e].cpu(), s[e].cpu(), cfg.block) for e in range(E)]).to(cuda)
            packed = layout.bf16_experts(dq(w.gate, w.gate_scale), dq(w.up, w.up_scale), dq(w.down, w.down_scale))
        else:
            packed = layout.fp8_experts(w.gate, w.gate_scale, w.up, w.up_scale, w.down, w.down_scale, cfg.block)
        router = w.router
    else:
        w = S.make_gpt_oss(cfg, seed=3, device=cuda)
        packed = layout.gpt_oss_mxfp4_experts(w.gu_blocks, w.gu_scales, w.gu_bias, w.dn_blocks, w.dn_scales,
                                              w.dn_bias, cfg.alpha, cfg.limit)
        router = w.router
    x = S.make_hidden(T, cfg.hidden, seed=11 + T, device=cuda)
    scores, idx = torch.topk(torch.softmax(torch.nn.functional.linear(x, router).float(), -1), cfg.top_k, -1)
    if cfg.family == "gpt_oss":
        scores = scores.bfloat16()
    one = ops.expert_layer(packed, x, idx, scores.contiguous(), num_experts=cfg.experts)
    perm = ops.permute(idx, cfg.experts)
    contrib = X.run_experts(packed, x, perm, scores.contiguous(), K=cfg.top_k, num_experts=cfg.experts,
                            expert_begin=0)
    sep = ops.combine(contrib, perm.inverse, idx, order=_lib.ORDER_EXPERT)
    assert torch.equal(one, sep)
    assert _lib.device_status(cuda.index) == 0


@pytest.mark.parametrize("T", [16, 2048])
def test_gpt_oss_efficient_layer_keeps_fp32_intermediates(cuda, T):
    """numerics="efficient" for GPT-OSS MXFP4 (the reference's fused
    grouped_mxfp4 path): fp32 gate/up epilogue with fp32 biases and one bf16
    rounding of the intermediate, fp32 down + bias, each slot's row scaled
    and rounded to bf16, fp32 slot-order reduce. Against the float64
    restatement of that algorithm
    (oracle.gpt_oss_layer_efficient): only fp32 summation order differs, so
    relative L2 <= 2e-3 and max |error| <= 2^-6 max |ref|."""
    cfg = S.CONFIGS["gpt-oss-20b"]
    w = S.make_gpt_oss(cfg, seed=41)
    x = S.make_hidden(T, cfg.hidden, seed=42 + T)
    _, scores, idx = oracle.gpt_oss_router(x, w.router, w.router_bias, cfg.top_k)
    m = gpt_module(cfg, w, cuda, "efficient")
    out = m(x.to(cuda), idx.to(cuda), scores.to(cuda)).cpu()
    ref = oracle.gpt_oss_layer_efficient(x, idx, scores, w.gu_blocks, w.gu_scales, w.gu_bias, w.dn_blocks,
                                         w.dn_scales, w.dn_bias, cfg.alpha, cfg.limit)
    r, mx = rel_l2(out, ref), max_abs(out, ref)
    print(f"\ngpt-oss-20b efficient T={T}: rel_l2={r:.2e} max_abs={mx:.2e}")
    assert out.isfinite().all()
    assert r <= 2e-3 and mx <= 2 ** -6 * float(ref.float().abs().max())
    assert _lib.device_status(cuda.index) == 0


def test_fp32_down_epilogue_and_slot_order_combine_exact(cuda):
    """EPI_DOWN_F32 writes acc + bias unrounded and b200moe_combine_f32 sums
    bf16(w * row) over a token's slots in fp32: with integer data, integer
    biases and power-of-two weights the GEMM and every product are exact, the
    bf16 roundings are those of the exact products, and the fp32 sum of two
    of them is exact, so both are bit-exact."""
    from moe_serving_profile_b200 import layout, ops
    g = torch.Generator().manual_seed(5)
    E, H, I, T, K = 4, 256, 192, 40, 2
    wv = torch.randint(-4, 5, (E, H, I), generator=g).bfloat16()
    bias = torch.randint(-8, 9, (E, H), generator=g).bfloat16()
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).long()
    wts = torch.pow(2.0, torch.randint(-3, 2, (T, K), generator=g).float())
    counts, offsets, perm, inv = oracle.permute(idx, E)
    R = T * K
    act = torch.zeros(R, 256, dtype=torch.bfloat16)
    act[:, :I] = torch.randint(-3, 4, (R, I), generator=g).bfloat16()
    w2 = torch.zeros(E, 256, 256, dtype=torch.bfloat16)
    w2[:, :H, :I] = wv
    b2 = torch.zeros(E, 256, dtype=torch.bfloat16)
    b2[:, :H] = bias
    y = torch.zeros(R, H, dtype=torch.float32, device=cuda)
    ops.expert_gemm(offsets=offsets.to(cuda), expert_begin=0, n_experts=E, max_rows=R, wfmt=_lib.W_BF16,
                    planes=1, feat_pad=256, n_feat=H, k_pad=256, weight=w2.to(cuda), b_src=act.to(cuda),
                    k_valid=I, epilogue=_lib.EPI_DOWN_F32, bias=b2.to(cuda), out=y)
    e_of_row = torch.repeat_interleave(torch.arange(E), counts.long())
    exact = torch.einsum("ri,rhi->rh", act[:, :I].double(), wv.double()[e_of_row]) + bias.double()[e_of_row]
    assert torch.equal(y.cpu(), exact.float())
    out = ops.combine_f32(y, inv.to(cuda), idx.to(cuda), wts.to(cuda))
    want = (exact[inv.long()].view(T, K, H) * wts.double()[..., None]).to(torch.bfloat16).double().sum(1)
    assert torch.equal(out.cpu(), want.to(torch.bfloat16))
    assert _lib.device_status(cuda.index) == 0
