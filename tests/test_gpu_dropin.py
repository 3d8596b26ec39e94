"""The modules dropped into Transformers' own MoE blocks, as the reference's
record_qwen3 / record_gpt_oss builders do (moe_serving/qwen3_parallel.py:172-174
swaps ``block.mlp.experts``; gpt_oss_parallel.py:371-372 likewise; the
routers are hooked at qwen3_parallel.py:42-44 and gpt_oss_parallel.py:256-258).

A Transformers 5.5 ``Qwen3MoeSparseMoeBlock`` and ``GptOssMLP`` (tiny
configs) run once with their own router and experts (bf16 weights equal to
the dequantised FP8 / decoded MXFP4 weights), then with ``mlp.gate`` /
``mlp.router`` replaced by this package's router modules and ``mlp.experts``
by its ParallelExperts holding the quantised weights. A forward hook of the
reference's RoutingRecorder kind (it keeps the router's outputs) sees the
same expert indices from both routers, and the block outputs agree within
the BF16 layer tolerance (relative L2 <= 1e-2, max |error| <= 2^-5 max |ref|).
"""

from types import SimpleNamespace

import pytest
import torch

from moe_serving_profile_b200 import _lib, gpt_oss, qwen3
from moe_serving_profile_b200 import synthetic as S
from moe_serving_profile_b200.parallel import ParallelGroup
from moe_serving_profile_b200.router import GptOssRouter, Qwen3Router
from oracle import oracle
from tests.conftest import max_abs, rel_l2

pytestmark = pytest.mark.gpu


class _Recorder:
    """Keeps what a router returns, as RoutingRecorder._hook does."""

    def __init__(self):
        self.calls = []

    def __call__(self, module, inputs, output):
        self.calls.append(tuple(t.detach().clone() for t in output))


def _close(out, ref):
    r, m = rel_l2(out, ref), max_abs(out, ref)
    assert r <= 1e-2 and m <= 2 ** -5 * float(ref.float().abs().max()), (r, m)


def test_qwen3_moe_block_with_b200_modules(cuda):
    from transformers.models.qwen3_moe.configuration_qwen3_moe import Qwen3MoeConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeSparseMoeBlock

    lc = S.CONFIGS["qwen3-tiny"]
    conf = Qwen3MoeConfig(hidden_size=lc.hidden, num_experts=lc.experts, num_experts_per_tok=lc.top_k,
                          moe_intermediate_size=lc.inter, norm_topk_prob=True, hidden_act="silu")
    w = S.make_qwen(lc, seed=21)
    deq = lambda q, s: torch.stack([oracle.dequant_fp8(q[e], s[e], lc.block) for e in range(lc.experts)])
    hf = Qwen3MoeSparseMoeBlock(conf).to(cuda, torch.bfloat16)
    with torch.no_grad():
        hf.gate.weight.copy_(w.router)
        hf.experts.gate_up_proj.copy_(torch.cat([deq(w.gate, w.gate_scale), deq(w.up, w.up_scale)], 1))
        hf.experts.down_proj.copy_(deq(w.down, w.down_scale))
    ours = Qwen3MoeSparseMoeBlock(conf).to(cuda, torch.bfloat16)
    ours.gate = Qwen3Router(conf).to(cuda)
    ours.gate.weight.data = w.router.to(cuda)
    ours.experts = qwen3.ParallelExperts(conf, ParallelGroup(1), "reference")
    for e, mods in enumerate(ours.experts.local):
        mods["gate_proj"] = qwen3.ExpertProjection(w.gate[e].to(cuda), w.gate_scale[e].to(cuda), lc.block)
        mods["up_proj"] = qwen3.ExpertProjection(w.up[e].to(cuda), w.up_scale[e].to(cuda), lc.block)
        mods["down_proj"] = qwen3.ExpertProjection(w.down[e].to(cuda), w.down_scale[e].to(cuda), lc.block)
    rec_hf, rec_ours = _Recorder(), _Recorder()
    hf.gate.register_forward_hook(rec_hf)
    ours.gate.register_forward_hook(rec_ours)
    x = S.make_hidden(2 * 32, lc.hidden, seed=22).view(2, 32, lc.hidden).to(cuda)
    with torch.inference_mode():
        ref = hf(x)
        out = ours(x)
    assert out.shape == ref.shape and out.dtype == torch.bfloat16
    (p0, s0, i0), (p1, s1, i1) = rec_hf.calls[0], rec_ours.calls[0]
    assert torch.equal(i0, i1) and torch.equal(s0, s1) and torch.equal(p0, p1)
    _close(out.reshape(-1, lc.hidden), ref.reshape(-1, lc.hidden))
    assert _lib.device_status(cuda.index) == 0


def test_gpt_oss_mlp_with_b200_modules(cuda):
    from transformers.models.gpt_oss.configuration_gpt_oss import GptOssConfig
    from transformers.models.gpt_oss.modeling_gpt_oss import GptOssMLP

    lc = S.LayerConfig("gpt-oss-probe", "gpt_oss", 256, 8, 2, 256, "mxfp4", (64,), norm_topk=False)
    conf = GptOssConfig(hidden_size=lc.hidden, intermediate_size=lc.inter, num_local_experts=lc.experts,
                        num_experts_per_tok=lc.top_k, num_hidden_layers=1)
    w = S.make_gpt_oss(lc, seed=23)
    dec = lambda b, s: torch.stack([oracle.decode_mxfp4(b[e], s[e]) for e in range(lc.experts)])
    hf = GptOssMLP(conf).to(cuda, torch.bfloat16)
    with torch.no_grad():
        hf.router.weight.copy_(w.router)
        hf.router.bias.copy_(w.router_bias)
        hf.experts.gate_up_proj.copy_(dec(w.gu_blocks, w.gu_scales).transpose(1, 2))
        hf.experts.gate_up_proj_bias.copy_(w.gu_bias)
        hf.experts.down_proj.copy_(dec(w.dn_blocks, w.dn_scales).transpose(1, 2))
        hf.experts.down_proj_bias.copy_(w.dn_bias)
    ours = GptOssMLP(conf).to(cuda, torch.bfloat16)
    ours.router = GptOssRouter(conf).to(cuda)
    ours.router.weight.data = w.router.to(cuda)
    ours.router.bias.data = w.router_bias.to(cuda)
    ours.experts = gpt_oss.ParallelExperts(SimpleNamespace(num_local_experts=lc.experts,
                                                           swiglu_alpha=lc.alpha, swiglu_limit=lc.limit),
                                           ParallelGroup(1), "mxfp4", "reference")
    for name, t in (("gate_up_proj_blocks", w.gu_blocks), ("gate_up_proj_scales", w.gu_scales),
                    ("gate_up_proj_bias", w.gu_bias), ("down_proj_blocks", w.dn_blocks),
                    ("down_proj_scales", w.dn_scales), ("down_proj_bias", w.dn_bias)):
        ours.experts.register_buffer(name, t.to(cuda))
    rec_hf, rec_ours = _Recorder(), _Recorder()
    hf.router.register_forward_hook(rec_hf)
    ours.router.register_forward_hook(rec_ours)
    x = S.make_hidden(2 * 32, lc.hidden, seed=24).view(2, 32, lc.hidden).to(cuda)
    with torch.inference_mode():
        ref, ref_scores = hf(x)
        out, scores = ours(x)
    (l0, s0, i0), (l1, s1, i1) = rec_hf.calls[0], rec_ours.calls[0]
    assert torch.equal(i0, i1) and torch.equal(s0, s1)
    assert torch.equal(scores, ref_scores)
    _close(out.reshape(-1, lc.hidden), ref.reshape(-1, lc.hidden))
    assert _lib.device_status(cuda.index) == 0


def test_safetensors_checkpoint_through_the_kernels(cuda, tmp_path):
    """Experts read straight from a safetensors checkpoint onto the GPU
    (loader.qwen3_fp8_experts / gpt_oss_mxfp4_experts, the loading path of
    qwen3_parallel.py:180-242 and gpt_oss_parallel.py:394-452) give the layer
    output of the same weights packed from the modules, bit for bit, and the
    oracle's within the BF16 layer tolerance."""
    from safetensors.torch import save_file

    from moe_serving_profile_b200 import experts as X
    from moe_serving_profile_b200 import layout, loader

    lc = S.CONFIGS["qwen3-tiny"]
    w = S.make_qwen(lc, seed=31)
    tensors = {}
    for e in range(lc.experts):
        for proj, wt, sc in (("gate_proj", w.gate, w.gate_scale), ("up_proj", w.up, w.up_scale),
                             ("down_proj", w.down, w.down_scale)):
            name = f"model.layers.5.mlp.experts.{e}.{proj}"
            tensors[name + ".weight"] = wt[e].contiguous()
            tensors[name + ".weight_scale_inv"] = sc[e].contiguous()
    save_file(tensors, str(tmp_path / "model.safetensors"))
    got = loader.qwen3_fp8_experts(tmp_path, layer=5, start=0, count=lc.experts, block=lc.block, device=cuda)
    want = layout.fp8_experts(w.gate.to(cuda), w.gate_scale.to(cuda), w.up.to(cuda), w.up_scale.to(cuda),
                              w.down.to(cuda), w.down_scale.to(cuda), lc.block)
    x = S.make_hidden(64, lc.hidden, seed=32)
    _, scores, idx, _ = oracle.qwen_router(x, w.router, lc.top_k, True)
    args = (x.to(cuda), idx.to(cuda), scores.to(cuda))
    out = X.layer_forward(got, *args, num_experts=lc.experts, expert_begin=0)
    assert torch.equal(out, X.layer_forward(want, *args, num_experts=lc.experts, expert_begin=0))
    ref = oracle.qwen_layer(x, idx, scores, w.gate, w.gate_scale, w.up, w.up_scale, w.down, w.down_scale,
                            lc.block)
    _close(out.cpu(), ref)

    gc = S.LayerConfig("gpt-oss-probe", "gpt_oss", 256, 8, 2, 256, "mxfp4", (64,), norm_topk=False)
    wg = S.make_gpt_oss(gc, seed=33)
    p = "model.layers.0.mlp.experts."
    save_file({p + "gate_up_proj_blocks": wg.gu_blocks.contiguous(), p + "gate_up_proj_scales": wg.gu_scales,
               p + "gate_up_proj_bias": wg.gu_bias, p + "down_proj_blocks": wg.dn_blocks.contiguous(),
               p + "down_proj_scales": wg.dn_scales, p + "down_proj_bias": wg.dn_bias},
              str(tmp_path / "gpt.safetensors"))
    (tmp_path / "gpt").mkdir()
    (tmp_path / "gpt.safetensors").rename(tmp_path / "gpt" / "model.safetensors")
    got = loader.gpt_oss_mxfp4_experts(tmp_path / "gpt", layer=0, start=0, count=gc.experts, device=cuda)
    want = layout.gpt_oss_mxfp4_experts(*(t.to(cuda) for t in (wg.gu_blocks, wg.gu_scales, wg.gu_bias,
                                                                 wg.dn_blocks, wg.dn_scales, wg.dn_bias)),
                                        gc.alpha, gc.limit)
    xg = S.make_hidden(64, gc.hidden, seed=34)
    _, sg, ig = oracle.gpt_oss_router(xg, wg.router, wg.router_bias, gc.top_k)
    argsg = (xg.to(cuda), ig.to(cuda), sg.to(cuda))
    outg = X.layer_forward(got, *argsg, num_experts=gc.experts, expert_begin=0)
    assert torch.equal(outg, X.layer_forward(want, *argsg, num_experts=gc.experts, expert_begin=0))
    refg = oracle.gpt_oss_layer(xg, ig, sg, wg.gu_blocks, wg.gu_scales, wg.gu_bias, wg.dn_blocks, wg.dn_scales,
                                wg.dn_bias, gc.alpha, gc.limit)
    _close(outg.cpu(), refg)
    assert _lib.device_status(cuda.index) == 0
