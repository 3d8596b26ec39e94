"""Generate golden fixtures by running the reference's own modules on CPU.

Run in a container where the reference project (moe_serving) is importable:

    python tests/golden/make_golden.py /path/to/MoE_Serving_Profile

Inputs are regenerated from seeds by moe_serving_profile_b200.synthetic, so a
fixture stores only the seed, a checksum of the inputs and the reference's
outputs:
  * routers: transformers' Qwen3MoeTopKRouter / GptOssTopKRouter (the
    reference hooks these; transformers 5.5.0 stands in for the pinned 5.20.0
    tree, which is not vendored) and moe_serving.moe.route;
  * expert layers: moe_serving.qwen3_parallel.ParallelExperts and
    moe_serving.gpt_oss_parallel.ParallelExperts with ParallelGroup(1) in
    "reference" and "fast" numerics;
  * the reference's ordering contract: per-expert (slot, token) row lists of
    parallel_numerics.ordered_expert_merge and each contribution row;
  * moe_serving.moe.simulate_ranks over two in-process ranks (token
    all-to-all) with bf16 experts.
The fixtures are small (.pt, tens of KB each).
"""

from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path
from types import SimpleNamespace

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from moe_serving_profile_b200 import synthetic as S  # noqa: E402

# Small configs used by the fixtures (name -> LayerConfig, tokens, seed).
QWEN_CASES = {
    "qwen3_tiny": (S.CONFIGS["qwen3-tiny"], 64, 0),
    # non-128 block scales and sizes that do not fill a tile, as the
    # reference's own qwen3 worker fixture (16x16 blocks, H=32, I=24)
    "qwen3_block16": (S.LayerConfig("qwen3-block16", "qwen3", 32, 4, 2, 24, "fp8", (13,),
                                    block=(16, 16)), 13, 1),
}
GPT_CASES = {
    "gpt_oss_small": (S.LayerConfig("gpt-oss-small", "gpt_oss", 256, 4, 2, 256, "mxfp4", (16,),
                                    norm_topk=False), 16, 2),
    "gpt_oss_tiny": (S.LayerConfig("gpt-oss-tiny", "gpt_oss", 32, 4, 2, 32, "mxfp4", (7,),
                                   norm_topk=False), 7, 3),
}


def checksum(*tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        t = t.detach().cpu().contiguous()
        h.update(t.view(torch.uint8).numpy().tobytes() if t.dtype != torch.bool else t.numpy().tobytes())
    return h.hexdigest()


def qwen_inputs(cfg, T, seed):
    w = S.make_qwen(cfg, seed)
    x = S.make_hidden(T, cfg.hidden, seed + 100)
    return w, x


def gpt_inputs(cfg, T, seed):
    w = S.make_gpt_oss(cfg, seed)
    x = S.make_hidden(T, cfg.hidden, seed + 100)
    return w, x


def order_rows(indices):
    """(expert, slots, tokens) of parallel_numerics.py:21-23."""
    rows = []
    for expert in torch.unique(indices, sorted=True).tolist():
        slots, tokens = torch.where(indices.T == expert)
        rows.append((expert, slots, tokens))
    return rows


def gen_qwen(name, cfg, T, seed, ref):
    from transformers import Qwen3MoeConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeTopKRouter

    w, x = qwen_inputs(cfg, T, seed)
    hf = Qwen3MoeConfig(hidden_size=cfg.hidden, num_experts=cfg.experts, num_experts_per_tok=cfg.top_k,
                        moe_intermediate_size=cfg.inter, norm_topk_prob=cfg.norm_topk)
    router = Qwen3MoeTopKRouter(hf)
    router.weight.data = w.router.clone()
    with torch.no_grad():
        probs, scores, indices = router(x)
        logits = torch.nn.functional.linear(x, w.router)
    out = {"probs": probs, "scores": scores, "indices": indices, "logits": logits}
    conf = SimpleNamespace(num_experts=cfg.experts, hidden_act="silu")
    for numerics in ("reference", "fast"):
        experts = ref.qwen3.ParallelExperts(conf, ref.ParallelGroup(1), numerics=numerics)
        for e, mods in enumerate(experts.local):
            mods["gate_proj"] = ref.qwen3.ExpertProjection(w.gate[e], w.gate_scale[e], cfg.block)
            mods["up_proj"] = ref.qwen3.ExpertProjection(w.up[e], w.up_scale[e], cfg.block)
            mods["down_proj"] = ref.qwen3.ExpertProjection(w.down[e], w.down_scale[e], cfg.block)
        with torch.no_grad():
            out[f"out_{numerics}"] = experts(x, indices, scores)
            if numerics == "reference":
                contrib, perm = [], []
                for expert, slots, tokens in order_rows(indices):
                    values = experts.project(expert, x[tokens])
                    contrib.append((values * scores[tokens, slots, None]).to(x.dtype))
                    perm.append(tokens * cfg.top_k + slots)
                out["contrib"] = torch.cat(contrib)
                out["perm_src"] = torch.cat(perm).to(torch.int32)
                out["dequant_gate0"] = ref.qwen3.dequantize_blocks(w.gate[0], w.gate_scale[0], cfg.block,
                                                                  torch.bfloat16)[:, :64].clone()
    bias_out = None
    if cfg.zipf_bias:
        bias_out = w.router_bias
    torch.save({"kind": "qwen3", "config": cfg.__dict__, "tokens": T, "seed": seed,
                "input_sha": checksum(x, w.router, w.gate, w.gate_scale, w.up, w.down),
                "router_bias": bias_out, **out}, HERE / f"{name}.pt")


def gen_gpt(name, cfg, T, seed, ref):
    from transformers import GptOssConfig
    from transformers.models.gpt_oss.modeling_gpt_oss import GptOssTopKRouter

    w, x = gpt_inputs(cfg, T, seed)
    hf = GptOssConfig(hidden_size=cfg.hidden, num_local_experts=cfg.experts,
                      num_experts_per_tok=cfg.top_k, intermediate_size=cfg.inter)
    router = GptOssTopKRouter(hf)
    router.weight.data = w.router.clone()
    router.bias.data = w.router_bias.clone()
    with torch.no_grad():
        logits, scores, indices = router(x)
    out = {"logits": logits, "scores": scores, "indices": indices}
    conf = SimpleNamespace(num_local_experts=cfg.experts, swiglu_alpha=cfg.alpha, swiglu_limit=cfg.limit)
    for numerics in ("reference", "fast"):
        experts = ref.gpt.ParallelExperts(conf, ref.ParallelGroup(1), storage="mxfp4", numerics=numerics)
        experts.register_buffer("gate_up_proj_blocks", w.gu_blocks.clone())
        experts.register_buffer("gate_up_proj_scales", w.gu_scales.clone())
        experts.register_buffer("gate_up_proj_bias", w.gu_bias.clone())
        experts.register_buffer("down_proj_blocks", w.dn_blocks.clone())
        experts.register_buffer("down_proj_scales", w.dn_scales.clone())
        experts.register_buffer("down_proj_bias", w.dn_bias.clone())
        with torch.no_grad():
            out[f"out_{numerics}"] = experts(x, indices, scores)
            if numerics == "reference":
                contrib, perm = [], []
                for expert, slots, tokens in order_rows(indices):
                    values = experts.project(expert, x[tokens])
                    contrib.append((values * scores[tokens, slots, None]).to(x.dtype))
                    perm.append(tokens * cfg.top_k + slots)
                out["contrib"] = torch.cat(contrib)
                out["perm_src"] = torch.cat(perm).to(torch.int32)
                out["decoded_gate_up0"] = experts.projection("gate_up_proj", 0, torch.bfloat16)[:, :64].clone()
    torch.save({"kind": "gpt_oss", "config": cfg.__dict__, "tokens": T, "seed": seed,
                "input_sha": checksum(x, w.router, w.router_bias, w.gu_blocks, w.gu_scales, w.dn_blocks),
                **out}, HERE / f"{name}.pt")


def gen_native(ref):
    """moe.route + simulate_ranks (two ranks, 3 + 4 tokens, bf16 experts)."""
    g = torch.Generator().manual_seed(4)
    E, H, I, K = 8, 64, 32, 2
    gate_up = (torch.randn(E, 2 * I, H, generator=g) * 0.1).to(torch.bfloat16)
    down = (torch.randn(E, H, I, generator=g) * 0.1).to(torch.bfloat16)
    gate = (torch.randn(E, H, generator=g) * 0.1).to(torch.bfloat16)
    tokens = torch.randn(7, H, generator=g).to(torch.bfloat16)
    banks = [ref.moe.LocalSwiGLUExperts(gate_up[:4], down[:4]),
             ref.moe.LocalSwiGLUExperts(gate_up[4:], down[4:])]
    with torch.no_grad():
        index, weight = ref.moe.route(tokens, gate, K, True)
        left, right = ref.moe.simulate_ranks([tokens[:3], tokens[3:]], gate, banks, K)
    torch.save({"kind": "native", "gate_up": gate_up, "down": down, "gate": gate, "tokens": tokens,
                "top_k": K, "index": index, "weight": weight, "rank_outputs": [left, right]},
               HERE / "native_a2a.pt")


def main(reference_root: str) -> None:
    sys.path.insert(0, reference_root)
    from moe_serving import gpt_oss_parallel, moe, qwen3_parallel

    ref = SimpleNamespace(qwen3=qwen3_parallel, gpt=gpt_oss_parallel, moe=moe,
                          ParallelGroup=gpt_oss_parallel.ParallelGroup)
    torch.set_num_threads(1)
    for name, (cfg, T, seed) in QWEN_CASES.items():
        gen_qwen(name, cfg, T, seed, ref)
    for name, (cfg, T, seed) in GPT_CASES.items():
        gen_gpt(name, cfg, T, seed, ref)
    gen_native(ref)
    for p in sorted(HERE.glob("*.pt")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MOE_SERVING_REFERENCE")
    if not root:
        sys.exit("usage: make_golden.py <reference checkout> (or set MOE_SERVING_REFERENCE)")
    main(root)
