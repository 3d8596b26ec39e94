"""Pin the CPU oracle to the reference: fixtures in tests/golden were produced
by the reference's own modules (tests/golden/make_golden.py). CPU only."""

import pytest
import torch

from tests.conftest import GOLDEN, load_golden, tie_free_rows
from moe_serving_profile_b200 import synthetic as S
from oracle import oracle
from tests.golden.make_golden import GPT_CASES, QWEN_CASES, checksum, gpt_inputs, qwen_inputs


@pytest.mark.parametrize("name", list(QWEN_CASES))
def test_qwen_oracle_matches_reference(name):
    cfg, T, seed = QWEN_CASES[name]
    g = load_golden(name)
    w, x = qwen_inputs(cfg, T, seed)
    assert checksum(x, w.router, w.gate, w.gate_scale, w.up, w.down) == g["input_sha"]

    probs, scores, indices, logits = oracle.qwen_router(x, w.router, cfg.top_k, cfg.norm_topk)
    assert torch.equal(probs, g["probs"]) and torch.equal(scores, g["scores"])
    assert torch.equal(indices, g["indices"]) and torch.equal(logits, g["logits"])

    # fixed-order logits of the kernels: within one bf16 ulp of torch's GEMM
    fixed = oracle.router_logits(x, w.router, None, 0)
    diff = (fixed - g["logits"].float()).abs()
    ulp = g["logits"].float().abs().clamp_min(2 ** -126) * 2 ** -7
    assert bool((diff <= ulp).all())

    # selection: value-descending, lower-id-first top-k equals torch.topk on tie-free rows
    sel = oracle.topk(g["probs"], cfg.top_k)
    free = tie_free_rows(g["probs"], cfg.top_k)
    assert torch.equal(sel[free], g["indices"][free])

    # permutation in the reference's (expert, slot, token) order
    counts, offsets, perm, inv = oracle.permute(g["indices"], cfg.experts)
    assert torch.equal(perm, g["perm_src"])
    assert torch.equal(counts, torch.bincount(g["indices"].flatten(), minlength=cfg.experts).int())
    assert torch.equal(inv[perm.long()], torch.arange(perm.numel(), dtype=torch.int32))

    # ordered combine of the reference's own contribution rows is bit-exact
    out = oracle.combine(g["contrib"], inv, g["indices"])
    assert torch.equal(out, g["out_reference"])

    # FP8 block dequantisation, bit-exact
    deq = oracle.dequant_fp8(w.gate[0], w.gate_scale[0], cfg.block)
    assert torch.equal(deq[:, :64], g["dequant_gate0"])

    # whole layer through the torch restatement, bit-exact on CPU
    layer = oracle.qwen_layer(x, g["indices"], g["scores"], w.gate, w.gate_scale, w.up, w.up_scale,
                              w.down, w.down_scale, cfg.block)
    assert torch.equal(layer, g["out_reference"])


@pytest.mark.parametrize("name", list(GPT_CASES))
def test_gpt_oss_oracle_matches_reference(name):
    cfg, T, seed = GPT_CASES[name]
    g = load_golden(name)
    w, x = gpt_inputs(cfg, T, seed)
    assert checksum(x, w.router, w.router_bias, w.gu_blocks, w.gu_scales, w.dn_blocks) == g["input_sha"]

    logits, scores, indices = oracle.gpt_oss_router(x, w.router, w.router_bias, cfg.top_k)
    assert torch.equal(logits, g["logits"]) and torch.equal(scores, g["scores"])
    assert torch.equal(indices, g["indices"])
    fixed = oracle.router_logits(x, w.router, w.router_bias, 1)
    ulp = g["logits"].float().abs().clamp_min(2 ** -126) * 2 ** -7
    assert bool(((fixed - g["logits"].float()).abs() <= ulp).all())
    free = tie_free_rows(g["logits"], cfg.top_k)
    assert torch.equal(oracle.topk(g["logits"].float(), cfg.top_k)[free], g["indices"][free])

    # exact MXFP4 decode (C) == transformers' decode used by the reference
    dec = oracle.decode_mxfp4(w.gu_blocks[0], w.gu_scales[0])      # [2I, H]
    assert torch.equal(dec.T[:, :64], g["decoded_gate_up0"])
    assert torch.equal(oracle.decode_mxfp4_torch(w.gu_blocks[0], w.gu_scales[0]), dec)

    counts, offsets, perm, inv = oracle.permute(g["indices"], cfg.experts)
    assert torch.equal(perm, g["perm_src"])
    assert torch.equal(oracle.combine(g["contrib"], inv, g["indices"]), g["out_reference"])

    layer = oracle.gpt_oss_layer(x, g["indices"], g["scores"], w.gu_blocks, w.gu_scales, w.gu_bias,
                                 w.dn_blocks, w.dn_scales, w.dn_bias, cfg.alpha, cfg.limit)
    assert torch.equal(layer, g["out_reference"])


def test_native_route_and_all_to_all_match_reference():
    g = load_golden("native_a2a")
    index, weight, _ = oracle.native_route(g["tokens"], g["gate"], g["top_k"], True)
    assert torch.equal(index, g["index"]) and torch.equal(weight, g["weight"])
    outs = oracle.routed_forward_ranks([g["tokens"][:3], g["tokens"][3:]], g["gate"], g["gate_up"],
                                       g["down"], g["top_k"])
    for a, b in zip(outs, g["rank_outputs"]):
        assert torch.equal(a, b)


def test_rank_slot_combine_order_matches_all_to_all():
    """ORDER_RANK_SLOT combine (C) reproduces moe.py's dest-sorted index_add_."""
    g = load_golden("native_a2a")
    tokens, K = g["tokens"], g["top_k"]
    index, weight, _ = oracle.native_route(tokens, g["gate"], K, True)
    E, epr = g["gate"].shape[0], g["gate"].shape[0] // 2
    flat = index.reshape(-1)
    order = torch.argsort(torch.div(flat, epr, rounding_mode="floor"), stable=True)
    rows = torch.randn(flat.numel(), tokens.shape[1]).to(torch.bfloat16)   # rows in send order
    token_index = torch.arange(tokens.shape[0]).repeat_interleave(K)
    ref = tokens.new_zeros(tokens.shape)
    ref.index_add_(0, token_index[order], rows * weight.reshape(-1)[order].unsqueeze(-1).to(rows.dtype))
    inverse = torch.empty(flat.numel(), dtype=torch.int32)
    inverse[order] = torch.arange(flat.numel(), dtype=torch.int32)
    out = oracle.combine(rows, inverse, index, order=1, experts_per_rank=epr, weights=weight.float())
    assert torch.equal(out, ref)
    assert E == 8


def test_synthetic_quantisers_roundtrip():
    w = torch.randn(256, 256) * 0.02
    q, s = S.quantize_fp8_blocks(w)
    deq = oracle.dequant_torch(q, s, (128, 128), torch.float32)
    assert float((deq - w).norm() / w.norm()) < 0.05
    b, sc = S.quantize_mxfp4(w)
    dec = oracle.decode_mxfp4(b, sc).float()
    assert float((dec - w).norm() / w.norm()) < 0.15


def test_oracle_slot_sum_matches_torch_cuda():
    """oracle.slot_sum (four fp32 accumulators, slot k into a[k % 4], then
    ((a0 + a1) + a2) + a3) reproduces torch's CUDA sum over the slot
    dimension, recorded on a B200 by tests/golden/make_slot_sum_golden.py on
    values whose bf16 result depends on the summation order (K = 1 .. 32); a
    plain left-to-right fp32 sum does not."""
    g = torch.load(GOLDEN / "slot_sum_torch_cuda.pt", weights_only=False)
    order_visible = 0
    for name, c in g["cases"].items():
        got = oracle.slot_sum(c["values"])
        assert torch.equal(got.view(torch.int16), c["sum"].view(torch.int16)), name
        seq = torch.zeros(c["values"][:, 0].shape)
        for k in range(c["values"].shape[1]):
            seq = seq + c["values"][:, k].float()
        order_visible += int(not torch.equal(seq.bfloat16(), c["sum"]))
    assert order_visible >= 6


def test_oracle_selection_matches_torch_cuda():
    """The oracle's top-k (slot order of equal values included) and its
    butterfly sum reproduce torch's CUDA topk / sum, recorded on a B200 by
    tests/golden/make_router_golden.py on tie-heavy logits: rows of repeated
    values, all-equal rows and a coarse value grid."""
    g = torch.load(GOLDEN / "router_torch_cuda.pt", weights_only=False)
    for name, c in g["cases"].items():
        K = c["K"]
        keys = c["logits"].float() if c["kind"] == "gpt" else c["probs"]
        idx = oracle.topk(keys, K)
        assert torch.equal(idx, c["indices"]), name
        if c["kind"] != "gpt":
            top = torch.gather(c["probs"], 1, idx)
            s = oracle.butterfly_sum(top)
            if K & (K - 1) == 0:   # pinned for powers of two
                assert torch.equal(s, c["sums"]), name
                assert torch.equal(top / s[:, None], c["scores"]), name
