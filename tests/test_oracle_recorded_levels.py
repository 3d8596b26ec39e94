"""The efficient-mode restatements against the reference's recorded
validation of those paths (CPU only).

The hub kernels behind the reference's efficient numerics (the finegrained-fp8
``matmul_grouped`` of grouped_fp8 and triton's ``matmul_ogs`` of
grouped_mxfp4) are not vendored, so their outputs cannot be compared bit for
bit. The reference's own four-GPU check of those paths
(tests/helpers/check_grouped_ep.py in the reference project) recorded the
relative L2 of each against the module's weight-only numerics on seeded
synthetic layers (tests/validation_results/efficient_grouped_ep.json there).
The same check rebuilt here (same shapes, value distributions, routing and
seed; CPU draws, so the values themselves differ) puts the oracle's
restatements at the recorded error levels: the error is set by the
algorithm's roundings (e4m3 activations; bf16 intermediates and scatter rows),
not by the particular draws.
"""

import pytest
import torch

from oracle import oracle

# relative L2 of the efficient path against the weight-only module, by
# token count, as recorded by the reference (ep_size 4)
RECORDED = {
    "gpt_oss": {4: 0.002918464597314596, 97: 0.0028776179533451796, 1: 0.002996075665578246},
    "qwen3_moe": {4: 0.04718032106757164, 97: 0.04467129707336426, 1: 0.046134304255247116},
}


def _routing(tokens):
    x = torch.randn(tokens, 256).bfloat16()
    idx = torch.stack([torch.randperm(4)[:2] for _ in range(tokens)])
    if tokens == 1:
        idx[:] = torch.tensor([0, 1])
    w = torch.softmax(torch.randn(tokens, 2), -1)
    return x, idx, w


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


def test_fused_mxfp4_restatement_has_the_recorded_error():
    """grouped_mxfp4 against the fp32 module (x.float(), MXFP4 decoded
    exactly, fp32 biases): 4 experts, H = I = 256, top-2, random e2m1 codes
    with scale 2^-7, biases N(0, 0.01)."""
    torch.manual_seed(12)
    bufs = {}
    for proj, n in (("gu", 512), ("dn", 256)):
        bufs[proj] = (torch.randint(0, 256, (4, n, 8, 16), dtype=torch.uint8),
                      torch.full((4, n, 8), 120, dtype=torch.uint8), torch.randn(4, n) * 0.01)
    (gb, gs, gbias), (db, ds, dbias) = bufs["gu"], bufs["dn"]
    for tokens in (4, 97, 1):
        x, idx, w = _routing(tokens)
        eff = oracle.gpt_oss_layer_efficient(x, idx, w, gb, gs, gbias, db, ds, dbias, 1.702, 7.0)
        ref = torch.zeros(tokens, 256)
        for e in range(4):
            t, s = torch.where(idx == e)
            if t.numel() == 0:
                continue
            gu = x.float()[t] @ oracle.decode_mxfp4_torch(gb[e], gs[e], torch.float32).T + gbias[e]
            gate, up = gu[:, 0::2].clamp(max=7.0), gu[:, 1::2].clamp(min=-7.0, max=7.0)
            a = (up + 1) * (gate * torch.sigmoid(gate * 1.702))
            y = a @ oracle.decode_mxfp4_torch(db[e], ds[e], torch.float32).T + dbias[e]
            ref.index_add_(0, t, y * w[t, s, None])
        r = _rel(eff, ref)
        assert abs(r / RECORDED["gpt_oss"][tokens] - 1) < 0.15, (tokens, r)


def test_w8a8_restatement_has_the_recorded_error():
    """grouped_fp8 against the weight-only module: 4 experts of 256 x 256
    e4m3 weights (N(0, 0.05) cast, scales 1 per 128 x 128 block), top-2."""
    torch.manual_seed(12)
    mats = {p: [] for p in ("gate", "up", "down")}
    for _ in range(4):
        for p in ("gate", "up", "down"):
            mats[p].append((torch.randn(256, 256) * 0.05).to(torch.float8_e4m3fn))
    g, u, d = (torch.stack(mats[p]) for p in ("gate", "up", "down"))
    s = torch.ones(4, 2, 2)
    for tokens in (4, 97, 1):
        x, idx, w = _routing(tokens)
        ref = oracle.qwen_layer(x, idx, w, g, s, u, s, d, s, (128, 128))
        eff = oracle.qwen_w8a8_layer(x, idx, w, g, s, u, s, d, s, (128, 128))
        r = _rel(eff, ref)
        # 97 tokens average over many rows; 1 and 4 tokens over a handful
        tol = 0.10 if tokens == 97 else 0.25
        assert abs(r / RECORDED["qwen3_moe"][tokens] - 1) < tol, (tokens, r)


@pytest.mark.parametrize("family", ["gpt_oss", "qwen3_moe"])
def test_recorded_levels_are_the_references(family):
    """The recorded figures are the reference's own acceptance-passing values
    (its bar: gpt_oss < 0.03, qwen3_moe < 0.08)."""
    bar = 0.03 if family == "gpt_oss" else 0.08
    assert all(0 < v < bar for v in RECORDED[family].values())
