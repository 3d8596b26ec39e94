"""Seeded synthetic MoE-layer workloads (no checkpoints or datasets exist here).

Each named config has the shapes of one benchmark layer:

=================  ======  =====  ==  =====  =======  ======================
name               hidden  E      K   inter  weights  batches (tokens)
=================  ======  =====  ==  =====  =======  ======================
qwen3-tiny         256     8      2   128    fp8-128  64
qwen3-30b-a3b      2048    128    8   768    fp8-128  1, 8, 64, 512, 4096
gpt-oss-20b        2880    32     4   2880   mxfp4    1, 16, 64, 2048
gpt-oss-120b       2880    128    4   2880   mxfp4    64, 8192
qwen3-235b-a22b    4096    128    8   1536   fp8-128  256, 16384
=================  ======  =====  ==  =====  =======  ======================

Weights are drawn N(0, 0.02) and quantised: FP8 E4M3 with one fp32 scale per
128x128 block (scale = block absmax / 448, dequantised as q * scale), or MXFP4
(32-value groups, ue8m0 scale 2^ceil(log2(absmax / 6)), e2m1 round to
nearest). GPT-OSS biases are N(0, 0.01). Activations are N(0, 1) bf16 and the
router weight N(0, 0.02) bf16. qwen3-235b-a22b adds a fixed per-expert router
bias that follows a Zipf(1.1) ranking, which skews the expert load to a
coefficient of variation near 0.5; the Qwen router has no bias, so this is a
harness-side deviation applied identically to the oracle and the kernels.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch


@dataclass(frozen=True)
class LayerConfig:
    name: str
    family: str            # "qwen3" or "gpt_oss"
    hidden: int
    experts: int
    top_k: int
    inter: int
    storage: str           # "fp8" or "mxfp4"
    batches: tuple
    norm_topk: bool = True
    zipf_bias: bool = False
    alpha: float = 1.702
    limit: float = 7.0
    block: tuple = (128, 128)


CONFIGS = {
    c.name: c
    for c in (
        LayerConfig("qwen3-tiny", "qwen3", 256, 8, 2, 128, "fp8", (64,)),
        LayerConfig("qwen3-30b-a3b", "qwen3", 2048, 128, 8, 768, "fp8", (1, 8, 64, 512, 4096)),
        LayerConfig("gpt-oss-20b", "gpt_oss", 2880, 32, 4, 2880, "mxfp4", (1, 16, 64, 2048),
                    norm_topk=False),
        LayerConfig("gpt-oss-120b", "gpt_oss", 2880, 128, 4, 2880, "mxfp4", (64, 8192),
                    norm_topk=False),
        LayerConfig("qwen3-235b-a22b", "qwen3", 4096, 128, 8, 1536, "fp8", (256, 16384),
                    zipf_bias=True),
    )
}

# Router-bias temperature giving expert_load_cv ~ 0.5 for qwen3-235b-a22b.
ZIPF_TAU = 0.245


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def quantize_fp8_blocks(w: torch.Tensor, block=(128, 128)):
    """fp32 [rows, cols] -> (e4m3 [rows, cols], fp32 scales [ceil(rows/br), ceil(cols/bc)])."""
    rows, cols = w.shape
    br, bc = block
    nbr, nbc = -(-rows // br), -(-cols // bc)
    pad = torch.zeros(nbr * br, nbc * bc, device=w.device, dtype=torch.float32)
    pad[:rows, :cols] = w
    blocks = pad.view(nbr, br, nbc, bc)
    amax = blocks.abs().amax(dim=(1, 3)).clamp_min(1e-12)
    scale = amax / 448.0
    q = (blocks / scale[:, None, :, None]).view(nbr * br, nbc * bc)[:rows, :cols]
    return q.to(torch.float8_e4m3fn), scale


_E2M1_MID = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)


def quantize_mxfp4(w: torch.Tensor):
    """fp32 [rows, K] (K % 32 == 0) -> (blocks u8 [rows, K/32, 16], scales u8 [rows, K/32])."""
    rows, K = w.shape
    g = w.view(rows, K // 32, 32)
    amax = g.abs().amax(dim=-1).clamp_min(1e-30)
    e = torch.ceil(torch.log2(amax / 6.0)).clamp(-127, 127)
    scales = (e + 127).to(torch.uint8)
    v = g / torch.exp2(e)[..., None]
    mids = torch.tensor(_E2M1_MID, device=w.device)
    mag = torch.bucketize(v.abs(), mids).to(torch.uint8)   # 0..7
    code = mag | ((v < 0).to(torch.uint8) << 3)
    packed = code[..., 0::2] | (code[..., 1::2] << 4)
    return packed.contiguous(), scales.contiguous()


@dataclass
class QwenLayerWeights:
    router: torch.Tensor        # bf16 [E, H]
    router_bias: torch.Tensor | None
    gate: torch.Tensor          # e4m3 [E, I, H]
    gate_scale: torch.Tensor    # fp32 [E, I/128, H/128]
    up: torch.Tensor
    up_scale: torch.Tensor
    down: torch.Tensor          # e4m3 [E, H, I]
    down_scale: torch.Tensor
    block: tuple = (128, 128)


@dataclass
class GptOssLayerWeights:
    router: torch.Tensor        # bf16 [E, H]
    router_bias: torch.Tensor   # bf16 [E]
    gu_blocks: torch.Tensor     # u8 [E, 2I, H/32, 16] (interleaved gate/up rows)
    gu_scales: torch.Tensor     # u8 [E, 2I, H/32]
    gu_bias: torch.Tensor       # bf16 [E, 2I]
    dn_blocks: torch.Tensor     # u8 [E, H, I/32, 16]
    dn_scales: torch.Tensor     # u8 [E, H, I/32]
    dn_bias: torch.Tensor       # bf16 [E, H]
    alpha: float = 1.702
    limit: float = 7.0


def zipf_router_bias(E: int, seed: int, device, s: float = 1.1, tau: float = ZIPF_TAU) -> torch.Tensor:
    ranks = torch.randperm(E, generator=_gen(seed, "cpu")).to(torch.float64) + 1.0
    bias = tau * (-s * torch.log(ranks))
    bias = bias - bias.mean()
    return bias.to(torch.bfloat16).to(device)


def make_qwen(cfg: LayerConfig, seed: int = 0, device="cpu") -> QwenLayerWeights:
    g = _gen(seed, device)
    E, H, I = cfg.experts, cfg.hidden, cfg.inter
    router = (torch.randn(E, H, generator=g, device=device) * 0.02).to(torch.bfloat16)
    mats = {"gate": [], "up": [], "down": []}
    scales = {"gate": [], "up": [], "down": []}
    for _ in range(E):
        for name, shape in (("gate", (I, H)), ("up", (I, H)), ("down", (H, I))):
            w = torch.randn(*shape, generator=g, device=device) * 0.02
            q, s = quantize_fp8_blocks(w, cfg.block)
            mats[name].append(q)
            scales[name].append(s)
    bias = zipf_router_bias(E, seed + 1, device) if cfg.zipf_bias else None
    return QwenLayerWeights(router, bias, torch.stack(mats["gate"]), torch.stack(scales["gate"]),
                            torch.stack(mats["up"]), torch.stack(scales["up"]),
                            torch.stack(mats["down"]), torch.stack(scales["down"]), cfg.block)


def make_gpt_oss(cfg: LayerConfig, seed: int = 0, device="cpu") -> GptOssLayerWeights:
    g = _gen(seed, device)
    E, H, I = cfg.experts, cfg.hidden, cfg.inter
    router = (torch.randn(E, H, generator=g, device=device) * 0.02).to(torch.bfloat16)
    router_bias = (torch.randn(E, generator=g, device=device) * 0.01).to(torch.bfloat16)
    gu_b, gu_s, dn_b, dn_s = [], [], [], []
    for _ in range(E):
        b, s = quantize_mxfp4(torch.randn(2 * I, H, generator=g, device=device) * 0.02)
        gu_b.append(b)
        gu_s.append(s)
        b, s = quantize_mxfp4(torch.randn(H, I, generator=g, device=device) * 0.02)
        dn_b.append(b)
        dn_s.append(s)
    gu_bias = (torch.randn(E, 2 * I, generator=g, device=device) * 0.01).to(torch.bfloat16)
    dn_bias = (torch.randn(E, H, generator=g, device=device) * 0.01).to(torch.bfloat16)
    return GptOssLayerWeights(router, router_bias, torch.stack(gu_b), torch.stack(gu_s), gu_bias,
                              torch.stack(dn_b), torch.stack(dn_s), dn_bias, cfg.alpha, cfg.limit)


def make_hidden(T: int, H: int, seed: int = 0, device="cpu") -> torch.Tensor:
    return torch.randn(T, H, generator=_gen(seed, device), device=device).to(torch.bfloat16)


def expert_load_cv(counts: torch.Tensor) -> float:
    """std(counts, biased) / mean(counts) (moe_serving/moe.py:47-52)."""
    c = counts.float()
    m = c.mean()
    return 0.0 if float(m) == 0 else float(c.std(unbiased=False) / m)


def algorithmic_bytes(cfg: LayerConfig, T: int, counts: torch.Tensor) -> int:
    """Compulsory HBM bytes of one layer call: weights of the used experts
    (values + scales + biases), router weight, hidden in / out, routing."""
    used = int((counts > 0).sum())
    H, I, E = cfg.hidden, cfg.inter, cfg.experts
    if cfg.storage == "fp8":
        br, bc = cfg.block
        per = 3 * H * I + 4 * (2 * math.ceil(I / br) * math.ceil(H / bc)
                               + math.ceil(H / br) * math.ceil(I / bc))
    else:
        per = (3 * H * I) // 2 + (3 * H * I) // 32 + 2 * (2 * I + H)
    return used * per + E * H * 2 + 2 * T * H * 2 + T * cfg.top_k * 8


def algorithmic_flops(cfg: LayerConfig, T: int) -> int:
    return 2 * T * cfg.top_k * 3 * cfg.hidden * cfg.inter + 2 * T * cfg.hidden * cfg.experts
