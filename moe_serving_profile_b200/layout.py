"""Device layout of the expert weights (built once, at load time).

Every format is stored per local expert as ``[E_loc][planes][feat_pad][k_pad]``
(K contiguous), the layout the grouped GEMM streams with TMA:

* gate/up (planes = 2): plane 0 holds the gate rows, plane 1 the up rows, both
  padded to ``I_p = ceil(I / 128) * 128`` features and ``H_k = ceil(H / 64) * 64``
  reduction columns. GPT-OSS stores gate/up interleaved (even / odd columns,
  moe_serving/gpt_oss_parallel.py:198); it is de-interleaved here, once.
* down (planes = 1): ``[E_loc][H_f][I_p]`` with ``H_f = ceil(H / 128) * 128``.

Formats:

* FP8 (Qwen3 block-scaled E4M3, moe_serving/qwen3_parallel.py:48-70): bytes as
  stored, fp32 block scales ``[E_loc][planes][ceil(rows/br)][ceil(cols/bc)]``
  (gate and up keep their own scale grids, as the reference's separate
  ``ExpertProjection`` modules do).
* MXFP4 (GPT-OSS, moe_serving/gpt_oss_parallel.py:183-193): e2m1 bytes, 16
  per 32-value group, ue8m0 scales ``[E_loc][planes][feat_pad][k_pad / 32]``;
  padding groups get scale 127 (2^0) so padded zeros stay zeros.
* BF16: K-major bf16 (GPT-OSS bf16 storage is N-major ``[E, H, 2I]`` and is
  transposed here).

Padding is zero-filled; the kernels never read outside the padded arrays.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from moe_serving_profile_b200 import _lib


def _ceil(v: int, m: int) -> int:
    return (v + m - 1) // m * m


@dataclass
class ExpertWeights:
    fmt: int
    n_experts: int
    hidden: int
    inter: int
    w1: torch.Tensor
    w2: torch.Tensor
    s1: torch.Tensor | None = None
    s2: torch.Tensor | None = None
    b1: torch.Tensor | None = None
    b2: torch.Tensor | None = None
    block: tuple[int, int] = (128, 128)
    gated_epilogue: int = _lib.EPI_SWIGLU
    alpha: float = 1.702
    limit: float = 7.0

    @property
    def i_pad(self) -> int:
        return _ceil(self.inter, 128)

    @property
    def h_k(self) -> int:
        return _ceil(self.hidden, 64)

    @property
    def h_f(self) -> int:
        return _ceil(self.hidden, 128)

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in
                   (self.w1, self.w2, self.s1, self.s2, self.b1, self.b2) if t is not None)


def _check_dims(hidden: int, inter: int) -> None:
    if hidden % 8 or inter % 8:
        raise NotImplementedError(
            f"hidden ({hidden}) and intermediate ({inter}) sizes must be multiples of 8")


def fp8_experts(gate: torch.Tensor, gate_scale: torch.Tensor, up: torch.Tensor,
                up_scale: torch.Tensor, down: torch.Tensor, down_scale: torch.Tensor,
                block: tuple[int, int]) -> ExpertWeights:
    """gate/up: e4m3 [E, I, H] with scales [E, ceil(I/br), ceil(H/bc)];
    down: e4m3 [E, H, I] with scales [E, ceil(H/br), ceil(I/bc)]."""
    E, inter, hidden = gate.shape
    _check_dims(hidden, inter)
    br, bc = block
    if bc % 16:
        raise NotImplementedError(f"FP8 scale blocks must be a multiple of 16 columns, got {bc}")
    dev = gate.device
    I_p, H_k, H_f = _ceil(inter, 128), _ceil(hidden, 64), _ceil(hidden, 128)
    w1 = torch.zeros(E, 2, I_p, H_k, device=dev, dtype=torch.uint8)
    w1[:, 0, :inter, :hidden] = gate.view(torch.uint8)
    w1[:, 1, :inter, :hidden] = up.view(torch.uint8)
    w2 = torch.zeros(E, H_f, I_p, device=dev, dtype=torch.uint8)
    w2[:, :hidden, :inter] = down.view(torch.uint8)
    s1 = torch.stack([gate_scale.float(), up_scale.float()], dim=1).contiguous()
    s2 = down_scale.float().contiguous()
    return ExpertWeights(_lib.W_FP8, E, hidden, inter, w1, w2, s1=s1, s2=s2, block=(br, bc))


def bf16_experts(gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor,
                 gate_bias: torch.Tensor | None = None, up_bias: torch.Tensor | None = None,
                 down_bias: torch.Tensor | None = None,
                 gated_epilogue: int = _lib.EPI_SWIGLU, alpha: float = 1.702,
                 limit: float = 7.0) -> ExpertWeights:
    """K-major bf16: gate/up [E, I, H], down [E, H, I]."""
    E, inter, hidden = gate.shape
    _check_dims(hidden, inter)
    dev = gate.device
    I_p, H_k, H_f = _ceil(inter, 128), _ceil(hidden, 64), _ceil(hidden, 128)
    w1 = torch.zeros(E, 2, I_p, H_k, device=dev, dtype=torch.bfloat16)
    w1[:, 0, :inter, :hidden] = gate
    w1[:, 1, :inter, :hidden] = up
    w2 = torch.zeros(E, H_f, I_p, device=dev, dtype=torch.bfloat16)
    w2[:, :hidden, :inter] = down
    b1 = b2 = None
    if gate_bias is not None:
        b1 = torch.zeros(E, 2, I_p, device=dev, dtype=torch.bfloat16)
        b1[:, 0, :inter] = gate_bias
        b1[:, 1, :inter] = up_bias
    if down_bias is not None:
        b2 = torch.zeros(E, H_f, device=dev, dtype=torch.bfloat16)
        b2[:, :hidden] = down_bias
    return ExpertWeights(_lib.W_BF16, E, hidden, inter, w1, w2, b1=b1, b2=b2,
                         gated_epilogue=gated_epilogue, alpha=alpha, limit=limit)


def gpt_oss_mxfp4_experts(gu_blocks: torch.Tensor, gu_scales: torch.Tensor,
                          gu_bias: torch.Tensor, dn_blocks: torch.Tensor,
                          dn_scales: torch.Tensor, dn_bias: torch.Tensor, alpha: float,
                          limit: float) -> ExpertWeights:
    """GPT-OSS packed experts: gate_up blocks [E, 2I, H/32, 16] u8 (interleaved
    gate/up rows), scales [E, 2I, H/32]; down blocks [E, H, I/32, 16]."""
    E, two_i, G, _ = gu_blocks.shape
    inter = two_i // 2
    hidden = G * 32
    _check_dims(hidden, inter)
    if dn_blocks.shape[1] != hidden or dn_blocks.shape[2] * 32 != inter:
        raise ValueError("down_proj blocks do not match gate_up_proj blocks")
    dev = gu_blocks.device
    I_p, H_k, H_f = _ceil(inter, 128), _ceil(hidden, 64), _ceil(hidden, 128)
    G1 = H_k // 32
    w1 = torch.zeros(E, 2, I_p, G1 * 16, device=dev, dtype=torch.uint8)
    s1 = torch.full((E, 2, I_p, G1), 127, device=dev, dtype=torch.uint8)
    gu = gu_blocks.reshape(E, two_i, G * 16)
    w1[:, 0, :inter, : G * 16] = gu[:, 0::2]
    w1[:, 1, :inter, : G * 16] = gu[:, 1::2]
    s1[:, 0, :inter, :G] = gu_scales[:, 0::2]
    s1[:, 1, :inter, :G] = gu_scales[:, 1::2]
    b1 = torch.zeros(E, 2, I_p, device=dev, dtype=torch.bfloat16)
    b1[:, 0, :inter] = gu_bias[:, 0::2].to(torch.bfloat16)
    b1[:, 1, :inter] = gu_bias[:, 1::2].to(torch.bfloat16)
    G2 = dn_blocks.shape[2]
    G2p = I_p // 32
    w2 = torch.zeros(E, H_f, G2p * 16, device=dev, dtype=torch.uint8)
    s2 = torch.full((E, H_f, G2p), 127, device=dev, dtype=torch.uint8)
    w2[:, :hidden, : G2 * 16] = dn_blocks.reshape(E, hidden, G2 * 16)
    s2[:, :hidden, :G2] = dn_scales
    b2 = torch.zeros(E, H_f, device=dev, dtype=torch.bfloat16)
    b2[:, :hidden] = dn_bias.to(torch.bfloat16)
    return ExpertWeights(_lib.W_MXFP4, E, hidden, inter, w1, w2, s1=s1, s2=s2, b1=b1, b2=b2,
                         gated_epilogue=_lib.EPI_CLAMP_SWIGLU, alpha=alpha, limit=limit)


def gpt_oss_bf16_experts(gate_up: torch.Tensor, gate_up_bias: torch.Tensor,
                         down: torch.Tensor, down_bias: torch.Tensor, alpha: float,
                         limit: float) -> ExpertWeights:
    """GPT-OSS bf16 storage: gate_up [E, H, 2I] (interleaved columns), down [E, I, H]."""
    gate = gate_up[:, :, 0::2].transpose(1, 2)
    up = gate_up[:, :, 1::2].transpose(1, 2)
    return bf16_experts(gate, up, down.transpose(1, 2), gate_up_bias[:, 0::2],
                        gate_up_bias[:, 1::2], down_bias,
                        gated_epilogue=_lib.EPI_CLAMP_SWIGLU, alpha=alpha, limit=limit)
