"""Device layout of the expert weights (built once, at load time).

Logically every format is ``[E_loc][planes][feat_pad][k_pad]`` (K
contiguous): gate/up (planes = 2) holds the gate rows in plane 0 and the up
rows in plane 1, both padded to ``I_p = ceil(I / 128) * 128`` features and
``H_k = ceil(H / 64) * 64`` reduction columns; down (planes = 1) is
``[E_loc][H_f][I_p]`` with ``H_f = ceil(H / 128) * 128``. GPT-OSS stores
gate/up interleaved (even / odd columns, moe_serving/gpt_oss_parallel.py:198);
it is de-interleaved here, once. Padding is zero (MXFP4 padding groups get
scale 127 = 2^0).

* BF16 weights stay in that layout (the GEMM streams 128-byte-swizzled tiles
  of it with TMA).
* Quantised weights (FP8 block-scaled E4M3, moe_serving/qwen3_parallel.py:48-70;
  MXFP4 E2M1 with ue8m0 group scales, gpt_oss_parallel.py:183-193) are packed
  into one contiguous blob per (expert, feature tile, 64-column k-block), the
  unit the GEMM converts, so each k-block arrives with a single bulk copy:
  ``[E_loc][feat_tiles][k_pad / 64][blob_bytes]``. A feature tile is 64
  features of a gated pair (rows 0-63 gate, 64-127 up) or 128 features of a
  single projection. A blob is 128 rows of 64 bytes (e4m3) or 32 bytes
  (e2m1 pairs), each row's 16-byte chunks permuted (chunk c of row r stored at
  c ^ ((r >> 1) & 3), resp. c ^ ((r >> 2) & 1)) so that one lane per row reads
  shared memory without bank conflicts, followed by the k-block's scales:
  FP8 with block scales covering whole 64 x 64 halves, the two fp32 scales of
  rows 0-63 and 64-127 plus 8 zero bytes; other FP8 blocks, 128 x 4 fp32
  (row, 16-column chunk); MXFP4, 128 x 2 ue8m0 bytes (row, 32-column group).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from moe_serving_profile_b200 import _lib


def _ceil(v: int, m: int) -> int:
    return (v + m - 1) // m * m


@dataclass
class ExpertWeights:
    """One layer's local experts in device layout: w1 (gate/up) and w2 (down)
    are bf16 [E, planes, F_p, K_p] for BF16 weights and packed blobs
    [E, feature tiles, K_p / 64, blob bytes] for FP8 / MXFP4 (scales inside)."""

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


def _tile_rows(w: torch.Tensor, planes: int) -> torch.Tensor:
    """[E, planes, F_p, C] -> [E, feat_tiles, 128, C]: a gated tile stacks 64
    gate rows over the 64 up rows of the same features; a single-plane tile
    takes 128 rows."""
    E, P, Fp, C = w.shape
    if planes == 2:
        return w.reshape(E, 2, Fp // 64, 64, C).permute(0, 2, 1, 3, 4).reshape(E, Fp // 64, 128, C)
    return w.reshape(E, Fp // 128, 128, C)


def _swizzle_sel(row_bytes: int) -> torch.Tensor:
    r = torch.arange(128)
    return ((r >> 1) & 3) if row_bytes == 64 else ((r >> 2) & 1)


def _kblock_rows(t: torch.Tensor, row_bytes: int) -> torch.Tensor:
    """[E, FT, 128, nkb * row_bytes] bytes -> [E, FT, nkb, 128 * row_bytes]
    with each row's 16-byte chunk c stored at position c ^ sel(row)."""
    E, FT, R, C = t.shape
    nkb, nch = C // row_bytes, row_bytes // 16
    t = t.reshape(E, FT, R, nkb, nch, 16).permute(0, 1, 3, 2, 4, 5)      # [E, FT, nkb, 128, nch, 16]
    src = torch.arange(nch)[None, :] ^ _swizzle_sel(row_bytes)[:, None]  # position p holds chunk p ^ sel
    idx = src.reshape(1, 1, 1, R, nch, 1).expand(E, FT, nkb, R, nch, 16).to(t.device)
    return torch.gather(t, 4, idx).reshape(E, FT, nkb, R * row_bytes)


def _fp8_blob_scales(s: torch.Tensor, planes: int, n_feat: int, feat_pad: int, k_pad: int,
                     block: tuple[int, int]) -> torch.Tensor:
    """Scale section of each FP8 blob: [E, FT, nkb, 16 or 2048] bytes."""
    E, P, nbr, nbc = s.shape
    br, bc = block
    feat_tile = 64 if planes == 2 else 128
    FT = feat_pad // feat_tile
    nkb = k_pad // 64
    dev = s.device
    s = s.float()
    if br % 64 == 0 and bc % 64 == 0:
        ft = torch.arange(FT, device=dev)
        sci = torch.clamp(torch.arange(nkb, device=dev) // (bc // 64), max=nbc - 1)
        out = torch.zeros(E, FT, nkb, 4, device=dev)
        for h in range(2):
            pl = h if planes == 2 else 0
            f = ft * feat_tile + (0 if planes == 2 else 64 * h)
            sri = torch.clamp(torch.clamp(f, max=n_feat - 1) // br, max=nbr - 1)
            out[..., h] = s[:, pl][:, sri][:, :, sci]
        return out.view(torch.uint8).reshape(E, FT, nkb, 16)
    r = torch.arange(128, device=dev)
    pl = (r // 64) if planes == 2 else torch.zeros_like(r)
    f = torch.arange(FT, device=dev)[:, None] * feat_tile + ((r % 64) if planes == 2 else r)[None, :]
    sri = torch.clamp(torch.clamp(f, max=n_feat - 1) // br, max=nbr - 1)          # [FT, 128]
    k0 = torch.arange(nkb, device=dev)[:, None] * 64 + torch.arange(4, device=dev)[None, :] * 16
    sci = torch.clamp(k0 // bc, max=nbc - 1)                                        # [nkb, 4]
    vals = s[:, pl[None, :].expand(FT, 128), sri]                                   # [E, FT, 128, nbc]
    out = vals[:, :, None, :, :].expand(E, FT, nkb, 128, nbc)
    idx = sci[None, None, :, None, :].expand(E, FT, nkb, 128, 4)
    return torch.gather(out, 4, idx).contiguous().view(torch.uint8).reshape(E, FT, nkb, 2048)


def pack_fp8_blobs(w: torch.Tensor, s: torch.Tensor, planes: int, n_feat: int,
                   block: tuple[int, int]) -> torch.Tensor:
    """e4m3 bytes [E, planes, F_p, k_pad] + fp32 block scales [E, planes, nbr, nbc]
    -> blobs [E, FT, k_pad / 64, 8192 + scale section]."""
    data = _kblock_rows(_tile_rows(w.view(torch.uint8), planes), 64)
    scales = _fp8_blob_scales(s, planes, n_feat, w.shape[2], w.shape[3], block)
    return torch.cat([data, scales], dim=-1).contiguous()


def pack_mxfp4_blobs(w: torch.Tensor, s: torch.Tensor, planes: int) -> torch.Tensor:
    """e2m1 pairs [E, planes, F_p, k_pad / 2] + ue8m0 scales [E, planes, F_p, k_pad / 32]
    -> blobs [E, FT, k_pad / 64, 4096 + 256]."""
    data = _kblock_rows(_tile_rows(w, planes), 32)
    st = _tile_rows(s, planes)                                    # [E, FT, 128, G]
    E, FT, R, G = st.shape
    sc = st.reshape(E, FT, R, G // 2, 2).permute(0, 1, 3, 2, 4).reshape(E, FT, G // 2, R * 2)
    return torch.cat([data, sc], dim=-1).contiguous()


def unpack_blob_rows(blobs: torch.Tensor, row_bytes: int, planes: int) -> torch.Tensor:
    """Inverse of the data part of the packing: blobs -> [E, planes, F_p, nkb * row_bytes]."""
    E, FT, nkb, _ = blobs.shape
    R, nch = 128, row_bytes // 16
    d = blobs[..., : R * row_bytes].reshape(E, FT, nkb, R, nch, 16)
    src = torch.arange(nch)[None, :] ^ _swizzle_sel(row_bytes)[:, None]   # involution
    idx = src.reshape(1, 1, 1, R, nch, 1).expand(E, FT, nkb, R, nch, 16).to(blobs.device)
    d = torch.gather(d, 4, idx).permute(0, 1, 3, 2, 4, 5).reshape(E, FT, R, nkb * row_bytes)
    if planes == 2:
        return d.reshape(E, FT, 2, 64, -1).permute(0, 2, 1, 3, 4).reshape(E, 2, FT * 64, -1)
    return d.reshape(E, 1, FT * 128, -1)


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
    return ExpertWeights(_lib.W_FP8, E, hidden, inter,
                         pack_fp8_blobs(w1, s1, 2, inter, (br, bc)),
                         pack_fp8_blobs(w2.unsqueeze(1), s2.unsqueeze(1), 1, hidden, (br, bc)),
                         block=(br, bc))


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
    return ExpertWeights(_lib.W_MXFP4, E, hidden, inter, pack_mxfp4_blobs(w1, s1, 2),
                         pack_mxfp4_blobs(w2.unsqueeze(1), s2.unsqueeze(1), 1), b1=b1, b2=b2,
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
