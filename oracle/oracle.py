"""CPU oracle of the MoE expert layer — TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this module, and only as the checker or as the timed CPU baseline; the
product package never does.

Two halves:
* exact stages (codecs, dequantisation, fixed-order router logits, top-k,
  permutation, ordered combine): ``liboracle.so`` built from oracle.c;
* floating-point expert math: a torch restatement of the reference's own
  sequence of operations, each function citing the reference file:line it
  follows. On CPU tensors this reproduces the reference's results bit for bit
  (pinned by tests/test_oracle_golden.py against fixtures produced by the
  reference modules themselves).
"""

from __future__ import annotations

import ctypes
import subprocess
from ctypes import POINTER, c_float, c_int, c_int64, c_long, c_uint8, c_uint16
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"


def build(force: bool = False) -> Path:
    src = HERE / "oracle.c"
    if force or not LIB.exists() or LIB.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-shared", "-fPIC",
                        "-o", str(LIB), str(src), "-lm"], check=True)
    return LIB


def _load() -> ctypes.CDLL:
    build()
    lib = ctypes.CDLL(str(LIB))
    vp = ctypes.c_void_p
    lib.oracle_dequant_fp8.argtypes = [vp, vp, c_int, c_int, c_int, c_int, vp]
    lib.oracle_decode_mxfp4.argtypes = [vp, vp, c_int, c_int, vp]
    lib.oracle_router_logits.argtypes = [vp, c_long, vp, vp, c_int, c_int, c_int, c_int, vp]
    lib.oracle_topk.argtypes = [vp, c_int, c_int, c_int, vp]
    lib.oracle_permute.argtypes = [vp, c_int, c_int, c_int, vp, vp, vp, vp]
    lib.oracle_permute.restype = c_int
    lib.oracle_combine.argtypes = [vp, c_long, vp, vp, c_int, c_int, c_int, c_int, c_int, c_int64,
                                   c_int64, c_int, vp, vp]
    lib.oracle_f32_to_e4m3.argtypes = [ctypes.c_float]
    lib.oracle_f32_to_e4m3.restype = ctypes.c_uint8
    lib.oracle_act_quant_fp8.argtypes = [vp, c_long, vp, c_int, c_int, c_int, c_int, vp, vp]
    return lib


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = _load()
    return _lib


def _np(t: torch.Tensor, dtype) -> np.ndarray:
    return np.ascontiguousarray(t.detach().cpu().contiguous().view(dtype).numpy())


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def _bf16_tensor(a: np.ndarray, shape) -> torch.Tensor:
    return torch.from_numpy(a.astype(np.int16, copy=False).reshape(shape)).view(torch.bfloat16)


# --------------------------------------------------------------------------- exact stages
def dequant_fp8(w: torch.Tensor, scales: torch.Tensor, block) -> torch.Tensor:
    """bf16(fp32(w) * scale) per block (moe_serving/qwen3_parallel.py:48-53)."""
    rows, cols = w.shape
    wa = _np(w, torch.uint8)
    sa = np.ascontiguousarray(scales.detach().float().cpu().numpy())
    out = np.empty(rows * cols, np.uint16)
    lib().oracle_dequant_fp8(_p(wa), _p(sa), rows, cols, block[0], block[1], _p(out))
    return _bf16_tensor(out, (rows, cols))


def decode_mxfp4(blocks: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """[..., G, 16] u8 + [..., G] u8 -> bf16 [..., G * 32] (before the transpose
    of transformers' _convert_moe_packed_tensors)."""
    *pre, G, _ = blocks.shape
    rows = int(np.prod(pre)) if pre else 1
    ba = _np(blocks, torch.uint8)
    sa = _np(scales, torch.uint8)
    out = np.empty(rows * G * 32, np.uint16)
    lib().oracle_decode_mxfp4(_p(ba), _p(sa), rows, G, _p(out))
    return _bf16_tensor(out, (*pre, G * 32))


def router_logits(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None, mode: int) -> torch.Tensor:
    """Fixed-order fp32 logits; mode 0 bf16, 1 bf16 with bias, 2 fp32 (float32 tensor)."""
    T, H = x.shape
    E = w.shape[0]
    xa, wa = _np(x, torch.int16), _np(w, torch.int16)
    ba = _np(bias, torch.int16) if bias is not None else None
    out = np.empty(T * E, np.float32)
    lib().oracle_router_logits(_p(xa), H, _p(wa), _p(ba) if ba is not None else None, T, H, E, mode,
                               _p(out))
    return torch.from_numpy(out.reshape(T, E))


def topk(values: torch.Tensor, k: int) -> torch.Tensor:
    """torch.topk(values, k).indices as computed on CUDA (k <= 32), including
    the slot order of equal values (oracle.c states the rule)."""
    T, E = values.shape
    va = np.ascontiguousarray(values.detach().float().cpu().numpy())
    out = np.empty(T * k, np.int64)
    lib().oracle_topk(_p(va), T, E, k, _p(out))
    return torch.from_numpy(out.reshape(T, k))


def butterfly_sum(v: torch.Tensor) -> torch.Tensor:
    """Row sums of v [T, K] (float32) in the order torch's CUDA sum over a row
    of K values uses (xor-butterfly over the next power of two, zero padded):
    ((v0 + v4) + (v2 + v6)) + ((v1 + v5) + (v3 + v7)) at K = 8. Pinned against
    torch's outputs by tests/golden/router_torch_cuda.pt for K = 2 and 8."""
    T, K = v.shape
    P = 1
    while P < K:
        P <<= 1
    lanes = torch.zeros(T, P, dtype=torch.float32)
    lanes[:, :K] = v.float()
    ids = torch.arange(P)
    o = P >> 1
    while o >= 1:
        lanes = lanes + lanes[:, ids ^ o]
        o >>= 1
    return lanes[:, 0]


def qwen_select(probs: torch.Tensor, k: int, normalize: bool):
    """torch.topk of the fp32 probabilities on CUDA (slot order of ties
    included) and the renormalised scores (transformers
    qwen3_moe/modeling_qwen3_moe.py:266-269)."""
    idx = topk(probs, k)
    top = torch.gather(probs.float().cpu(), 1, idx)
    if normalize:
        top = top / butterfly_sum(top)[:, None]
    return idx, top


def permute(indices: torch.Tensor, num_experts: int):
    """(counts, offsets, perm_src, inverse) in (expert, slot, token) order."""
    T, K = indices.shape
    ia = _np(indices.to(torch.int64), torch.int64)
    counts = np.empty(num_experts, np.int32)
    offsets = np.empty(num_experts + 1, np.int32)
    perm = np.zeros(T * K, np.int32)
    inv = np.empty(T * K, np.int32)
    lib().oracle_permute(_p(ia), T, K, num_experts, _p(counts), _p(offsets), _p(perm), _p(inv))
    return tuple(torch.from_numpy(a) for a in (counts, offsets, perm, inv))


def combine(rows: torch.Tensor, inverse: torch.Tensor, indices: torch.Tensor, *, order: int = 0,
            experts_per_rank: int = 1, lo: int = 0, hi: int = 1 << 62,
            weights: torch.Tensor | None = None) -> torch.Tensor:
    """Ordered bf16 combine (parallel_numerics.py:26-35, moe.py:123-136)."""
    T, K = indices.shape
    H = rows.shape[1]
    ra = _np(rows, torch.int16)
    inv = _np(inverse.to(torch.int32), torch.int32)
    ia = _np(indices.to(torch.int64), torch.int64)
    wa = np.ascontiguousarray(weights.detach().float().cpu().numpy()) if weights is not None else None
    out = np.empty(T * H, np.uint16)
    lib().oracle_combine(_p(ra), rows.stride(0), _p(inv), _p(ia), T, K, H, order, experts_per_rank,
                         lo, hi, int(weights is not None), _p(wa) if wa is not None else None,
                         _p(out))
    return _bf16_tensor(out, (T, H))


def slot_sum(values: torch.Tensor) -> torch.Tensor:
    """bf16 [T, K, H] -> bf16 [T, H]: torch's CUDA ``sum(1)`` over the slot
    dimension, restated. With the slots strided (H elements apart) each
    output is reduced by one thread with four fp32 accumulators in flight:
    slot k adds into a[k % 4] in ascending k, then ((a0 + a1) + a2) + a3,
    one rounding to bf16. Pinned to torch's recorded CUDA outputs
    (tests/golden/slot_sum_torch_cuda.pt)."""
    T, K, H = values.shape
    acc = torch.zeros(4, T, H, dtype=torch.float32)
    for k in range(K):
        acc[k % 4] = acc[k % 4] + values[:, k].float()
    return (((acc[0] + acc[1]) + acc[2]) + acc[3]).to(torch.bfloat16)


def w8a8_local_combine(rows: torch.Tensor, inverse: torch.Tensor, indices: torch.Tensor,
                       weights: torch.Tensor | None, lo: int = 0, hi: int = 1 << 62) -> torch.Tensor:
    """The local combine of grouped_fp8 (moe_serving/efficient_kernels.py:269-273):
    contribution rows in permuted order times bf16 routing weights (one bf16
    rounding), rows of dropped slots and of experts outside [lo, hi) zero,
    then slot_sum over each token's K slots."""
    T, K = indices.shape
    inv = inverse.long().reshape(-1)
    e = indices.reshape(-1).long()
    valid = (inv >= 0) & (e >= lo) & (e < hi)
    vals = rows[inv.clamp(min=0)]
    if weights is not None:
        vals = vals * weights.reshape(-1, 1).to(torch.bfloat16)
    vals = vals.masked_fill(~valid[:, None], 0)
    return slot_sum(vals.reshape(T, K, -1))


def f32_to_e4m3_c(values: torch.Tensor) -> torch.Tensor:
    """e4m3fn codes (uint8) of fp32 values from the C encoder (round to
    nearest even, saturating at +-448)."""
    f = lib().oracle_f32_to_e4m3
    flat = values.detach().float().cpu().reshape(-1).tolist()
    return torch.tensor([f(v) for v in flat], dtype=torch.uint8).reshape(values.shape)


def act_quant_fp8_c(x: torch.Tensor, k_pad: int | None = None, rows_src: torch.Tensor | None = None,
                    src_div: int = 1) -> tuple[torch.Tensor, torch.Tensor]:
    """The C restatement of ``act_quant_fp8``: (e4m3 codes as uint8 [rows, k_pad],
    fp32 scales [rows, ceil(k_pad / 128)])."""
    k_valid = x.shape[1]
    k_pad = k_valid if k_pad is None else k_pad
    xa = _np(x.to(torch.bfloat16), torch.int16)
    ma = _np(rows_src.to(torch.int32), torch.int32) if rows_src is not None else None
    rows = rows_src.numel() if rows_src is not None else x.shape[0]
    groups = -(-k_pad // 128)
    q = np.empty(rows * k_pad, np.uint8)
    sc = np.empty(rows * groups, np.float32)
    lib().oracle_act_quant_fp8(_p(xa), k_valid, _p(ma) if ma is not None else None, src_div, rows, k_valid,
                               k_pad, _p(q), _p(sc))
    return torch.from_numpy(q.reshape(rows, k_pad)), torch.from_numpy(sc.reshape(rows, groups))


# --------------------------------------------------------------------------- reference FP math (torch)
def qwen_router(h: torch.Tensor, weight: torch.Tensor, top_k: int, norm_topk_prob: bool):
    """Qwen3MoeTopKRouter.forward (transformers qwen3_moe/modeling_qwen3_moe.py:263-272)."""
    logits = F.linear(h, weight)
    probs = torch.softmax(logits, dtype=torch.float, dim=-1)
    top_value, top_index = torch.topk(probs, top_k, dim=-1)
    if norm_topk_prob:
        top_value = top_value / top_value.sum(dim=-1, keepdim=True)
    return probs, top_value.to(probs.dtype), top_index, logits


def gpt_oss_router(h: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, top_k: int):
    """GptOssTopKRouter.forward (transformers gpt_oss/modeling_gpt_oss.py:126-131)."""
    logits = F.linear(h, weight, bias)
    top_value, top_index = torch.topk(logits, top_k, dim=-1)
    scores = torch.softmax(top_value, dim=1, dtype=top_value.dtype)
    return logits, scores, top_index


def native_route(h: torch.Tensor, gate_weight: torch.Tensor, top_k: int, renormalize: bool):
    """moe_serving/moe.py:97-107."""
    scores = torch.softmax(F.linear(h.float(), gate_weight.float()), dim=-1)
    weight, index = torch.topk(scores, top_k, dim=-1)
    if renormalize:
        weight = weight / weight.sum(dim=-1, keepdim=True).clamp_min(1e-20)
    return index.to(torch.int64), weight.to(h.dtype), scores


def qwen_project(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor,
                 w_down: torch.Tensor) -> torch.Tensor:
    """moe_serving/qwen3_parallel.py:84-94 with materialised bf16 weights."""
    gate, up = F.linear(x, torch.cat((w_gate, w_up), dim=0)).chunk(2, dim=-1)
    return F.linear(F.silu(gate) * up, w_down)


def gpt_oss_project(x: torch.Tensor, w_gate_up: torch.Tensor, b_gate_up: torch.Tensor,
                    w_down: torch.Tensor, b_down: torch.Tensor, alpha: float,
                    limit: float) -> torch.Tensor:
    """moe_serving/gpt_oss_parallel.py:195-204: w_gate_up [H, 2I] (interleaved
    columns), w_down [I, H]."""
    gate_up = x @ w_gate_up + b_gate_up
    gate, up = gate_up[..., ::2], gate_up[..., 1::2]
    gate = gate.clamp(max=limit)
    up = up.clamp(min=-limit, max=limit)
    glu = gate * torch.sigmoid(gate * alpha)
    return ((up + 1) * glu) @ w_down + b_down


def ordered_expert_merge(hidden: torch.Tensor, indices: torch.Tensor, weights: torch.Tensor,
                         project) -> torch.Tensor:
    """moe_serving/parallel_numerics.py:13-36 on one rank: experts ascending,
    rows in (slot, token) order, contribution bf16(y * w), bf16 index_add_."""
    result = torch.zeros_like(hidden)
    for expert in torch.unique(indices, sorted=True).tolist():
        slots, tokens = torch.where(indices.T == expert)
        values = project(expert, hidden[tokens])
        result.index_add_(0, tokens, (values * weights[tokens, slots, None]).to(hidden.dtype))
    return result


def qwen_layer(hidden, indices, weights, gate_w, gate_s, up_w, up_s, down_w, down_s, block):
    """Reference-numerics Qwen3 expert layer (FP8 block storage) on one rank."""
    cache = {}

    def project(e, x):
        if e not in cache:
            cache[e] = (dequant_torch(gate_w[e], gate_s[e], block), dequant_torch(up_w[e], up_s[e], block),
                        dequant_torch(down_w[e], down_s[e], block))
        g, u, d = cache[e]
        return qwen_project(x, g, u, d)

    return ordered_expert_merge(hidden, indices, weights, project)


def dequant_torch(w: torch.Tensor, scales: torch.Tensor, block, dtype=torch.bfloat16) -> torch.Tensor:
    """Torch form of moe_serving/qwen3_parallel.py:48-53 (works on any device)."""
    rows, cols = w.shape
    br, bc = block
    expanded = scales.float().repeat_interleave(br, 0).repeat_interleave(bc, 1)
    return (w.float() * expanded[:rows, :cols]).to(dtype)


def act_quant_fp8(x: torch.Tensor, k_pad: int | None = None, rows_src: torch.Tensor | None = None,
                  src_div: int = 1) -> tuple[torch.Tensor, torch.Tensor]:
    """Dynamic per-(row, 128-column group) FP8 activation quantisation of the
    W8A8 path (moe_serving/efficient_kernels.py:243-274 quantises the
    activations inside the hub ``matmul_grouped``, which is not vendored in
    the reference): s = amax / 448 per group (1 for an all-zero group),
    q = e4m3fn(x / s) with round-to-nearest-even, saturating at +-448.
    Columns k_valid .. k_pad - 1 quantise zeros."""
    xf = x.float()
    if rows_src is not None:
        xf = xf[rows_src.long() // src_div]
    rows, k = xf.shape
    k_pad = k if k_pad is None else k_pad
    groups = -(-k_pad // 128)
    xp = torch.zeros(rows, groups * 128, dtype=torch.float32)
    xp[:, :k] = xf
    g = xp.view(rows, groups, 128)
    amax = g.abs().amax(-1)
    scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    q = (g / scale[..., None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return q.view(rows, groups * 128)[:, :k_pad].contiguous(), scale


def w8a8_matmul(q: torch.Tensor, q_scale: torch.Tensor, w: torch.Tensor, w_scale: torch.Tensor,
                block) -> torch.Tensor:
    """One expert's W8A8 product in float64, the math of the hub
    finegrained-fp8 ``matmul_grouped`` that grouped_fp8 calls
    (moe_serving/efficient_kernels.py:255-265):
    D[n, f] = sum_g w_scale[f // br, g] * q_scale[n, g] * sum_{k in g} W[f, k] * q[n, k]
    over 128-column groups g. q: e4m3 [n, k_pad]; w: e4m3 [F, K] (K <= k_pad);
    w_scale: [ceil(F / br), ceil(K / 128)]. Returns float64 [n, F]."""
    br, bc = block
    assert bc == 128, "W8A8 groups are 128 columns"
    n, k_pad = q.shape
    F, K = w.shape
    groups = q_scale.shape[1]
    qf = torch.zeros(n, groups * 128, dtype=torch.float64)
    qf[:, :k_pad] = q.double()
    wf = torch.zeros(F, groups * 128, dtype=torch.float64)
    wf[:, :K] = w.double()
    sw = w_scale.double().repeat_interleave(br, 0)[:F]                     # [F, >= groups]
    out = torch.zeros(n, F, dtype=torch.float64)
    for g in range(groups):
        part = qf[:, g * 128:(g + 1) * 128] @ wf[:, g * 128:(g + 1) * 128].T
        gs = min(g, sw.shape[1] - 1)
        out += part * q_scale[:, g].double()[:, None] * sw[:, gs][None, :]
    return out


def qwen_w8a8_project(x: torch.Tensor, gate_w, gate_s, up_w, up_s, down_w, down_s, block,
                      k_pad_h: int, k_pad_i: int) -> torch.Tensor:
    """One expert of grouped_fp8 (moe_serving/efficient_kernels.py:255-265):
    dynamic FP8 quantisation of the token rows, W8A8 gate/up with a bf16
    output, bf16(silu(gate)) * up in bf16, quantisation of the activation,
    W8A8 down with a bf16 output."""
    q, qs = act_quant_fp8(x, k_pad=k_pad_h)
    gate = w8a8_matmul(q, qs, gate_w, gate_s, block).to(torch.bfloat16)
    up = w8a8_matmul(q, qs, up_w, up_s, block).to(torch.bfloat16)
    act = F.silu(gate.float()).to(torch.bfloat16) * up
    q2, qs2 = act_quant_fp8(act, k_pad=k_pad_i)
    return w8a8_matmul(q2, qs2, down_w, down_s, block).to(torch.bfloat16)


def qwen_w8a8_layer(hidden, indices, weights, gate_w, gate_s, up_w, up_s, down_w, down_s, block,
                    k_pad_h: int | None = None, k_pad_i: int | None = None):
    """W8A8 Qwen3 expert layer on one rank, grouped_fp8
    (moe_serving/efficient_kernels.py:243-273): each routed (token, slot)
    row through qwen_w8a8_project, the contributions bf16(y * bf16(w)),
    summed over each token's slots by slot_sum (fp32, one rounding)."""
    T, K = indices.shape
    H = hidden.shape[1]
    inter = gate_w.shape[1]
    k_pad_h = -(-H // 64) * 64 if k_pad_h is None else k_pad_h
    k_pad_i = -(-inter // 128) * 128 if k_pad_i is None else k_pad_i
    values = torch.zeros(T, K, H, dtype=torch.bfloat16)
    for e in torch.unique(indices, sorted=True).tolist():
        tok, slot = torch.where(indices == e)
        y = qwen_w8a8_project(hidden[tok], gate_w[e], gate_s[e], up_w[e], up_s[e], down_w[e], down_s[e],
                              block, k_pad_h, k_pad_i)
        values[tok, slot] = y * weights[tok, slot, None].to(torch.bfloat16)
    return slot_sum(values)


_E2M1 = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]


def decode_mxfp4_torch(blocks: torch.Tensor, scales: torch.Tensor, dtype=torch.bfloat16) -> torch.Tensor:
    """Torch form of the MXFP4 decode: [..., G, 16] -> [..., G*32] (any device)."""
    lut = torch.tensor(_E2M1, dtype=dtype, device=blocks.device)
    *pre, G, B = blocks.shape
    b = blocks.to(torch.int64)
    out = torch.empty(*pre, G, B * 2, dtype=dtype, device=blocks.device)
    out[..., 0::2] = lut[b & 15]
    out[..., 1::2] = lut[b >> 4]
    exp = scales.to(torch.int32) - 127
    out = torch.ldexp(out, exp[..., None])
    return out.reshape(*pre, G * B * 2)


def gpt_oss_layer(hidden, indices, weights, gu_blocks, gu_scales, gu_bias, dn_blocks, dn_scales,
                  dn_bias, alpha, limit):
    """Reference-numerics GPT-OSS expert layer (MXFP4 storage) on one rank:
    per used expert, decode (the transposed [H, 2I] / [I, H] matrices) then
    ``project`` (moe_serving/gpt_oss_parallel.py:183-204)."""

    def project(e, x):
        wgu = decode_mxfp4_torch(gu_blocks[e], gu_scales[e]).transpose(0, 1).contiguous()
        wdn = decode_mxfp4_torch(dn_blocks[e], dn_scales[e]).transpose(0, 1).contiguous()
        return gpt_oss_project(x, wgu, gu_bias[e], wdn, dn_bias[e], alpha, limit)

    return ordered_expert_merge(hidden, indices, weights, project)


def gpt_oss_layer_efficient(hidden, indices, weights, gu_blocks, gu_scales, gu_bias, dn_blocks, dn_scales,
                            dn_bias, alpha, limit):
    """The reference's efficient GPT-OSS numerics (grouped_mxfp4,
    moe_serving/efficient_kernels.py:157-206, with biases made fp32 at
    gpt_oss_parallel.py:438-446), restated from the published algorithm of the
    fused MXFP4 matmul it calls (the hub kernel is not vendored, so this
    restatement is not pinned to its outputs): per routed (token, slot), in
    float64 standing in for fp32 accumulation, gu = x W_gu^T + b_gu; gate =
    min(gu[0::2], limit), up = clamp(gu[1::2], -limit, limit); the
    intermediate bf16(gate / (1 + exp(-alpha gate)) * (up + 1)); y = a W_dn^T +
    b_dn; each (token, slot) row rounded to bf16 after the routing weight,
    bf16(w[t, k] * y), as the published matmul_ogs stores its gamma-scaled
    scatter rows in the output dtype before the grouped reduction; out[t] =
    bf16(sum over slots of those rows). On the reference's own check of this
    path (tests/helpers/check_grouped_ep.py shapes) the restatement's relative
    L2 against the fp32 module is 0.0028-0.0030, the hub kernel's recorded
    0.0029-0.0030 (tests/validation_results/efficient_grouped_ep.json);
    without the per-slot rounding it is 0.0023."""
    T, K = indices.shape
    x = hidden.double()
    out = torch.zeros(T, hidden.shape[1], dtype=torch.float64)
    wd = weights.double()
    for e in torch.unique(indices, sorted=True).tolist():
        rows = torch.nonzero(indices == e)          # (token, slot) pairs, token-major
        t, k = rows[:, 0], rows[:, 1]
        wgu = decode_mxfp4_torch(gu_blocks[e], gu_scales[e], torch.float64)   # [2I, H]
        wdn = decode_mxfp4_torch(dn_blocks[e], dn_scales[e], torch.float64)   # [H, I]
        gu = x[t] @ wgu.T + gu_bias[e].double()
        gate = gu[:, 0::2].clamp(max=limit)
        up = gu[:, 1::2].clamp(min=-limit, max=limit)
        a = (gate / (1 + torch.exp(-alpha * gate)) * (up + 1)).to(torch.bfloat16).double()
        y = a @ wdn.T + dn_bias[e].double()
        out.index_put_((t,), (y * wd[t, k, None]).to(torch.bfloat16).double(), accumulate=True)
    return out.to(torch.bfloat16)


def routed_forward_ranks(hiddens, gate_weight, gate_up, down, top_k, renormalize=True,
                         routes=None):
    """moe_serving/moe.py:171-224 (simulate_ranks) with the exchange of
    moe_serving/distributed.py:49-67: token all-to-all EP over len(hiddens)
    in-process ranks, SwiGLU experts gate_up [E, 2I, H], down [E, H, I] run
    per expert on the owning rank (moe.py:73-81); returns per-rank outputs.
    ``routes`` (a list of per-rank (index, weight)) replaces the router."""
    ep = len(hiddens)
    E = gate_weight.shape[0]
    epr = E // ep
    packed = []
    for r, hidden in enumerate(hiddens):
        if routes is None:
            index, weight, _ = native_route(hidden, gate_weight, top_k, renormalize)
        else:
            index, weight = routes[r]
        flat_index = index.reshape(-1)
        token_index = torch.arange(hidden.shape[0]).repeat_interleave(top_k)
        dest = torch.div(flat_index, epr, rounding_mode="floor")
        local = flat_index - dest * epr
        order = torch.argsort(dest, stable=True)
        packed.append(dict(hidden=hidden, weight=weight.reshape(-1), token_index=token_index,
                           order=order, send_hidden=hidden[token_index[order]],
                           send_expert=local[order],
                           send_counts=torch.bincount(dest, minlength=ep)))

    def exchange(payloads, splits):
        received = []
        for d in range(ep):
            chunks, counts = [], []
            for s_ in range(ep):
                count = int(splits[s_][d])
                start = int(splits[s_][:d].sum())
                chunks.append(payloads[s_][start:start + count])
                counts.append(count)
            received.append((torch.cat(chunks), torch.tensor(counts)))
        return received

    recv_h = exchange([p["send_hidden"] for p in packed], [p["send_counts"] for p in packed])
    recv_e = exchange([p["send_expert"] for p in packed], [p["send_counts"] for p in packed])
    computed, counts = [], []
    for rank, ((rows, _), (ids, rc)) in enumerate(zip(recv_h, recv_e)):
        out = rows.new_empty(rows.shape[0], down.shape[1])
        for e in ids.unique().tolist():
            mask = ids == e
            g, u = F.linear(rows[mask], gate_up[rank * epr + e]).chunk(2, dim=-1)
            out[mask] = F.linear(F.silu(g) * u, down[rank * epr + e])
        computed.append(out)
        counts.append(rc)
    returned = exchange(computed, counts)
    outs = []
    for p, (rows, _) in zip(packed, returned):
        combined = p["hidden"].new_zeros(p["hidden"].shape)
        combined.index_add_(0, p["token_index"][p["order"]],
                            rows * p["weight"][p["order"]].unsqueeze(-1).to(rows.dtype))
        outs.append(combined)
    return outs
