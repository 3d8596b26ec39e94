"""The expert layer pipeline on one GPU: permute -> gate/up GEMM -> down GEMM.

``run_experts`` computes, for the experts of one rank, the contribution row
``bf16(bf16(y) * w)`` of every (token, slot) routed to them, in the global
permuted row order (expert-major, then slot, then token). The caller combines
the rows (``ops.combine``) after any expert-parallel exchange.

Launch shapes (the token tile) come from ``tile_policy``, which depends only
on T, K and the global expert count — not on the expert-parallel size. Each
output element is one fp32 tensor-core accumulation over K in increasing
order, so a token's expert outputs are bitwise the same whether its experts
run on 1 or 8 GPUs.
"""

from __future__ import annotations

import math
from functools import lru_cache

import torch

from moe_serving_profile_b200 import _lib, ops
from moe_serving_profile_b200.layout import ExpertWeights


@lru_cache(maxsize=None)
def _sm_count(device: int) -> int:
    return torch.cuda.get_device_properties(device).multi_processor_count


def tile_policy(T: int, K: int, num_experts: int, max_tile: int = 256, cover: float = 1.5) -> int:
    """Token tile (the MMA N) for one grouped GEMM launch: the smallest power
    of two in [16, max_tile] covering ``cover`` x the mean rows per expert, so
    that one tile usually holds an expert's rows (a second, nearly empty tile
    costs a whole tile's k-block loop: 512 tokens with 32-token tiles took
    2.3x the time of 64-token tiles on B200; the W8A8 gate/up GEMM at 512
    tokens: 64-token tiles 138 us, 32-token tiles 150 us)."""
    rows = cover * T * K / num_experts
    bn = 16
    while bn < max_tile and bn < rows:
        bn *= 2
    return min(bn, max_tile)


def _max_tile(w: ExpertWeights) -> int:
    # quantised weights: at most 160 tokens, the largest tile whose two
    # accumulator slots fit beside the converted-weight stages in tensor
    # memory. (256-row tiles exist, with the converted weights in shared
    # memory instead, but measured no faster: both operands then come from
    # shared memory, whose operand bandwidth holds a 128 x 256 x 16 MMA to
    # 171 cycles against 138 with the weights in tensor memory.)
    return 256 if w.fmt == _lib.W_BF16 else 160


def run_experts(w: ExpertWeights, hidden: torch.Tensor, perm: ops.Permutation,
                weights: torch.Tensor | None, *, K: int, num_experts: int, expert_begin: int,
                contrib: torch.Tensor | None = None, b_map_div: int | None = None,
                tile_tokens: int | None = None) -> torch.Tensor:
    """Contribution rows [T*K, H] (rows of other ranks' experts are left as given).

    ``hidden`` rows are gathered through ``perm.perm_src // K``; ``weights``
    ([T, K], fp32 or bf16) scale the down projection's rows, or are skipped
    when None (the token all-to-all path scales at combine time).
    ``tile_tokens`` (default: the rows of ``hidden``) is the batch the token
    tile is chosen for; with the global batch, outputs are bitwise those of
    one GPU running it whole.
    """
    T, H = hidden.shape
    if H != w.hidden:
        raise ValueError(f"hidden size {H} does not match the experts' {w.hidden}")
    tokens = T if tile_tokens is None else tile_tokens
    act = gate_up(w, hidden, perm, K=K, num_experts=num_experts, expert_begin=expert_begin,
                  b_map_div=b_map_div, tokens=tokens)
    return down(w, act, perm, weights, K=K, num_experts=num_experts, expert_begin=expert_begin,
                contrib=contrib, tokens=tokens)


def gate_up(w: ExpertWeights, hidden: torch.Tensor, perm: ops.Permutation, *, K: int,
            num_experts: int, expert_begin: int, b_map_div: int | None = None,
            tokens: int | None = None, out: torch.Tensor | None = None,
            epilogue: int | None = None) -> torch.Tensor:
    """Gated projection of every routed row: act [T*K, I_p] bf16."""
    T = hidden.shape[0] if tokens is None else tokens
    R = perm.perm_src.numel()
    dev = hidden.device
    bn = tile_policy(T, K, num_experts, _max_tile(w))
    div = K if b_map_div is None else b_map_div
    act = torch.empty(R, w.i_pad, device=dev, dtype=torch.bfloat16) if out is None else out
    if bn >= 64 or w.fmt != _lib.W_BF16:
        # gather the routed rows once into permuted order: large token tiles
        # read them as plain 2D tiles instead of per-row gathers, and the
        # decode kernel of quantised weights reads contiguous rows only
        b_src = ops.gather_rows(hidden, perm.perm_src, div, offsets=perm.offsets,
                                expert_lo=expert_begin, expert_hi=expert_begin + w.n_experts)
        b_map, b_div = None, 1
    else:
        b_src, b_map, b_div = hidden, perm.perm_src, div
    ops.expert_gemm(offsets=perm.offsets, expert_begin=expert_begin, n_experts=w.n_experts,
                    max_rows=R, wfmt=w.fmt, planes=2, feat_pad=w.i_pad, n_feat=w.inter,
                    k_pad=w.h_k, weight=w.w1, fp8_block=w.block, b_src=b_src,
                    k_valid=hidden.shape[1], b_map=b_map, b_div=b_div,
                    epilogue=w.gated_epilogue if epilogue is None else epilogue, bias=w.b1,
                    alpha=w.alpha, limit=w.limit, out=act, token_tile=bn)
    return act


def down(w: ExpertWeights, act: torch.Tensor, perm: ops.Permutation,
         weights: torch.Tensor | None, *, K: int, num_experts: int, expert_begin: int,
         contrib: torch.Tensor | None = None, tokens: int) -> torch.Tensor:
    """Down projection of the gated rows, scaled by the routing weights."""
    R = perm.perm_src.numel()
    dev = act.device
    bn = tile_policy(tokens, K, num_experts, _max_tile(w))
    if contrib is None:
        contrib = torch.empty(R, w.hidden, device=dev, dtype=torch.bfloat16)
    ops.expert_gemm(offsets=perm.offsets, expert_begin=expert_begin, n_experts=w.n_experts,
                    max_rows=R, wfmt=w.fmt, planes=1, feat_pad=w.h_f, n_feat=w.hidden,
                    k_pad=w.i_pad, weight=w.w2, fp8_block=w.block, b_src=act,
                    k_valid=w.inter, epilogue=_lib.EPI_DOWN, bias=w.b2,
                    row_weight=None if weights is None else weights.reshape(-1),
                    row_src=perm.perm_src, out=contrib, token_tile=bn)
    return contrib


def run_experts_w8a8(w: ExpertWeights, hidden: torch.Tensor, perm: ops.Permutation,
                     weights: torch.Tensor | None, *, K: int, num_experts: int, expert_begin: int,
                     contrib: torch.Tensor | None = None,
                     b_map_div: int | None = None) -> torch.Tensor:
    """``run_experts`` in the reference's efficient FP8 numerics (W8A8,
    moe_serving/efficient_kernels.py:243-274): the routed token rows and the
    gated activations are quantised to e4m3 per (row, 128-column group) and
    multiplied with the e4m3 weights on the tensor cores; FP32 block scales
    of both sides are applied per group in fp32. With ``weights`` the rows
    are bf16(bf16(y) * w); grouped_fp8's own combine takes them unscaled
    (weights None) and scales them by bf16(w) in the slot-sum combine."""
    if w.fmt != _lib.W_FP8 or w.block[1] != 128 or w.block[0] % 64:
        raise ValueError("W8A8 needs FP8 weights with scale blocks of 128 columns (rows a multiple of 64)")
    T, H = hidden.shape
    if H != w.hidden:
        raise ValueError(f"hidden size {H} does not match the experts' {w.hidden}")
    R = perm.perm_src.numel()
    dev = hidden.device
    bn = tile_policy(T, K, num_experts, 128)
    div = K if b_map_div is None else b_map_div
    # only this rank's rows are quantised (other ranks' rows are never read)
    lo, hi = expert_begin, expert_begin + w.n_experts
    local = dict(offsets=perm.offsets, expert_lo=lo, expert_hi=hi) if (lo, hi) != (0, num_experts) else {}
    q, qs = ops.act_quant_fp8(hidden, k_pad=w.h_k, rows_src=perm.perm_src, src_div=div, **local)
    act = torch.empty(R, w.i_pad, device=dev, dtype=torch.bfloat16)
    ops.w8a8_gemm(offsets=perm.offsets, expert_begin=expert_begin, n_experts=w.n_experts, max_rows=R,
                  planes=2, feat_pad=w.i_pad, n_feat=w.inter, k_pad=w.h_k, weight=w.w1,
                  fp8_block=w.block, q=q, q_scale=qs, epilogue=_lib.EPI_SWIGLU, out=act,
                  token_tile=bn)
    q2, qs2 = ops.act_quant_fp8(act[:, :w.inter], k_pad=w.i_pad, **local)
    if contrib is None:
        contrib = torch.empty(R, w.hidden, device=dev, dtype=torch.bfloat16)
    ops.w8a8_gemm(offsets=perm.offsets, expert_begin=expert_begin, n_experts=w.n_experts, max_rows=R,
                  planes=1, feat_pad=w.h_f, n_feat=w.hidden, k_pad=w.i_pad, weight=w.w2,
                  fp8_block=w.block, q=q2, q_scale=qs2, epilogue=_lib.EPI_DOWN,
                  row_weight=None if weights is None else weights.reshape(-1),
                  row_src=perm.perm_src, out=contrib, token_tile=bn)
    return contrib


def run_experts_mxfp4_efficient(w: ExpertWeights, hidden: torch.Tensor, perm: ops.Permutation,
                                weights: torch.Tensor, indices: torch.Tensor, *, K: int, num_experts: int,
                                expert_begin: int) -> torch.Tensor:
    """The reference's fused MXFP4 experts (grouped_mxfp4, matmul_ogs with a
    fused clamped SwiGLU and fp32 biases; moe_serving/efficient_kernels.py:157-206,
    biases made fp32 at gpt_oss_parallel.py:438-446): the gate/up epilogue
    works in fp32 and rounds once to bf16, the down projection keeps
    acc + bias in fp32, each (token, slot) row is scaled by its routing
    weight and rounded to bf16 (the output dtype matmul_ogs stores it in),
    and each token's rows are summed in fp32 in slot order, rounded once.
    Returns this rank's [T, H] bf16 partial (its experts only)."""
    T, H = hidden.shape
    act = gate_up(w, hidden, perm, K=K, num_experts=num_experts, expert_begin=expert_begin, tokens=T,
                  epilogue=_lib.EPI_CLAMP_SWIGLU_F32)
    R = perm.perm_src.numel()
    bn = tile_policy(T, K, num_experts, _max_tile(w))
    y = torch.empty(R, w.hidden, device=hidden.device, dtype=torch.float32)
    ops.expert_gemm(offsets=perm.offsets, expert_begin=expert_begin, n_experts=w.n_experts,
                    max_rows=R, wfmt=w.fmt, planes=1, feat_pad=w.h_f, n_feat=w.hidden,
                    k_pad=w.i_pad, weight=w.w2, fp8_block=w.block, b_src=act,
                    k_valid=w.inter, epilogue=_lib.EPI_DOWN_F32, bias=w.b2, out=y, token_tile=bn)
    return ops.combine_f32(y, perm.inverse, indices, weights, expert_lo=expert_begin,
                           expert_hi=expert_begin + w.n_experts)


def check_inputs(hidden: torch.Tensor, indices: torch.Tensor, weights: torch.Tensor) -> tuple:
    if hidden.dtype != torch.bfloat16:
        raise ValueError(f"b200 experts compute in bfloat16, got hidden {hidden.dtype}")
    if hidden.dim() != 2:
        raise ValueError("hidden must be [tokens, hidden]")
    if hidden.stride(1) != 1 or hidden.stride(0) % 8:
        hidden = hidden.contiguous()
    indices = indices.to(torch.int64).contiguous()
    weights = weights.contiguous()
    if weights.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError(f"routing weights must be float32 or bfloat16, got {weights.dtype}")
    if indices.shape != weights.shape or indices.shape[0] != hidden.shape[0]:
        raise ValueError("indices / routing weights / hidden shapes disagree")
    return hidden, indices, weights


def layer_forward(w: ExpertWeights, hidden: torch.Tensor, indices: torch.Tensor,
                  weights: torch.Tensor, *, num_experts: int, expert_begin: int,
                  parallel=None, numerics: str = "reference") -> torch.Tensor:
    """Replicated-token expert layer: the reference's ``ParallelExperts.forward``.

    numerics "reference": contributions of all experts reach every rank and
    are combined in ascending global expert order (bitwise independent of the
    EP size, the contract of moe_serving/parallel_numerics.py:13-36).
    numerics "fast": each rank combines its own experts and the partial sums
    are all-reduced (moe_serving/qwen3_parallel.py:105-118).
    numerics "efficient": FP8 weights run the W8A8 experts of the reference's
    grouped_fp8 (moe_serving/efficient_kernels.py:243-274) with its fp32
    slot-sum combine; GPT-OSS MXFP4 weights its fused path (grouped_mxfp4,
    :157-206: fp32 epilogues and an fp32 slot-order scatter-reduce); the
    rank partials of both are all-reduced.
    """
    hidden, indices, weights = check_inputs(hidden, indices, weights)
    T, K = indices.shape
    if T == 0:
        return torch.empty_like(hidden)
    size = 1 if parallel is None else parallel.size
    fused_mx = numerics == "efficient" and w.fmt == _lib.W_MXFP4 and \
        w.gated_epilogue == _lib.EPI_CLAMP_SWIGLU
    if size == 1 and numerics in ("reference", "fast") or (
            size == 1 and numerics == "efficient" and w.fmt == _lib.W_BF16):
        # one library call: permutation, gather, both GEMMs and the ordered
        # combine (the same kernels and results as the separate calls)
        return ops.expert_layer(w, hidden, indices, weights, num_experts=num_experts,
                                expert_begin=expert_begin)
    perm = ops.permute(indices, num_experts)
    if fused_mx:
        # GPT-OSS MXFP4: the fused path's fp32 epilogues and fp32 slot-order
        # scatter-reduce (grouped_mxfp4), then the all-reduce of the rank
        # partials (efficient_kernels.py:206)
        part = run_experts_mxfp4_efficient(w, hidden, perm, weights, indices, K=K,
                                           num_experts=num_experts, expert_begin=expert_begin)
        return part if size == 1 else parallel.reduce(part)
    if numerics == "efficient" and w.fmt == _lib.W_FP8:
        # W8A8 experts (grouped_fp8) with its local combine: unscaled rows
        # times bf16 routing weights, fp32 sum over each token's slots, one
        # rounding (efficient_kernels.py:269-273), then the all-reduce of the
        # rank partials (:274)
        y = run_experts_w8a8(w, hidden, perm, None, K=K, num_experts=num_experts, expert_begin=expert_begin)
        part = ops.combine(y, perm.inverse, indices, order=_lib.ORDER_SLOT_SUM, expert_lo=expert_begin,
                           expert_hi=expert_begin + w.n_experts, weights=weights)
        return part if size == 1 else parallel.reduce(part)
    if numerics == "efficient":
        # BF16 weights: the weight-only experts; the rank-local partial sums
        # are all-reduced, the reference's efficient EP exchange
        # (efficient_kernels.py:206, 274).
        contrib = run_experts(w, hidden, perm, weights, K=K, num_experts=num_experts,
                              expert_begin=expert_begin)
        if size == 1:
            return ops.combine(contrib, perm.inverse, indices, order=_lib.ORDER_EXPERT)
        return parallel.combine_reduce(contrib, perm.inverse, indices, expert_begin,
                                       expert_begin + w.n_experts)
    if numerics == "reference":
        g = parallel.gather_rows_buffer(hidden.device, hidden.shape[1], T * K)
        if g is not None:
            # The down GEMM writes this rank's experts' rows into its gather
            # area; every rank copies them to the same rows of the others'
            # areas over NVLink, then combines all rows in global expert order.
            contrib = g.area_a[:T * K]
            run_experts(w, hidden, perm, weights, K=K, num_experts=num_experts,
                        expert_begin=expert_begin, contrib=contrib)
            ops.ep_gather(g, perm.offsets, expert_begin, expert_begin + w.n_experts, T * K)
            return ops.combine(contrib, perm.inverse, indices, order=_lib.ORDER_EXPERT)
        # Rows of other ranks' experts start at zero, so a SUM all-reduce is an
        # exact gather of every expert's contribution rows.
        contrib = torch.zeros(T * K, hidden.shape[1], device=hidden.device, dtype=torch.bfloat16)
        run_experts(w, hidden, perm, weights, K=K, num_experts=num_experts,
                    expert_begin=expert_begin, contrib=contrib)
        parallel.reduce(contrib)
        return ops.combine(contrib, perm.inverse, indices, order=_lib.ORDER_EXPERT)
    if numerics == "fast":
        contrib = run_experts(w, hidden, perm, weights, K=K, num_experts=num_experts,
                              expert_begin=expert_begin)
        # combine of the local experts + SUM over the group: one NVLink kernel
        # (parallel.combine_reduce) or combine + NCCL all-reduce
        return parallel.combine_reduce(contrib, perm.inverse, indices, expert_begin,
                                       expert_begin + w.n_experts)
    raise ValueError(f"numerics must be reference, fast or efficient, got {numerics!r}")
