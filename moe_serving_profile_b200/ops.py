"""Torch-facing wrappers of the b200moe C ABI.

Each function takes CUDA tensors, allocates its outputs with torch's caching
allocator and enqueues the kernels on the current stream of the tensors'
device. Nothing here synchronises the host. Tensors on any other device are
rejected: the library has no CPU implementation.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from moe_serving_profile_b200 import _lib
from moe_serving_profile_b200._lib import check, lib


def _dev(t: torch.Tensor, what: str) -> int:
    if not t.is_cuda:
        raise ValueError(f"{what} must be a CUDA tensor (b200moe has no CPU path), got {t.device}")
    return t.device.index


def _stream(device: int) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _bf16_rows(t: torch.Tensor, what: str) -> None:
    if t.dtype != torch.bfloat16:
        raise ValueError(f"{what} must be bfloat16, got {t.dtype}")
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{what} must be a 2D tensor with contiguous rows")


# --------------------------------------------------------------------------- router
@dataclass
class RouterOut:
    logits: torch.Tensor     # bf16 [T,E] (qwen3 / gpt_oss) or fp32 [T,E] (native)
    probs: torch.Tensor | None   # fp32 [T,E] (qwen3)
    scores: torch.Tensor     # fp32 [T,K] (qwen3) or bf16 [T,K]
    indices: torch.Tensor    # int64 [T,K]
    counts: torch.Tensor     # int32 [E]


def router(mode: int, hidden: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None,
           top_k: int, normalize: bool, logits: torch.Tensor | None = None) -> RouterOut:
    """Fused router; with ``logits`` given, only the selection stage runs."""
    device = _dev(weight if logits is None else logits, "router input")
    E = weight.shape[0] if weight is not None else logits.shape[1]
    if logits is None:
        _bf16_rows(hidden, "hidden")
        _bf16_rows(weight, "router weight")
        if not weight.is_contiguous():
            raise ValueError("router weight must be contiguous")
        T, H = hidden.shape
        if weight.shape[1] != H:
            raise ValueError(f"router weight {tuple(weight.shape)} does not match hidden size {H}")
        ldt = torch.float32 if mode == _lib.ROUTER_NATIVE else torch.bfloat16
        logits_t = torch.empty(T, E, device=hidden.device, dtype=ldt)
        given = 0
    else:
        T, H = logits.shape[0], 0
        want = torch.float32 if mode == _lib.ROUTER_NATIVE else torch.bfloat16
        if logits.dtype != want or not logits.is_contiguous():
            raise ValueError(f"logits must be contiguous {want}")
        logits_t = logits
        given = 1
    if bias is not None:
        if bias.dtype != torch.bfloat16 or not bias.is_contiguous():
            raise ValueError("router bias must be contiguous bfloat16")
    dev = logits_t.device
    probs = torch.empty(T, E, device=dev, dtype=torch.float32) if mode == _lib.ROUTER_QWEN3 else None
    sdt = torch.float32 if mode == _lib.ROUTER_QWEN3 else torch.bfloat16
    scores = torch.empty(T, top_k, device=dev, dtype=sdt)
    indices = torch.empty(T, top_k, device=dev, dtype=torch.int64)
    counts = torch.empty(E, device=dev, dtype=torch.int32)
    check(
        lib.b200moe_router(
            device, _stream(device), mode,
            _ptr(hidden) if given == 0 else None, hidden.stride(0) if given == 0 else 0,
            _ptr(weight) if given == 0 else None, _ptr(bias),
            T, H, E, top_k, int(normalize),
            _ptr(logits_t), _ptr(probs), _ptr(scores), _ptr(indices), _ptr(counts), given,
        ),
        "router",
    )
    return RouterOut(logits_t, probs, scores, indices, counts)


def route_record(indices: torch.Tensor, scores: torch.Tensor,
                 out_indices: torch.Tensor | None = None,
                 out_scores: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """(int16 expert ids, fp16 routing weights) of one router call, on the device."""
    device = _dev(indices, "indices")
    if indices.dtype != torch.int64 or not indices.is_contiguous():
        raise ValueError("indices must be contiguous int64")
    if scores.dtype not in (torch.float32, torch.bfloat16) or not scores.is_contiguous():
        raise ValueError("scores must be contiguous float32 or bfloat16")
    if scores.shape != indices.shape:
        raise ValueError("indices and scores shapes differ")
    if out_indices is None:
        out_indices = torch.empty(indices.shape, device=indices.device, dtype=torch.int16)
    if out_scores is None:
        out_scores = torch.empty(indices.shape, device=indices.device, dtype=torch.float16)
    check(
        lib.b200moe_route_record(device, _stream(device), _ptr(indices), _ptr(scores),
                                 int(scores.dtype == torch.bfloat16), indices.numel(),
                                 _ptr(out_indices), _ptr(out_scores)),
        "route_record",
    )
    return out_indices, out_scores


def act_quant_fp8(x: torch.Tensor, k_pad: int | None = None, rows_src: torch.Tensor | None = None,
                  src_div: int = 1, offsets: torch.Tensor | None = None, expert_lo: int = 0,
                  expert_hi: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """Dynamic FP8 activation quantisation of the W8A8 FP8 path: e4m3 ``q``
    [rows, k_pad] and fp32 ``scales`` [rows, ceil(k_pad / 128)], one scale per
    row and 128-column group (amax / 448). With ``rows_src`` (int32), row r
    quantises ``x[rows_src[r] // src_div]`` (the permuted-row gather). With
    ``offsets`` (the permutation's device offsets), only the rows
    [offsets[expert_lo], offsets[expert_hi]) are written."""
    device = _dev(x, "x")
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be a 2-D bfloat16 tensor with unit column stride")
    k_valid = x.shape[1]
    k_pad = k_valid if k_pad is None else k_pad
    rows = x.shape[0]
    if rows_src is not None:
        _dev(rows_src, "rows_src")
        if rows_src.dtype != torch.int32 or not rows_src.is_contiguous() or rows_src.dim() != 1:
            raise ValueError("rows_src must be contiguous 1-D int32")
        rows = rows_src.numel()
    if offsets is not None:
        _dev(offsets, "offsets")
        if offsets.dtype != torch.int32 or not 0 <= expert_lo <= expert_hi < offsets.numel():
            raise ValueError("offsets must be int32 with 0 <= expert_lo <= expert_hi < offsets.numel()")
    q = torch.empty((rows, k_pad), device=x.device, dtype=torch.float8_e4m3fn)
    s = torch.empty((rows, -(-k_pad // 128)), device=x.device, dtype=torch.float32)
    check(
        lib.b200moe_act_quant_fp8(device, _stream(device), _ptr(x), x.stride(0), _ptr(rows_src),
                                  int(src_div), rows, k_valid, k_pad, _ptr(q), _ptr(s), _ptr(offsets),
                                  int(expert_lo), int(expert_hi)),
        "act_quant_fp8",
    )
    return q, s


# --------------------------------------------------------------------------- permutation
@dataclass
class Permutation:
    counts: torch.Tensor     # int32 [E]
    offsets: torch.Tensor    # int32 [E+1]
    perm_src: torch.Tensor   # int32 [T*K]: permuted row -> t*K + k
    inverse: torch.Tensor    # int32 [T*K]: t*K + k -> permuted row (-1 dropped)


def permute(indices: torch.Tensor, num_experts: int) -> Permutation:
    device = _dev(indices, "indices")
    if indices.dtype != torch.int64 or indices.dim() != 2 or not indices.is_contiguous():
        raise ValueError("indices must be a contiguous int64 [T, K] tensor")
    T, K = indices.shape
    dev = indices.device
    counts = torch.empty(num_experts, device=dev, dtype=torch.int32)
    offsets = torch.empty(num_experts + 1, device=dev, dtype=torch.int32)
    perm_src = torch.empty(T * K, device=dev, dtype=torch.int32)
    inverse = torch.empty(T * K, device=dev, dtype=torch.int32)
    nbytes = ctypes.c_size_t(0)
    check(lib.b200moe_permute_workspace(T, K, num_experts, ctypes.byref(nbytes)), "permute_workspace")
    ws = torch.empty(max(nbytes.value, 1), device=dev, dtype=torch.uint8)
    check(
        lib.b200moe_permute(
            device, _stream(device), _ptr(indices), T, K, num_experts, _ptr(counts), _ptr(offsets),
            _ptr(perm_src), _ptr(inverse), _ptr(ws), nbytes.value,
        ),
        "permute",
    )
    return Permutation(counts, offsets, perm_src, inverse)


def permute_noalloc(indices: torch.Tensor, num_experts: int, out: Permutation) -> Permutation:
    """``permute`` into caller-owned buffers, with no allocation in the call:
    the chunk histograms use the library's fixed per-device scratch
    (``_lib.PERMUTE_SCRATCH_BYTES``). Calls on one device must not overlap in
    time; shapes needing more scratch raise NotImplementedError."""
    device = _dev(indices, "indices")
    if indices.dtype != torch.int64 or indices.dim() != 2 or not indices.is_contiguous():
        raise ValueError("indices must be a contiguous int64 [T, K] tensor")
    T, K = indices.shape
    want = {"counts": num_experts, "offsets": num_experts + 1, "perm_src": T * K, "inverse": T * K}
    for name, n in want.items():
        t = getattr(out, name)
        if t.dtype != torch.int32 or not t.is_contiguous() or t.numel() != n or t.device != indices.device:
            raise ValueError(f"out.{name} must be a contiguous int32 tensor of {n} elements on {indices.device}")
    check(
        lib.b200moe_permute_noalloc(
            device, _stream(device), _ptr(indices), T, K, num_experts, _ptr(out.counts),
            _ptr(out.offsets), _ptr(out.perm_src), _ptr(out.inverse),
        ),
        "permute_noalloc",
    )
    return out


# --------------------------------------------------------------------------- grouped GEMM
def expert_gemm(*, offsets: torch.Tensor, expert_begin: int, n_experts: int, max_rows: int,
                wfmt: int, planes: int, feat_pad: int, n_feat: int, k_pad: int,
                weight: torch.Tensor, fp8_block: tuple[int, int] = (128, 128),
                b_src: torch.Tensor, k_valid: int, b_map: torch.Tensor | None = None,
                b_rows: int | None = None,
                b_div: int = 1, epilogue: int, bias: torch.Tensor | None = None,
                alpha: float = 1.702, limit: float = 7.0, row_weight: torch.Tensor | None = None,
                row_src: torch.Tensor | None = None, out: torch.Tensor,
                token_tile: int = 0, split_k: int = 0) -> torch.Tensor:
    device = _dev(weight, "weight")
    _bf16_rows(b_src, "activations")
    if epilogue == _lib.EPI_DOWN_F32:
        if out.dtype != torch.float32 or out.dim() != 2 or out.stride(1) != 1:
            raise ValueError("the fp32 down epilogue writes a 2D float32 output with contiguous rows")
    else:
        _bf16_rows(out, "output")
    a = _lib.GemmArgs()
    a.offsets = _ptr(offsets)
    a.expert_begin = expert_begin
    a.n_experts = n_experts
    a.max_rows = max_rows
    a.token_tile = token_tile
    a.split_k = split_k
    a.wfmt = wfmt
    a.planes = planes
    a.feat_pad = feat_pad
    a.n_feat = n_feat
    a.k_pad = k_pad
    a.weight = _ptr(weight)
    a.sc_br, a.sc_bc = fp8_block
    a.b_src = _ptr(b_src)
    a.ldb = b_src.stride(0)
    a.b_rows = b_src.shape[0] if b_rows is None else b_rows
    a.k_valid = k_valid
    a.b_map = _ptr(b_map)
    a.b_div = b_div
    a.epilogue = epilogue
    a.bias = _ptr(bias)
    a.alpha = alpha
    a.limit = limit
    if row_weight is not None:
        a.row_weight = _ptr(row_weight)
        a.row_weight_bf16 = int(row_weight.dtype == torch.bfloat16)
        a.row_src = _ptr(row_src)
    a.out = _ptr(out)
    a.ldo = out.stride(0)
    check(lib.b200moe_expert_gemm(device, _stream(device), ctypes.byref(a)), "expert_gemm")
    return out


def expert_layer(w, hidden: torch.Tensor, indices: torch.Tensor, weights: torch.Tensor, *,
                 num_experts: int, expert_begin: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
    """The single-GPU expert layer in one call (b200moe_expert_layer):
    permutation, row gather, gate/up and down grouped GEMMs and the
    global-expert-order combine of the experts in ``w`` (a
    layout.ExpertWeights). The workspace is one allocation of the caching
    allocator per call."""
    device = _dev(hidden, "hidden")
    _bf16_rows(hidden, "hidden")
    T, K = indices.shape
    if out is None:
        out = torch.empty(T, w.hidden, device=hidden.device, dtype=torch.bfloat16)
    _bf16_rows(out, "output")
    a = _lib.LayerArgs()
    a.indices = _ptr(indices)
    a.weights = _ptr(weights)
    a.weights_bf16 = int(weights.dtype == torch.bfloat16)
    a.T, a.K, a.E = T, K, num_experts
    a.expert_begin = expert_begin
    a.hidden = _ptr(hidden)
    a.ldh = hidden.stride(0)
    a.H, a.I = w.hidden, w.inter
    a.wfmt, a.n_experts = w.fmt, w.n_experts
    a.w1, a.w2, a.b1, a.b2 = _ptr(w.w1), _ptr(w.w2), _ptr(w.b1), _ptr(w.b2)
    a.sc_br, a.sc_bc = w.block
    a.gated_epilogue = w.gated_epilogue
    a.alpha, a.limit = w.alpha, w.limit
    a.out = _ptr(out)
    a.ldo = out.stride(0)
    nbytes = lib.b200moe_layer_workspace(ctypes.byref(a))
    ws = torch.empty(max(nbytes, 256), device=hidden.device, dtype=torch.uint8)
    check(lib.b200moe_expert_layer(device, _stream(device), ctypes.byref(a), _ptr(ws), nbytes),
          "expert_layer")
    return out


def w8a8_gemm(*, offsets: torch.Tensor, expert_begin: int, n_experts: int, max_rows: int,
              planes: int, feat_pad: int, n_feat: int, k_pad: int, weight: torch.Tensor,
              fp8_block: tuple[int, int] = (128, 128), q: torch.Tensor, q_scale: torch.Tensor,
              epilogue: int, row_weight: torch.Tensor | None = None,
              row_src: torch.Tensor | None = None, out: torch.Tensor,
              token_tile: int = 0) -> torch.Tensor:
    """W8A8 grouped GEMM: packed FP8 weight blobs times e4m3 permuted rows
    ``q`` [rows, k_pad] with per-(row, 128-column) scales ``q_scale``
    (``act_quant_fp8``'s outputs)."""
    device = _dev(weight, "weight")
    _bf16_rows(out, "output")
    if q.dtype != torch.float8_e4m3fn or q.dim() != 2 or not q.is_contiguous() or q.shape[1] != k_pad:
        raise ValueError(f"q must be contiguous float8_e4m3fn [rows, {k_pad}]")
    groups = -(-k_pad // 128)
    if (q_scale.dtype != torch.float32 or not q_scale.is_contiguous()
            or tuple(q_scale.shape) != (q.shape[0], groups)):
        raise ValueError(f"q_scale must be contiguous float32 [{q.shape[0]}, {groups}]")
    a = _lib.GemmArgs()
    a.offsets = _ptr(offsets)
    a.expert_begin = expert_begin
    a.n_experts = n_experts
    a.max_rows = max_rows
    a.token_tile = token_tile
    a.wfmt = _lib.W_FP8
    a.planes = planes
    a.feat_pad = feat_pad
    a.n_feat = n_feat
    a.k_pad = k_pad
    a.weight = _ptr(weight)
    a.sc_br, a.sc_bc = fp8_block
    a.b_rows = q.shape[0]
    a.b_div = 1
    a.epilogue = epilogue
    if row_weight is not None:
        a.row_weight = _ptr(row_weight)
        a.row_weight_bf16 = int(row_weight.dtype == torch.bfloat16)
        a.row_src = _ptr(row_src)
    a.out = _ptr(out)
    a.ldo = out.stride(0)
    check(lib.b200moe_w8a8_gemm(device, _stream(device), ctypes.byref(a), _ptr(q), _ptr(q_scale)),
          "w8a8_gemm")
    return out


# --------------------------------------------------------------------------- combine
def combine(rows: torch.Tensor, inverse: torch.Tensor, indices: torch.Tensor, *, order: int,
            experts_per_rank: int = 1, expert_lo: int = 0, expert_hi: int = 1 << 30,
            weights: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    device = _dev(indices, "indices")
    T, K = indices.shape
    H = rows.shape[1]
    _bf16_rows(rows, "contribution rows")
    if out is None:
        out = torch.empty(T, H, device=indices.device, dtype=torch.bfloat16)
    _bf16_rows(out, "output")
    wbf16 = int(weights is not None and weights.dtype == torch.bfloat16)
    check(
        lib.b200moe_combine(
            device, _stream(device), _ptr(rows), rows.stride(0), _ptr(inverse), _ptr(indices),
            T, K, H, order, experts_per_rank, expert_lo, expert_hi, int(weights is not None),
            _ptr(weights), wbf16, _ptr(out), out.stride(0),
        ),
        "combine",
    )
    return out


def append_shared_slot(indices: torch.Tensor, weights: torch.Tensor, score_logit: torch.Tensor,
                       shared_expert: int) -> tuple[torch.Tensor, torch.Tensor]:
    """The routing of [T, K] extended by slot K = ``shared_expert`` with
    weight bf16(sigmoid(score_logit)) (b200moe_append_shared_slot):
    int64 [T, K + 1] expert ids and bf16 [T, K + 1] weights. score_logit is
    the bf16 [T, 1] (or [T]) output of F.linear(hidden, score)."""
    device = _dev(indices, "indices")
    if indices.dtype != torch.int64 or indices.dim() != 2 or not indices.is_contiguous():
        raise ValueError("indices must be a contiguous int64 [T, K] tensor")
    T, K = indices.shape
    if weights.shape != indices.shape or weights.dtype not in (torch.float32, torch.bfloat16) \
            or not weights.is_contiguous():
        raise ValueError("weights must be a contiguous fp32 or bf16 tensor shaped like indices")
    logit = score_logit.reshape(T, -1)
    if logit.dtype != torch.bfloat16 or logit.shape[1] != 1 or logit.device != indices.device:
        raise ValueError("score_logit must be the bf16 [T, 1] score on the indices' device")
    out_idx = torch.empty(T, K + 1, device=indices.device, dtype=torch.int64)
    out_w = torch.empty(T, K + 1, device=indices.device, dtype=torch.bfloat16)
    check(lib.b200moe_append_shared_slot(device, _stream(device), _ptr(indices), _ptr(weights),
                                         int(weights.dtype == torch.bfloat16), _ptr(logit), logit.stride(0),
                                         T, K, shared_expert, _ptr(out_idx), _ptr(out_w)),
          "append_shared_slot")
    return out_idx, out_w


def combine_f32(rows: torch.Tensor, inverse: torch.Tensor, indices: torch.Tensor, weights: torch.Tensor,
                *, expert_lo: int = 0, expert_hi: int = 1 << 30,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 out[t] = fp32 sum over the token's slots in order of
    bf16(w * rows[inverse]) (fp32 rows of the fp32 down epilogue, each scaled
    row rounded to bf16 as matmul_ogs stores it; b200moe_combine_f32)."""
    device = _dev(indices, "indices")
    T, K = indices.shape
    if rows.dtype != torch.float32 or rows.dim() != 2 or rows.stride(1) != 1:
        raise ValueError("rows must be a 2D float32 tensor with contiguous rows")
    H = rows.shape[1]
    if out is None:
        out = torch.empty(T, H, device=indices.device, dtype=torch.bfloat16)
    _bf16_rows(out, "output")
    check(lib.b200moe_combine_f32(device, _stream(device), _ptr(rows), rows.stride(0), _ptr(inverse),
                                  _ptr(indices), T, K, H, expert_lo, expert_hi, _ptr(weights),
                                  int(weights.dtype == torch.bfloat16), _ptr(out), out.stride(0)),
          "combine_f32")
    return out


def combine_allreduce(rows: torch.Tensor, inverse: torch.Tensor, indices: torch.Tensor, *,
                      expert_lo: int, expert_hi: int, peers, t_cap: int, rank: int,
                      weights: torch.Tensor | None = None, out: torch.Tensor | None = None,
                      timeout_ns: int = 0) -> torch.Tensor:
    """Fused expert-order combine of [expert_lo, expert_hi) and a SUM over the
    ranks whose exchange buffers are ``peers`` (device addresses, this rank's
    at ``rank``); see b200moe_combine_allreduce."""
    device = _dev(indices, "indices")
    T, K = indices.shape
    H = rows.shape[1]
    _bf16_rows(rows, "contribution rows")
    if out is None:
        out = torch.empty(T, H, device=indices.device, dtype=torch.bfloat16)
    _bf16_rows(out, "output")
    arr = (ctypes.c_void_p * len(peers))(*peers)
    wbf16 = int(weights is not None and weights.dtype == torch.bfloat16)
    check(
        lib.b200moe_combine_allreduce(
            device, _stream(device), _ptr(rows), rows.stride(0), _ptr(inverse), _ptr(indices),
            T, K, H, expert_lo, expert_hi, int(weights is not None), _ptr(weights), wbf16,
            len(peers), rank, arr, t_cap, _ptr(out), out.stride(0), timeout_ns,
        ),
        "combine_allreduce",
    )
    return out


# --------------------------------------------------------------------------- peer-memory row exchanges
def _peer_array(buf):
    return (ctypes.c_void_p * len(buf.peers))(*buf.peers)


def a2a_counts(buf, counts: torch.Tensor, recv_offsets: torch.Tensor, E: int) -> torch.Tensor:
    """Exchange this rank's per-expert row counts (int32 [E]) with every rank
    of ``buf`` (a parallel.PeerRows) and write the receive segments of this
    rank's experts into ``recv_offsets`` (int32 [E / world + 1])."""
    device = _dev(counts, "counts")
    if counts.dtype != torch.int32 or counts.numel() != E or not counts.is_contiguous():
        raise ValueError(f"counts must be contiguous int32 [{E}]")
    if recv_offsets.dtype != torch.int32 or recv_offsets.numel() != E // buf.world + 1:
        raise ValueError(f"recv_offsets must be int32 [{E // buf.world + 1}]")
    check(lib.b200moe_a2a_counts(device, _stream(device), _peer_array(buf), buf.world, buf.rank, E,
                                 _ptr(counts), _ptr(recv_offsets), buf.cap_a, buf.cap_b,
                                 buf.timeout_ns), "a2a_counts")
    return recv_offsets


def a2a_dispatch(buf, hidden: torch.Tensor, indices: torch.Tensor, perm: "Permutation", E: int) -> None:
    """Push every routed row of this rank into its expert owner's receive area."""
    device = _dev(hidden, "hidden")
    _bf16_rows(hidden, "hidden")
    T, K = indices.shape
    if indices.dtype != torch.int64 or not indices.is_contiguous():
        raise ValueError("indices must be contiguous int64")
    check(lib.b200moe_a2a_dispatch(device, _stream(device), _peer_array(buf), buf.world, buf.rank, E,
                                   _ptr(hidden), hidden.stride(0), hidden.shape[1], _ptr(indices),
                                   _ptr(perm.perm_src), _ptr(perm.offsets), T * K, K, buf.cap_a,
                                   buf.timeout_ns), "a2a_dispatch")


def a2a_return(buf, y: torch.Tensor, E: int) -> None:
    """Push every computed row (receive order, [cap_a, H]) back to its source."""
    device = _dev(y, "y")
    _bf16_rows(y, "y")
    check(lib.b200moe_a2a_return(device, _stream(device), _peer_array(buf), buf.world, buf.rank, E,
                                 _ptr(y), y.stride(0), y.shape[1], buf.cap_a, buf.cap_b,
                                 buf.timeout_ns), "a2a_return")


def ep_gather(buf, offsets: torch.Tensor, expert_lo: int, expert_hi: int, rows_total: int) -> None:
    """Copy rows [offsets[expert_lo], offsets[expert_hi]) of this rank's area A
    to the same rows of every other rank's area A."""
    device = _dev(offsets, "offsets")
    check(lib.b200moe_ep_gather(device, _stream(device), _peer_array(buf), buf.world, buf.rank,
                                buf.hidden, _ptr(offsets), expert_lo, expert_hi, rows_total,
                                buf.cap_a, buf.timeout_ns), "ep_gather")


def gather_rows(src: torch.Tensor, index_map: torch.Tensor, div: int = 1,
                out: torch.Tensor | None = None, offsets: torch.Tensor | None = None,
                expert_lo: int = 0, expert_hi: int = 0) -> torch.Tensor:
    """out[i] = src[index_map[i] // div] for bf16 rows; with ``offsets``
    (a permutation's), only rows [offsets[expert_lo], offsets[expert_hi])."""
    device = _dev(src, "src")
    _bf16_rows(src, "src")
    n = index_map.numel()
    H = src.shape[1]
    if out is None:
        out = torch.empty(n, H, device=src.device, dtype=torch.bfloat16)
    if offsets is not None:
        check(
            lib.b200moe_gather_rows_range(
                device, _stream(device), _ptr(src), src.stride(0), _ptr(index_map), div, n, H,
                _ptr(out), out.stride(0), _ptr(offsets), expert_lo, expert_hi,
            ),
            "gather_rows_range",
        )
        return out
    check(
        lib.b200moe_gather_rows(
            device, _stream(device), _ptr(src), src.stride(0), _ptr(index_map), div, n, H,
            _ptr(out), out.stride(0),
        ),
        "gather_rows",
    )
    return out


# --------------------------------------------------------------------------- token all-to-all
@dataclass
class RecvPlan:
    offsets: torch.Tensor    # int32 [el+1]: expert-major segment starts
    map_in: torch.Tensor     # int32 [rows]: expert-major position -> arrival row
    map_back: torch.Tensor   # int32 [rows]: arrival row -> expert-major position


def a2a_recv_plan(counts: torch.Tensor, ep: int, experts_per_rank: int, rows: int) -> RecvPlan:
    """Transposition of received [source][expert] row segments into expert-major
    order; ``counts`` is int32 [ep * experts_per_rank] (source-major)."""
    device = _dev(counts, "counts")
    if counts.dtype != torch.int32 or not counts.is_contiguous() or counts.numel() != ep * experts_per_rank:
        raise ValueError("counts must be a contiguous int32 tensor of ep * experts_per_rank elements")
    dev = counts.device
    offsets = torch.empty(experts_per_rank + 1, device=dev, dtype=torch.int32)
    map_in = torch.empty(rows, device=dev, dtype=torch.int32)
    map_back = torch.empty(rows, device=dev, dtype=torch.int32)
    check(
        lib.b200moe_a2a_recv_plan(
            device, _stream(device), _ptr(counts), ep, experts_per_rank, rows, _ptr(offsets),
            _ptr(map_in), _ptr(map_back),
        ),
        "a2a_recv_plan",
    )
    return RecvPlan(offsets, map_in, map_back)
