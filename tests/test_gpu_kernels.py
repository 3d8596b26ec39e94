"""Kernel-level parity on the GPU, called through the C ABI (ops wrappers).

Integer and ordering stages are compared bit-exactly with the C oracle.
The grouped GEMM is checked bit-exactly on integer-valued data (every fp32
partial sum is exact, so any summation order gives the same result) across
token tiles and weight formats, and its dequantisers are probed exactly with
one-hot activations.
"""

import pytest
import torch
import torch.nn.functional as F

from moe_serving_profile_b200 import _lib, layout, ops
from moe_serving_profile_b200 import synthetic as S
from oracle import oracle

pytestmark = pytest.mark.gpu


def _status_clean(dev):
    assert _lib.device_status(dev.index) == 0


# ------------------------------------------------------------------ router
# (family, T, H, E, K) of every workload: qwen3-tiny, qwen3-30b-a3b,
# gpt-oss-20b, gpt-oss-120b and qwen3-235b-a22b (with its Zipf router bias)
ROUTER_SHAPES = (
    [("qwen3-tiny", 64)] + [("qwen3-30b-a3b", t) for t in (1, 8, 64, 512, 4096)]
    + [("gpt-oss-20b", t) for t in (1, 16, 64, 2048)] + [("gpt-oss-120b", t) for t in (64, 8192)]
    + [("qwen3-235b-a22b", t) for t in (256, 16384)])


def _router_inputs(name, T, cuda):
    cfg = S.CONFIGS[name]
    g = torch.Generator().manual_seed(T * 131 + cfg.hidden)
    x = torch.randn(T, cfg.hidden, generator=g).bfloat16().to(cuda)
    w = (torch.randn(cfg.experts, cfg.hidden, generator=g) * 0.02).bfloat16().to(cuda)
    if cfg.family == "gpt_oss":
        b = (torch.randn(cfg.experts, generator=g) * 0.01).bfloat16().to(cuda)
    else:
        b = S.zipf_router_bias(cfg.experts, T, cuda) if cfg.zipf_bias else None
    return cfg, x, w, b


def _router_module(cfg, w, b, cuda, logits):
    from types import SimpleNamespace

    from moe_serving_profile_b200.router import GptOssRouter, Qwen3Router
    if cfg.family == "gpt_oss":
        r = GptOssRouter(SimpleNamespace(num_experts_per_tok=cfg.top_k, num_local_experts=cfg.experts,
                                         hidden_size=cfg.hidden), logits=logits).to(cuda)
        r.bias.data = b
    else:
        r = Qwen3Router(SimpleNamespace(num_experts_per_tok=cfg.top_k, num_experts=cfg.experts,
                                        norm_topk_prob=cfg.norm_topk, hidden_size=cfg.hidden),
                        logits=logits).to(cuda)
        r.bias = b
    r.weight.data = w
    return r


def _reference_router(cfg, x, w, b):
    """The reference's router on the same device: Transformers' forward, i.e.
    torch's F.linear, softmax, topk and sum (oracle.qwen_router /
    gpt_oss_router; the Zipf bias of qwen3-235b-a22b enters F.linear)."""
    if cfg.family == "gpt_oss":
        logits, scores, idx = oracle.gpt_oss_router(x, w, b, cfg.top_k)
        return logits, scores, idx
    logits = F.linear(x, w, b)
    probs = torch.softmax(logits, dtype=torch.float, dim=-1)
    top, idx = torch.topk(probs, cfg.top_k, dim=-1)
    if cfg.norm_topk:
        top = top / top.sum(dim=-1, keepdim=True)
    return probs, top, idx


def _bits(t):
    return t.contiguous().view(torch.int16 if t.element_size() == 2 else torch.int32)


@pytest.mark.parametrize("name,T", ROUTER_SHAPES)
def test_exact_router_equals_reference_router(cuda, name, T):
    """Default ("exact") routing is the reference's router bit for bit at every
    workload shape: probabilities (or logits), scores and expert indices,
    including the slot order of tied values, on every row."""
    cfg, x, w, b = _router_inputs(name, T, cuda)
    first, scores, idx = _router_module(cfg, w, b, cuda, "exact")(x)
    r_first, r_scores, r_idx = _reference_router(cfg, x, w, b)
    assert torch.equal(idx, r_idx), f"{int((idx != r_idx).any(-1).sum())}/{T} rows differ"
    assert torch.equal(_bits(first), _bits(r_first))
    assert torch.equal(_bits(scores), _bits(r_scores))
    # the fused fixed-order logits on the same inputs (informational): rows
    # whose indices differ from the reference's come from near-ties of logits
    # one bf16 ulp apart
    _, _, f_idx = _router_module(cfg, w, b, cuda, "fused")(x)
    agree = float((f_idx == r_idx).all(-1).float().mean())
    print(f"\n{name} T={T}: fused-logits routing equals the reference on {agree:.4%} of rows")
    _status_clean(cuda)


@pytest.mark.parametrize("T,H,E,K", [(1, 2048, 128, 8), (64, 2048, 128, 8), (4096, 2048, 128, 8),
                                     (64, 256, 8, 2), (13, 4096, 128, 8)])
def test_fused_router_logits_bit_exact(cuda, T, H, E, K):
    """The fixed-order logits kernel against the C oracle; the selection on
    its logits against torch's softmax / topk / sum of the same logits."""
    g = torch.Generator().manual_seed(T + H)
    x = torch.randn(T, H, generator=g).bfloat16()
    w = (torch.randn(E, H, generator=g) * 0.02).bfloat16()
    out = ops.router(_lib.ROUTER_QWEN3, x.to(cuda), w.to(cuda), None, K, True)
    ref_logits = oracle.router_logits(x, w, None, 0)
    assert torch.equal(out.logits.float().cpu(), ref_logits)
    probs = torch.softmax(out.logits, dtype=torch.float, dim=-1)
    top, idx = torch.topk(probs, K, dim=-1)
    assert torch.equal(out.indices, idx)
    assert torch.equal(_bits(out.probs), _bits(probs))
    assert torch.equal(_bits(out.scores), _bits(top / top.sum(-1, keepdim=True)))
    assert torch.equal(out.indices.cpu(), oracle.topk(probs.cpu(), K))
    assert torch.equal(out.counts.cpu().long(), torch.bincount(out.indices.cpu().flatten(), minlength=E))
    _status_clean(cuda)


@pytest.mark.parametrize("T", [1, 16, 64, 2048])
def test_gpt_oss_fused_router_bit_exact(cuda, T):
    H, E, K = 2880, 32, 4
    g = torch.Generator().manual_seed(T)
    x = torch.randn(T, H, generator=g).bfloat16()
    w = (torch.randn(E, H, generator=g) * 0.02).bfloat16()
    b = (torch.randn(E, generator=g) * 0.01).bfloat16()
    out = ops.router(_lib.ROUTER_GPT_OSS, x.to(cuda), w.to(cuda), b.to(cuda), K, False)
    ref_logits = oracle.router_logits(x, w, b, 1)
    assert torch.equal(out.logits.float().cpu(), ref_logits)
    top, idx = torch.topk(out.logits, K, dim=-1)
    assert torch.equal(out.indices, idx)
    assert torch.equal(_bits(out.scores), _bits(torch.softmax(top, dim=1, dtype=top.dtype)))
    _status_clean(cuda)


def test_native_router_bit_exact(cuda):
    """moe.route (fp32): fixed-order logits against the oracle, and the
    exact path (F.linear fp32 logits) against the reference's route."""
    from moe_serving_profile_b200.router import native_route
    T, H, E, K = 37, 512, 16, 3
    g = torch.Generator().manual_seed(7)
    x = torch.randn(T, H, generator=g).bfloat16()
    w = (torch.randn(E, H, generator=g) * 0.05).bfloat16()
    out = ops.router(_lib.ROUTER_NATIVE, x.to(cuda), w.to(cuda), None, K, True)
    ref = oracle.router_logits(x, w, None, 2)
    assert torch.equal(out.logits.cpu(), ref)
    for renorm in (True, False):
        idx, wt = native_route(x.to(cuda), w.to(cuda), K, renorm)
        r_idx, r_wt, _ = oracle.native_route(x.to(cuda), w.to(cuda), K, renorm)
        assert torch.equal(idx, r_idx) and torch.equal(_bits(wt), _bits(r_wt))
    _status_clean(cuda)


def _tie_logits(T, E, dtype, seed):
    """Rows of repeated values, all-equal rows, a coarse value grid and plain rows."""
    g = torch.Generator().manual_seed(seed)
    lg = (torch.randn(T, E, generator=g) * 0.9)
    q = T // 4
    lg[:q] = lg[:q, :max(1, E // 8)].repeat(1, 8)[:, :E]       # each value 8 times
    lg[q:q + 8] = 0.0                                            # all tied
    lg[q + 8:2 * q] = (torch.randint(0, 24, (2 * q - q - 8, E), generator=g).float() / 8 - 1.5)
    return lg.to(dtype)


@pytest.mark.parametrize("E,K", [(128, 8), (8, 2), (32, 4), (128, 4), (512, 32), (64, 6)])
def test_selection_reproduces_torch_topk_with_ties(cuda, E, K):
    """Selection alone on caller logits: indices (including the slot order of
    equal values), probabilities and scores equal torch's softmax / topk / sum
    on CUDA bit for bit, on tie-heavy rows; the C oracle restates the rule."""
    logits = _tie_logits(1024, E, torch.bfloat16, E * 37 + K).to(cuda)
    out = ops.router(_lib.ROUTER_QWEN3, None, None, None, K, True, logits=logits)
    probs = torch.softmax(logits, dtype=torch.float, dim=-1)
    top, idx = torch.topk(probs, K, dim=-1)
    assert torch.equal(out.indices, idx), f"{int((out.indices != idx).any(-1).sum())} rows differ"
    assert torch.equal(out.indices.cpu(), oracle.topk(probs.cpu(), K))
    assert torch.equal(_bits(out.probs), _bits(probs))
    if K & (K - 1) == 0:   # the butterfly sum order is pinned for powers of two
        assert torch.equal(_bits(out.scores), _bits(top / top.sum(-1, keepdim=True)))
    else:
        assert torch.allclose(out.scores, top / top.sum(-1, keepdim=True), rtol=2e-7, atol=0)
    # GPT-OSS: top-k on the bf16 logits, softmax over the k values in bf16
    bias = torch.zeros(E, device=cuda, dtype=torch.bfloat16)
    out = ops.router(_lib.ROUTER_GPT_OSS, None, None, bias, K, False, logits=logits)
    top, idx = torch.topk(logits, K, dim=-1)
    assert torch.equal(out.indices, idx)
    assert torch.equal(_bits(out.scores), _bits(torch.softmax(top, dim=1, dtype=top.dtype)))
    # NATIVE: fp32 logits
    lf = _tie_logits(1024, E, torch.float32, E + K).to(cuda)
    out = ops.router(_lib.ROUTER_NATIVE, None, None, None, K, True, logits=lf)
    top, idx = torch.topk(torch.softmax(lf, dim=-1), K, dim=-1)
    assert torch.equal(out.indices, idx)
    want = (top / top.sum(-1, keepdim=True).clamp_min(1e-20)).to(torch.bfloat16)
    if K & (K - 1) == 0:
        assert torch.equal(_bits(out.scores), _bits(want))
    _status_clean(cuda)


# ------------------------------------------------------------------ permutation
@pytest.mark.parametrize("T,K,E", [(1, 8, 128), (13, 2, 4), (64, 8, 128), (1023, 8, 128),
                                   (4096, 8, 128), (16384, 8, 128), (2048, 4, 32), (8192, 4, 128),
                                   (3000, 3, 1000)])
def test_permute_bit_exact(cuda, T, K, E):
    g = torch.Generator().manual_seed(T * K + E)
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).long()
    p = ops.permute(idx.to(cuda), E)
    counts, offsets, perm, inv = oracle.permute(idx, E)
    assert torch.equal(p.counts.cpu(), counts) and torch.equal(p.offsets.cpu(), offsets)
    assert torch.equal(p.perm_src.cpu(), perm) and torch.equal(p.inverse.cpu(), inv)
    _status_clean(cuda)


def test_permute_skewed_and_invalid_ids(cuda):
    T, K, E = 5000, 8, 64
    g = torch.Generator().manual_seed(11)
    idx = torch.randint(0, 4, (T, K), generator=g)       # heavy skew, repeated ids
    idx[7, 3] = E + 5
    idx[100, 0] = -1
    p = ops.permute(idx.to(cuda), E)
    counts, offsets, perm, inv = oracle.permute(idx, E)
    n = int(offsets[-1])
    assert torch.equal(p.counts.cpu(), counts) and torch.equal(p.offsets.cpu(), offsets)
    assert torch.equal(p.perm_src.cpu()[:n], perm[:n]) and torch.equal(p.inverse.cpu(), inv)
    assert _lib.device_status(cuda.index) & _lib.STATUS_BAD_INDEX


def test_permute_empty(cuda):
    p = ops.permute(torch.empty(0, 8, dtype=torch.int64, device=cuda), 128)
    assert int(p.offsets[-1]) == 0 and int(p.counts.sum()) == 0


# ------------------------------------------------------------------ combine / gather
@pytest.mark.parametrize("order", [0, 1])
@pytest.mark.parametrize("scale", [False, True])
def test_combine_bit_exact(cuda, order, scale):
    T, K, E, H = 777, 8, 128, 2880
    g = torch.Generator().manual_seed(5 + order)
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).long()
    rows = torch.randn(T * K, H, generator=g).bfloat16()
    wts = torch.rand(T, K, generator=g)
    counts, offsets, perm, inv = oracle.permute(idx, E)
    lo, hi = (16, 80) if scale else (0, E)
    out = ops.combine(rows.to(cuda), inv.to(cuda), idx.to(cuda), order=order, experts_per_rank=16,
                      expert_lo=lo, expert_hi=hi, weights=wts.to(cuda) if scale else None)
    ref = oracle.combine(rows, inv, idx, order=order, experts_per_rank=16, lo=lo, hi=hi,
                         weights=wts if scale else None)
    assert torch.equal(out.cpu(), ref)


@pytest.mark.parametrize("T,K,H,wdtype,lo,hi", [
    (777, 8, 2048, torch.float32, 0, 128), (300, 8, 2880, torch.bfloat16, 16, 80),
    (129, 4, 2880, torch.float32, 0, 128), (64, 6, 512, torch.float32, 32, 96),
    (33, 1, 256, torch.bfloat16, 0, 128), (5, 32, 1024, torch.float32, 0, 128)])
def test_combine_slot_sum_equals_torch(cuda, T, K, H, wdtype, lo, hi):
    """Order SLOT_SUM against grouped_fp8's own combine run with torch on the
    same GPU (efficient_kernels.py:269-273: rows times bf16 weights, masked
    rows zero, values[inverse].reshape(T, K, H).sum(1)) and against the
    oracle, bit for bit, on rows whose exponents make the fp32 summation order
    visible in the bf16 result; dropped slots and rank ranges included."""
    from tests.golden.make_slot_sum_golden import spread_values

    E = 128
    g = torch.Generator().manual_seed(T * K + H)
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).long()
    idx[3, 0] = -1                                          # a dropped slot
    wts = (torch.rand(T, K, generator=g) * 1.5).to(wdtype)
    wts[::2] = wts[::2, :1].clone()        # equal weights: the scaled +B / -B pair cancels
    counts, offsets, perm, inv = oracle.permute(idx, E)
    # token t's slot k holds values[t, k] (a token's slots share the +B / -B pair)
    values = spread_values(T, K, H, seed=H + K).reshape(T * K, H)
    rows = torch.zeros(T * K, H, dtype=torch.bfloat16)
    kept = inv >= 0
    rows[inv[kept].long()] = values[kept]
    out = ops.combine(rows.to(cuda), inv.to(cuda), idx.to(cuda), order=_lib.ORDER_SLOT_SUM,
                      expert_lo=lo, expert_hi=hi, weights=wts.to(cuda))
    unscaled = ops.combine(rows.to(cuda), inv.to(cuda), idx.to(cuda), order=_lib.ORDER_SLOT_SUM,
                           expert_lo=lo, expert_hi=hi)
    _status_clean(cuda)
    # the reference's expression, torch on the GPU
    r, ic, w = rows.to(cuda), inv.long().to(cuda), wts.to(cuda)
    e = idx.to(cuda).reshape(-1)
    valid = (ic >= 0) & (e >= lo) & (e < hi)
    vals = r[ic.clamp(min=0)] * w.reshape(-1, 1).to(torch.bfloat16)
    vals.masked_fill_(~valid[:, None], 0)
    want = vals.reshape(T, K, H).sum(1)
    assert torch.equal(out, want)
    plain = r[ic.clamp(min=0)].masked_fill(~valid[:, None], 0).reshape(T, K, H).sum(1)
    assert torch.equal(unscaled, plain)
    assert torch.equal(out.cpu(), oracle.w8a8_local_combine(rows, inv, idx, wts, lo, hi))


def _p2p_buffer(cuda, t_cap, H, world):
    import ctypes
    ptr = ctypes.c_void_p()
    nbytes = _lib.lib.b200moe_p2p_buffer_bytes(t_cap, H, world)
    _lib.check(_lib.lib.b200moe_p2p_alloc(cuda.index, nbytes, ctypes.byref(ptr)), "p2p_alloc")
    return ptr.value


@pytest.mark.parametrize("scale", [False, True])
def test_combine_allreduce_single_rank_equals_combine(cuda, scale):
    """One rank: the fused kernel's partial is the expert-order combine and
    the rank sum is that partial (one bf16 rounding of an exact value), so it
    equals b200moe_combine bit for bit, in consecutive calls (epochs 1, 2, 3)."""
    T, K, E, H = 300, 8, 128, 2048
    g = torch.Generator().manual_seed(11)
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).long()
    rows = torch.randn(T * K, H, generator=g).bfloat16().to(cuda)
    wts = torch.rand(T, K, generator=g).to(cuda)
    counts, offsets, perm, inv = oracle.permute(idx, E)
    inv, idx = inv.to(cuda), idx.to(cuda)
    buf = _p2p_buffer(cuda, 512, H, 1)
    try:
        ref = ops.combine(rows, inv, idx, order=_lib.ORDER_EXPERT, expert_lo=16, expert_hi=80,
                          weights=wts if scale else None)
        for _ in range(3):
            out = ops.combine_allreduce(rows, inv, idx, expert_lo=16, expert_hi=80, peers=[buf],
                                        t_cap=512, rank=0, weights=wts if scale else None)
            assert torch.equal(out, ref)
        _status_clean(cuda)
    finally:
        torch.cuda.synchronize(cuda)
        _lib.lib.b200moe_p2p_free(cuda.index, buf)


def test_combine_allreduce_peer_timeout_sets_status(cuda):
    """A peer that never signals: every block's wait gives up after the
    timeout, the kernel returns, the status word says PEER_TIMEOUT and the
    context stays usable (no fault, no hang)."""
    import ctypes
    T, K, E, H = 64, 2, 8, 256
    idx = torch.randint(0, E, (T, K))
    counts, offsets, perm, inv = oracle.permute(idx, E)
    rows = torch.ones(T * K, H, dtype=torch.bfloat16, device=cuda)
    bufs = [_p2p_buffer(cuda, T, H, 2), _p2p_buffer(cuda, T, H, 2)]   # "rank 1": nobody signals
    out = torch.full((T, H), 7.0, dtype=torch.bfloat16, device=cuda)
    try:
        ops.combine_allreduce(rows, inv.to(cuda), idx.to(cuda), expert_lo=0, expert_hi=E, peers=bufs,
                              t_cap=T, rank=0, out=out, timeout_ns=20_000_000)
        torch.cuda.synchronize(cuda)
        st = ctypes.c_int()
        _lib.check(_lib.lib.b200moe_device_status(cuda.index, 1, ctypes.byref(st)), "status")
        assert st.value & _lib.STATUS_PEER_TIMEOUT
        assert bool((out == 7.0).all())   # rows are not written after a timeout
        assert float((torch.ones(4, device=cuda) * 2).sum()) == 8.0   # the context still runs kernels
    finally:
        torch.cuda.synchronize(cuda)
        for b in bufs:
            _lib.lib.b200moe_p2p_free(cuda.index, b)


def test_gather_rows_range_only_touches_the_experts_rows(cuda):
    T, K, E, H = 300, 4, 16, 512
    g = torch.Generator().manual_seed(3)
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).long()
    counts, offsets, perm, inv = oracle.permute(idx, E)
    src = torch.randn(T, H, generator=g).bfloat16().to(cuda)
    full = ops.gather_rows(src, perm.to(cuda), K)
    out = torch.full((T * K, H), 5.0, dtype=torch.bfloat16, device=cuda)
    ops.gather_rows(src, perm.to(cuda), K, out=out, offsets=offsets.to(cuda), expert_lo=4, expert_hi=11)
    r0, r1 = int(offsets[4]), int(offsets[11])
    assert torch.equal(out[r0:r1], full[r0:r1])
    assert bool((out[:r0] == 5.0).all()) and bool((out[r1:] == 5.0).all())


def test_gather_rows_exact(cuda):
    src = torch.randn(50, 2048).bfloat16()
    m = torch.randint(0, 400, (333,), dtype=torch.int32)
    out = ops.gather_rows(src.to(cuda), m.to(cuda), div=8)
    assert torch.equal(out.cpu(), src[(m // 8).long()])


# ------------------------------------------------------------------ grouped GEMM, exact integer data
def _int_case(fmt, E, feat, K, T, topk, seed):
    """Integer-valued weights / activations: all fp32 partial sums exact."""
    g = torch.Generator().manual_seed(seed)
    if fmt == _lib.W_FP8:
        wv = torch.randint(-8, 9, (E, feat, K), generator=g).float()
    elif fmt == _lib.W_MXFP4:
        codes = torch.randint(0, 16, (E, feat, K), generator=g)
        lut = torch.tensor([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6])
        wv = lut[codes] * 2.0                           # scale 2^1 (ue8m0 128)
    else:
        wv = torch.randint(-8, 9, (E, feat, K), generator=g).float()
    x = torch.randint(-3, 4, (T, K), generator=g).float()
    idx = torch.stack([torch.randperm(E, generator=g)[:topk] for _ in range(T)]).long()
    return g, wv, x, idx


def _pack_weight(fmt, wv, planes=1):
    """Integer-valued weights [E * planes, feat, K] -> the GEMM's weight
    argument (bf16 tiles or packed blobs) and the padded feature count."""
    EP, feat, K = wv.shape
    E = EP // planes
    Fp, Kp = -(-feat // 128) * 128, -(-K // 64) * 64
    if fmt == _lib.W_FP8:
        w = torch.zeros(EP, Fp, Kp, dtype=torch.uint8)
        w[:, :feat, :K] = wv.to(torch.float8_e4m3fn).view(torch.uint8)
        scale = torch.ones(E, planes, -(-feat // 128), -(-K // 128))
        return layout.pack_fp8_blobs(w.reshape(E, planes, Fp, Kp), scale, planes, feat, (128, 128)), Fp
    if fmt == _lib.W_MXFP4:
        w = torch.zeros(EP, Fp, Kp // 2, dtype=torch.uint8)
        b, s = S.quantize_mxfp4(torch.nn.functional.pad(wv, (0, Kp - K)).reshape(-1, Kp))
        w[:, :feat] = b.reshape(EP, feat, Kp // 2)
        sc = torch.full((EP, Fp, Kp // 32), 127, dtype=torch.uint8)
        sc[:, :feat] = s.reshape(EP, feat, Kp // 32)
        return layout.pack_mxfp4_blobs(w.reshape(E, planes, Fp, Kp // 2),
                                       sc.reshape(E, planes, Fp, Kp // 32), planes), Fp
    w = torch.zeros(EP, Fp, Kp, dtype=torch.bfloat16)
    w[:, :feat, :K] = wv.bfloat16()
    return w.reshape(E, planes, Fp, Kp), Fp


@pytest.mark.parametrize("fmt", [_lib.W_FP8, _lib.W_MXFP4, _lib.W_BF16])
@pytest.mark.parametrize("tile,split", [(16, 1), (32, 0), (64, 1), (128, 1), (160, 1), (256, 1), (0, 0)])
def test_down_gemm_integer_exact(cuda, fmt, tile, split):
    E, feat, K, T, topk = 6, 296, 448, 150, 3
    g, wv, x, idx = _int_case(fmt, E, feat, K, T, topk, seed=fmt * 10 + tile + split)
    w, Fp = _pack_weight(fmt, wv)
    counts, offsets, perm, inv = oracle.permute(idx, E)
    R = T * topk
    act = torch.zeros(R, -(-K // 64) * 64).bfloat16()
    act[:, :K] = x[(perm // topk).long()].bfloat16()
    out = torch.zeros(R, feat, dtype=torch.bfloat16, device=cuda)
    call = lambda: ops.expert_gemm(
        offsets=offsets.to(cuda), expert_begin=0, n_experts=E, max_rows=R, wfmt=fmt,
        planes=1, feat_pad=Fp, n_feat=feat, k_pad=act.shape[1], weight=w.to(cuda),
        b_src=act.to(cuda), k_valid=K, epilogue=_lib.EPI_DOWN, out=out, token_tile=tile, split_k=split)
    call()
    # exact result: y[r, f] = sum_k act[r, k] * w[e(r), f, k]
    e_of_row = torch.repeat_interleave(torch.arange(E), counts.long())
    ref = torch.einsum("rk,rfk->rf", act[:, :K].double(), wv.double()[e_of_row]).to(torch.bfloat16)
    assert torch.equal(out.cpu(), ref)
    _status_clean(cuda)


def test_gemm_rejects_split_k(cuda):
    """Split-K is not implemented: the host refuses it (NotImplementedError)
    before any launch."""
    E, feat, K, T, topk = 2, 128, 512, 64, 1
    g, wv, x, idx = _int_case(_lib.W_FP8, E, feat, K, T, topk, seed=1)
    w, Fp = _pack_weight(_lib.W_FP8, wv)
    counts, offsets, perm, inv = oracle.permute(idx, E)
    out = torch.zeros(T, feat, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(NotImplementedError):
        ops.expert_gemm(offsets=offsets.to(cuda), expert_begin=0, n_experts=E, max_rows=T,
                        wfmt=_lib.W_FP8, planes=1, feat_pad=Fp, n_feat=feat, k_pad=K,
                        weight=w.to(cuda), b_src=x.bfloat16().to(cuda), k_valid=K,
                        epilogue=_lib.EPI_DOWN, out=out, token_tile=128, split_k=4)


@pytest.mark.parametrize("fmt", [_lib.W_FP8, _lib.W_MXFP4, _lib.W_BF16])
@pytest.mark.parametrize("tile,split", [(16, 1), (64, 1), (128, 1), (160, 1), (256, 1)])
def test_gated_gemm_integer_exact(cuda, fmt, tile, split):
    """Gate/up planes with exact pre-activations; SwiGLU epilogue vs torch."""
    E, inter, H, T, topk = 5, 200, 320, 97, 2
    g, wv, x, idx = _int_case(fmt, E, 2 * inter, H, T, topk, seed=99 + tile)
    w, Ip = _pack_weight(fmt, wv.reshape(E, 2, inter, H).reshape(E * 2, inter, H), planes=2)
    counts, offsets, perm, inv = oracle.permute(idx, E)
    R = T * topk
    out = torch.zeros(R, Ip, dtype=torch.bfloat16, device=cuda)
    xb = x.bfloat16()
    k_pad = -(-H // 64) * 64
    ops.expert_gemm(offsets=offsets.to(cuda), expert_begin=0, n_experts=E, max_rows=R, wfmt=fmt,
                    planes=2, feat_pad=Ip, n_feat=inter, k_pad=k_pad, weight=w.to(cuda),
                    b_src=xb.to(cuda), k_valid=H, b_map=perm.to(cuda), b_div=topk,
                    epilogue=_lib.EPI_SWIGLU, out=out, token_tile=tile, split_k=split)
    e_of_row = torch.repeat_interleave(torch.arange(E), counts.long())
    xr = x[(perm // topk).long()].double()
    pre = torch.einsum("rk,rfk->rf", xr, wv.double()[e_of_row])       # [R, 2I] exact
    gate, up = pre[:, :inter].bfloat16(), pre[:, inter:].bfloat16()
    ref = (torch.nn.functional.silu(gate) * up)                          # torch bf16 semantics
    got = out.cpu()[:, :inter]
    mism = (got != ref)
    assert float(mism.float().mean()) < 1e-3
    assert float((got.float() - ref.float()).abs().max()) <= float(ref.float().abs().max()) * 2 ** -7
    _status_clean(cuda)


@pytest.mark.parametrize("planes", [1, 2])
@pytest.mark.parametrize("tile", [0, 256])
def test_fp8_per_chunk_scales_exact(cuda, planes, tile):
    """FP8 scale blocks that do not cover whole 64 x 64 halves (32 x 32 here)
    travel as per-(row, 16-column chunk) scales inside each blob; with
    power-of-two scales every dequantised weight and partial sum is exact.
    tile 256: contiguous permuted rows through the shared-memory A stages."""
    E, feat, K, T, topk, (br, bc) = 3, 200, 320, 90, 2, (32, 32)
    g, wv, x, idx = _int_case(_lib.W_FP8, E, planes * feat, K, T, topk, seed=31 + planes)
    wv = wv.reshape(E, planes, feat, K)
    Fp, Kp = -(-feat // 128) * 128, -(-K // 64) * 64
    nbr, nbc = -(-feat // br), -(-K // bc)
    scale = torch.pow(2.0, torch.randint(-2, 3, (E, planes, nbr, nbc), generator=g).float())
    w = torch.zeros(E, planes, Fp, Kp, dtype=torch.uint8)
    w[:, :, :feat, :K] = wv.to(torch.float8_e4m3fn).view(torch.uint8)
    blobs = layout.pack_fp8_blobs(w, scale, planes, feat, (br, bc))
    weff = wv * scale.repeat_interleave(br, 2)[:, :, :feat].repeat_interleave(bc, 3)[..., :K]
    counts, offsets, perm, inv = oracle.permute(idx, E)
    R = T * topk
    e_of_row = torch.repeat_interleave(torch.arange(E), counts.long())
    xr = x[(perm // topk).long()]
    out = torch.zeros(R, Fp if planes == 2 else feat, dtype=torch.bfloat16, device=cuda)
    if tile == 256:
        rows = torch.zeros(R, Kp, dtype=torch.bfloat16)
        rows[:, :K] = xr.bfloat16()
        src = dict(b_src=rows.to(cuda), token_tile=256)
    else:
        src = dict(b_src=x.bfloat16().to(cuda), b_map=perm.to(cuda), b_div=topk)
    ops.expert_gemm(offsets=offsets.to(cuda), expert_begin=0, n_experts=E, max_rows=R,
                    wfmt=_lib.W_FP8, planes=planes, feat_pad=Fp, n_feat=feat, k_pad=Kp,
                    weight=blobs.to(cuda), fp8_block=(br, bc), k_valid=K,
                    epilogue=_lib.EPI_SWIGLU if planes == 2 else _lib.EPI_DOWN, out=out, **src)
    pre = torch.einsum("rk,rpfk->rpf", xr.double(), weff.double()[e_of_row])   # [R, planes, feat]
    got = out.cpu()[:, :feat]
    if planes == 1:
        assert torch.equal(got, pre[:, 0].bfloat16())
    else:
        ref = torch.nn.functional.silu(pre[:, 0].bfloat16()) * pre[:, 1].bfloat16()
        assert float((got != ref).float().mean()) < 1e-3
        assert float((got.float() - ref.float()).abs().max()) <= float(ref.float().abs().max()) * 2 ** -7
    _status_clean(cuda)


@pytest.mark.parametrize("fmt", [_lib.W_FP8, _lib.W_MXFP4])
@pytest.mark.parametrize("planes", [1, 2])
def test_256_row_tiles_cut_evenly_integer_exact(cuda, fmt, planes):
    """Quantised weights at 256-row token tiles (weights converted into
    shared-memory operand stages): an expert with more rows than one tile is
    cut into equal tiles rounded up to 16 rows (700 rows -> 240 + 240 + 220),
    each tile's MMA N its own row count; other experts get one tile each.
    Contiguous permuted rows, integer data, exact results."""
    E, feat, K, T, topk = 4, 200, 320, 700, 2
    g, wv, x, _ = _int_case(fmt, E, planes * feat, K, T, topk, seed=7 + planes + fmt)
    # every token routes to expert 0 and one of experts 1..3
    idx = torch.stack([torch.zeros(T, dtype=torch.long), torch.randint(1, E, (T,), generator=g)], 1)
    w, Fp = _pack_weight(fmt, wv.reshape(E * planes, feat, K), planes=planes)
    counts, offsets, perm, inv = oracle.permute(idx, E)
    assert int(counts[0]) == T
    R = T * topk
    Kp = -(-K // 64) * 64
    xr = x[(perm // topk).long()]
    rows = torch.zeros(R, Kp, dtype=torch.bfloat16)
    rows[:, :K] = xr.bfloat16()
    out = torch.zeros(R, Fp if planes == 2 else feat, dtype=torch.bfloat16, device=cuda)
    ops.expert_gemm(offsets=offsets.to(cuda), expert_begin=0, n_experts=E, max_rows=R, wfmt=fmt,
                    planes=planes, feat_pad=Fp, n_feat=feat, k_pad=Kp, weight=w.to(cuda),
                    b_src=rows.to(cuda), k_valid=K,
                    epilogue=_lib.EPI_SWIGLU if planes == 2 else _lib.EPI_DOWN, out=out, token_tile=256)
    e_of_row = torch.repeat_interleave(torch.arange(E), counts.long())
    pre = torch.einsum("rk,rpfk->rpf", xr.double(), wv.reshape(E, planes, feat, K).double()[e_of_row])
    got = out.cpu()[:, :feat]
    if planes == 1:
        assert torch.equal(got, pre[:, 0].bfloat16())
    else:
        ref = torch.nn.functional.silu(pre[:, 0].bfloat16()) * pre[:, 1].bfloat16()
        assert float((got != ref).float().mean()) < 1e-3
        assert float((got.float() - ref.float()).abs().max()) <= float(ref.float().abs().max()) * 2 ** -7
    _status_clean(cuda)


# ------------------------------------------------------------------ dequantisers, exact
@pytest.mark.parametrize("storage", ["fp8", "mxfp4"])
def test_dequant_exact_via_one_hot(cuda, storage):
    """With one-hot activation rows the down GEMM outputs single dequantised
    weights, which must equal the oracle's bit for bit."""
    H, I, E = 256, 192, 2
    if storage == "fp8":
        cfg = S.LayerConfig("probe", "qwen3", H, E, 1, I, "fp8", (1,))
        wq = S.make_qwen(cfg, seed=5)
        w = oracle.dequant_fp8(wq.down[1], wq.down_scale[1], (128, 128))         # [H, I]
        from moe_serving_profile_b200.layout import fp8_experts
        lay = fp8_experts(wq.gate, wq.gate_scale, wq.up, wq.up_scale, wq.down, wq.down_scale, (128, 128))
        fmt, w2 = _lib.W_FP8, lay.w2
    else:
        cfg = S.LayerConfig("probe", "gpt_oss", H, E, 1, I, "mxfp4", (1,))
        wg = S.make_gpt_oss(cfg, seed=6)
        w = oracle.decode_mxfp4(wg.dn_blocks[1], wg.dn_scales[1])                 # [H, I]
        from moe_serving_profile_b200.layout import gpt_oss_mxfp4_experts
        lay = gpt_oss_mxfp4_experts(wg.gu_blocks, wg.gu_scales, wg.gu_bias, wg.dn_blocks, wg.dn_scales,
                                    wg.dn_bias, 1.702, 7.0)
        fmt, w2 = _lib.W_MXFP4, lay.w2
    R = I                                                  # one row per reduction index, expert 1
    act = torch.zeros(R, lay.i_pad, dtype=torch.bfloat16)
    act[torch.arange(I), torch.arange(I)] = 1.0
    offsets = torch.tensor([0, 0, R], dtype=torch.int32)
    out = torch.zeros(R, H, dtype=torch.bfloat16, device=cuda)
    ops.expert_gemm(offsets=offsets.to(cuda), expert_begin=0, n_experts=E, max_rows=R, wfmt=fmt,
                    planes=1, feat_pad=lay.h_f, n_feat=H, k_pad=lay.i_pad, weight=w2.to(cuda),
                    fp8_block=lay.block, b_src=act.to(cuda), k_valid=I, epilogue=_lib.EPI_DOWN, out=out)
    assert torch.equal(out.cpu(), w.T.contiguous())


def test_backend_check_runtime_accepts_this_device(cuda):
    from moe_serving_profile_b200 import backend

    backend.check_runtime("qwen3", cuda, torch.bfloat16, "fp8")
    backend.check_runtime("gpt_oss", cuda, torch.bfloat16, "mxfp4")
