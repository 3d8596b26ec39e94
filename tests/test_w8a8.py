"""W8A8 FP8 path: dynamic per-(row, 128-column) activation quantisation
(moe_serving/efficient_kernels.py:243-274).

CPU tests check the oracle's defining properties and the C ABI's argument
checks; GPU tests compare ``b200moe_act_quant_fp8`` with the oracle bit for
bit (e4m3 codes and fp32 scales), including the permuted-row gather, padded
columns, all-zero groups and values that saturate, and the W8A8 grouped GEMM
(``b200moe_w8a8_gemm``) and layer with the float64 oracle within the stated
tolerance.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from moe_serving_profile_b200 import _lib
from oracle import oracle


def _codes(q: torch.Tensor) -> torch.Tensor:
    return q.cpu().view(torch.uint8)


def test_oracle_quant_properties():
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(37, 300, generator=g) * 5).to(torch.bfloat16)
    x[4, 128:256] = 0                      # an all-zero group
    q, s = oracle.act_quant_fp8(x, k_pad=320)
    assert q.shape == (37, 320) and s.shape == (37, 3)
    assert (_codes(q)[:, 300:] == 0).all()          # padded columns quantise zeros
    assert s[4, 1] == 1.0 and (_codes(q)[4, 128:256] == 0).all()
    # every nonzero group's amax element lands on +-448 and the rest within half an e4m3 step
    qp, xp = torch.zeros(37, 384), torch.zeros(37, 384)
    qp[:, :320] = q.float()
    xp[:, :300] = x.float()
    qg, xg = qp.view(37, 3, 128), xp.view(37, 3, 128)
    assert (qg.abs().amax(-1)[s != 1.0] == 448.0).all()
    err = (qg * s[..., None] - xg).abs()
    assert (err <= xg.abs() * 2.0 ** -4 + s[..., None] * 2.0 ** -10).all()
    # the gather form equals gathering first
    src = torch.tensor([5, 0, 72, 9, 9], dtype=torch.int32)
    q2, s2 = oracle.act_quant_fp8(x, k_pad=320, rows_src=src, src_div=2)
    q3, s3 = oracle.act_quant_fp8(x[src.long() // 2], k_pad=320)
    assert torch.equal(_codes(q2), _codes(q3)) and torch.equal(s2, s3)


def test_e4m3_encoder_c_matches_torch():
    """The C e4m3 encoder (written from the format's definition) agrees with
    torch's float8_e4m3fn conversion on every code, the midpoints between
    neighbouring codes (ties to even), values just off them, subnormals and
    saturation."""
    codes = torch.arange(256, dtype=torch.uint8)
    vals = codes.view(torch.float8_e4m3fn).float()
    finite = vals[vals.isfinite()].unique()
    pos = finite[finite >= 0]
    mids = (pos[1:] + pos[:-1]) / 2
    probes = torch.cat([finite, mids, mids * (1 + 2 ** -20), mids * (1 - 2 ** -20), -mids,
                        torch.tensor([447.9, 448.0, 460.0, 1e6, 2.0 ** -10, 2.0 ** -11, 3 * 2.0 ** -11]),
                        torch.randn(4000, generator=torch.Generator().manual_seed(5)) * 100])
    got = oracle.f32_to_e4m3_c(probes)
    want = probes.clamp(-448.0, 448.0).to(torch.float8_e4m3fn).view(torch.uint8)
    # +-0 may differ only in sign for values that round to zero
    zero = (want & 0x7f) == 0
    assert torch.equal(got[~zero], want[~zero]) and ((got[zero] & 0x7f) == 0).all()


def test_act_quant_oracles_agree():
    """The torch oracle and the plain-C restatement of the activation
    quantiser give the same codes and scales (gather, padding, all-zero
    groups, one huge value flushing its neighbours)."""
    g = torch.Generator().manual_seed(9)
    x = (torch.randn(40, 300, generator=g) * torch.rand(40, 1, generator=g) * 30).to(torch.bfloat16)
    x[3, :128] = 0
    x[5, 7] = 3.0e38
    src = torch.randint(0, 80, (57,), generator=g, dtype=torch.int32)
    for rows_src, div in ((None, 1), (src, 2)):
        qt, st = oracle.act_quant_fp8(x, k_pad=320, rows_src=rows_src, src_div=div)
        qc, scc = oracle.act_quant_fp8_c(x, k_pad=320, rows_src=rows_src, src_div=div)
        assert torch.equal(st, scc)
        assert torch.equal(_codes(qt), qc)


def test_act_quant_argument_checks():
    L = _lib.lib
    # no rows: nothing to enqueue, no pointer needed
    assert L.b200moe_act_quant_fp8(0, None, None, 128, None, 1, 0, 128, 128, None, None, None, 0, 0) == _lib.OK
    # k_pad not a multiple of 16, k_valid not a multiple of 4, k_valid > k_pad, ldx < k_valid
    assert L.b200moe_act_quant_fp8(0, None, None, 128, None, 1, 4, 128, 120, None, None, None, 0, 0) == _lib.ERR_INVALID
    assert L.b200moe_act_quant_fp8(0, None, None, 128, None, 1, 4, 126, 128, None, None, None, 0, 0) == _lib.ERR_INVALID
    assert L.b200moe_act_quant_fp8(0, None, None, 256, None, 1, 4, 256, 128, None, None, None, 0, 0) == _lib.ERR_INVALID
    assert L.b200moe_act_quant_fp8(0, None, None, 64, None, 1, 4, 128, 128, None, None, None, 0, 0) == _lib.ERR_INVALID
    assert L.b200moe_act_quant_fp8(0, None, None, 128, None, 0, 4, 128, 128, 1, 1, None, 0, 0) == _lib.ERR_INVALID
    # a row range that runs backwards
    assert L.b200moe_act_quant_fp8(0, None, None, 128, None, 1, 4, 128, 128, 1, 1, 1, 3, 2) == _lib.ERR_INVALID


CASES = [  # rows, k_valid, k_pad, gather divisor (0 = no gather)
    (1, 2048, 2048, 0),
    (257, 2048, 2048, 8),
    (1000, 768, 768, 4),
    (64, 2880, 2944, 0),
    (33, 300, 320, 0),
]


@pytest.mark.gpu
@pytest.mark.parametrize("rows,k_valid,k_pad,div", CASES)
def test_act_quant_matches_oracle(cuda, rows, k_valid, k_pad, div):
    from moe_serving_profile_b200 import ops

    g = torch.Generator().manual_seed(rows * 7 + k_valid)
    src_rows = rows if not div else max(1, rows // 2)
    x = (torch.randn(src_rows, k_valid, generator=g) * torch.rand(src_rows, 1, generator=g) * 20)
    x = x.to(torch.bfloat16)
    x[0, : min(128, k_valid)] = 0                                 # an all-zero group
    if src_rows > 1:
        x[1, 5] = 3.0e38                                          # a group dominated by one huge value
        x[1, 6] = 1.0e-30                                         # which flushes its neighbours to 0
    src = None
    if div:
        src = torch.randint(0, src_rows * div, (rows,), generator=g, dtype=torch.int32)
    q_ref, s_ref = oracle.act_quant_fp8(x, k_pad=k_pad, rows_src=src, src_div=max(div, 1))
    q, s = ops.act_quant_fp8(x.to(cuda), k_pad=k_pad,
                             rows_src=None if src is None else src.to(cuda), src_div=max(div, 1))
    torch.cuda.synchronize()
    assert torch.equal(s.cpu(), s_ref)
    assert torch.equal(_codes(q), _codes(q_ref))


@pytest.mark.gpu
def test_act_quant_strided_rows(cuda):
    """Rows of a wider buffer (ldx > k_valid), e.g. the activated half of a gate/up output."""
    from moe_serving_profile_b200 import ops

    g = torch.Generator().manual_seed(11)
    wide = (torch.randn(90, 1536, generator=g) * 3).to(torch.bfloat16)
    q_ref, s_ref = oracle.act_quant_fp8(wide[:, :768].contiguous())
    q, s = ops.act_quant_fp8(wide.to(cuda)[:, :768])
    torch.cuda.synchronize()
    assert torch.equal(s.cpu(), s_ref) and torch.equal(_codes(q), _codes(q_ref))


# ------------------------------------------------------------------ W8A8 grouped GEMM
#
# Tolerance of the GEMM against the float64 oracle (same e4m3 codes and
# scales on both sides; only the fp32 summation inside the tensor core and the
# fp32 promotion differ, so bf16 outputs differ by rounding): relative L2
# <= 4e-3 and max |error| <= 2^-6 * max |oracle|. The layer is also held to
# the reference's own acceptance bar for efficient FP8 against its
# dequantise-then-BF16 numerics, relative L2 < 0.08
# (tests/helpers/check_grouped_fp8.py:42).

W8A8_REL_L2 = 4e-3
W8A8_MAX_ABS_FRAC = 2 ** -6


def test_w8a8_oracle_equals_scaled_product():
    """The grouped restatement equals the plain product of the dequantised
    operands (scales folded in), for ragged K and 64-row scale blocks."""
    g = torch.Generator().manual_seed(4)
    x = (torch.randn(9, 300, generator=g) * 2).to(torch.bfloat16)
    q, qs = oracle.act_quant_fp8(x, k_pad=320)
    w = (torch.randn(70, 300, generator=g) * 40).clamp(-448, 448).to(torch.float8_e4m3fn)
    ws = torch.rand(2, 3, generator=g) + 0.5
    d = oracle.w8a8_matmul(q, qs, w, ws, (64, 128))
    xa = q.double()[:, :300] * qs.double().repeat_interleave(128, 1)[:, :300]
    wa = w.double() * ws.double().repeat_interleave(64, 0)[:70].repeat_interleave(128, 1)[:, :300]
    assert torch.allclose(d, xa @ wa.T, rtol=1e-12, atol=1e-12)


def test_w8a8_layer_oracle_meets_reference_bar():
    """The W8A8 restatement stays within the reference's own acceptance bar
    (relative L2 < 0.08) of the dequantise-then-BF16 layer on the tiny
    Qwen3 layer."""
    from moe_serving_profile_b200 import synthetic as S

    cfg = S.CONFIGS["qwen3-tiny"]
    w = S.make_qwen(cfg, seed=0)
    x = S.make_hidden(64, cfg.hidden, seed=100)
    idx = oracle.topk(oracle.router_logits(x, w.router, None, 0), cfg.top_k)
    sc = torch.softmax(torch.randn(64, cfg.top_k, generator=torch.Generator().manual_seed(1)), -1)
    ref = oracle.qwen_layer(x, idx, sc, w.gate, w.gate_scale, w.up, w.up_scale, w.down, w.down_scale,
                            cfg.block)
    out = oracle.qwen_w8a8_layer(x, idx, sc, w.gate, w.gate_scale, w.up, w.up_scale, w.down,
                                 w.down_scale, cfg.block)
    r = float((out.float() - ref.float()).norm() / ref.float().norm())
    assert out.isfinite().all() and 0 < r < 0.08


def test_w8a8_gemm_argument_checks():
    """Rejections happen on the host, before any device work."""
    L = _lib.lib
    fake = 0x10000

    def args(**kw):
        a = _lib.GemmArgs()
        a.offsets, a.weight, a.out = fake, fake, fake
        a.expert_begin, a.n_experts, a.max_rows = 0, 8, 128
        a.wfmt, a.planes, a.epilogue = _lib.W_FP8, 2, _lib.EPI_SWIGLU
        a.feat_pad, a.n_feat, a.k_pad = 128, 128, 256
        a.sc_br, a.sc_bc = 128, 128
        a.b_rows, a.b_div, a.ldo = 128, 1, 128
        for k, v in kw.items():
            setattr(a, k, v)
        return ctypes.byref(a)

    def rc(**kw):
        return L.b200moe_w8a8_gemm(0, None, args(**kw), fake, fake)

    assert L.b200moe_w8a8_gemm(0, None, args(max_rows=0), None, None) == _lib.OK
    assert rc(wfmt=_lib.W_BF16) == _lib.ERR_INVALID                 # FP8 weights only
    assert rc(sc_bc=64) == _lib.ERR_INVALID                         # 128-column scale groups
    assert rc(sc_br=32) == _lib.ERR_INVALID
    assert rc(epilogue=_lib.EPI_CLAMP_SWIGLU) == _lib.ERR_INVALID   # no GPT-OSS epilogue
    assert rc(planes=1) == _lib.ERR_INVALID                         # gated epilogue needs two planes
    assert rc(bias=fake) == _lib.ERR_INVALID
    assert rc(b_map=fake) == _lib.ERR_INVALID
    assert rc(token_tile=160) == _lib.ERR_INVALID
    assert rc(k_pad=96) == _lib.ERR_INVALID
    assert rc(n_feat=132) == _lib.ERR_INVALID
    assert L.b200moe_w8a8_gemm(0, None, args(), fake + 8, fake) == _lib.ERR_INVALID  # unaligned q


def _gemm_case(cuda, E, H, I, T, K, tile, seed, empty_expert=False):
    from moe_serving_profile_b200 import layout, ops
    from moe_serving_profile_b200 import synthetic as S

    cfg = S.LayerConfig("w8a8-case", "qwen3", H, E, K, I, "fp8", (T,))
    w = S.make_qwen(cfg, seed=seed)
    x = S.make_hidden(T, H, seed=seed + 100)
    g = torch.Generator().manual_seed(seed)
    lo = 1 if empty_expert else 0
    idx = torch.stack([torch.randperm(E - lo, generator=g)[:K] + lo for _ in range(T)]).to(torch.int64)
    wts = torch.softmax(torch.randn(T, K, generator=g), -1)
    packed = layout.fp8_experts(w.gate.to(cuda), w.gate_scale.to(cuda), w.up.to(cuda),
                                w.up_scale.to(cuda), w.down.to(cuda), w.down_scale.to(cuda), cfg.block)
    perm = ops.permute(idx.to(cuda), E)
    R = T * K
    q, qs = ops.act_quant_fp8(x.to(cuda), k_pad=packed.h_k, rows_src=perm.perm_src, src_div=K)
    act = torch.full((R, packed.i_pad), float("nan"), device=cuda, dtype=torch.bfloat16)
    ops.w8a8_gemm(offsets=perm.offsets, expert_begin=0, n_experts=E, max_rows=R, planes=2,
                  feat_pad=packed.i_pad, n_feat=I, k_pad=packed.h_k, weight=packed.w1, q=q, q_scale=qs,
                  epilogue=_lib.EPI_SWIGLU, out=act, token_tile=tile)
    q2, qs2 = ops.act_quant_fp8(act[:, :I], k_pad=packed.i_pad)
    out = torch.full((R, H), float("nan"), device=cuda, dtype=torch.bfloat16)
    ops.w8a8_gemm(offsets=perm.offsets, expert_begin=0, n_experts=E, max_rows=R, planes=1,
                  feat_pad=packed.h_f, n_feat=H, k_pad=packed.i_pad, weight=packed.w2, q=q2,
                  q_scale=qs2, epilogue=_lib.EPI_DOWN, row_weight=wts.reshape(-1).to(cuda),
                  row_src=perm.perm_src, out=out, token_tile=tile)
    torch.cuda.synchronize()
    assert _lib.device_status(cuda.index) == 0
    offs = perm.offsets.cpu().tolist()
    src = perm.perm_src.cpu().long()
    act_c, q2_c, qs2_c, out_c = act.cpu(), q2.cpu(), qs2.cpu(), out.cpu()
    act_ref = torch.zeros(R, I, dtype=torch.bfloat16)
    out_ref = torch.zeros(R, H, dtype=torch.bfloat16)
    for e in range(E):
        a, b = offs[e], offs[e + 1]
        if a == b:
            continue
        qe, qse = oracle.act_quant_fp8(x[src[a:b] // K], k_pad=packed.h_k)
        gate = oracle.w8a8_matmul(qe, qse, w.gate[e], w.gate_scale[e], cfg.block).to(torch.bfloat16)
        up = oracle.w8a8_matmul(qe, qse, w.up[e], w.up_scale[e], cfg.block).to(torch.bfloat16)
        act_ref[a:b] = torch.nn.functional.silu(gate.float()).to(torch.bfloat16) * up
        # the down GEMM is checked on the GPU's own quantised activations
        y = oracle.w8a8_matmul(q2_c[a:b], qs2_c[a:b], w.down[e], w.down_scale[e], cfg.block)
        rw = wts.reshape(-1)[src[a:b]]
        out_ref[a:b] = (y.to(torch.bfloat16) * rw[:, None]).to(torch.bfloat16)
    for got, ref, what in ((act_c[:, :I], act_ref, "gate/up"), (out_c, out_ref, "down")):
        r = float((got.float() - ref.float()).norm() / ref.float().norm())
        m = float((got.float() - ref.float()).abs().max())
        bound = W8A8_MAX_ABS_FRAC * float(ref.float().abs().max())
        print(f"\n{what} E{E} H{H} I{I} T{T} K{K} tile {tile}: rel_l2={r:.2e} max_abs={m:.2e} (bound {bound:.2e})")
        assert got.isfinite().all(), what
        assert r <= W8A8_REL_L2 and m <= bound, (what, r, m)


@pytest.mark.gpu
@pytest.mark.parametrize("tile", [16, 32, 64, 128])
def test_w8a8_gemm_tiles_match_oracle(cuda, tile):
    """Tiny Qwen3 layer shapes (H 256, 8 experts, top-2, I 128, 64 tokens)
    at every token tile; expert 0 receives no rows."""
    _gemm_case(cuda, 8, 256, 128, 64, 2, tile, seed=tile, empty_expert=True)


@pytest.mark.gpu
@pytest.mark.parametrize("E,H,I,T,K", [
    (16, 2048, 768, 200, 4),     # Qwen3-30B-A3B expert shapes, ~50 rows per expert
    (4, 320, 256, 37, 2),        # odd 64-column k-block count (a one-k-block last group)
])
def test_w8a8_gemm_shapes_match_oracle(cuda, E, H, I, T, K):
    _gemm_case(cuda, E, H, I, T, K, 0, seed=E + H)


@pytest.mark.gpu
@pytest.mark.parametrize("cfg_name,T", [("qwen3-tiny", 64), ("qwen3-30b-a3b", 64), ("qwen3-30b-a3b", 512)])
def test_w8a8_layer_matches_oracle(cuda, cfg_name, T):
    """``ParallelExperts(numerics="efficient")`` against the W8A8 oracle layer
    (GEMM tolerance, relative L2 <= 1e-2 after the combine) and against the
    dequantise-then-BF16 reference layer (the reference's bar, < 0.08)."""
    from types import SimpleNamespace

    from moe_serving_profile_b200 import qwen3
    from moe_serving_profile_b200 import synthetic as S
    from moe_serving_profile_b200.parallel import ParallelGroup

    cfg = S.CONFIGS[cfg_name]
    w = S.make_qwen(cfg, seed=3)
    x = S.make_hidden(T, cfg.hidden, seed=103)
    idx = oracle.topk(oracle.router_logits(x, w.router, None, 0), cfg.top_k)
    sc = torch.softmax(torch.randn(T, cfg.top_k, generator=torch.Generator().manual_seed(T)), -1)
    m = qwen3.ParallelExperts(SimpleNamespace(num_experts=cfg.experts, hidden_act="silu"),
                              ParallelGroup(1), "efficient")
    for e, mods in enumerate(m.local):
        mods["gate_proj"] = qwen3.ExpertProjection(w.gate[e].to(cuda), w.gate_scale[e].to(cuda), cfg.block)
        mods["up_proj"] = qwen3.ExpertProjection(w.up[e].to(cuda), w.up_scale[e].to(cuda), cfg.block)
        mods["down_proj"] = qwen3.ExpertProjection(w.down[e].to(cuda), w.down_scale[e].to(cuda), cfg.block)
    out = m(x.to(cuda), idx.to(cuda), sc.to(cuda)).cpu()
    assert _lib.device_status(cuda.index) == 0
    want = oracle.qwen_w8a8_layer(x, idx, sc, w.gate, w.gate_scale, w.up, w.up_scale, w.down,
                                  w.down_scale, cfg.block)
    ref = oracle.qwen_layer(x, idx, sc, w.gate, w.gate_scale, w.up, w.up_scale, w.down, w.down_scale,
                            cfg.block)
    r_w8 = float((out.float() - want.float()).norm() / want.float().norm())
    r_ref = float((out.float() - ref.float()).norm() / ref.float().norm())
    print(f"\n{cfg_name} T{T}: vs W8A8 oracle {r_w8:.2e}, vs reference numerics {r_ref:.2e}")
    assert out.isfinite().all()
    assert r_w8 <= 1e-2 and r_ref < 0.08
