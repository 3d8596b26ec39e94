"""Host-side checks that need no GPU.

* the C-ABI library loads and exports every function ``include/b200moe.h``
  declares, and the ctypes binding registers each of them;
* arguments the C ABI rejects on the host (before any CUDA call) give the
  documented status codes;
* the torch wrappers refuse CPU tensors (there is no CPU path);
* the load-time weight layouts (padding, GPT-OSS gate/up de-interleave,
  MXFP4 scale padding) and the token-tile policy.
"""

import ctypes
import json
import re

import pytest
import torch

from moe_serving_profile_b200 import _lib, layout, ops
from moe_serving_profile_b200.experts import tile_policy
from tests.conftest import ROOT

HEADER = ROOT / "include" / "b200moe.h"


def _declared() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(b200moe_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    names = _declared()
    assert len(names) >= 11
    for n in names:
        assert hasattr(_lib.lib, n), f"{n} declared in the header but not exported"
    assert sorted(_lib.EXPORTED) == names
    assert _lib.version().startswith("b200moe")
    assert _lib.lib.b200moe_gemm_args_size() == ctypes.sizeof(_lib.GemmArgs)


def test_binding_constants_match_the_header():
    """Every status, format, epilogue, router mode and combine order of the
    header has the same value in the ctypes binding."""
    header = (ROOT / "include" / "b200moe.h").read_text()
    consts = dict(re.findall(r"^#define B200MOE_([A-Z0-9_]+) (\d+)\b", header, re.M))
    checked = 0
    for name, value in consts.items():
        if name == "H_":
            continue
        assert getattr(_lib, name) == int(value), name
        checked += 1
    assert checked >= 20 and consts["ORDER_SLOT_SUM"] == "2"


def test_permute_workspace_is_host_arithmetic():
    n = ctypes.c_size_t(0)
    assert _lib.lib.b200moe_permute_workspace(64, 8, 128, ctypes.byref(n)) == _lib.OK
    assert n.value == 0                                  # single-CTA path, no workspace
    assert _lib.lib.b200moe_permute_workspace(4096, 8, 128, ctypes.byref(n)) == _lib.OK
    assert n.value == 32 * 128 * 4                       # 32 chunks of 1024 assignments
    assert _lib.lib.b200moe_permute_workspace(-1, 8, 128, ctypes.byref(n)) == _lib.ERR_INVALID


FAKE = 0x10000   # a 16-byte aligned non-NULL address; never dereferenced by a rejected call


def test_c_abi_rejections_before_any_cuda_call():
    L = _lib.lib
    assert L.b200moe_permute(0, None, FAKE, 4, 2, 2000, FAKE, FAKE, FAKE, FAKE, None, 0) == _lib.ERR_UNSUPPORTED
    assert L.b200moe_permute(0, None, FAKE, 4, 0, 8, FAKE, FAKE, FAKE, FAKE, None, 0) == _lib.ERR_INVALID
    # 1 MiB of fixed scratch: 2049 chunks at E = 128 is one chunk too many
    assert L.b200moe_permute_noalloc(0, None, FAKE, 2049 * 128, 8, 128, FAKE, FAKE, FAKE, FAKE) == _lib.ERR_UNSUPPORTED
    assert "scratch" in L.b200moe_last_error().decode()
    assert L.b200moe_router(0, None, 7, FAKE, 64, FAKE, None, 4, 64, 8, 2, 1, FAKE, FAKE, FAKE, FAKE, None, 0) == _lib.ERR_INVALID
    assert L.b200moe_router(0, None, 0, FAKE, 64, FAKE, None, 4, 64, 600, 2, 1, FAKE, FAKE, FAKE, FAKE, None, 0) == _lib.ERR_UNSUPPORTED
    assert L.b200moe_expert_gemm(0, None, None) == _lib.ERR_INVALID


def _gemm_args(**over):
    a = _lib.GemmArgs(offsets=FAKE, expert_begin=0, n_experts=8, max_rows=64, token_tile=0,
                      split_k=0, wfmt=_lib.W_BF16, planes=1, feat_pad=256, n_feat=256, k_pad=128,
                      weight=FAKE, b_src=FAKE, ldb=128, b_rows=64, k_valid=128, b_div=1,
                      epilogue=_lib.EPI_DOWN, out=FAKE, ldo=256)
    for k, v in over.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("over,code", [
    ({"split_k": 2}, _lib.ERR_UNSUPPORTED),
    ({"n_experts": 2000}, _lib.ERR_UNSUPPORTED),
    ({"feat_pad": 200}, _lib.ERR_INVALID),
    ({"k_valid": 130}, _lib.ERR_INVALID),
    ({"ldo": 250, "n_feat": 250}, _lib.ERR_INVALID),
    ({"out": FAKE + 8}, _lib.ERR_INVALID),
    ({"planes": 2}, _lib.ERR_INVALID),                   # down epilogue with two planes
    ({"wfmt": _lib.W_FP8}, _lib.ERR_INVALID),             # fp8 without scales
    ({"token_tile": 48}, _lib.ERR_INVALID),
])
def test_gemm_argument_rejections(over, code):
    a = _gemm_args(**over)
    assert _lib.lib.b200moe_expert_gemm(0, None, ctypes.byref(a)) == code


def test_check_maps_status_codes_to_exceptions():
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_INVALID, "x")
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.ERR_UNSUPPORTED, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.ERR_CUDA, "x")


def test_wrappers_refuse_cpu_tensors():
    idx = torch.zeros(4, 2, dtype=torch.int64)
    with pytest.raises(ValueError, match="CUDA"):
        ops.permute(idx, 8)
    with pytest.raises(ValueError, match="CUDA"):
        ops.gather_rows(torch.zeros(4, 64, dtype=torch.bfloat16), torch.zeros(4, dtype=torch.int32), 1)


def test_w8a8_paths_refuse_before_device_work():
    """The efficient (W8A8) path checks its inputs on the host: CPU tensors,
    a q that is not e4m3 of the padded width, and non-FP8 expert weights are
    refused before anything is enqueued."""
    from types import SimpleNamespace

    from moe_serving_profile_b200 import experts as X
    from moe_serving_profile_b200 import qwen3
    from moe_serving_profile_b200.parallel import ParallelGroup

    with pytest.raises(ValueError, match="CUDA"):
        ops.act_quant_fp8(torch.zeros(4, 128, dtype=torch.bfloat16))
    kw = dict(offsets=torch.zeros(9, dtype=torch.int32), expert_begin=0, n_experts=8, max_rows=8, planes=2,
              feat_pad=128, n_feat=128, k_pad=256, weight=torch.zeros(16, dtype=torch.uint8),
              q=torch.zeros(8, 256, dtype=torch.float8_e4m3fn), q_scale=torch.zeros(8, 2),
              epilogue=_lib.EPI_SWIGLU, out=torch.zeros(8, 128, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="CUDA"):
        ops.w8a8_gemm(**kw)
    g, u, d = (torch.zeros(2, 128, 256, dtype=torch.bfloat16), torch.zeros(2, 128, 256, dtype=torch.bfloat16),
               torch.zeros(2, 256, 128, dtype=torch.bfloat16))
    w = layout.bf16_experts(g, u, d)
    perm = ops.Permutation(*(torch.zeros(n, dtype=torch.int32) for n in (2, 3, 8, 8)))
    with pytest.raises(ValueError, match="FP8"):
        X.run_experts_w8a8(w, torch.zeros(4, 256, dtype=torch.bfloat16), perm, None, K=2, num_experts=2,
                           expert_begin=0)
    m = qwen3.ParallelExperts(SimpleNamespace(num_experts=2, hidden_act="silu"), ParallelGroup(1), "efficient")
    for e, mods in enumerate(m.local):
        mods["gate_proj"] = qwen3.ExpertProjection(g[e])
        mods["up_proj"] = qwen3.ExpertProjection(u[e])
        mods["down_proj"] = qwen3.ExpertProjection(d[e])
    with pytest.raises(ValueError, match="block FP8"):
        m.prepare()
    # the refusal repeats on every call: nothing was packed or released by the first
    x, idx, wts = torch.zeros(3, 256, dtype=torch.bfloat16), torch.zeros(3, 2, dtype=torch.int64), torch.zeros(3, 2)
    for _ in range(2):
        with pytest.raises(ValueError, match="block FP8"):
            m(x, idx, wts)
    assert m.packed is None and m.local is not None
    with pytest.raises(ValueError):
        qwen3.ParallelExperts(SimpleNamespace(num_experts=2, hidden_act="silu"), ParallelGroup(1), "exact")


def test_efficient_numerics_dispatch(monkeypatch):
    """numerics="efficient" runs the W8A8 experts (with the slot-sum combine)
    for FP8 weights, the fused
    MXFP4 path (fp32 epilogues, the reference's grouped_mxfp4) for GPT-OSS
    MXFP4 weights and the weight-only experts for BF16; GPT-OSS needs MXFP4
    storage for it, as the reference's check_runtime does."""
    from types import SimpleNamespace

    from moe_serving_profile_b200 import experts as X
    from moe_serving_profile_b200 import gpt_oss
    from moe_serving_profile_b200.parallel import ParallelGroup

    calls, orders = [], []
    monkeypatch.setattr(X.ops, "permute", lambda idx, E: SimpleNamespace(inverse=None))
    monkeypatch.setattr(X.ops, "combine", lambda contrib, inverse, idx, order, **k: orders.append(order) or contrib)
    monkeypatch.setattr(X, "run_experts", lambda *a, **k: calls.append("weight_only") or "rows")
    monkeypatch.setattr(X, "run_experts_w8a8", lambda *a, **k: calls.append("w8a8") or "rows")
    # one GPU: BF16 weights take the single-call layer; GPT-OSS MXFP4 the
    # fused path with fp32 epilogues (grouped_mxfp4)
    monkeypatch.setattr(X.ops, "expert_layer", lambda *a, **k: calls.append("weight_only") or "rows")
    monkeypatch.setattr(X, "run_experts_mxfp4_efficient", lambda *a, **k: calls.append("mxfp4_f32") or "rows")
    for fmt, want in ((_lib.W_FP8, "w8a8"), (_lib.W_MXFP4, "mxfp4_f32"), (_lib.W_BF16, "weight_only")):
        out = X.layer_forward(SimpleNamespace(fmt=fmt, n_experts=4, gated_epilogue=_lib.EPI_CLAMP_SWIGLU),
                              torch.zeros(3, 64, dtype=torch.bfloat16),
                              torch.zeros(3, 2, dtype=torch.int64), torch.zeros(3, 2), num_experts=4,
                              expert_begin=0, numerics="efficient")
        assert out == "rows" and calls[-1] == want
        if fmt == _lib.W_FP8:
            # grouped_fp8's local combine: bf16-weighted rows, fp32 slot sum
            assert orders[-1] == _lib.ORDER_SLOT_SUM
    # two ranks, W8A8: the rank's experts [4, 8) are combined locally (slot
    # sum, routing weights applied there, not in the down GEMM), then the
    # [T, H] partials are all-reduced (efficient_kernels.py:269-274)
    seen = {}
    monkeypatch.setattr(X, "run_experts_w8a8",
                        lambda w, h, perm, weights, **k: seen.update(gemm_weights=weights) or "rows")
    monkeypatch.setattr(X.ops, "combine",
                        lambda rows, inverse, idx, order, **k: seen.update(order=order, **k) or "partial")
    group = SimpleNamespace(size=2, reduce=lambda t: seen.update(reduced=t) or "reduced")
    wts = torch.rand(3, 2)
    out = X.layer_forward(SimpleNamespace(fmt=_lib.W_FP8, n_experts=4, gated_epilogue=_lib.EPI_SWIGLU),
                          torch.zeros(3, 64, dtype=torch.bfloat16), torch.zeros(3, 2, dtype=torch.int64), wts,
                          num_experts=8, expert_begin=4, parallel=group, numerics="efficient")
    assert out == "reduced" and seen["reduced"] == "partial" and seen["gemm_weights"] is None
    assert seen["order"] == _lib.ORDER_SLOT_SUM and (seen["expert_lo"], seen["expert_hi"]) == (4, 8)
    assert seen["weights"] is wts
    conf = SimpleNamespace(num_local_experts=4, swiglu_alpha=1.702, swiglu_limit=7.0)
    gpt_oss.ParallelExperts(conf, ParallelGroup(1), "mxfp4", "efficient")
    with pytest.raises(ValueError, match="mxfp4"):
        gpt_oss.ParallelExperts(conf, ParallelGroup(1), "bf16", "efficient")


@pytest.mark.parametrize("T,K,E,bn", [(1, 8, 128, 16), (64, 8, 128, 16), (512, 8, 128, 64),
                                      (4096, 8, 128, 256), (2048, 4, 32, 256), (16, 4, 32, 16),
                                      (64, 4, 32, 16), (256, 8, 128, 32), (1024, 8, 128, 128)])
def test_tile_policy(T, K, E, bn):
    assert tile_policy(T, K, E) == bn
    assert tile_policy(T, K, E, 160) == min(bn, 160)


@pytest.mark.parametrize("T,bn", [(1, 16), (64, 16), (512, 64), (4096, 128), (16384, 128)])
def test_w8a8_tile_policy(T, bn):
    """The W8A8 launch caps the tile at 128 rows (four 128-column TMEM group
    buffers fill the 512 columns); Qwen3-30B-A3B: top-8 of 128 experts. A
    smaller cover picks smaller tiles."""
    assert tile_policy(T, 8, 128, 128) == bn
    assert tile_policy(512, 8, 128, 128, cover=1.0) == 32


def test_fp8_layout_pads_with_zeros():
    E, I, H = 2, 136, 200
    g = torch.Generator().manual_seed(0)
    mk = lambda *s: torch.randint(0, 255, s, generator=g, dtype=torch.uint8).view(torch.float8_e4m3fn)
    gate, up, down = mk(E, I, H), mk(E, I, H), mk(E, H, I)
    sc = lambda r, c: torch.rand(E, (r + 127) // 128, (c + 127) // 128, generator=g)
    w = layout.fp8_experts(gate, sc(I, H), up, sc(I, H), down, sc(H, I), (128, 128))
    # blobs: [E, feature tiles, k-blocks, 128 rows x 64 B + 16 B of scales]
    assert w.w1.shape == (E, 256 // 64, 256 // 64, 8208) and w.w2.shape == (E, 256 // 128, 256 // 64, 8208)
    w1 = layout.unpack_blob_rows(w.w1, 64, 2)
    w2 = layout.unpack_blob_rows(w.w2, 64, 1)[:, 0]
    assert torch.equal(w1[:, 0, :I, :H], gate.view(torch.uint8))
    assert torch.equal(w1[:, 1, :I, :H], up.view(torch.uint8))
    assert int(w1[:, :, I:].sum()) == 0 and int(w1[:, :, :, H:].sum()) == 0
    assert torch.equal(w2[:, :H, :I], down.view(torch.uint8)) and int(w2[:, H:].sum()) == 0


def test_gpt_oss_mxfp4_layout_deinterleaves_gate_up():
    E, I, H = 2, 64, 96
    g = torch.Generator().manual_seed(1)
    gu_b = torch.randint(0, 255, (E, 2 * I, H // 32, 16), generator=g, dtype=torch.uint8)
    gu_s = torch.randint(100, 140, (E, 2 * I, H // 32), generator=g, dtype=torch.uint8)
    gu_bias = torch.randn(E, 2 * I, generator=g)
    dn_b = torch.randint(0, 255, (E, H, I // 32, 16), generator=g, dtype=torch.uint8)
    dn_s = torch.randint(100, 140, (E, H, I // 32), generator=g, dtype=torch.uint8)
    dn_bias = torch.randn(E, H, generator=g)
    w = layout.gpt_oss_mxfp4_experts(gu_b, gu_s, gu_bias, dn_b, dn_s, dn_bias, 1.702, 7.0)
    assert w.i_pad == 128 and w.h_k == 128 and w.h_f == 128
    assert w.w1.shape == (E, 2, 2, 4352) and w.w2.shape == (E, 1, 2, 4352)
    w1 = layout.unpack_blob_rows(w.w1, 32, 2)
    assert torch.equal(w1[:, 0, :I, : H // 2], gu_b[:, 0::2].reshape(E, I, H // 2))
    assert torch.equal(w1[:, 1, :I, : H // 2], gu_b[:, 1::2].reshape(E, I, H // 2))
    # scales after the data: [128 rows][2 groups] per (tile, k-block)
    s1 = w.w1[..., 4096:].reshape(E, 2, 2, 2, 64, 2)        # [E, ft, kb, plane, row, group]
    s1 = s1.permute(0, 3, 1, 4, 2, 5).reshape(E, 2, 128, 4)  # [E, plane, feature, group]
    assert torch.equal(s1[:, 1, :I, : H // 32], gu_s[:, 1::2])
    assert bool((s1[:, :, I:] == 127).all()) and bool((s1[:, :, :, H // 32:] == 127).all())
    assert torch.equal(w.b1[:, 0, :I], gu_bias[:, 0::2].bfloat16())
    assert w.gated_epilogue == _lib.EPI_CLAMP_SWIGLU


# ------------------------------------------------------------------ native runtime host logic
def test_expert_plan_and_stats():
    from moe_serving_profile_b200 import native

    p = native.ExpertPlan(128, 8, 3)
    assert (p.experts_per_rank, p.expert_start, p.expert_end) == (16, 48, 64)
    dest, local = p.owner(torch.tensor([0, 17, 127]))
    assert dest.tolist() == [0, 1, 7] and local.tolist() == [0, 1, 15]
    with pytest.raises(ValueError):
        native.ExpertPlan(10, 4, 0)
    st = native.RoutingStats(counts=torch.tensor([2, 2, 0, 4]))
    assert st.expert_dead_fraction == 0.25
    assert abs(st.expert_load_cv - float(torch.tensor([2., 2., 0., 4.]).std(unbiased=False) / 2)) < 1e-7


def test_exchange_inplace_groups_by_source():
    from moe_serving_profile_b200 import native

    p0 = torch.tensor([[0], [1], [2]])          # rank 0 sends 1 row to 0, 2 rows to 1
    p1 = torch.tensor([[10], [11], [12]])       # rank 1 sends 2 rows to 0, 1 row to 1
    (r0, c0), (r1, c1) = native.exchange_inplace([p0, p1], [[1, 2], [2, 1]])
    assert r0.flatten().tolist() == [0, 10, 11] and c0.tolist() == [1, 2]
    assert r1.flatten().tolist() == [1, 2, 12] and c1.tolist() == [2, 1]


def test_empty_problems_return_ok_without_device_work():
    L = _lib.lib
    # T = 0 / n = 0 / no rows: nothing to enqueue, so no pointer is needed and no CUDA call runs
    assert L.b200moe_combine(0, None, None, 8, None, None, 0, 8, 64, 1, 16, 0, 128, 1, None, 1, None, 64) == _lib.OK
    assert L.b200moe_gather_rows(0, None, None, 64, None, 1, 0, 64, None, 64) == _lib.OK
    a = _lib.GemmArgs(max_rows=0)
    assert L.b200moe_expert_gemm(0, None, ctypes.byref(a)) == _lib.OK


def test_backend_checks_and_metadata():
    from moe_serving_profile_b200 import backend

    with pytest.raises(ValueError, match="CUDA"):
        backend.check_runtime("qwen3", "cpu", torch.bfloat16, "fp8")
    with pytest.raises(ValueError):
        backend.check_runtime("qwen3", "cuda", torch.float16, "fp8")
    with pytest.raises(ValueError):
        backend.check_runtime("gpt_oss", "cuda", torch.bfloat16, "fp8")
    with pytest.raises(ValueError):
        backend.check_runtime("llama", "cuda", torch.bfloat16, "fp8")
    m = backend.backend_metadata("gpt_oss", "reference")
    assert "mxfp4" in m["experts"] and "ordered" in m["expert_parallel"]
    assert "fp8" in backend.backend_metadata("qwen3", "fast")["experts"]
    assert "w8a8" in backend.backend_metadata("qwen3", "efficient")["experts"]
    m = backend.backend_metadata("gpt_oss", "efficient")
    assert "mxfp4" in m["experts"] and "weight_only" in m["experts"]
    assert m["expert_parallel"] == "local_combine_then_all_reduce"
    with pytest.raises(ValueError):
        backend.backend_metadata("qwen3", "exact")


def test_two_shot_exchange_needs_a_group_size_dividing_1024():
    """Above 16 MiB pushed per rank the fused exchange runs two-shot, whose
    row-to-owner slots need the group size to divide 1024: 3 ranks are
    refused (before any device work), 4 pass the argument checks."""
    peers = (ctypes.c_void_p * 4)(*([0x1000] * 4))
    fake = ctypes.c_void_p(0x1000)
    args = lambda world: (0, None, fake, 2048, fake, fake, 4000, 8, 2048, 0, 128, 0, None, 0, world, 0,
                          peers, 8192, fake, 2048, 0)
    assert _lib.lib.b200moe_combine_allreduce(*args(3)) == _lib.ERR_UNSUPPORTED
    assert _lib.lib.b200moe_combine_allreduce(*args(4)) != _lib.ERR_UNSUPPORTED


def test_checkpoint_loader_packs_what_layout_packs(tmp_path):
    """Load-time preparation from a safetensors checkpoint (sharded, with an
    index) gives the same packed experts as packing the same tensors directly,
    for one expert-parallel rank's slice (CPU)."""
    from safetensors.torch import save_file

    from moe_serving_profile_b200 import loader
    from moe_serving_profile_b200 import synthetic as S

    cfg = S.LayerConfig("probe", "qwen3", 256, 4, 2, 128, "fp8", (1,))
    w = S.make_qwen(cfg, seed=2)
    shard_a, shard_b, index = {}, {}, {}
    for e in range(cfg.experts):
        for proj, wt, sc in (("gate_proj", w.gate, w.gate_scale), ("up_proj", w.up, w.up_scale),
                             ("down_proj", w.down, w.down_scale)):
            name = f"model.layers.3.mlp.experts.{e}.{proj}"
            shard = shard_a if e < 2 else shard_b
            shard[name + ".weight"] = wt[e].contiguous()
            shard[name + ".weight_scale_inv"] = sc[e].contiguous()
            index[name + ".weight"] = index[name + ".weight_scale_inv"] = "a.safetensors" if e < 2 \
                else "b.safetensors"
    save_file(shard_a, str(tmp_path / "a.safetensors"))
    save_file(shard_b, str(tmp_path / "b.safetensors"))
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": index}))
    got = loader.qwen3_fp8_experts(tmp_path, layer=3, start=2, count=2, block=cfg.block, device="cpu")
    want = layout.fp8_experts(w.gate[2:4], w.gate_scale[2:4], w.up[2:4], w.up_scale[2:4],
                              w.down[2:4], w.down_scale[2:4], cfg.block)
    assert torch.equal(got.w1, want.w1) and torch.equal(got.w2, want.w2)
    assert (got.n_experts, got.hidden, got.inter) == (2, 256, 128)


def test_checkpoint_loader_gpt_oss_slices_the_expert_axis(tmp_path):
    from safetensors.torch import save_file

    from moe_serving_profile_b200 import loader
    from moe_serving_profile_b200 import synthetic as S

    cfg = S.LayerConfig("probe", "gpt_oss", 128, 4, 2, 64, "mxfp4", (1,))
    w = S.make_gpt_oss(cfg, seed=4)
    p = "model.layers.0.mlp.experts."
    save_file({p + "gate_up_proj_blocks": w.gu_blocks.contiguous(), p + "gate_up_proj_scales": w.gu_scales,
               p + "gate_up_proj_bias": w.gu_bias, p + "down_proj_blocks": w.dn_blocks.contiguous(),
               p + "down_proj_scales": w.dn_scales, p + "down_proj_bias": w.dn_bias},
              str(tmp_path / "model.safetensors"))
    got = loader.gpt_oss_mxfp4_experts(tmp_path, layer=0, start=1, count=2, device="cpu")
    want = layout.gpt_oss_mxfp4_experts(w.gu_blocks[1:3], w.gu_scales[1:3], w.gu_bias[1:3],
                                        w.dn_blocks[1:3], w.dn_scales[1:3], w.dn_bias[1:3], 1.702, 7.0)
    assert torch.equal(got.w1, want.w1) and torch.equal(got.w2, want.w2)
    assert torch.equal(got.b1, want.b1) and torch.equal(got.b2, want.b2)


def test_shared_expert_joins_the_routed_pack_when_it_fits():
    """MoELayer's joint pack (host arithmetic on CPU tensors): the shared
    expert is expert E, zero-padded to the routed experts' intermediate; the
    routed pack becomes a view of the joint one; a wider shared expert keeps
    its own launch."""
    from moe_serving_profile_b200 import native

    E, H, I = 4, 128, 256
    g = torch.Generator().manual_seed(3)
    gate_up = torch.randn(E, 2 * I, H, generator=g).bfloat16()
    down = torch.randn(E, H, I, generator=g).bfloat16()
    w = lambda *s: torch.randn(*s, generator=g).bfloat16()
    experts = native.LocalSwiGLUExperts(gate_up, down)
    before = experts.weights.w1.clone(), experts.weights.w2.clone()
    sg, su, sd = w(192, H), w(192, H), w(H, 192)
    joint = native._joint_weights(experts, native.SharedSwiGLU(sg, su, sd, w(1, H)))
    assert joint.n_experts == E + 1 and joint.inter == I and joint.i_pad == experts.weights.i_pad
    assert torch.equal(joint.w1[:E], before[0]) and torch.equal(joint.w2[:E], before[1])
    assert experts.weights.w1.data_ptr() == joint.w1.data_ptr() and experts.weights.n_experts == E
    assert torch.equal(joint.w1[E, 0, :192, :H], sg) and torch.equal(joint.w1[E, 1, :192, :H], su)
    assert not joint.w1[E, :, 192:].any() and not joint.w2[E, :, 192:].any()
    assert torch.equal(joint.w2[E, :H, :192], sd)
    wide = native.SharedSwiGLU(w(384, H), w(384, H), w(H, 384), w(1, H))
    assert native._joint_weights(native.LocalSwiGLUExperts(gate_up, down), wide) is None


def test_append_shared_slot_refuses_bad_shapes():
    idx = torch.zeros(3, 2, dtype=torch.int64)
    with pytest.raises(ValueError):
        ops.append_shared_slot(idx, torch.zeros(3, 2), torch.zeros(3, 1, dtype=torch.bfloat16), 4)
