"""W8A8 FP8 path: dynamic per-(row, 128-column) activation quantisation
(moe_serving/efficient_kernels.py:243-274).

CPU tests check the oracle's defining properties and the C ABI's argument
checks; GPU tests compare ``b200moe_act_quant_fp8`` with the oracle bit for
bit (e4m3 codes and fp32 scales), including the permuted-row gather, padded
columns, all-zero groups and values that saturate.
"""

from __future__ import annotations

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


def test_act_quant_argument_checks():
    L = _lib.lib
    # no rows: nothing to enqueue, no pointer needed
    assert L.b200moe_act_quant_fp8(0, None, None, 128, None, 1, 0, 128, 128, None, None) == _lib.OK
    # k_pad not a multiple of 16, k_valid not a multiple of 4, k_valid > k_pad, ldx < k_valid
    assert L.b200moe_act_quant_fp8(0, None, None, 128, None, 1, 4, 128, 120, None, None) == _lib.ERR_INVALID
    assert L.b200moe_act_quant_fp8(0, None, None, 128, None, 1, 4, 126, 128, None, None) == _lib.ERR_INVALID
    assert L.b200moe_act_quant_fp8(0, None, None, 256, None, 1, 4, 256, 128, None, None) == _lib.ERR_INVALID
    assert L.b200moe_act_quant_fp8(0, None, None, 64, None, 1, 4, 128, 128, None, None) == _lib.ERR_INVALID
    assert L.b200moe_act_quant_fp8(0, None, None, 128, None, 0, 4, 128, 128, 1, 1) == _lib.ERR_INVALID


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
