"""Property tests of the oracle's integer and ordering stages against the
reference's own definitions, at random shapes (CPU only): the permutation is
the order of ``torch.where(indices.T == e)`` over ascending experts
(moe_serving/parallel_numerics.py:21-26), and the expert-order combine is the
bf16 ``index_add_`` of each expert's contribution rows in turn
(parallel_numerics.py:26-36), restricted to a rank's expert range."""

import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from oracle import oracle


@st.composite
def routings(draw):
    """[T, K] expert ids, distinct within a row (a router's top-k), with an
    optional sprinkling of dropped ids (negative or >= E)."""
    T = draw(st.integers(0, 48))
    K = draw(st.integers(1, 8))
    E = draw(st.integers(K, 24))
    g = torch.Generator().manual_seed(draw(st.integers(0, 2 ** 31 - 1)))
    if T:
        idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).long()
    else:
        idx = torch.empty(0, K, dtype=torch.long)
    if draw(st.booleans()) and T:
        drop = torch.rand(T, K, generator=g) < 0.15
        idx[drop] = torch.where(torch.rand(T, K, generator=g) < 0.5, -1, E + 3)[drop]
    return idx, E, g


def _where_order(idx: torch.Tensor, E: int) -> torch.Tensor:
    T, K = idx.shape
    parts = []
    for e in range(E):
        slots, tokens = torch.where(idx.T == e)
        parts.append(tokens * K + slots)
    return torch.cat(parts) if parts else torch.empty(0, dtype=torch.long)


@settings(max_examples=80, deadline=None)
@given(routings())
def test_permutation_is_the_reference_where_order(case):
    idx, E, _ = case
    T, K = idx.shape
    counts, offsets, perm, inv = oracle.permute(idx, E)
    valid = (idx >= 0) & (idx < E)
    n = int(valid.sum())
    assert int(offsets[-1]) == n and int(offsets[0]) == 0
    assert torch.equal(counts.long(), torch.bincount(idx[valid], minlength=E)[:E])
    assert torch.equal(perm[:n].long(), _where_order(idx, E))
    flat_valid = valid.reshape(-1)
    assert bool((inv[~flat_valid] == -1).all())
    assert torch.equal(inv[perm[:n].long()].long(), torch.arange(n))


@settings(max_examples=60, deadline=None)
@given(routings(), st.integers(0, 2), st.booleans())
def test_expert_order_combine_is_index_add_per_expert(case, split, scaled):
    idx, E, g = case
    T, K = idx.shape
    H = 16
    counts, offsets, perm, inv = oracle.permute(idx, E)
    n = int(offsets[-1])
    rows = torch.randn(max(n, 1), H, generator=g).to(torch.bfloat16)
    weights = torch.rand(T, K, generator=g)
    # a rank's expert range: all experts, the lower half or the upper half
    lo, hi = [(0, E), (0, E // 2), (E // 2, E)][split]
    got = oracle.combine(rows, inv, idx, order=0, lo=lo, hi=hi, weights=weights if scaled else None)
    ref = torch.zeros(T, H, dtype=torch.bfloat16)
    pos = 0
    for e in range(E):
        slots, tokens = torch.where(idx.T == e)
        values = rows[pos:pos + tokens.numel()]
        pos += tokens.numel()
        if not lo <= e < hi or tokens.numel() == 0:
            continue
        contrib = (values * weights[tokens, slots, None]).to(torch.bfloat16) if scaled else values
        ref.index_add_(0, tokens, contrib)
    assert torch.equal(got, ref)
