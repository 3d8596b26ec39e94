"""b200moe_permute_noalloc against b200moe_permute, through the C ABI.

The no-allocation entry point keeps its chunk histograms in one fixed device
array per device, so its results must not depend on what an earlier call left
there. Each test makes two calls in a row on one stream with different shapes
and compares both with the workspace entry point bit for bit. The file is
named to be collected last, so the tests also run after every other GPU test
has used the device.
"""

import pytest
import torch

from moe_serving_profile_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _ids(T, K, E, seed, skew=False):
    g = torch.Generator().manual_seed(seed)
    if skew:
        return torch.randint(0, max(1, E // 16), (T, K), generator=g)
    return torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).long()


def _buffers(T, K, E, dev):
    return ops.Permutation(
        torch.full((E,), -7, device=dev, dtype=torch.int32),
        torch.full((E + 1,), -7, device=dev, dtype=torch.int32),
        torch.full((T * K,), -7, device=dev, dtype=torch.int32),
        torch.full((T * K,), -7, device=dev, dtype=torch.int32),
    )


def _same(a: ops.Permutation, b: ops.Permutation):
    n = int(b.offsets[-1])
    assert torch.equal(a.counts, b.counts) and torch.equal(a.offsets, b.offsets)
    assert torch.equal(a.perm_src[:n], b.perm_src[:n]) and torch.equal(a.inverse, b.inverse)


# (T, K, E) pairs: the multi-kernel path (T*K > 8192) with different chunk
# counts and expert counts back to back, and the single-CTA path next to it.
CASES = [
    ((4096, 8, 128), (3000, 6, 64)),
    ((16384, 8, 128), (1500, 4, 256)),
    ((64, 8, 128), (9000, 8, 128)),
]


@pytest.mark.parametrize("first,second", CASES)
def test_noalloc_matches_workspace_permute(cuda, first, second):
    _lib.device_status(cuda.index)            # start from a clean status word
    idx1 = _ids(*first, seed=sum(first)).to(cuda)
    idx2 = _ids(*second, seed=sum(second), skew=True).to(cuda)
    ref1 = ops.permute(idx1, first[2])
    ref2 = ops.permute(idx2, second[2])
    out1 = _buffers(*first, cuda)
    out2 = _buffers(*second, cuda)
    torch.cuda.synchronize(cuda)
    before = torch.cuda.memory_stats(cuda).get("allocation.all.allocated", 0)
    ops.permute_noalloc(idx1, first[2], out1)
    ops.permute_noalloc(idx2, second[2], out2)
    after = torch.cuda.memory_stats(cuda).get("allocation.all.allocated", 0)
    assert after == before, "the no-allocation path allocated through torch"
    torch.cuda.synchronize(cuda)
    _same(out1, ref1)
    _same(out2, ref2)
    assert _lib.device_status(cuda.index) == 0


def test_noalloc_dropped_ids_and_empty(cuda):
    _lib.device_status(cuda.index)
    T, K, E = 5000, 8, 64
    idx = _ids(T, K, E, seed=3, skew=True)
    idx[7, 3] = E + 5
    idx[100, 0] = -1
    idx = idx.to(cuda)
    ref = ops.permute(idx, E)
    assert _lib.device_status(cuda.index) & _lib.STATUS_BAD_INDEX
    out = _buffers(T, K, E, cuda)
    ops.permute_noalloc(idx, E, out)
    assert _lib.device_status(cuda.index) & _lib.STATUS_BAD_INDEX
    _same(out, ref)
    empty = _buffers(0, K, E, cuda)
    ops.permute_noalloc(torch.empty(0, K, dtype=torch.int64, device=cuda), E, empty)
    assert int(empty.offsets.abs().sum()) == 0 and int(empty.counts.abs().sum()) == 0


def test_noalloc_rejects_beyond_scratch(cuda):
    # 1 MiB of scratch holds 2048 chunks of 1024 assignments at E = 128
    T, K, E = 2048 * 1024 // 8 + 1, 8, 128
    idx = torch.zeros(1, K, dtype=torch.int64, device=cuda)   # never read: rejected on the host
    rc = _lib.lib.b200moe_permute_noalloc(cuda.index, None, idx.data_ptr(), T, K, E, idx.data_ptr(),
                                          idx.data_ptr(), idx.data_ptr(), idx.data_ptr())
    assert rc == _lib.ERR_UNSUPPORTED
    assert "scratch" in _lib.lib.b200moe_last_error().decode()
