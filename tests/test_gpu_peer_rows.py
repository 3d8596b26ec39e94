"""Peer-memory row exchanges (b200moe_a2a_counts / dispatch / return and
b200moe_ep_gather) with every rank's buffer on one GPU.

The ranks' kernels run one after another on one GPU, so no kernel may wait
for another that has not run yet: before every call each buffer's flag table
is preset to an epoch above the call's, so every wait is satisfied either by
the preset or by a rank that ran earlier in the sequence, and each
rank's count board is preset with all ranks' counts (each rank then rewrites
its own row with the same values). What is checked is the placement and the
data movement: every row lands where the receiving rank's grouped GEMMs and
the source's combine expect it. The all-to-all output of every rank must
equal native.simulate_routed (the NCCL-free one-process reference path, the
same expert kernels) bit for bit, over two calls in a row; the gather must
leave every rank's area holding every rank's rows.
"""

import ctypes
from types import SimpleNamespace

import pytest
import torch

from moe_serving_profile_b200 import _lib, native, ops
from moe_serving_profile_b200._lib import check, lib
from moe_serving_profile_b200.parallel import PEER_ROWS_HEADER_BYTES, _DeviceRows

pytestmark = pytest.mark.gpu

FLAG_WORDS = 5 * 8          # PeerRowsHeader.flags [phase][source]
BOARD_OFFSET = 256          # PeerRowsHeader.board [8][1024] int32, byte offset


class _I32:
    def __init__(self, ptr, rows, cols):
        self.__cuda_array_interface__ = {"shape": (rows, cols), "typestr": "<i4",
                                         "data": (ptr, False), "version": 3, "strides": None}


def _view(ptr, rows, cols, typestr, device):
    """A tensor aliasing rows x cols of bf16 ("<i2") or int32 ("<i4") at ptr."""
    if typestr == "<i2":
        return torch.as_tensor(_DeviceRows(ptr, rows, cols), device=device).view(torch.bfloat16)
    return torch.as_tensor(_I32(ptr, rows, cols), device=device)


def _buffers(world, H, cap_a, cap_b, device):
    """One zeroed buffer per emulated rank on ``device``, flags preset."""
    nbytes = lib.b200moe_peer_rows_bytes(H, cap_a, cap_b)
    ptrs = []
    for _ in range(world):
        p = ctypes.c_void_p()
        check(lib.b200moe_p2p_alloc(device.index, nbytes, ctypes.byref(p)), "p2p_alloc")
        ptrs.append(p.value)
    bufs = []
    for r in range(world):
        base = ptrs[r] + PEER_ROWS_HEADER_BYTES
        b = SimpleNamespace(peers=ptrs, world=world, rank=r, cap_a=cap_a, cap_b=cap_b, hidden=H,
                            timeout_ns=0, local=ptrs[r])
        b.area_a = _view(base, cap_a, H, "<i2", device)
        b.area_b = _view(base + cap_a * H * 2, cap_b, H, "<i2", device) if cap_b else None
        b.flags = _view(ptrs[r], 1, FLAG_WORDS, "<i4", device)
        b.board = _view(ptrs[r] + BOARD_OFFSET, 8, 1024, "<i4", device)
        b.flags.fill_(1 << 20)
        bufs.append(b)
    return bufs


def _free(bufs, device):
    torch.cuda.synchronize(device)
    for p in bufs[0].peers:
        lib.b200moe_p2p_free(device.index, p)


def _experts(E, H, I, world, seed, device):
    g = torch.Generator().manual_seed(seed)
    gate_up = (torch.randn(E, 2 * I, H, generator=g) * 0.02).bfloat16()
    down = (torch.randn(E, H, I, generator=g) * 0.02).bfloat16()
    gate = (torch.randn(E, H, generator=g) * 0.02).bfloat16()
    el = E // world
    banks = [native.LocalSwiGLUExperts(gate_up[r * el:(r + 1) * el].to(device),
                                       down[r * el:(r + 1) * el].to(device)) for r in range(world)]
    return gate.to(device), banks, g


@pytest.mark.parametrize("world,tokens", [(1, [40]), (2, [64, 48]), (4, [16, 0, 64, 33]),
                                          (8, [8, 3, 0, 20, 8, 1, 15, 9])])
def test_a2a_emulated_ranks_equal_one_process_run(cuda, world, tokens):
    E, H, I, K = 128, 1024, 256, 8
    gate, banks, g = _experts(E, H, I, world, seed=world, device=cuda)
    el = E // world
    t_cap = max(tokens)
    bufs = _buffers(world, H, world * t_cap * K, t_cap * K, cuda)
    try:
        for call in range(2):
            hs = [torch.randn(t, H, generator=g).bfloat16().to(cuda) for t in tokens]
            routes = [native.route(h, gate, K, True) if h.shape[0] else
                      (torch.empty(0, K, dtype=torch.int64, device=cuda),
                       torch.empty(0, K, dtype=torch.bfloat16, device=cuda)) for h in hs]
            sim = native.simulate_routed(hs, [r[0] for r in routes], [r[1] for r in routes], banks, E)
            perms = [ops.permute(r[0], E) for r in routes]
            for b in bufs:
                b.flags.fill_(1 << 20)   # a rank's signal of the last call lowered its slots
                for s in range(world):
                    b.board[s, :E] = perms[s].counts
            recv = [torch.empty(el + 1, dtype=torch.int32, device=cuda) for _ in range(world)]
            for r in range(world):
                ops.a2a_counts(bufs[r], perms[r].counts, recv[r], E)
            for r in range(world):
                ops.a2a_dispatch(bufs[r], hs[r], routes[r][0], perms[r], E)
            ys = [native.run_experts_received(banks[r].weights, bufs[r].area_a, recv[r],
                                              tile_tokens=sum(tokens), K=K, num_experts=E)
                  for r in range(world)]
            for r in range(world):
                ops.a2a_return(bufs[r], ys[r], E)
            for r in range(world):
                T = tokens[r]
                out = ops.combine(bufs[r].area_b[:T * K], perms[r].inverse, routes[r][0],
                                  order=_lib.ORDER_RANK_SLOT, experts_per_rank=el,
                                  weights=routes[r][1].to(torch.bfloat16).contiguous())
                assert torch.equal(out, sim[r]), f"call {call} rank {r} differs"
            # receive offsets: this rank's experts' rows from every source, expert-major
            for r in range(world):
                tot = sum(p.counts.long() for p in perms)[r * el:(r + 1) * el]
                want = torch.cat([torch.zeros(1, dtype=torch.long, device=cuda), tot.cumsum(0)])
                assert torch.equal(recv[r].long(), want)
        assert _lib.device_status(cuda.index) == 0
    finally:
        _free(bufs, cuda)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_gather_emulated_ranks_fill_every_area(cuda, world):
    """Each rank's area A starts with only its experts' rows (at their global
    permuted positions); after every rank's gather, every area holds all rows."""
    E, H, T, K = 64, 512, 96, 4
    g = torch.Generator().manual_seed(world)
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).to(cuda)
    perm = ops.permute(idx, E)
    rows = torch.randn(T * K, H, generator=g).bfloat16().to(cuda)
    bufs = _buffers(world, H, T * K, 0, cuda)
    el = E // world
    try:
        for call in range(2):
            rows = rows + 1
            off = perm.offsets.long().tolist()
            for r, b in enumerate(bufs):
                b.flags.fill_(1 << 20)
                b.area_a.zero_()
                lo, hi = off[r * el], off[(r + 1) * el]
                b.area_a[lo:hi] = rows[lo:hi]
            for r, b in enumerate(bufs):
                ops.ep_gather(b, perm.offsets, r * el, (r + 1) * el, T * K)
            for r, b in enumerate(bufs):
                assert torch.equal(b.area_a[:T * K], rows), f"call {call} rank {r}"
        assert _lib.device_status(cuda.index) == 0
    finally:
        _free(bufs, cuda)
