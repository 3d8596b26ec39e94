"""Expert-parallel process groups with the reference's contract.

``ParallelGroup(size)`` splits the world into contiguous blocks of ``size``
ranks (moe_serving/gpt_oss_parallel.py:53-103): rank r belongs to block
r // size, its position in the block is ``rank``, and every rank creates every
block's group in the same order. Tokens are replicated within a block.
"""

from __future__ import annotations

import ctypes
import os

import torch
import torch.distributed as dist

# Largest batch the fused combine + all-reduce exchanges (its buffers hold
# this many rows); larger batches use combine + the NCCL all-reduce.
P2P_MAX_ROWS = 8192
# Above this many pushed bytes per rank the fused exchange runs two-shot.
P2P_ONE_SHOT_BYTES = 16 << 20


class _IpcBuffers:
    """One cudaMalloc'd buffer per rank of a group, mapped into the other
    ranks with CUDA IPC (plain peer loads and stores over NVLink). Created
    collectively, outside CUDA graph capture; ``close`` is collective too."""

    def __init__(self, group, rank: int, size: int, device: torch.device, nbytes: int):
        from moe_serving_profile_b200._lib import check, lib

        self.group, self.rank, self.size, self.device = group, rank, size, device
        dev = device.index
        ptr = ctypes.c_void_p()
        check(lib.b200moe_p2p_alloc(dev, nbytes, ctypes.byref(ptr)), "p2p_alloc")
        self.local = ptr.value
        handle = ctypes.create_string_buffer(64)
        check(lib.b200moe_p2p_export(dev, self.local, handle), "p2p_export")
        handles = [None] * size
        dist.all_gather_object(handles, handle.raw, group=group)
        self.peers = []
        for i, h in enumerate(handles):
            if i == rank:
                self.peers.append(self.local)
                continue
            q = ctypes.c_void_p()
            check(lib.b200moe_p2p_import(dev, h, ctypes.byref(q)), "p2p_import")
            self.peers.append(q.value)
        dist.barrier(group=group)   # every buffer mapped everywhere before first use

    def close(self) -> None:
        from moe_serving_profile_b200._lib import lib

        if self.peers is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)   # no rank still reads a peer's buffer
        for i, q in enumerate(self.peers):
            if i != self.rank:
                lib.b200moe_p2p_close(self.device.index, q)
        dist.barrier(group=self.group)
        lib.b200moe_p2p_free(self.device.index, self.local)
        self.peers = None


class PeerExchange(_IpcBuffers):
    """Exchange buffers of the fused combine + all-reduce
    (b200moe_combine_allreduce)."""

    def __init__(self, group, rank: int, size: int, device: torch.device, t_cap: int, hidden: int):
        from moe_serving_profile_b200._lib import lib

        self.t_cap, self.hidden = t_cap, hidden
        super().__init__(group, rank, size, device, lib.b200moe_p2p_buffer_bytes(t_cap, hidden, size))


class _DeviceRows:
    """A device address range seen by torch through __cuda_array_interface__."""

    def __init__(self, ptr: int, rows: int, cols: int):
        self.__cuda_array_interface__ = {"shape": (rows, cols), "typestr": "<i2",
                                         "data": (ptr, False), "version": 3, "strides": None}


PEER_ROWS_HEADER_BYTES = 65536   # b200moe_peer_rows_bytes's header (include/b200moe.h)


class PeerRows(_IpcBuffers):
    """Row-exchange buffers of the peer-memory token all-to-all and the
    replicated-token exact gather (b200moe_a2a_* / b200moe_ep_gather): per
    rank a header, area A [cap_a, hidden] (received / gathered rows) and
    area B [cap_b, hidden] (returned rows), both exposed as bf16 tensors that
    alias the buffer (valid until ``close``)."""

    def __init__(self, group, rank: int, size: int, device: torch.device, hidden: int, cap_a: int,
                 cap_b: int, timeout_ns: int = 0):
        from moe_serving_profile_b200._lib import lib

        self.world, self.hidden, self.cap_a, self.cap_b = size, hidden, cap_a, cap_b
        self.timeout_ns = timeout_ns
        super().__init__(group, rank, size, device, lib.b200moe_peer_rows_bytes(hidden, cap_a, cap_b))
        base = self.local + PEER_ROWS_HEADER_BYTES
        with torch.cuda.device(device):
            self.area_a = torch.as_tensor(_DeviceRows(base, cap_a, hidden), device=device).view(torch.bfloat16)
            self.area_b = torch.as_tensor(_DeviceRows(base + cap_a * hidden * 2, cap_b, hidden),
                                          device=device).view(torch.bfloat16)

    def close(self) -> None:
        self.area_a = self.area_b = None
        super().close()


class ParallelGroup:
    def __init__(self, size: int):
        world = dist.get_world_size() if dist.is_initialized() else 1
        grank = dist.get_rank() if dist.is_initialized() else 0
        if size < 1 or world % size:
            raise ValueError(f"Parallel size {size} must divide world size {world}")
        self.size = size
        self.rank = grank % size
        self.start_rank = grank - self.rank
        self.group = None
        self._exchange = None
        self._gather = None
        if size > 1:
            for first in range(0, world, size):
                g = dist.new_group(list(range(first, first + size)))
                if first == self.start_rank:
                    self.group = g

    def reduce(self, tensor: torch.Tensor) -> torch.Tensor:
        """In-place SUM over the group (NCCL all-reduce on GPUs)."""
        if self.size > 1:
            dist.all_reduce(tensor, group=self.group)
        return tensor

    def combine_reduce(self, rows: torch.Tensor, inverse: torch.Tensor, indices: torch.Tensor,
                       expert_lo: int, expert_hi: int,
                       weights: torch.Tensor | None = None) -> torch.Tensor:
        """SUM over the group of each rank's expert-order combine of its
        experts [expert_lo, expert_hi): the fused NVLink kernel when the
        exchange fits (B200MOE_P2P=0 turns it off), else combine + all-reduce."""
        from moe_serving_profile_b200 import _lib, ops

        T, H = indices.shape[0], rows.shape[1]
        ex = self._peer_exchange(rows.device, H, T)
        if ex is not None:
            return ops.combine_allreduce(rows, inverse, indices, expert_lo=expert_lo,
                                         expert_hi=expert_hi, peers=ex.peers, t_cap=ex.t_cap,
                                         rank=self.rank, weights=weights)
        partial = ops.combine(rows, inverse, indices, order=_lib.ORDER_EXPERT,
                              expert_lo=expert_lo, expert_hi=expert_hi, weights=weights)
        return self.reduce(partial)

    def gather_rows_buffer(self, device: torch.device, hidden: int, rows: int):
        """This rank's exact-gather buffers (a PeerRows for b200moe_ep_gather)
        when ``rows`` contribution rows fit them and the NVLink path is on,
        else None. They hold P2P_MAX_ROWS tokens x 8 slots of rows."""
        if (self.size == 1 or self.size > 8 or device.type != "cuda"
                or os.environ.get("B200MOE_P2P", "1") == "0"):
            return None
        cap = P2P_MAX_ROWS * 8
        if rows > cap:
            return None
        g = self._gather
        if g is None or g.hidden != hidden or g.device != device:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("the NVLink exchange buffers are created by an eager call "
                                   "before CUDA graph capture")
            if g is not None:
                g.close()
            g = self._gather = PeerRows(self.group, self.rank, self.size, device, hidden, cap, 0)
        return g

    def _peer_exchange(self, device: torch.device, hidden: int, T: int):
        if (self.size == 1 or self.size > 8 or device.type != "cuda"
                or os.environ.get("B200MOE_P2P", "1") == "0"):
            return None
        t_cap = P2P_MAX_ROWS
        if T > t_cap:
            return None
        if T * hidden * 2 * (self.size - 1) > P2P_ONE_SHOT_BYTES and 1024 % self.size:
            return None   # the two-shot exchange needs a group size of 2, 4 or 8
        ex = self._exchange
        if ex is None or ex.hidden != hidden or ex.device != device:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("the NVLink exchange buffers are created by an eager call "
                                   "before CUDA graph capture")
            if ex is not None:
                ex.close()
            ex = self._exchange = PeerExchange(self.group, self.rank, self.size, device, t_cap, hidden)
        return ex

    def close(self) -> None:
        """Release the NVLink exchange buffers (collective)."""
        if self._exchange is not None:
            self._exchange.close()
            self._exchange = None
        if self._gather is not None:
            self._gather.close()
            self._gather = None

    def broadcast(self, tensor: torch.Tensor, owner: int = 0) -> torch.Tensor:
        if self.size > 1:
            dist.broadcast(tensor, src=self.start_rank + owner, group=self.group)
        return tensor

    def gather(self, tensor: torch.Tensor, dim: int) -> torch.Tensor:
        if self.size == 1:
            return tensor
        parts = [torch.empty_like(tensor, memory_format=torch.contiguous_format)
                 for _ in range(self.size)]
        dist.all_gather(parts, tensor.contiguous(), group=self.group)
        return torch.cat(parts, dim=dim)

    def all_to_all(self, out: torch.Tensor, inp: torch.Tensor, out_splits=None,
                   in_splits=None) -> torch.Tensor:
        if self.size == 1:
            out.copy_(inp)
            return out
        dist.all_to_all_single(out, inp, output_split_sizes=out_splits,
                               input_split_sizes=in_splits, group=self.group)
        return out
