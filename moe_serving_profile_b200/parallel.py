"""Expert-parallel process groups with the reference's contract.

``ParallelGroup(size)`` splits the world into contiguous blocks of ``size``
ranks (moe_serving/gpt_oss_parallel.py:53-103): rank r belongs to block
r // size, its position in the block is ``rank``, and every rank creates every
block's group in the same order. Tokens are replicated within a block.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


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
