"""Routing records: every router call's expert ids and routing weights, kept
compact on the device and read back once per step.

The reference's recorders capture each router's output through a forward
hook and convert and copy it at every layer (int16 ids and fp16 weights in
moe_serving/record_routing.py:71-77; ``RoutingRecorder`` in
moe_serving/gpt_oss_parallel.py:247-300). Here the hook runs one small
kernel (``b200moe_route_record``) per router call that writes the int16 /
fp16 copy on the device, and ``end()`` moves the whole step to pinned host
memory with one copy per dtype, waiting only for that copy.

Usage::

    rec = RoutingRecords.attach(model)   # every Qwen3Router / GptOssRouter in it
    rec.begin()
    model(...)
    step = rec.end()    # {layer name: {"indices": int16 [T, K], "scores": fp16 [T, K]}}
    rec.close()
"""

from __future__ import annotations

import torch
from torch import nn

from moe_serving_profile_b200 import ops
from moe_serving_profile_b200.router import GptOssRouter, Qwen3Router


class RoutingRecords:
    def __init__(self, routers: dict[str, nn.Module]):
        self._pending: list[tuple[str, torch.Tensor, torch.Tensor]] = []
        self._handles = [m.register_forward_hook(self._hook(name)) for name, m in routers.items()]

    @classmethod
    def attach(cls, model: nn.Module) -> "RoutingRecords":
        return cls({name: m for name, m in model.named_modules()
                    if isinstance(m, (Qwen3Router, GptOssRouter))})

    def _hook(self, name: str):
        def hook(_module, _inputs, output):
            _first, scores, indices = output
            ids, w = ops.route_record(indices.contiguous(), scores.contiguous())
            self._pending.append((name, ids, w))

        return hook

    def begin(self) -> None:
        self._pending = []

    def end(self) -> dict[str, dict[str, torch.Tensor]]:
        """The step's records on the host, by router name (a router called
        twice in a step keeps its last call)."""
        pending, self._pending = self._pending, []
        if not pending:
            return {}
        ids = torch.cat([i.reshape(-1) for _, i, _ in pending])
        ws = torch.cat([w.reshape(-1) for _, _, w in pending])
        host_ids = torch.empty(ids.shape, dtype=torch.int16, pin_memory=True)
        host_ws = torch.empty(ws.shape, dtype=torch.float16, pin_memory=True)
        host_ids.copy_(ids, non_blocking=True)
        host_ws.copy_(ws, non_blocking=True)
        done = torch.cuda.Event()
        done.record()
        done.synchronize()
        out, o = {}, 0
        for name, i, _ in pending:
            n = i.numel()
            out[name] = {"indices": host_ids[o:o + n].reshape(i.shape),
                         "scores": host_ws[o:o + n].reshape(i.shape)}
            o += n
        return out

    def close(self) -> None:
        for h in self._handles:
            h.remove()
        self._handles.clear()
