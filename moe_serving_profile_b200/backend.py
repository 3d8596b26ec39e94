"""Runtime checks, backend labels and weight preparation for the b200 experts.

Mirrors the reference's backend hooks (moe_serving/efficient_kernels.py):
``check_runtime`` fails at model-build time, with no fallback, when the b200
path cannot run (:277-288); ``backend_metadata`` names the kernels a run used,
for the recorders' metadata (:291-302); ``prepare_fp8`` / ``prepare_mxfp4``
pack a layer's experts once after loading (:136-154, :217-240).
"""

from __future__ import annotations

import torch

NUMERICS = ("reference", "fast", "efficient")
STORAGE = {"qwen3": ("fp8", "bf16"), "gpt_oss": ("mxfp4", "bf16")}


def check_runtime(family: str, device, dtype: torch.dtype, storage: str) -> None:
    """Raise unless the b200 experts can run: a CUDA sm_100 device, bf16
    compute, a supported expert storage, and the compiled library present."""
    if family not in STORAGE:
        raise ValueError(f"unknown model family {family!r}")
    dev = torch.device(device)
    if dev.type != "cuda":
        raise ValueError("the b200 experts require a CUDA device (there is no CPU path)")
    if dtype != torch.bfloat16:
        raise ValueError(f"the b200 experts compute in bfloat16, got {dtype}")
    if storage not in STORAGE[family]:
        raise ValueError(f"b200 {family} experts support storage {STORAGE[family]}, got {storage!r}")
    major, minor = torch.cuda.get_device_capability(dev)
    if (major, minor) != (10, 0):
        raise ValueError(f"the b200 kernels are built for sm_100a, device is sm_{major}{minor}")
    from moe_serving_profile_b200 import _lib  # raises ImportError if the library is missing

    _lib.version()


def backend_metadata(family: str, numerics: str) -> dict:
    """Labels of the kernels one layer call runs (the reference's keys)."""
    if numerics not in NUMERICS:
        raise ValueError(f"numerics must be one of {NUMERICS}, got {numerics!r}")
    weights = "mxfp4_e2m1_ue8m0" if family == "gpt_oss" else "fp8_e4m3_block128"
    kind = "w8a8_dynamic_act_128" if numerics == "efficient" and family == "qwen3" else "weight_only"
    return {
        "experts": f"b200_tcgen05_grouped_{weights}_{kind}",
        "router": "b200_fused_router",
        "permutation": "b200_counting_sort",
        "combine": "b200_ordered_bf16_combine",
        "expert_parallel": ("replicated_tokens_zero_fill_all_reduce_ordered_combine"
                            if numerics == "reference" else "local_combine_then_all_reduce"),
    }


def prepare_fp8(experts) -> None:
    """Pack a Qwen3 ``ParallelExperts`` layer once (its per-expert modules are released)."""
    experts.prepare()


def prepare_mxfp4(experts, config=None) -> None:
    """Pack a GPT-OSS ``ParallelExperts`` layer once (the packed buffers are released)."""
    experts.prepare()
