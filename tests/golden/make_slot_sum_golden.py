"""Record torch's CUDA sum over the slot dimension of [T, K, H] bf16 tensors.

The reference's W8A8 path (grouped_fp8, moe_serving/efficient_kernels.py:269-273)
combines a token's K contribution rows with
``values[inverse].reshape(T, K, H).sum(1)``: torch's CUDA reduction kernel
with an fp32 accumulator, whose summation order over the strided slot
dimension is not documented. This script records its outputs on values with
widely spread exponents (so that fp32 rounding depends on the order) for
several K, so the oracle's restatement (oracle.slot_sum) is pinned on CPU.
It needs only torch and a CUDA device (no reference checkout):

    python tests/golden/make_slot_sum_golden.py [out.pt]   # default tests/golden/slot_sum_torch_cuda.pt
"""

import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


def spread_values(T: int, K: int, H: int, seed: int) -> torch.Tensor:
    """bf16 values sign * 2^e * (1 + m / 128), e in [-8, 8], and in each
    (token, column) with K > 1 a pair of slots holding +B and -B with
    B = 2^[16, 24] (1 + m / 128): whether small values are added before,
    between or after the pair changes the fp32 sum by more than a bf16 ulp,
    so the output shows the summation order. Zeros of both signs too."""
    g = torch.Generator().manual_seed(seed)
    e = torch.randint(-8, 9, (T, K, H), generator=g).float()
    m = torch.randint(0, 128, (T, K, H), generator=g).float()
    s = torch.where(torch.rand(T, K, H, generator=g) < 0.5, -1.0, 1.0)
    v = s * torch.exp2(e) * (1 + m / 128)
    if K > 1:
        big = torch.exp2(torch.randint(16, 25, (T, H), generator=g).float()) * \
            (1 + torch.randint(0, 128, (T, H), generator=g).float() / 128)
        i = torch.randint(0, K, (T, H), generator=g)
        j = (i + torch.randint(1, K, (T, H), generator=g)) % K
        v.scatter_(1, i[:, None], big[:, None])
        v.scatter_(1, j[:, None], -big[:, None])
    v[T // 8: T // 8 + 1] = 0.0
    v[T // 8 + 1: T // 8 + 2] = -0.0
    return v.to(torch.bfloat16)


def main(path: Path) -> None:
    dev = torch.device("cuda", 0)
    out = {"device": torch.cuda.get_device_name(dev), "torch": str(torch.__version__), "cases": {}}
    shapes = [(32, K, 32) for K in (1, 2, 3, 4, 5, 6, 8, 9, 16, 32)] + [(8, 8, 2048), (8, 4, 2880)]
    for T, K, H in shapes:
        v = spread_values(T, K, H, seed=K * 1000 + H)
        s = v.to(dev).sum(1)
        # wide rows run torch's kernel with vectorised outputs; every column
        # is summed alike, so the first 256 columns are kept
        c = min(H, 256)
        out["cases"][f"T{T}_K{K}_H{H}"] = {"values": v[..., :c].clone(), "sum": s.cpu()[..., :c].clone()}
    torch.save(out, path)
    print("wrote", path)


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else HERE / "slot_sum_torch_cuda.pt")
