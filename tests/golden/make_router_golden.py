"""Record torch's CUDA router operations on tie-heavy logits as fixtures.

The reference's routers (transformers Qwen3MoeTopKRouter / GptOssTopKRouter,
moe_serving/moe.py:97-107) select experts with torch's softmax, topk and sum.
On the GPU these are torch's CUDA kernels, whose slot order for equal values
and whose summation order are not documented; this script records them so the
oracle's restatement (oracle.topk, oracle.butterfly_sum) is pinned on CPU.
It needs only torch and a CUDA device (no reference checkout):

    python tests/golden/make_router_golden.py [out.pt]   # default tests/golden/router_torch_cuda.pt
"""

import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
ROWS = 256


def tie_logits(E: int, seed: int, dtype) -> torch.Tensor:
    """Rows of repeated values, all-equal rows, a coarse value grid, plain rows."""
    g = torch.Generator().manual_seed(seed)
    lg = torch.randn(ROWS, E, generator=g) * 0.9
    q = ROWS // 4
    lg[:q] = lg[:q, :max(1, E // 8)].repeat(1, 8)[:, :E]
    lg[q:q + 8] = 0.0
    lg[q + 8:2 * q] = torch.randint(0, 24, (q - 8, E), generator=g).float() / 8 - 1.5
    return lg.to(dtype)


def main(path: Path) -> None:
    dev = torch.device("cuda", 0)
    out = {"device": torch.cuda.get_device_name(dev), "torch": str(torch.__version__), "cases": {}}
    for kind, E, K in (("qwen", 128, 8), ("qwen", 8, 2), ("qwen", 64, 6), ("gpt", 32, 4),
                       ("gpt", 128, 4), ("native", 16, 8)):
        dtype = torch.float32 if kind == "native" else torch.bfloat16
        lg = tie_logits(E, E * 100 + K, dtype).to(dev)
        case = {"kind": kind, "K": K, "logits": lg.cpu()}
        if kind == "gpt":
            top, idx = torch.topk(lg, K, dim=-1)
            case.update(indices=idx.cpu(), scores=torch.softmax(top, dim=1, dtype=top.dtype).cpu())
        else:
            probs = torch.softmax(lg, dtype=torch.float, dim=-1)
            top, idx = torch.topk(probs, K, dim=-1)
            case.update(probs=probs.cpu(), indices=idx.cpu(), sums=top.sum(dim=-1).cpu(),
                        scores=(top / top.sum(dim=-1, keepdim=True)).cpu())
        out["cases"][f"{kind}_E{E}_K{K}"] = case
    torch.save(out, path)
    print("wrote", path)


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else HERE / "router_torch_cuda.pt")
