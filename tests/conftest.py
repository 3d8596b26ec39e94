import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a)")


def load_golden(name: str) -> dict:
    return torch.load(GOLDEN / f"{name}.pt", weights_only=False)


@pytest.fixture(scope="session")
def cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    return torch.device("cuda", 0)


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def max_abs(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((a.float().cpu() - b.float().cpu()).abs().max())


def tie_free_rows(values: torch.Tensor, k: int) -> torch.Tensor:
    """Rows whose k+1 largest values are pairwise distinct (no top-k tie)."""
    v = values.float().cpu()
    kk = min(k + 1, v.shape[1])
    top = torch.topk(v, kk, dim=-1).values
    return (top[:, :-1] != top[:, 1:]).all(dim=-1)
