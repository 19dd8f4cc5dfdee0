import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REPO / "qwen3tts-streaming_b200"))
sys.path.insert(0, str(REPO / "oracle"))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built q3s library")


def load_golden(name: str) -> dict:
    import torch

    with np.load(GOLDEN / f"{name}.npz") as z:
        d = {k: z[k] for k in z.files}
    if "logits_u16" in d:
        bits = torch.from_numpy(d.pop("logits_u16").view(np.int16))
        d["logits_bf16"] = bits.view(torch.bfloat16)
        d["logits"] = d["logits_bf16"].float().numpy()
    return d


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def q3s_lib(cuda_device):
    import q3s

    return q3s.load_library()
