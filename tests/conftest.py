"""Shared fixtures. The oracle (`oracle/`, numpy float32) is the checker for every
numerical test; it is pinned to the reference's own outputs by test_oracle_golden.py.

Markers: `gpu` tests need an sm_100 (B200) device and call the CUDA path through the
C ABI; everything else runs on CPU.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

GOLDEN = REPO / "tests" / "golden"

# Parity bar for the bf16-weight CUDA path against the fp32 oracle on the same
# bf16-rounded weights: max-abs logit error and cosine similarity per step.
LOGIT_ATOL = 3e-2
LOGIT_MIN_COS = 0.9999


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU; runs the CUDA path")
    config.addinivalue_line("markers", "slow: runs the full 24-layer model")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


def golden_npz(name: str):
    return np.load(GOLDEN / name)


def golden_json(name: str):
    return json.loads((GOLDEN / name).read_text())


@pytest.fixture(scope="session")
def full_cfg():
    from qweninfer_b200 import synthetic
    return synthetic.full_config()


@pytest.fixture(scope="session")
def state_fp32(full_cfg):
    from qweninfer_b200 import synthetic
    return {k: v.numpy() for k, v in synthetic.synthetic_state(full_cfg, 0).items()}


@pytest.fixture(scope="session")
def state_bf16w(state_fp32):
    from oracle import bf16_round
    return {k: bf16_round(v) for k, v in state_fp32.items()}


@pytest.fixture(scope="session")
def oracle_bf16w(state_bf16w, full_cfg):
    from oracle import OracleModel
    return OracleModel(state_bf16w, vars(full_cfg))


@pytest.fixture(scope="session")
def ckpt_bf16(full_cfg):
    from qweninfer_b200 import synthetic
    return synthetic.checkpoint_dir(full_cfg, 0, torch.bfloat16)


@pytest.fixture(scope="session")
def gpu_model(ckpt_bf16):
    from qweninfer_b200.models.qwen2 import Qwen2
    return Qwen2.from_pretrained(ckpt_bf16, dtype=torch.bfloat16, device="cuda")


def logit_report(got: np.ndarray, ref: np.ndarray) -> tuple[float, float]:
    """(max-abs difference, cosine similarity) of two logit vectors."""
    got = np.asarray(got, dtype=np.float64).ravel()
    ref = np.asarray(ref, dtype=np.float64).ravel()
    cos = float(got @ ref / (np.linalg.norm(got) * np.linalg.norm(ref)))
    return float(np.abs(got - ref).max()), cos


def top2_margin(logits: np.ndarray) -> float:
    part = np.partition(np.asarray(logits, dtype=np.float64).ravel(), -2)
    return float(part[-1] - part[-2])
