import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "glm-flash-lite_b200")
GOLDEN = os.path.join(REPO, "tests", "golden")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

# Parity bar of the path: layer outputs within max-abs 2e-3 x RMS(output).
TOL_MAXABS_REL_RMS = 2e-3


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


def load_golden(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz"), allow_pickle=False))


def golden_bank(d):
    """Rebuild the ExpertBank of a golden fixture (trellis from SplitMix64, checked against the stored SHA-256)."""
    from glmx import synth
    H, I, E, shared = int(d["H"]), int(d["I"]), int(d["E"]), bool(int(d["shared"]))
    b = synth.ExpertBank(H, I, E, shared, (3, 3, 3), np.zeros(0, np.uint8),
                         [d[f"suh{p}"] for p in range(3)], [d[f"svh{p}"] for p in range(3)])
    b.trellis = synth.splitmix_bytes(int(d["seed"]), b.e_total * b.expert_bytes)
    assert synth.sha256(b.trellis) == str(d["trellis_sha256"]), "trellis regeneration does not match the fixture"
    return b


def parity(a, ref):
    """(max-abs / RMS(ref), rel-RMS) of a against ref."""
    a = np.asarray(a, np.float64); ref = np.asarray(ref, np.float64)
    rms = float(np.sqrt(np.mean(ref * ref))) or 1e-30
    d = a - ref
    return float(np.max(np.abs(d))) / rms, float(np.sqrt(np.mean(d * d))) / rms


def cuda_ok():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
