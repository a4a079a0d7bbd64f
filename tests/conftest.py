import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


def load_golden(name: str) -> dict:
    return torch.load(os.path.join(GOLDEN, f"{name}.pt"), weights_only=True)


SSD_CASES = ["ssd_c0_fp32", "ssd_ragged_fp32", "ssd_threshold_fp32", "ssd_nosoftplus_fp32",
             "ssd_bf16_c1slice", "ssd_bf16_groups"]
SSU_CASES = ["ssu_bf16", "ssu_fp32_groups"]


# Tolerances (north_star): fp32 within rel 1e-4; bf16 within atol 2e-2 / rel 1e-2.
def assert_fp32_close(actual, expected, what=""):
    a, e = actual.double().cpu(), expected.double().cpu()
    scale = e.abs().max().item()
    tol = 1e-4 * e.abs() + 1e-5 * scale + 1e-12
    err = (a - e).abs()
    bad = err > tol
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {e.numel()} elements outside rel 1e-4 "
                           f"(max abs err {err.max().item():.3e}, max |ref| {scale:.3e})")


def assert_bf16_close(actual, expected, what=""):
    a, e = actual.double().cpu(), expected.double().cpu()
    tol = 2e-2 + 1e-2 * e.abs()
    err = (a - e).abs()
    bad = err > tol
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {e.numel()} elements outside atol 2e-2 / rel 1e-2 "
                           f"(max abs err {err.max().item():.3e})")


def assert_bf16_operand_close(actual, expected, what=""):
    """An fp32 result of a problem whose inputs are 16-bit, computed with 16-bit
    tensor-core operands (the backward's state-side products): within rel 1e-2 of each
    element plus 5e-3 of the tensor's largest magnitude (the north star's bf16 rel 1e-2,
    with an absolute term scaled to the tensor instead of a fixed 2e-2)."""
    a, e = actual.double().cpu(), expected.double().cpu()
    scale = e.abs().max().item()
    tol = 1e-2 * e.abs() + 5e-3 * scale + 1e-12
    err = (a - e).abs()
    bad = err > tol
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {e.numel()} elements outside rel 1e-2 + 5e-3 max "
                           f"(max abs err {err.max().item():.3e}, max |ref| {scale:.3e})")


def assert_close_for(dtype):
    return assert_fp32_close if dtype == torch.float32 else assert_bf16_close
