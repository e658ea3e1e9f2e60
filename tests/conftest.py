"""Shared pytest configuration.

Tests marked ``gpu`` need a B200 (sm_100) and the built CUDA library; every
other test runs on CPU.  ``-m "not gpu"`` is the CPU suite, ``-m gpu`` the
parity suite.
"""
from __future__ import annotations

import functools
import os
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
REF = ROOT / "baseline" / "_ref"
GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU and the built liblthc_b200.so")
    config.addinivalue_line("markers", "slow: full-size (benchmark-configuration) cases")


@functools.lru_cache(maxsize=1)
def _cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available() and torch.cuda.get_device_capability(0)[0] == 10
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_ok():
        return
    skip = pytest.mark.skip(reason="no sm_100 GPU in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def _device_error_word(request):
    """After every GPU test: the library's device error word must be clear.  A
    kernel whose bounded wait gave up sets it and returns without finishing its
    work, so a test that passed with the word set would hide a timeout."""
    yield
    if "gpu" not in request.keywords or not _cuda_ok():
        return
    import ctypes

    import torch

    from flowmatching_lthc_b200 import _lib

    if _lib._lib is None:  # the test never loaded the library
        return
    st = ctypes.c_int(-1)
    _lib.call("lthc_device_status", ctypes.byref(st), torch.cuda.current_stream().cuda_stream)
    assert st.value == 0, "a bounded device-side wait gave up during this test (LTHC_ERR_TIMEOUT)"


def reference_root() -> Path | None:
    """Where the reference package (tongtongliang/flowmatching_lthc) can be
    imported from: an explicit checkout named by LTHC_REFERENCE, else the copy
    installed under baseline/_ref.  None when neither exists."""
    for cand in (os.environ.get("LTHC_REFERENCE"), REF):
        if cand and (Path(cand) / "flowmatching_lthc" / "__init__.py").exists():
            return Path(cand)
    return None


def reference_available() -> bool:
    return reference_root() is not None


def import_reference():
    root = reference_root()
    if root is None:
        pytest.skip("reference package not importable (set LTHC_REFERENCE or install it under baseline/_ref)")
    if str(root) not in sys.path:
        sys.path.insert(0, str(root))
    sys.dont_write_bytecode = True  # the reference checkout may be read-only
    import flowmatching_lthc.models.local_thc as L  # noqa: F401
    return L


def close_16bit(a: torch.Tensor, b: torch.Tensor, max_frac: float = 0.02) -> bool:
    """a and b (same 16-bit dtype and shape) differ by at most one unit in the last
    place (plus 1e-4 of b's largest magnitude, for sums that cancel), on at most
    max_frac of the elements: the tolerance of the tensor-core materialisation
    backward, whose position sums are accumulated by the tensor core."""
    a, b = a.detach().cpu(), b.detach().cpu()
    if a.shape != b.shape or a.dtype != b.dtype:
        return False
    af, bf = a.float(), b.float()
    eps = {torch.bfloat16: 2.0**-7, torch.float16: 2.0**-10}[a.dtype]
    bound = eps * torch.maximum(af.abs(), bf.abs()) + 1e-4 * bf.abs().max()
    return bool(((af - bf).abs() <= bound).all()) and (af != bf).float().mean().item() <= max_frac
