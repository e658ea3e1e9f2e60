"""The C-ABI library loads and exports every entry point the header declares, and
its host-side argument validation answers with the documented status codes.
No kernel is launched: every call here fails validation or is an empty batch."""
from __future__ import annotations

import ctypes
import re

import pytest

from conftest import ROOT
from flowmatching_lthc_b200 import _lib

HEADER = ROOT / "include" / "lthc_b200.h"


def declared() -> list[str]:
    return re.findall(r"^LTHC_API\s+[\w\s\*]+?\b(lthc_\w+)\s*\(", HEADER.read_text(), flags=re.M)


def test_library_exports_every_declared_symbol():
    names = declared()
    assert len(names) >= 20
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    for n in names:
        assert hasattr(lib, n), f"{n} declared in lthc_b200.h but not exported"
    assert set(names) == set(_lib.SIGNATURES), "ctypes signature table out of sync with the header"


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.lthc_version() == 100
    for code in range(9):
        assert lib.lthc_status_string(code)
    assert lib.lthc_status_string(99) == b"unknown status"


P = 256  # a 16-byte aligned non-null address that is never dereferenced


@pytest.mark.parametrize("call, status", [
    (lambda L: L.lthc_read_fwd(None, P, 0, P, 1, 16, 768, 1, None), 1),
    (lambda L: L.lthc_read_fwd(P, P, 0, P, 1, 16, 7, 1, None), 2),
    (lambda L: L.lthc_read_fwd(P, P, 0, P, 1, 16, 768, 9, None), 3),
    (lambda L: L.lthc_read_fwd(P + 2, P, 0, P, 1, 16, 768, 1, None), 4),
    (lambda L: L.lthc_write_fwd(P, P, 5, P, 1, 16, 768, 1, None), 3),
    (lambda L: L.lthc_write_add_fwd(P, P, P, 0, P, -1, 16, 768, 1, None), 2),
    (lambda L: L.lthc_materialise_fwd(P, _lib.ptr_array([P] * 13), _lib.ptr_array([P] * 13), 0, 13, P, 1, 16, 768, 1,
                                      None), 2),
    (lambda L: L.lthc_materialise_fwd(P, None, None, 0, 12, P, 1, 16, 768, 1, None), 1),
    (lambda L: L.lthc_lazy_update_fwd(P, P, P, 0, P, 0, P, 4, 12, 1, None), 2),
    (lambda L: L.lthc_weight_grad(P, _lib.ptr_array([P]), 0, P, P, 1 << 20, 1, 16, 768, 1, None), 2),
    (lambda L: L.lthc_final_norm_modulate_fwd(P, P, 0, P, P, 1536, P, 2, 4096, 1032, 1e-6, 1, None), 2),
    (lambda L: L.lthc_final_norm_modulate_fwd(P, P, 0, P, P, 512, P, 2, 4096, 768, 1e-6, 1, None), 2),
    (lambda L: L.lthc_final_norm_modulate_fwd(P, P, 7, P, P, 1536, P, 2, 4096, 768, 1e-6, 1, None), 3),
    (lambda L: L.lthc_final_norm_modulate_fwd(P + 8, P, 0, P, P, 1536, P, 2, 4096, 768, 1e-6, 1, None), 4),
    (lambda L: L.lthc_final_norm_modulate_fwd(P, None, 0, P, P, 1536, P, 2, 4096, 768, 1e-6, 1, None), 1),
    (lambda L: L.lthc_final_norm_modulate_bwd(P, P, 0, P, 1536, P, None, None, None, None, P, 1 << 30, 2, 4096, 768,
                                              1e-6, 1, None), 1),
    (lambda L: L.lthc_branch_lazy_fwd(P, P, P, P, 4608, P, 0, P, 0, P, P, 2, 256, 770, 1, None), 2),
    (lambda L: L.lthc_branch_lazy_fwd(P, P, P, P, 700, P, 0, P, 0, P, P, 2, 256, 768, 1, None), 2),
    (lambda L: L.lthc_branch_lazy_fwd(P, P, P, P, 4608, P, 0, P, 6, P, P, 2, 256, 768, 1, None), 3),
    (lambda L: L.lthc_branch_lazy_fwd(P, P, P + 4, P, 4608, P, 0, P, 0, P, P, 2, 256, 768, 1, None), 4),
    (lambda L: L.lthc_branch_lazy_fwd(P, None, P, P, 4608, P, 0, P, 0, P, P, 2, 256, 768, 1, None), 1),
    (lambda L: L.lthc_branch_lazy_bwd(None, None, P, P, P, 4608, P, 0, P, 0, P, P, P, P, P, P, 1 << 30, 2, 256, 768,
                                      1, None), 1),
    (lambda L: L.lthc_branch_lazy_bwd(P, P, P, P, P, 4612, P, 0, P, 0, P, P, P, P, P, P, 1 << 30, 2, 256, 768, 1,
                                      None), 2),
])
def test_validation_errors(call, status):
    lib = _lib.load()
    assert call(lib) == status
    assert lib.lthc_last_error_message()


def test_empty_batch_is_a_successful_no_op():
    lib = _lib.load()
    assert lib.lthc_read_fwd(P, P, 0, P, 0, 16, 768, 1, None) == 0
    assert lib.lthc_write_add_fwd(P, P, P, 0, P, 0, 16, 768, 1, None) == 0
    assert lib.lthc_materialise12_fwd(P, _lib.ptr_array([P] * 12), _lib.ptr_array([P] * 12), 0, P, 0, 16, 768, 1,
                                      None) == 0
    assert lib.lthc_lazy_update_fwd(P, P, P, 0, P, 0, P, 0, 768, 1, None) == 0
    assert lib.lthc_final_norm_modulate_fwd(P, P, 0, P, P, 1536, P, 0, 4096, 768, 1e-6, 1, None) == 0
    assert lib.lthc_final_norm_modulate_bwd(P, P, 0, P, 1536, P, P, None, None, None, None, 0, 0, 4096, 768, 1e-6, 1,
                                            None) == 0
    assert lib.lthc_branch_lazy_fwd(P, P, P, P, 4608, P, 0, P, 0, P, P, 0, 256, 768, 1, None) == 0
    assert lib.lthc_branch_lazy_bwd(None, P, P, P, P, 4608, P, 0, P, 0, P, P, None, None, None, None, 0, 2, 0, 768, 1,
                                    None) == 0


def test_workspace_queries():
    lib = _lib.load()
    assert lib.lthc_materialise_bwd_workspace_bytes(0, 16, 768, 12) == 0
    n12 = lib.lthc_materialise_bwd_workspace_bytes(64, 16, 768, 12)
    n1 = lib.lthc_materialise_bwd_workspace_bytes(64, 16, 768, 1)
    assert n12 > 0 and n12 % (12 * 768 * 16 * 4) == 0 and n1 * 12 == n12
    assert lib.lthc_weight_grad_workspace_bytes(64, 16, 768, 12) == n12
    assert lib.lthc_read_bwd_workspace_bytes(64, 16, 768) == n1
    assert lib.lthc_lazy_update_bwd_workspace_bytes(64 * 256, 768) % (768 * 4) == 0
    assert lib.lthc_final_norm_modulate_bwd_workspace_bytes(0, 4096, 768) == 0
    nf = lib.lthc_final_norm_modulate_bwd_workspace_bytes(64, 4096, 768)
    assert nf > 0 and nf % (64 * 3 * 768 * 4) == 0
    assert lib.lthc_branch_lazy_bwd_workspace_bytes(0, 256, 768) == 0
    nb = lib.lthc_branch_lazy_bwd_workspace_bytes(64, 256, 768)
    assert nb > 0 and nb % (64 * 2 * 768 * 4) == 0


def test_call_helper_raises_with_message():
    with pytest.raises(_lib.LthcError) as ei:
        _lib.call("lthc_read_fwd", P, P, 0, P, 1, 16, 12, 1, None)
    assert ei.value.status == 2 and "channels" in str(ei.value)
