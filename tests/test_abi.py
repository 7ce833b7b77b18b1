"""The C-ABI library builds, loads and exports every symbol the header declares.

CPU only: nothing here launches a kernel. coli_cuda_init on a machine without
a GPU must fail cleanly (return 0 with a reason), and calls before init must
return 0 rather than crash.
"""
import ctypes

import pytest

from conftest import load_pkg


@pytest.fixture(scope="module")
def pkg():
    p = load_pkg()
    p.build()
    return p


def test_header_symbols_exported(pkg):
    lib = pkg.load_library()
    names = pkg.header_symbols()
    assert len(names) >= 35
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header(pkg):
    from coli_cuda import SIGNATURES
    assert set(pkg.header_symbols()) == set(SIGNATURES)


def test_calls_before_init_fail_cleanly(pkg):
    lib = pkg.load_library()
    if not lib.coli_cuda_available():
        assert lib.coli_cuda_kv_ensure(0, 1, 2, 16, 256) == 0
        assert b"not ready" in lib.coli_cuda_last_error()
        assert lib.coli_cuda_gdn_state_ensure(0, 1, 32, 128, 128) == 0


def test_init_without_gpu_reports_reason(pkg):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = pkg.load_library()
    assert lib.coli_cuda_init(0) == 0
    assert lib.coli_cuda_last_error()
