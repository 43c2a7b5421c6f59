"""The C ABI library on the host: it loads, exports every declared symbol, and
its host-only utilities behave.  No device compute is called here."""
import ctypes
import os
import re

import numpy as np
import pytest

from conftest import REPO


def declared_symbols():
    src = open(os.path.join(REPO, "include", "uaii_moe.h")).read()
    return sorted(set(re.findall(r"UAII_MOE_API\s+[\w\s\*]+?\b(uaii_moe_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared_symbols()
    for n in ("uaii_moe_dispatch", "uaii_moe_router_f32", "uaii_moe_experts_swiglu", "uaii_moe_ffn_forward",
              "uaii_moe_dequant_rows", "uaii_moe_backend_create"):
        assert n in names


def test_library_exports_every_declared_symbol(um):
    lib = ctypes.CDLL(um.LIB_PATH)
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing
    assert set(um.EXPORTED) == set(declared_symbols())


def test_abi_version_and_ops(um):
    assert um.lib.uaii_moe_abi_version() == 1
    for op in (b"MoERouter", b"MoEExperts", b"MoEExpertsSwiGLU", b"MoEFFN"):
        assert um.lib.uaii_moe_supports_op(op) == 1
    for op in (b"MatMul", b"Attention", b""):
        assert um.lib.uaii_moe_supports_op(op) == 0


@pytest.mark.parametrize("fmt", [0, 1, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16])
def test_packed_nbytes_matches_reference_formula(um, oracle, fmt):
    for n in (256, 1024, 2816, 14336):
        assert um.packed_nbytes(fmt, n) == oracle.packed_nbytes(fmt, n)


@pytest.mark.parametrize("fmt,tol", [(7, 0.09), (11, 0.005), (14, 0.06), (16, 0.02)])
def test_quantizer_round_trip(um, oracle, fmt, tol):
    src = um.fill_normal((64, 1024), 1, 2, 0.0, 0.02)
    q = um.quantize_rows(fmt, src)
    assert q.shape == (64, um.packed_nbytes(fmt, 1024))
    back = oracle.dequant(fmt, q, 64, 1024)
    assert np.isfinite(back).all()
    assert np.abs(back - src).max() <= tol * np.abs(src).max()
    # deterministic
    assert np.array_equal(q, um.quantize_rows(fmt, src))


def test_quantizer_rejects_other_formats(um):
    with pytest.raises(um.UaiiMoeError) as e:
        um.quantize_rows(um.Q5_K, np.zeros((1, 256), np.float32))
    assert e.value.status == 7


def test_fill_normal_is_counter_based(um):
    a = um.fill_normal((3, 5000), 42, 7)
    b = um.fill_normal((15000,), 42, 7)
    assert np.array_equal(a.reshape(-1), b)
    c = um.fill_normal((10,), 42, 8)
    assert not np.array_equal(a.reshape(-1)[:10], c)
    big = um.fill_normal((1 << 21,), 1, 1)
    assert abs(float(big.mean())) < 5e-3 and abs(float(big.std()) - 1.0) < 5e-3


def test_backend_create_reports_errors_without_crashing(um):
    import torch
    if torch.cuda.is_available():
        pytest.skip("needs a host without a GPU")
    h = ctypes.c_void_p()
    st = um.lib.uaii_moe_backend_create(0, None, ctypes.byref(h))
    assert st != 0 and not h.value
    assert um.lib.uaii_moe_last_error()


def test_null_backend_is_invalid_argument(um):
    assert um.lib.uaii_moe_synchronize(None) == 1
    assert b"null backend" in um.lib.uaii_moe_last_error()
