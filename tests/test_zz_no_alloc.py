"""The allocation-free layer forward (uaii_moe_ffn_forward_noalloc).

Callers such as serving engines that pre-reserve HBM for their own pools, or
runtimes that own every device allocation, cannot let an operator call
cudaMalloc; this entry point runs the MoE FFN layer out of a fixed scratch
array compiled into the library.  Here it must give the same layer output as
the regular entry point (uaii_moe_ffn_forward) on two calls in a row -- the
second call finds the first call's leftovers in the shared scratch -- and it
must refuse work that does not fit its scratch.

This file is collected last so that, if it fails, a run that stops at the first
failure has already run every other test; it also passes on its own.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

REL_TOL = 2e-3  # the layer-output bar used by every parity test


def rel_err(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


def test_noalloc_forward_matches_regular_forward_twice(um, backend):
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    T, D, E, I, k = 12, 1024, 8, 2048, 2  # Mixtral formats (Q4_K gate/up, Q6_K down), reduced width
    x = um.fill_normal((T, D), 31, 1)
    w = um.fill_normal((E, D), 31, 2, 0.0, 0.02)
    G = um.quantize_rows(um.Q4_K, um.fill_normal((E * I, D), 31, 3, 0.0, 0.02))
    U = um.quantize_rows(um.Q4_K, um.fill_normal((E * I, D), 31, 4, 0.0, 0.02))
    Dn = um.quantize_rows(um.Q6_K, um.fill_normal((E * D, I), 31, 5, 0.0, 0.02))
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    xd, wd, Gd, Ud, Dd = (dev(a) for a in (x, w, G, U, Dn))
    L = um.make_layer(D, E, I, k, 1, wd, Gd, um.Q4_K, Ud, um.Q4_K, Dd, um.Q6_K)

    y_ref = torch.empty((T, D), device="cuda")
    p_ref = torch.empty((T, E), device="cuda")
    backend.ffn(L, xd, T, y_ref, p_ref)
    backend.synchronize()

    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # the second call reuses the scratch the first one left behind
        y = torch.full((T, D), float("nan"), device="cuda")
        p = torch.full((T, E), float("nan"), device="cuda")
        um.ffn_forward_noalloc(0, stream, L, xd, T, y, p)
        assert rel_err(y.cpu().numpy(), y_ref.cpu().numpy()) <= REL_TOL
        assert np.allclose(p.cpu().numpy(), p_ref.cpu().numpy(), rtol=1e-6, atol=0)


def test_noalloc_forward_rejects_oversized_and_host_arguments(um):
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    D, E, I, k = 1024, 8, 2048, 2
    w = torch.zeros((E, D), device="cuda")
    G = torch.zeros((E * I, um.packed_nbytes(um.Q4_K, D)), dtype=torch.uint8, device="cuda")
    Dn = torch.zeros((E * D, um.packed_nbytes(um.Q6_K, I)), dtype=torch.uint8, device="cuda")
    L = um.make_layer(D, E, I, k, 1, w, G, um.Q4_K, G, um.Q4_K, Dn, um.Q6_K)
    T = 4096  # needs far more than the fixed scratch
    x = torch.zeros((T, D), device="cuda")
    y = torch.zeros((T, D), device="cuda")
    with pytest.raises(um.UaiiMoeError) as e:
        um.ffn_forward_noalloc(0, None, L, x, T, y)
    assert e.value.status == 1 and "scratch" in e.value.message
    xh = np.zeros((2, D), np.float32)
    with pytest.raises(um.UaiiMoeError) as e:
        um.ffn_forward_noalloc(0, None, L, xh, 2, y)
    assert e.value.status == 1 and "device memory" in e.value.message
