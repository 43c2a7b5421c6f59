"""Failure detection on the device, without faulting it.

The tensor-core kernels bound every mbarrier wait; when a wait runs out the
kernel records a code in the backend's device error word and returns, and the
host turns the code into an error status at the next synchronisation.  The
self-test kernel makes that happen on purpose (its threads wait on a barrier
nothing arrives on, with a ~1 ms budget); the backend must report it and stay
usable for the next call.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def test_bounded_wait_timeout_is_reported_and_recoverable(um, backend, oracle):
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    with pytest.raises(um.UaiiMoeError) as e:
        backend.selftest_wait_timeout(2_000_000)  # ~1 ms of SM cycles
    assert e.value.status == um.INTERNAL
    assert "gave up waiting" in e.value.message and "code 9" in e.value.message
    # the error word was consumed and the context is intact: a normal layer runs and is right
    T, D, E, I, k = 8, 256, 4, 256, 2
    x = um.fill_normal((T, D), 5, 1)
    w = um.fill_normal((E, D), 5, 2, 0.0, 0.3)
    G = um.quantize_rows(um.Q4_0, um.fill_normal((E * I, D), 5, 3, 0.0, 0.02))
    U = um.quantize_rows(um.Q4_0, um.fill_normal((E * I, D), 5, 4, 0.0, 0.02))
    Dn = um.quantize_rows(um.Q4_0, um.fill_normal((E * D, I), 5, 5, 0.0, 0.02))
    _, pr, _ = oracle.router(x, w)
    y_ref, _, _ = oracle.experts_packed(x, G, um.Q4_0, U, um.Q4_0, Dn, um.Q4_0, pr, E, I, k, 1)
    y = np.empty_like(x)
    backend.ffn(um.make_layer(D, E, I, k, 1, w, G, um.Q4_0, U, um.Q4_0, Dn, um.Q4_0), x, T, y)
    assert np.abs(y - y_ref).max() / np.abs(y_ref).max() <= 2e-3


def test_selftest_budget_is_validated(um, backend):
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    with pytest.raises(um.UaiiMoeError) as e:
        backend.selftest_wait_timeout(10)
    assert e.value.status == um.INTERNAL or e.value.status == um.INVALID_ARGUMENT
