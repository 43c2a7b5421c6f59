"""The allocation-free layer forward (uaii_moe_ffn_forward_noalloc).

Callers such as serving engines that pre-reserve HBM for their own pools, or
runtimes that own every device allocation, cannot let an operator call
cudaMalloc; this entry point runs the MoE FFN layer out of a fixed scratch
array compiled into the library.  Here it must give the same layer output as
the regular entry point (uaii_moe_ffn_forward) on two calls in a row -- the
second call finds the first call's leftovers in the shared scratch.  Both
entry points run the same kernels with the same plan, so the outputs must be
equal bit for bit (a looser bar would hide a stale-scratch bug).  A call made
after the library's kernels have been loaded must leave the device's free
memory unchanged, and it must leave the caller's current device as it found
it.  It must refuse work that does not fit its scratch.

This file is collected last so that, if it fails, a run that stops at the first
failure has already run every other test; it also passes on its own.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")



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
    yr, pr = y_ref.cpu().numpy(), p_ref.cpu().numpy()
    outs = [(torch.full((T, D), float("nan"), device="cuda"), torch.full((T, E), float("nan"), device="cuda"))
            for _ in range(2)]
    for i, (y, p) in enumerate(outs):  # the second call reuses the scratch the first one left behind
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        um.ffn_forward_noalloc(0, stream, L, xd, T, y, p)
        torch.cuda.synchronize()
        if i > 0:  # the first call may load the library's kernels; a warmed call allocates nothing
            assert torch.cuda.mem_get_info()[0] == free0
        assert torch.cuda.current_device() == 0
        assert np.array_equal(y.cpu().numpy().view(np.uint32), yr.view(np.uint32))
        assert np.array_equal(p.cpu().numpy().view(np.uint32), pr.view(np.uint32))
    if torch.cuda.device_count() > 1:  # a caller working on another device gets it back
        y, p = outs[0]
        with torch.cuda.device(1):
            um.ffn_forward_noalloc(0, None, L, xd, T, y, p)
            assert torch.cuda.current_device() == 1
        assert np.array_equal(y.cpu().numpy().view(np.uint32), yr.view(np.uint32))


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
