"""The reference's own CudaBackend (libs/uaii-backends/src/cuda_backend.cpp, unmodified, built with
UAII_WITH_CUDA into oracle/_ref/libuaii_ref_cuda.so) with its CUDA native layer supplied by
universal-ai-inference_b200/plugin/uaii_cuda_native.cpp.  tests/reference_cuda_backend.py runs
it in a child process with device-resident tensors.

Bars against the oracle: probabilities within 1e-6 and the same top-1 expert (the device router's
logits are the reference's bit for bit), MoEExpertsSwiGLU and the packed MatMulRelu within 2e-3 of
the largest output (f16 tensor-core operands), the host-staged Softmax within 1e-6.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, REPO)
CUDA_SO = os.path.join(REPO, "oracle", "_ref", "libuaii_ref_cuda.so")

needs_build = pytest.mark.skipif(not os.path.exists(CUDA_SO),
                                 reason="reference CUDA backend not built (build() with the reference tree)")


def _run(*args):
    p = subprocess.run([sys.executable, os.path.join(HERE, "reference_cuda_backend.py"), *args],
                       capture_output=True, text=True, timeout=600)
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert p.returncode == 0 and lines, (p.returncode, p.stdout[-2000:], p.stderr[-2000:])
    return json.loads(lines[-1])


def _rel(y, ref):
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    return float(np.abs(y - ref).max() / np.abs(ref).max())


@needs_build
def test_native_layer_symbols_are_linked_into_the_reference_backend():
    out = subprocess.run(["nm", "-D", "--defined-only", CUDA_SO], capture_output=True, text=True, check=True)
    names = {ln.split()[-1] for ln in out.stdout.splitlines() if ln.strip()}
    assert "uaii_cuda_native_stats" in names
    # the reference's stub layer (native_unavailable.cpp without UAII_WITH_CUDA) is not in the library
    out = subprocess.run(["nm", "-C", "--defined-only", CUDA_SO], capture_output=True, text=True, check=True)
    assert "uaii::backends::native::cuda_dispatch" in out.stdout
    assert "uaii::backends::native::cuda_compiled" in out.stdout


@needs_build
def test_backend_reports_host_fallback_without_a_gpu():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    r = _run()
    assert r["create"][0] == 0 and r["native_available"] == 0
    assert "native init failed" in r["details"]


@pytest.mark.gpu
@needs_build
def test_reference_cuda_backend_runs_moe_ops_natively():
    from oracle import synth
    from oracle.oracle import Oracle
    sys.path.insert(0, HERE)
    import reference_cuda_backend as rcb

    T = 64
    r = _run("--T", str(T))
    assert r["create"][0] == 0 and r["native_available"] == 1, r["details"]
    assert "libuaii_moe" in r["details"]
    assert r["router"][0] == 0 and r["swiglu"][0] == 0 and r["matmul"][0] == 0 and r["sync"] == 0, r
    # three ops on the device, nothing declined; then the Softmax is declined and host-staged
    assert r["native_calls_before_softmax"] == [3, 0]
    assert r["softmax"][0] == 0 and r["native_calls"] == [3, 1]

    D, E, I, K = rcb.D, rcb.E, rcb.I, rcb.K
    x = synth.fill_normal((T, D), 5, 6, 0.0, 1.0)
    w = synth.fill_normal((E, D), 11, 1, 0.0, 0.02)
    G = synth.quantize_rows(rcb.Q4_K, synth.fill_normal((E * I, D), 11, 2, 0.0, 0.02))
    U = synth.quantize_rows(rcb.Q4_K, synth.fill_normal((E * I, D), 11, 3, 0.0, 0.02))
    Dn = synth.quantize_rows(rcb.Q6_K, synth.fill_normal((E * D, I), 11, 4, 0.0, 0.02))
    Bm = synth.quantize_rows(rcb.Q4_K, synth.fill_normal((rcb.MM_N, D), 11, 7, 0.0, 0.05))
    o = Oracle()
    _, probs, top = o.router(x, w)
    assert np.abs(np.asarray(r["probs"]) - probs).max() <= 1e-6
    assert np.array_equal(np.asarray(r["top"], np.float32), top.ravel())
    y, _, _ = o.experts_packed(x, G, rcb.Q4_K, U, rcb.Q4_K, Dn, rcb.Q6_K, probs, E, I, K)
    assert _rel(r["y"], y) <= 2e-3
    c = o.quant_gemm(x, Bm, rcb.Q4_K, rcb.MM_N, relu=True)
    assert _rel(r["c"], c) <= 2e-3
    e = np.exp(x.astype(np.float64) - x.max(axis=1, keepdims=True))
    assert np.abs(np.asarray(r["softmax_y"]) - e / e.sum(axis=1, keepdims=True)).max() <= 1e-6


def _session(tmp_path, *args):
    d = tmp_path / ("s_" + "_".join(a.strip("-") for a in args))
    d.mkdir()
    p = subprocess.run([sys.executable, os.path.join(HERE, "reference_runtime_session.py"), str(d), *args],
                       capture_output=True, text=True, timeout=600)
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert p.returncode == 0 and lines, (p.returncode, p.stdout[-2000:], p.stderr[-2000:])
    return json.loads(lines[-1])


@pytest.mark.gpu
@needs_build
def test_reference_cuda_session_with_native_layer_and_plugin(tmp_path):
    """A Session with backend "cuda" in the runtime built with the native layer: the backend
    reports native, the Session's host-resident tensors run through host dispatch
    (cuda_backend.cpp:189-192), where the operator plugin puts both MoE operators on the GPU.
    Against the stock CPU Session (f32 experts): probabilities within 1e-6, outputs within 2e-3."""
    plugin = os.path.join(REPO, "universal-ai-inference_b200", "libuaii_moe_plugin.so")
    if not os.path.exists(plugin):
        pytest.skip("plugin not built")
    ref = _session(tmp_path, "--keep-quantized", "0")
    got = _session(tmp_path, "--runtime", "cuda", "--backend", "cuda", "--plugin", "--const-weights")
    assert "CUDA backend (native)" in got["details"], got["details"]
    assert got["plugin_load"][0] == 0 and got["registered"] == [1, 1, 1]
    assert got["plugin_calls"] == [4, 0]
    assert np.abs(np.asarray(got["probs"]) - np.asarray(ref["probs"])).max() <= 1e-6
    y, r = np.asarray(got["y"], np.float64), np.asarray(ref["y"], np.float64)
    assert np.abs(y - r).max() / np.abs(r).max() <= 2e-3
