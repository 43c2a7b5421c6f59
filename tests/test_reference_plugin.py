"""The operator plugin (universal-ai-inference_b200/plugin/uaii_moe_plugin.cpp) inside the
reference's own runtime: a Session created from a .uaii.json MoE layer
(tests/reference_runtime_session.py, run in a child process) with and without the plugin.

Without the plugin the reference's host kernels run the layer (experts dequantized to f32
at load: its MoEExpertsSwiGLU reads f32 experts only).  With it, the same unmodified
Session dispatches MoERouter and MoEExpertsSwiGLU to the GPU with the experts kept packed.
Bars: probabilities within 1e-6 (the device router's logits are the reference's bit for
bit; the exponential differs by at most an ulp), outputs within 2e-3 of the largest
output (f16 tensor-core operands) or 1e-5 on the CUDA-core path (f32 experts).
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
RUNTIME_SO = os.path.join(REPO, "oracle", "_ref", "libuaii_ref_runtime.so")
PLUGIN_SO = os.path.join(REPO, "universal-ai-inference_b200", "libuaii_moe_plugin.so")

needs_build = pytest.mark.skipif(not (os.path.exists(RUNTIME_SO) and os.path.exists(PLUGIN_SO)),
                                 reason="reference runtime or plugin not built (build() with the reference tree)")


def _run(tmp_path, *args):
    d = tmp_path / ("run_" + "_".join(a.strip("-") for a in args))
    d.mkdir()
    p = subprocess.run([sys.executable, os.path.join(HERE, "reference_runtime_session.py"), str(d), *args],
                       capture_output=True, text=True, timeout=600)
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert p.returncode == 0 and lines, (p.returncode, p.stdout[-2000:], p.stderr[-2000:])
    return json.loads(lines[-1])


def _rel(y, ref):
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    return float(np.abs(y - ref).max() / np.abs(ref).max())


@needs_build
def test_plugin_exports_the_reference_plugin_abi():
    # the dynamic symbol table (the library itself only loads into a UAII host process)
    out = subprocess.run(["nm", "-D", "--defined-only", PLUGIN_SO], capture_output=True, text=True, check=True)
    names = {ln.split()[-1] for ln in out.stdout.splitlines() if ln.strip()}
    for sym in ("uaii_plugin_get_info", "uaii_plugin_init", "uaii_plugin_shutdown", "uaii_moe_plugin_stats"):
        assert sym in names, sym


@needs_build
def test_plugin_refuses_to_load_without_a_gpu(tmp_path):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    r = _run(tmp_path, "--plugin")
    assert r["plugin_load"][0] == 5 and "init failed" in r["plugin_load"][1]  # PluginError
    assert r["registered"] == [0, 0, 0]


@pytest.mark.gpu
@needs_build
def test_reference_session_runs_moe_on_the_gpu_through_the_plugin(tmp_path):
    ref = _run(tmp_path, "--keep-quantized", "0")
    got = _run(tmp_path, "--plugin")
    assert got["plugin_load"][0] == 0 and got["registered"] == [1, 1, 1]
    assert got["plugin_calls"] == [4, 0]  # 2 runs x (router, experts), nothing on the host kernels
    assert np.abs(np.asarray(got["probs"]) - np.asarray(ref["probs"])).max() <= 1e-6
    assert _rel(got["y"], ref["y"]) <= 2e-3


@pytest.mark.gpu
@needs_build
def test_plugin_with_cuda_backend_constant_weights_and_demo(tmp_path):
    ref = _run(tmp_path, "--keep-quantized", "0", "--demo")
    got = _run(tmp_path, "--plugin", "--backend", "cuda", "--const-weights", "--demo", "--runs", "3")
    assert ref["demo"] == [0, 1] and got["demo"] == [0, 1]
    # 3 runs x 2 ops, then the demo's MoERouter + MoEExperts and MoERouter + MoEExpertsSwiGLU
    assert got["plugin_calls"] == [10, 0]
    assert _rel(got["y"], ref["y"]) <= 2e-3


@pytest.mark.gpu
@needs_build
def test_plugin_with_f32_experts_matches_the_reference_kernel(tmp_path):
    ref = _run(tmp_path, "--keep-quantized", "0", "--T", "16")
    got = _run(tmp_path, "--plugin", "--keep-quantized", "0", "--T", "16")
    assert got["plugin_calls"] == [4, 0]
    assert _rel(got["y"], ref["y"]) <= 1e-5
