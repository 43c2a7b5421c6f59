"""Runs a MoE layer through the reference's own Session (oracle/_ref/libuaii_ref_runtime.so,
built from the unmodified reference sources) and prints one JSON line.

    python tests/reference_runtime_session.py OUT_DIR [--plugin] [--backend cpu|cuda]
        [--const-weights] [--demo] [--T 64] [--runtime stub|cuda]

The graph is a .uaii.json IR file (the reference's own format, include/uaii/ir/serialize.hpp)
with MoERouter -> MoEExpertsSwiGLU; its weights live in a GGUF file next to it and are
loaded by the Session through "file.gguf#tensor" weight refs (session.cpp:408-440), the
experts kept packed (keep_quantized_weights, naive allocation) or, with --keep-quantized 0,
dequantized to f32 at load: the reference's own MoEExpertsSwiGLU kernel reads f32 experts
only (transformer.cpp:560-608 indexes them as floats).  With --plugin the
repository's operator plugin (universal-ai-inference_b200/libuaii_moe_plugin.so) is
loaded first through the reference's plugin host, so the same Session runs the two MoE
operators on the GPU.  Run as a separate process: the reference runtime is loaded with
RTLD_GLOBAL (plugins resolve host symbols from the process) and its operator table keeps
a registered plugin until exit.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)

from gguf_writer import F32 as KV_F32, U32, GGML_F32, GGML_Q4_K, GGML_Q6_K, write_gguf  # noqa: E402
from oracle import synth  # noqa: E402

RUNTIME_SO = os.path.join(REPO, "oracle", "_ref", "libuaii_ref_runtime.so")
# the same runtime built with UAII_WITH_CUDA, its CUDA native layer from plugin/uaii_cuda_native.cpp
RUNTIME_CUDA_SO = os.path.join(REPO, "oracle", "_ref", "libuaii_ref_cuda.so")
PLUGIN_SO = os.path.join(REPO, "universal-ai-inference_b200", "libuaii_moe_plugin.so")
Q4_K, Q6_K = 14, 16
D, E, I, K = 512, 8, 1024, 2


def write_model(out_dir: str, seed: int = 11):
    rng_w = synth.fill_normal((E, D), seed, 1, 0.0, 0.02)
    G = synth.quantize_rows(Q4_K, synth.fill_normal((E * I, D), seed, 2, 0.0, 0.02))
    U = synth.quantize_rows(Q4_K, synth.fill_normal((E * I, D), seed, 3, 0.0, 0.02))
    Dn = synth.quantize_rows(Q6_K, synth.fill_normal((E * D, I), seed, 4, 0.0, 0.02))
    write_gguf(os.path.join(out_dir, "moe.gguf"), [("general.alignment", U32, 32)], [
        ("blk.0.ffn_gate_inp.weight", GGML_F32, (E, D), rng_w.tobytes()),
        ("blk.0.ffn_gate_exps.weight", GGML_Q4_K, (E, I, D), G.tobytes()),
        ("blk.0.ffn_up_exps.weight", GGML_Q4_K, (E, I, D), U.tobytes()),
        ("blk.0.ffn_down_exps.weight", GGML_Q6_K, (E, D, I), Dn.tobytes())])
    return rng_w, G, U, Dn


def write_graph(out_dir: str, T: int) -> str:
    def tensor(i, name, shape, weight="", quant="f32"):
        t = {"id": i, "name": name, "dtype": "f32", "shape": list(shape),
             "storage_hint": "external" if weight else "ram", "is_weight": bool(weight), "weight_ref": weight}
        if quant != "f32":
            t["quant_format"] = quant
        return t
    g = {
        "ir_version": {"major": 1, "minor": 0}, "name": "moe_layer", "producer": "uaii-b200-tests", "domain": "uaii",
        "tensors": [
            tensor(1, "x", (T, D)),
            tensor(2, "gate", (E, D), "moe.gguf#blk.0.ffn_gate_inp.weight"),
            tensor(3, "probs", (T, E)),
            tensor(4, "top_expert", (T, 1)),
            tensor(5, "gate_exps", (E, I, D), "moe.gguf#blk.0.ffn_gate_exps.weight", "q4_k"),
            tensor(6, "up_exps", (E, I, D), "moe.gguf#blk.0.ffn_up_exps.weight", "q4_k"),
            tensor(7, "down_exps", (E, D, I), "moe.gguf#blk.0.ffn_down_exps.weight", "q6_k"),
            tensor(8, "y", (T, D)),
        ],
        "nodes": [
            {"id": 1, "name": "router", "op_name": "MoERouter", "op_version": "1", "inputs": [1, 2],
             "outputs": [3, 4], "attributes": [{"key": "num_experts", "type": "int", "value": E}]},
            {"id": 2, "name": "experts", "op_name": "MoEExpertsSwiGLU", "op_version": "1",
             "inputs": [1, 5, 6, 7, 3], "outputs": [8],
             "attributes": [{"key": "num_experts", "type": "int", "value": E},
                            {"key": "top_k", "type": "int", "value": K}]},
        ],
        "inputs": [1], "outputs": [8, 3], "metadata": {},
    }
    path = os.path.join(out_dir, "moe.uaii.json")
    with open(path, "w") as f:
        json.dump(g, f)
    return path


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("out_dir")
    ap.add_argument("--plugin", action="store_true")
    ap.add_argument("--backend", default="cpu")
    ap.add_argument("--const-weights", action="store_true")
    ap.add_argument("--demo", action="store_true", help="also run the reference's MoE smoke demo")
    ap.add_argument("--T", type=int, default=64)
    ap.add_argument("--runs", type=int, default=2)
    ap.add_argument("--runtime", default="stub", choices=["stub", "cuda"],
                    help="stub: the reference's CUDA native layer stubbed out (its default build); cuda: the "
                         "runtime with the repository's native layer linked in")
    ap.add_argument("--keep-quantized", type=int, default=1,
                    help="1: experts stay packed (the reference's own MoEExpertsSwiGLU reads f32 experts "
                         "only, so without the plugin use 0: dequantized to f32 at load)")
    a = ap.parse_args()
    if a.const_weights:
        os.environ["UAII_MOE_CONST_WEIGHTS"] = "1"
    rt = ctypes.CDLL(RUNTIME_CUDA_SO if a.runtime == "cuda" else RUNTIME_SO, mode=ctypes.RTLD_GLOBAL)
    vp, cp, i32, sz = ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_size_t
    for name, res, args in (("urt_last_error", cp, []), ("urt_plugin_load", i32, [cp]),
                            ("urt_operator_registered", i32, [cp]), ("urt_moe_smoke_demo", i32, [vp]),
                            ("urt_session_create", i32, [cp, cp, cp, i32, i32, vp]),
                            ("urt_session_destroy", None, [vp]), ("urt_session_set_f32", i32, [vp, cp, vp, sz]),
                            ("urt_session_run", i32, [vp]), ("urt_session_get_f32", i32, [vp, cp, vp, sz, vp]),
                            ("urt_session_backend_details", cp, [vp])):
        f = getattr(rt, name)
        f.restype, f.argtypes = res, args
    out = {"plugin": a.plugin, "backend": a.backend, "keep_quantized": a.keep_quantized, "runtime": a.runtime}
    if a.plugin:
        st = rt.urt_plugin_load(PLUGIN_SO.encode())
        out["plugin_load"] = [st, rt.urt_last_error().decode()]
        out["registered"] = [rt.urt_operator_registered(op) for op in (b"MoERouter", b"MoEExperts", b"MoEExpertsSwiGLU")]
        if st != 0:
            print(json.dumps(out))
            return
    write_model(a.out_dir)
    path = write_graph(a.out_dir, a.T)
    sess = ctypes.c_void_p()
    st = rt.urt_session_create(path.encode(), a.backend.encode(), a.out_dir.encode(), a.keep_quantized, 0,
                               ctypes.byref(sess))
    if st != 0:
        out["error"] = [st, rt.urt_last_error().decode()]
        print(json.dumps(out))
        sys.exit(1)
    out["details"] = rt.urt_session_backend_details(sess).decode()
    x = synth.fill_normal((a.T, D), 5, 6, 0.0, 1.0)
    y = np.empty((a.T, D), np.float32)
    probs = np.empty((a.T, E), np.float32)
    n = ctypes.c_size_t()
    ms = []
    for _ in range(a.runs):
        assert rt.urt_session_set_f32(sess, b"x", x.ctypes.data, x.size) == 0, rt.urt_last_error()
        t0 = time.perf_counter()
        st = rt.urt_session_run(sess)
        ms.append((time.perf_counter() - t0) * 1e3)
        assert st == 0, rt.urt_last_error()
    assert rt.urt_session_get_f32(sess, b"y", y.ctypes.data, y.size, ctypes.byref(n)) == 0 and n.value == y.size
    assert rt.urt_session_get_f32(sess, b"probs", probs.ctypes.data, probs.size, ctypes.byref(n)) == 0
    rt.urt_session_destroy(sess)
    out.update({"T": a.T, "ms": ms, "y": y.tolist(), "probs": probs.tolist()})
    if a.demo:
        ok = ctypes.c_int(0)
        out["demo"] = [rt.urt_moe_smoke_demo(ctypes.byref(ok)), ok.value]
    if a.plugin:
        pl = ctypes.CDLL(PLUGIN_SO)
        dev, host = ctypes.c_uint64(), ctypes.c_uint64()
        pl.uaii_moe_plugin_stats(ctypes.byref(dev), ctypes.byref(host))
        out["plugin_calls"] = [dev.value, host.value]
    print(json.dumps(out))


if __name__ == "__main__":
    main()
