"""Runs MoE operators through the reference's own CudaBackend with device-resident tensors and
prints one JSON line.

    python tests/reference_cuda_backend.py [--T 64]

oracle/_ref/libuaii_ref_cuda.so is the reference runtime built from its unmodified sources with
UAII_WITH_CUDA, whose CUDA native layer (libs/uaii-backends/src/native_stubs.hpp:18-37) is the
repository's universal-ai-inference_b200/plugin/uaii_cuda_native.cpp over libuaii_moe.so.  The
script creates the backend through the reference factory, allocates device buffers with
CudaBackend::allocate, uploads with copy_h2d and calls IBackend::dispatch (cuda_backend.cpp:166-207)
for MoERouter, MoEExpertsSwiGLU on packed Q4_K / Q6_K experts, MatMulRelu with a packed Q4_K B,
and a Softmax that the native layer declines (CudaBackend stages it through the host kernels).
The counters of the native layer show which ops ran on the device.  Run as a separate process
so the reference runtime's globals live and die with it.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, REPO)

from oracle import synth  # noqa: E402

CUDA_SO = os.path.join(REPO, "oracle", "_ref", "libuaii_ref_cuda.so")
Q4_K, Q6_K = 14, 16
D, E, I, K = 512, 8, 1024, 2
MM_N = 384


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--T", type=int, default=64)
    a = ap.parse_args()
    T = a.T
    L = ctypes.CDLL(CUDA_SO)
    vp, i32, i64, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
    ull = ctypes.c_ulonglong
    for name, res, args in (
            ("ucb_last_error", ctypes.c_char_p, []), ("ucb_create", i32, [vp, vp, ctypes.c_char_p, sz]),
            ("ucb_destroy", None, [vp]), ("ucb_alloc", i32, [vp, sz, vp]), ("ucb_free", i32, [vp, vp]),
            ("ucb_h2d", i32, [vp, vp, vp, sz]), ("ucb_d2h", i32, [vp, vp, vp, sz]), ("ucb_sync", i32, [vp]),
            ("ucb_moe_router", i32, [vp, vp, vp, i64, i64, i64, vp, vp]),
            ("ucb_moe_swiglu", i32, [vp, vp, vp, i32, sz, vp, i32, sz, vp, i32, sz, vp, i64, i64, i64, i64, i64,
                                     vp]),
            ("ucb_matmul_packed", i32, [vp, vp, i64, i64, vp, i32, sz, i64, i32, vp]),
            ("ucb_softmax", i32, [vp, vp, i64, i64, vp]),
            ("uaii_cuda_native_stats", None, [vp, vp])):
        f = getattr(L, name)
        f.restype, f.argtypes = res, args

    def err():
        return L.ucb_last_error().decode()

    b = ctypes.c_void_p()
    native = ctypes.c_int(0)
    details = ctypes.create_string_buffer(512)
    st = L.ucb_create(ctypes.byref(b), ctypes.byref(native), details, 512)
    out = {"create": [st, err() if st else ""], "native_available": native.value, "details": details.value.decode()}
    if st != 0 or not native.value:
        print(json.dumps(out))
        return

    bufs = []

    def dev(arr=None, nbytes=None):
        n = int(arr.nbytes if arr is not None else nbytes)
        p = ctypes.c_void_p()
        assert L.ucb_alloc(b, n, ctypes.byref(p)) == 0, err()
        bufs.append(p.value)
        if arr is not None:
            assert L.ucb_h2d(b, arr.ctypes.data, p.value, n) == 0, err()
        return p.value

    def host(p, shape):
        h = np.empty(shape, np.float32)
        assert L.ucb_d2h(b, p, h.ctypes.data, h.nbytes) == 0, err()
        return h

    x = synth.fill_normal((T, D), 5, 6, 0.0, 1.0)
    w = synth.fill_normal((E, D), 11, 1, 0.0, 0.02)
    G = synth.quantize_rows(Q4_K, synth.fill_normal((E * I, D), 11, 2, 0.0, 0.02))
    U = synth.quantize_rows(Q4_K, synth.fill_normal((E * I, D), 11, 3, 0.0, 0.02))
    Dn = synth.quantize_rows(Q6_K, synth.fill_normal((E * D, I), 11, 4, 0.0, 0.02))
    Bm = synth.quantize_rows(Q4_K, synth.fill_normal((MM_N, D), 11, 7, 0.0, 0.05))
    dx, dw = dev(x), dev(w)
    dG, dU, dD, dB = dev(G), dev(U), dev(Dn), dev(Bm)
    dprobs, dtop = dev(nbytes=T * E * 4), dev(nbytes=T * 4)
    dy, dc, dsm = dev(nbytes=T * D * 4), dev(nbytes=T * MM_N * 4), dev(nbytes=T * D * 4)

    out["router"] = [L.ucb_moe_router(b, dx, dw, T, D, E, dprobs, dtop), err()]
    out["swiglu"] = [L.ucb_moe_swiglu(b, dx, dG, Q4_K, G.nbytes, dU, Q4_K, U.nbytes, dD, Q6_K, Dn.nbytes, dprobs,
                                      T, D, E, I, K, dy), err()]
    out["matmul"] = [L.ucb_matmul_packed(b, dx, T, D, dB, Q4_K, Bm.nbytes, MM_N, 1, dc), err()]
    out["sync"] = L.ucb_sync(b)
    dev_ops, declined = ull(), ull()
    L.uaii_cuda_native_stats(ctypes.byref(dev_ops), ctypes.byref(declined))
    out["native_calls_before_softmax"] = [dev_ops.value, declined.value]
    out["softmax"] = [L.ucb_softmax(b, dx, T, D, dsm), err()]
    L.uaii_cuda_native_stats(ctypes.byref(dev_ops), ctypes.byref(declined))
    out["native_calls"] = [dev_ops.value, declined.value]
    out.update({"T": T, "probs": host(dprobs, (T, E)).tolist(), "top": host(dtop, (T, 1)).ravel().tolist(),
                "y": host(dy, (T, D)).tolist(), "c": host(dc, (T, MM_N)).tolist(),
                "softmax_y": host(dsm, (T, D)).tolist()})
    for p in bufs:
        assert L.ucb_free(b, p) == 0, err()
    L.ucb_destroy(b)
    print(json.dumps(out))


if __name__ == "__main__":
    main()
