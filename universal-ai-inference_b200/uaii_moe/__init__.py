"""ctypes binding of libuaii_moe.so (the C ABI in include/uaii_moe.h).

This is the binding a maintainer of the reference's Python SDK would add beside
its own ctypes fallback (bindings/python/uaii/__init__.py in the reference):
every call goes straight to the C ABI, and array arguments may be torch tensors
(host or CUDA) or numpy arrays.  There is no Python compute path: if the shared
library is missing, importing this module raises.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, byref, c_char_p, c_double, c_float, c_int, c_int32, c_int64, c_size_t, c_uint64, c_void_p

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("UAII_MOE_LIB") or os.path.join(os.path.dirname(_HERE), "libuaii_moe.so")

# uaii::quant::QuantFormat values (include/uaii/quant/formats.hpp:10-29)
F32, F16 = 0, 1
Q4_0, Q4_1, Q5_0, Q5_1, Q8_0 = 7, 8, 9, 10, 11
Q2_K, Q3_K, Q4_K, Q5_K, Q6_K = 12, 13, 14, 15, 16
FORMAT_NAMES = {F32: "f32", F16: "f16", Q4_0: "q4_0", Q4_1: "q4_1", Q5_0: "q5_0", Q5_1: "q5_1",
                Q8_0: "q8_0", Q2_K: "q2_k", Q3_K: "q3_k", Q4_K: "q4_k", Q5_K: "q5_k", Q6_K: "q6_k"}
BLOCK = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q4_1: (32, 20), Q5_0: (32, 22), Q5_1: (32, 24),
         Q8_0: (32, 34), Q2_K: (256, 84), Q3_K: (256, 110), Q4_K: (256, 144), Q5_K: (256, 176),
         Q6_K: (256, 210)}

OK = 0
INVALID_ARGUMENT, NOT_FOUND, NOT_IMPLEMENTED, INTERNAL = 1, 2, 7, 8
STATUS_NAMES = {0: "Ok", 1: "InvalidArgument", 2: "NotFound", 3: "IoError", 4: "ConfigError",
                5: "PluginError", 6: "AbiMismatch", 7: "NotImplemented", 8: "Internal"}

DTYPE_UNKNOWN, DTYPE_F32, DTYPE_F16 = 0, 1, 2
ATTR_INT, ATTR_FLOAT, ATTR_BOOL = 1, 2, 3


class UaiiMoeError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status
        self.message = message


class Tensor(ctypes.Structure):
    _fields_ = [("dtype", c_int32), ("quant_format", c_int32), ("shape", POINTER(c_int64)),
                ("rank", c_uint64), ("data", c_void_p), ("nbytes", c_uint64)]


class Attr(ctypes.Structure):
    _fields_ = [("key", c_char_p), ("type", c_int32), ("i", c_int64), ("f", c_double)]


class Layer(ctypes.Structure):
    _fields_ = [("d_model", c_int64), ("n_experts", c_int64), ("d_ff", c_int64), ("top_k", c_int32),
                ("norm_topk", c_int32), ("router_w", c_void_p), ("gate_exps", c_void_p),
                ("gate_fmt", c_int32), ("up_exps", c_void_p), ("up_fmt", c_int32),
                ("down_exps", c_void_p), ("down_fmt", c_int32), ("shared_d_ff", c_int64),
                ("gate_shexp", c_void_p), ("gate_shexp_fmt", c_int32), ("up_shexp", c_void_p),
                ("up_shexp_fmt", c_int32), ("down_shexp", c_void_p), ("down_shexp_fmt", c_int32),
                ("gate_inp_shexp", c_void_p)]


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is not built; run `make -C {os.path.dirname(LIB_PATH)}` "
                          "(or __graft_entry__.build())")
    lib = ctypes.CDLL(LIB_PATH)
    sig = {
        "uaii_moe_abi_version": (c_int, []),
        "uaii_moe_last_error": (c_char_p, []),
        "uaii_moe_backend_create": (c_int, [c_int, c_void_p, POINTER(c_void_p)]),
        "uaii_moe_backend_destroy": (None, [c_void_p]),
        "uaii_moe_synchronize": (c_int, [c_void_p]),
        "uaii_moe_supports_op": (c_int, [c_char_p]),
        "uaii_moe_dispatch": (c_int, [c_void_p, c_char_p, c_char_p, POINTER(Tensor), c_size_t,
                                      POINTER(Tensor), c_size_t, POINTER(Attr), c_size_t]),
        "uaii_moe_dequant_rows": (c_int, [c_void_p, c_int, c_void_p, c_int64, c_int64, c_void_p]),
        "uaii_moe_router_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                        c_void_p, c_void_p, c_void_p]),
        "uaii_moe_experts_swiglu": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int,
                                            c_void_p, c_int, c_void_p, c_int64, c_int64, c_int64,
                                            c_int64, c_int, c_int, c_void_p]),
        "uaii_moe_ffn_forward": (c_int, [c_void_p, POINTER(Layer), c_void_p, c_int64, c_void_p, c_void_p]),
        "uaii_moe_ffn_forward_noalloc": (c_int, [c_int, c_void_p, POINTER(Layer), c_void_p, c_int64, c_void_p,
                                                 c_void_p]),
        "uaii_moe_register_weights": (c_int, [c_void_p, c_void_p, c_uint64]),
        "uaii_moe_release_weights": (c_int, [c_void_p, c_void_p]),
        "uaii_moe_set_expert_path": (c_int, [c_void_p, c_int]),
        "uaii_moe_backend_stream": (c_int, [c_void_p, POINTER(c_void_p)]),
        "uaii_moe_set_graphs": (c_int, [c_void_p, c_int]),
        "uaii_moe_route": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int, c_int, c_void_p,
                                   c_void_p]),
        "uaii_moe_quant_matmul": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_int, c_int64, c_int,
                                          c_void_p]),
        "uaii_moe_gguf_open": (c_int, [c_char_p, POINTER(c_void_p)]),
        "uaii_moe_gguf_close": (None, [c_void_p]),
        "uaii_moe_gguf_tensor_count": (c_int64, [c_void_p]),
        "uaii_moe_gguf_tensor_at": (c_int, [c_void_p, c_int64, POINTER(c_char_p), POINTER(c_void_p), POINTER(c_int),
                                            POINTER(c_int64), POINTER(c_int), POINTER(c_uint64)]),
        "uaii_moe_gguf_tensor": (c_int, [c_void_p, c_char_p, POINTER(c_void_p), POINTER(c_int), POINTER(c_int64),
                                         POINTER(c_int), POINTER(c_uint64)]),
        "uaii_moe_gguf_kv_int": (c_int, [c_void_p, c_char_p, POINTER(c_int64)]),
        "uaii_moe_gguf_kv_float": (c_int, [c_void_p, c_char_p, POINTER(c_double)]),
        "uaii_moe_gguf_kv_string": (c_int, [c_void_p, c_char_p, POINTER(c_char_p)]),
        "uaii_moe_gguf_moe_layer": (c_int, [c_void_p, c_int, c_int, c_void_p]),
        "uaii_moe_last_plan": (c_int, [c_void_p, POINTER(c_int), POINTER(c_int), POINTER(c_int)]),
        "uaii_moe_ep_dispatch": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p,
                                         c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
        "uaii_moe_ep_experts": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64,
                                        c_void_p]),
        "uaii_moe_ep_combine": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int64, c_void_p]),
        "uaii_moe_ep_combine_f16": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int64, c_void_p]),
        "uaii_moe_ep_experts_records_f16": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                                    c_void_p]),
        "uaii_moe_ep_dispatch_records": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_void_p,
                                                 c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
        "uaii_moe_ep_experts_records": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                                c_void_p]),
        "uaii_moe_selftest_wait_timeout": (c_int, [c_void_p, c_int64]),
        "uaii_moe_profile_enable": (c_int, [c_void_p, c_int]),
        "uaii_moe_profile_read": (c_int, [c_void_p, POINTER(c_double), POINTER(c_uint64), POINTER(c_uint64)]),
        "uaii_moe_packed_nbytes": (c_uint64, [c_int, c_int64]),
        "uaii_moe_quantize_rows": (c_int, [c_int, c_void_p, c_int64, c_int64, c_void_p]),
        "uaii_moe_fill_normal": (c_int, [c_void_p, c_int64, c_uint64, c_uint64, c_float, c_float]),
        "uaii_moe_decoder_create": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int,
                                            POINTER(c_void_p)]),
        "uaii_moe_decoder_destroy": (None, [c_void_p]),
        "uaii_moe_decoder_set_kv": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_int64]),
        "uaii_moe_decoder_fill_kv": (c_int, [c_void_p, c_int64, c_uint64]),
        "uaii_moe_decoder_step": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p]),
        "uaii_moe_decoder_generate": (c_int, [c_void_p, c_void_p, c_int64, c_void_p]),
        "uaii_moe_decoder_position": (c_int64, [c_void_p]),
        "uaii_moe_fill_normal_device": (c_int, [c_void_p, c_void_p, c_int64, c_uint64, c_uint64, c_float, c_float]),
        "uaii_moe_quantize_rows_device": (c_int, [c_void_p, c_int, c_void_p, c_int64, c_int64, c_void_p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()
EXPORTED = ("uaii_moe_abi_version", "uaii_moe_last_error", "uaii_moe_backend_create",
            "uaii_moe_backend_destroy", "uaii_moe_synchronize", "uaii_moe_supports_op",
            "uaii_moe_dispatch", "uaii_moe_dequant_rows", "uaii_moe_router_f32",
            "uaii_moe_experts_swiglu", "uaii_moe_ffn_forward", "uaii_moe_ffn_forward_noalloc",
            "uaii_moe_register_weights",
            "uaii_moe_release_weights",
            "uaii_moe_set_expert_path", "uaii_moe_set_graphs", "uaii_moe_route", "uaii_moe_backend_stream", "uaii_moe_quant_matmul", "uaii_moe_last_plan",
            "uaii_moe_gguf_open", "uaii_moe_gguf_close", "uaii_moe_gguf_tensor_count", "uaii_moe_gguf_tensor_at",
            "uaii_moe_gguf_tensor", "uaii_moe_gguf_kv_int", "uaii_moe_gguf_kv_float", "uaii_moe_gguf_kv_string",
            "uaii_moe_gguf_moe_layer", "uaii_moe_ep_dispatch", "uaii_moe_ep_experts",
            "uaii_moe_ep_combine", "uaii_moe_ep_dispatch_records", "uaii_moe_ep_experts_records",
            "uaii_moe_ep_experts_records_f16", "uaii_moe_ep_combine_f16",
            "uaii_moe_selftest_wait_timeout", "uaii_moe_profile_enable",
            "uaii_moe_profile_read",
            "uaii_moe_packed_nbytes", "uaii_moe_quantize_rows",
            "uaii_moe_fill_normal", "uaii_moe_decoder_create", "uaii_moe_decoder_destroy",
            "uaii_moe_decoder_set_kv", "uaii_moe_decoder_fill_kv", "uaii_moe_decoder_step",
            "uaii_moe_decoder_generate", "uaii_moe_decoder_position", "uaii_moe_fill_normal_device",
            "uaii_moe_quantize_rows_device")


def _check(status: int):
    if status != OK:
        raise UaiiMoeError(status, lib.uaii_moe_last_error().decode())


def ptr(a) -> int | None:
    """Address of a torch tensor, numpy array or raw int; None stays None."""
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if isinstance(a, np.ndarray):
        if not a.flags["C_CONTIGUOUS"]:
            raise ValueError("numpy array must be C-contiguous")
        return a.ctypes.data
    if hasattr(a, "data_ptr"):
        if not a.is_contiguous():
            raise ValueError("tensor must be contiguous")
        return a.data_ptr()
    raise TypeError(f"cannot take the address of {type(a)}")


def packed_nbytes(fmt: int, n: int) -> int:
    return int(lib.uaii_moe_packed_nbytes(fmt, n))


def quantize_rows(fmt: int, src: np.ndarray) -> np.ndarray:
    """f32 [rows, cols] -> GGUF bytes [rows, packed_nbytes(fmt, cols)] (uint8)."""
    src = np.ascontiguousarray(src, dtype=np.float32)
    cols = src.shape[-1]
    rows = src.size // cols
    out = np.empty(src.shape[:-1] + (packed_nbytes(fmt, cols),), dtype=np.uint8)
    _check(lib.uaii_moe_quantize_rows(fmt, src.ctypes.data, rows, cols, out.ctypes.data))
    return out


def fill_normal(shape, seed: int, stream: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(shape, dtype=np.float32)
    _check(lib.uaii_moe_fill_normal(out.ctypes.data, out.size, seed, stream, mean, std))
    return out


class Backend:
    """One device, one stream, a workspace and a weight cache (uaii_moe_backend)."""

    def __init__(self, device: int = 0, stream: int | None = None):
        h = c_void_p()
        _check(lib.uaii_moe_backend_create(device, stream, ctypes.byref(h)))
        self._h = h

    def close(self):
        if self._h:
            lib.uaii_moe_backend_destroy(self._h)
            self._h = c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stream(self) -> int:
        """cudaStream_t handle the backend queues its work on (its own stream if none was given)."""
        h = c_void_p()
        _check(lib.uaii_moe_backend_stream(self._h, ctypes.byref(h)))
        return int(h.value or 0)

    def synchronize(self):
        _check(lib.uaii_moe_synchronize(self._h))

    def set_expert_path(self, path: int):
        _check(lib.uaii_moe_set_expert_path(self._h, path))

    def set_graphs(self, on: bool):
        """CUDA-graph replay of repeated device-resident layer calls (default on)."""
        _check(lib.uaii_moe_set_graphs(self._h, int(on)))

    def last_plan(self) -> dict:
        """Schedule of the most recent expert-product call: tensor cores or not,
        which tensor-core schedule ("tcgen05", "warp_mma", "quad_mma", "quad_mma_i8" or None), slot
        tile width and down-projection K splits."""
        tc, bn, sp = c_int(), c_int(), c_int()
        _check(lib.uaii_moe_last_plan(self._h, byref(tc), byref(bn), byref(sp)))
        sched = {1: "tcgen05", 2: "warp_mma", 3: "quad_mma", 4: "quad_mma_i8"}.get(tc.value)
        return {"tensor_cores": bool(tc.value), "schedule": sched, "slot_tile": bn.value, "down_splits": sp.value}

    PHASES = ("router", "route", "gateup", "down", "shared", "combine")

    def profile_enable(self, on: bool = True):
        _check(lib.uaii_moe_profile_enable(self._h, int(on)))

    def profile_read(self):
        """{phase: (total_ms, calls)}, kernel launches since profile_enable."""
        ms = (c_double * 6)()
        calls = (c_uint64 * 6)()
        n = c_uint64()
        _check(lib.uaii_moe_profile_read(self._h, ms, calls, ctypes.byref(n)))
        return {p: (ms[i], int(calls[i])) for i, p in enumerate(self.PHASES)}, int(n.value)

    @property
    def handle(self):
        return self._h

    def register_weights(self, array):
        """Declare a weight buffer constant until release_weights(): a host buffer is
        uploaded once; for host and device buffers alike, layouts derived from the
        weights (padded rows) are made once and kept."""
        _check(lib.uaii_moe_register_weights(self._h, ptr(array), array.nbytes))

    def release_weights(self, array):
        _check(lib.uaii_moe_release_weights(self._h, ptr(array)))

    def dequant_rows(self, fmt: int, packed, rows: int, cols: int, out):
        _check(lib.uaii_moe_dequant_rows(self._h, fmt, ptr(packed), rows, cols, ptr(out)))

    def router(self, x, gate_w, T: int, D: int, E: int, probs, top, logits=None):
        _check(lib.uaii_moe_router_f32(self._h, ptr(x), ptr(gate_w), T, D, E, ptr(probs), ptr(top),
                                       ptr(logits)))

    def experts(self, x, gate, gfmt, up, ufmt, down, dfmt, probs, T, D, E, I, top_k, norm_topk, y):
        _check(lib.uaii_moe_experts_swiglu(self._h, ptr(x), ptr(gate), gfmt, ptr(up), ufmt, ptr(down),
                                           dfmt, ptr(probs), T, D, E, I, top_k, norm_topk, ptr(y)))

    def ffn(self, layer: Layer, x, T: int, y, probs=None):
        _check(lib.uaii_moe_ffn_forward(self._h, ctypes.byref(layer), ptr(x), T, ptr(y), ptr(probs)))

    # ---- expert parallelism (device tensors; see include/uaii_moe.h)
    def route(self, x, gate_w, T: int, D: int, E: int, k: int, norm_topk: int, ids, w):
        """The fused layer's token -> expert assignment: ids [T, k] int32 in rank order, weights [T, k]."""
        _check(lib.uaii_moe_route(self._h, ptr(x), ptr(gate_w), T, D, E, k, norm_topk, ptr(ids), ptr(w)))

    def quant_matmul(self, x, M: int, K: int, w, fmt: int, N: int, y, relu: bool = False):
        """y[M,N] = x[M,K] . dequant(w[N rows of K, fmt])^T (the MatMul op with a packed B)."""
        _check(lib.uaii_moe_quant_matmul(self._h, ptr(x), M, K, ptr(w), fmt, N, int(relu), ptr(y)))

    def ep_dispatch(self, layer: Layer, x, T: int, rank: int, world: int, send_x16, send_ids, send_w, send_token,
                    row_of, send_counts, send_entries, probs=None):
        _check(lib.uaii_moe_ep_dispatch(self._h, ctypes.byref(layer), ptr(x), T, rank, world, ptr(send_x16),
                                        ptr(send_ids), ptr(send_w), ptr(send_token), ptr(row_of), ptr(send_counts),
                                        ptr(send_entries), ptr(probs)))

    def ep_experts(self, layer: Layer, recv_x16, recv_ids, recv_w, rows: int, entries: int, y_part):
        _check(lib.uaii_moe_ep_experts(self._h, ctypes.byref(layer), ptr(recv_x16), ptr(recv_ids), ptr(recv_w),
                                       rows, entries, ptr(y_part)))

    def selftest_wait_timeout(self, budget_cycles: int):
        """Bounded-wait failure path on the device; raises UaiiMoeError (Internal) when it works."""
        _check(lib.uaii_moe_selftest_wait_timeout(self._h, budget_cycles))

    def ep_dispatch_records(self, layer: Layer, x, T: int, rank: int, world: int, send_rec, rec_bytes: int,
                            send_token, row_of, send_counts, send_entries, probs=None):
        """ep_dispatch with each row one record: f16 x, top_k int32 ids, top_k f32 weights."""
        _check(lib.uaii_moe_ep_dispatch_records(self._h, ctypes.byref(layer), ptr(x), T, rank, world, ptr(send_rec),
                                                rec_bytes, ptr(send_token), ptr(row_of), ptr(send_counts),
                                                ptr(send_entries), ptr(probs)))

    def ep_experts_records(self, layer: Layer, recv_rec, rec_bytes: int, rows: int, entries: int, y_part):
        _check(lib.uaii_moe_ep_experts_records(self._h, ctypes.byref(layer), ptr(recv_rec), rec_bytes, rows, entries,
                                               ptr(y_part)))

    def ep_experts_records_f16(self, layer: Layer, recv_rec, rec_bytes: int, rows: int, entries: int, y_part):
        """As ep_experts_records with y_part f16 [rows, d_model] (each row's sum rounded once)."""
        _check(lib.uaii_moe_ep_experts_records_f16(self._h, ctypes.byref(layer), ptr(recv_rec), rec_bytes, rows,
                                                   entries, ptr(y_part)))

    def ep_combine_f16(self, y_back, row_of, T: int, world: int, d_model: int, y):
        """As ep_combine with f16 returned rows (added in f32, rank order)."""
        _check(lib.uaii_moe_ep_combine_f16(self._h, ptr(y_back), ptr(row_of), T, world, d_model, ptr(y)))

    def ep_combine(self, y_back, row_of, T: int, world: int, d_model: int, y):
        _check(lib.uaii_moe_ep_combine(self._h, ptr(y_back), ptr(row_of), T, world, d_model, ptr(y)))

    def dispatch(self, op_name: str, inputs, outputs, attrs: dict | None = None, op_version="1"):
        """inputs/outputs: lists of tensor_desc(...) tuples; attrs: {key: int|float|bool}."""
        keep = []
        def mk(descs):
            arr = (Tensor * max(1, len(descs)))()
            for i, (dtype, qfmt, shape, data, nbytes) in enumerate(descs):
                shp = (c_int64 * len(shape))(*shape)
                keep.append(shp)
                arr[i] = Tensor(dtype, qfmt, ctypes.cast(shp, POINTER(c_int64)), len(shape), ptr(data), nbytes)
            return arr
        ins, outs = mk(inputs), mk(outputs)
        attrs = attrs or {}
        at = (Attr * max(1, len(attrs)))()
        for i, (k, v) in enumerate(attrs.items()):
            if isinstance(v, bool):
                at[i] = Attr(k.encode(), ATTR_BOOL, int(v), 0.0)
            elif isinstance(v, int):
                at[i] = Attr(k.encode(), ATTR_INT, v, 0.0)
            else:
                at[i] = Attr(k.encode(), ATTR_FLOAT, 0, float(v))
        _check(lib.uaii_moe_dispatch(self._h, op_name.encode(), op_version.encode(), ins, len(inputs),
                                     outs, len(outputs), at, len(attrs)))


def ffn_forward_noalloc(device: int, stream, layer: Layer, x, T: int, y, probs=None):
    """uaii_moe_ffn_forward_noalloc: the layer forward without any device allocation
    (fixed scratch inside the library; all arrays must be on the device)."""
    _check(lib.uaii_moe_ffn_forward_noalloc(device, stream, ctypes.byref(layer), ptr(x), T, ptr(y), ptr(probs)))


def f32_desc(a, shape=None):
    shape = tuple(shape if shape is not None else a.shape)
    n = int(np.prod(shape)) if shape else 0
    return (DTYPE_F32, F32, shape, a, 4 * n)


def packed_desc(a, fmt: int, shape):
    """Packed GGUF expert tensor [E, rows, cols] (dtype Unknown, quant_format = fmt)."""
    rows = int(np.prod(shape[:-1]))
    return (DTYPE_UNKNOWN, fmt, tuple(shape), a, rows * packed_nbytes(fmt, shape[-1]))


GGUF_SHEXP_GATE = 1


class GgufFile:
    """A GGUF file mapped read-only (uaii_moe_gguf_*).  Tensor data are numpy uint8
    views into the mapping; layers and views stay valid while this object is open."""

    def __init__(self, path: str):
        h = c_void_p()
        _check(lib.uaii_moe_gguf_open(os.fsencode(path), ctypes.byref(h)))
        self._h = h

    def close(self):
        if self._h:
            lib.uaii_moe_gguf_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    def _info(self, getter, *args):
        data, fmt, rank, nb = c_void_p(), c_int(), c_int(), c_uint64()
        shape = (c_int64 * 8)()
        _check(getter(self._h, *args, ctypes.byref(data), ctypes.byref(fmt), shape, ctypes.byref(rank),
                      ctypes.byref(nb)))
        return data.value, fmt.value, tuple(shape[i] for i in range(rank.value)), nb.value

    def tensors(self):
        """[(name, fmt, shape, nbytes)] in file order (fmt -1: type without a format)."""
        out = []
        for i in range(int(lib.uaii_moe_gguf_tensor_count(self._h))):
            name = c_char_p()
            data, fmt, shape, nb = self._info(lambda h, i_, *r: lib.uaii_moe_gguf_tensor_at(h, i_, ctypes.byref(name),
                                                                                          *r), i)
            out.append((name.value.decode(), fmt, shape, nb))
        return out

    def tensor(self, name: str):
        """(numpy uint8 view of the packed bytes, fmt, shape)."""
        data, fmt, shape, nb = self._info(lib.uaii_moe_gguf_tensor, name.encode())
        if not data:
            raise UaiiMoeError(NOT_IMPLEMENTED, f"{name}: tensor type without a format")
        arr = np.ctypeslib.as_array((ctypes.c_uint8 * nb).from_address(data))
        return arr, fmt, shape

    def kv_int(self, key: str) -> int:
        v = c_int64()
        _check(lib.uaii_moe_gguf_kv_int(self._h, key.encode(), ctypes.byref(v)))
        return v.value

    def kv_float(self, key: str) -> float:
        v = c_double()
        _check(lib.uaii_moe_gguf_kv_float(self._h, key.encode(), ctypes.byref(v)))
        return v.value

    def kv_str(self, key: str) -> str:
        v = c_char_p()
        _check(lib.uaii_moe_gguf_kv_string(self._h, key.encode(), ctypes.byref(v)))
        return v.value.decode()

    def moe_layer(self, block: int, shexp_gate: bool = False) -> "Layer":
        L = Layer()
        _check(lib.uaii_moe_gguf_moe_layer(self._h, block, GGUF_SHEXP_GATE if shexp_gate else 0, ctypes.byref(L)))
        L._keep = self  # the layer points into this mapping
        return L


class DecoderConfig(ctypes.Structure):
    _fields_ = [("n_layers", c_int64), ("d_model", c_int64), ("n_heads", c_int64), ("n_kv_heads", c_int64),
                ("head_dim", c_int64), ("vocab", c_int64), ("batch", c_int64), ("max_seq", c_int64),
                ("rope_theta", c_float), ("rms_eps", c_float), ("rope_mode", c_int32)]


class DecoderBlock(ctypes.Structure):
    _fields_ = [("attn_norm", c_void_p), ("wq", c_void_p), ("wq_fmt", c_int32), ("wk", c_void_p),
                ("wk_fmt", c_int32), ("wv", c_void_p), ("wv_fmt", c_int32), ("wo", c_void_p), ("wo_fmt", c_int32),
                ("ffn_norm", c_void_p), ("moe", Layer)]


class Decoder:
    """Batched greedy decode of a GGUF MoE transformer on the device (uaii_moe_decoder_*).

    blocks: list of dicts with attn_norm, wq, wk, wv, wo (+ *_fmt), ffn_norm and moe (a Layer);
    every array is device memory (torch CUDA tensors), kept alive by this object."""

    def __init__(self, backend: "Backend", n_layers, d_model, n_heads, n_kv_heads, vocab, batch, max_seq, blocks,
                 output_norm, token_embd, embd_fmt, output=None, output_fmt=0, head_dim=128, rope_theta=1e6,
                 rms_eps=1e-5, rope_mode=0):
        self._keep = [blocks, output_norm, token_embd, output]
        cfg = DecoderConfig(n_layers, d_model, n_heads, n_kv_heads, head_dim, vocab, batch, max_seq, rope_theta,
                            rms_eps, rope_mode)
        arr = (DecoderBlock * n_layers)()
        for i, b in enumerate(blocks):
            arr[i] = DecoderBlock(ptr(b["attn_norm"]), ptr(b["wq"]), b["wq_fmt"], ptr(b["wk"]), b["wk_fmt"],
                                  ptr(b["wv"]), b["wv_fmt"], ptr(b["wo"]), b["wo_fmt"], ptr(b["ffn_norm"]), b["moe"])
        self._cfg, self._arr = cfg, arr
        h = c_void_p()
        _check(lib.uaii_moe_decoder_create(backend.handle, ctypes.byref(cfg), arr, ptr(output_norm), ptr(token_embd),
                                           embd_fmt, ptr(output), output_fmt, ctypes.byref(h)))
        self._h = h
        self.batch, self.vocab = batch, vocab

    def close(self):
        if self._h:
            lib.uaii_moe_decoder_destroy(self._h)
            self._h = c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def position(self) -> int:
        return int(lib.uaii_moe_decoder_position(self._h))

    def set_kv(self, layer: int, k, v, n_pos: int):
        """K, V [batch, n_kv_heads, n_pos, head_dim] f32 (host or device) for positions [0, n_pos)."""
        _check(lib.uaii_moe_decoder_set_kv(self._h, layer, ptr(k), ptr(v), n_pos))

    def fill_kv(self, n_pos: int, seed: int = 0):
        _check(lib.uaii_moe_decoder_fill_kv(self._h, n_pos, seed))

    def step(self, tokens, logits=None, next_tokens=None):
        _check(lib.uaii_moe_decoder_step(self._h, ptr(tokens), ptr(logits), ptr(next_tokens)))

    def generate(self, tokens, steps: int, out):
        _check(lib.uaii_moe_decoder_generate(self._h, ptr(tokens), steps, ptr(out)))


def fill_normal_device(backend: "Backend", out, seed: int, stream: int, mean: float = 0.0, std: float = 1.0):
    """uaii_moe_fill_normal's draws written on the device (out: a CUDA f32 tensor)."""
    _check(lib.uaii_moe_fill_normal_device(backend.handle, ptr(out), out.numel(), seed, stream, mean, std))


def quantize_rows_device(backend: "Backend", fmt: int, src, dst):
    """GGUF blocks of the f32 rows src [rows, cols] into dst (CUDA tensors), as quantize_rows does."""
    rows, cols = src.shape
    _check(lib.uaii_moe_quantize_rows_device(backend.handle, fmt, ptr(src), rows, cols, ptr(dst)))


def make_layer(D, E, I, top_k, norm_topk, router_w, gate, gfmt, up, ufmt, down, dfmt,
               shared=None) -> Layer:
    """shared: None or (I_sh, gate_sh, gfmt, up_sh, ufmt, down_sh, dfmt, gate_inp_or_None)."""
    L = Layer()
    L.d_model, L.n_experts, L.d_ff, L.top_k, L.norm_topk = D, E, I, top_k, norm_topk
    L.router_w, L.gate_exps, L.gate_fmt = ptr(router_w), ptr(gate), gfmt
    L.up_exps, L.up_fmt, L.down_exps, L.down_fmt = ptr(up), ufmt, ptr(down), dfmt
    if shared is not None:
        I_sh, g, gf, u, uf, d, df, gi = shared
        L.shared_d_ff = I_sh
        L.gate_shexp, L.gate_shexp_fmt = ptr(g), gf
        L.up_shexp, L.up_shexp_fmt = ptr(u), uf
        L.down_shexp, L.down_shexp_fmt = ptr(d), df
        L.gate_inp_shexp = ptr(gi)
    return L
