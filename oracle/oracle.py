"""ctypes access to the CPU checkers -- TEST INFRASTRUCTURE ONLY.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs,
never by the product library.  Two checkers:

* ``Oracle``: oracle/libmoe_oracle.so, the C restatement (moe_oracle.c) of
  the reference path, pinned against the reference build and tests/golden/.
* ``Reference``: oracle/_ref/libuaii_ref.so, the reference's own sources
  compiled by oracle/Makefile; present when it was built (it is built where
  the reference tree exists and travels with the repository as a binary).
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_char_p, c_float, c_int, c_int64, c_size_t, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "libmoe_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libuaii_ref.so")


def _p(a):
    if a is None:
        return None
    assert isinstance(a, np.ndarray) and a.flags["C_CONTIGUOUS"], "numpy C-contiguous arrays only"
    return a.ctypes.data


class Oracle:
    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C {HERE} oracle`")
        L = ctypes.CDLL(path)
        sig = {
            "uo_f16_to_f32": (c_float, [ctypes.c_uint16]),
            "uo_packed_nbytes": (c_size_t, [c_int, c_int64]),
            "uo_dequant_row": (c_int, [c_int, c_void_p, c_int64, c_void_p]),
            "uo_dequant_rows": (c_int, [c_int, c_void_p, c_int64, c_int64, c_int64, c_void_p]),
            "uo_router_logits": (None, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p]),
            "uo_softmax_rows": (None, [c_void_p, c_int64, c_int64, c_void_p]),
            "uo_moe_router": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p]),
            "uo_topk_row": (None, [c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p]),
            "uo_moe_experts_swiglu": (c_int, [c_void_p] * 5 + [c_int64] * 4 + [c_int, c_int, c_void_p, c_void_p, c_void_p]),
            "uo_moe_experts_swiglu_packed": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int,
                                                     c_void_p] + [c_int64] * 4 + [c_int, c_int, c_void_p, c_void_p,
                                                                                  c_void_p]),
            "uo_shared_expert_packed": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int,
                                                c_void_p, c_int64, c_int64, c_int64, c_void_p]),
            "uo_quant_gemm": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_int, c_int64, c_int, c_void_p]),
            "uo_moe_experts_linear": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p]),
        }
        for n, (r, a) in sig.items():
            f = getattr(L, n)
            f.restype, f.argtypes = r, a
        self.L = L

    def packed_nbytes(self, fmt, n):
        return int(self.L.uo_packed_nbytes(fmt, n))

    def dequant(self, fmt, packed: np.ndarray, rows: int, cols: int) -> np.ndarray:
        out = np.empty((rows, cols), np.float32)
        st = self.L.uo_dequant_rows(fmt, _p(packed), rows, cols, 0, _p(out))
        if st != 0:
            raise ValueError(f"oracle dequant status {st}")
        return out

    def router(self, x, w):
        T, D = x.shape
        E = w.shape[0]
        lg = np.empty((T, E), np.float32)
        pr = np.empty((T, E), np.float32)
        top = np.empty((T, 1), np.float32)
        assert self.L.uo_moe_router(_p(x), _p(w), T, D, E, _p(lg), _p(pr), _p(top)) == 0
        return lg, pr, top

    def topk(self, probs_row: np.ndarray, k: int, norm: int = 1):
        ids = np.empty(k, np.int32)
        w = np.empty(k, np.float32)
        self.L.uo_topk_row(_p(probs_row), probs_row.shape[0], k, norm, _p(ids), _p(w))
        return ids, w

    def experts_f32(self, x, G, U, Dn, probs, top_k, norm=1):
        T, D = x.shape
        E, I, _ = G.shape
        y = np.empty((T, D), np.float32)
        ids = np.empty((T, max(1, min(top_k, E))), np.int32)
        w = np.empty_like(ids, dtype=np.float32)
        assert self.L.uo_moe_experts_swiglu(_p(x), _p(G), _p(U), _p(Dn), _p(probs), T, D, E, I, top_k, norm,
                                            _p(y), _p(ids), _p(w)) == 0
        return y, ids, w

    def experts_linear(self, x, W, top):
        """MoEExperts: y[b] = x[b] . W[top[b]]^T (top-1 linear experts, W [E, D, D])."""
        B, D = x.shape
        y = np.empty((B, D), np.float32)
        assert self.L.uo_moe_experts_linear(_p(x), _p(W), _p(top), B, D, W.shape[0], _p(y)) == 0
        return y

    def experts_packed(self, x, G, gf, U, uf, Dn, df, probs, E, I, top_k, norm=1):
        T, D = x.shape
        k = max(1, min(top_k, E))
        y = np.empty((T, D), np.float32)
        ids = np.empty((T, k), np.int32)
        w = np.empty((T, k), np.float32)
        assert self.L.uo_moe_experts_swiglu_packed(_p(x), _p(G), gf, _p(U), uf, _p(Dn), df, _p(probs), T, D, E,
                                                   I, top_k, norm, _p(y), _p(ids), _p(w)) == 0
        return y, ids, w

    def quant_gemm(self, a, b_packed, fmt, N, relu=False):
        """c[M,N] = a[M,K] . dequant(b_packed[N rows])^T (kernels::quant_gemm_f32), max(., 0) with relu."""
        M, K = a.shape
        c = np.empty((M, N), np.float32)
        assert self.L.uo_quant_gemm(_p(a), M, K, _p(b_packed), fmt, N, int(relu), _p(c)) == 0
        return c

    def shared_packed(self, x, G, gf, U, uf, Dn, df, wsg, Ish, y):
        T, D = x.shape
        assert self.L.uo_shared_expert_packed(_p(x), _p(G), gf, _p(U), uf, _p(Dn), df, _p(wsg), T, D, Ish,
                                              _p(y)) == 0
        return y


class Reference:
    """The reference's own compiled functions (oracle/_ref/libuaii_ref.so)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C {HERE} ref` where the reference tree exists")
        L = ctypes.CDLL(path)
        sig = {
            "uref_last_error": (c_char_p, []),
            "uref_dequant_row": (c_int, [c_int, c_void_p, c_int64, c_void_p]),
            "uref_moe_router": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p]),
            "uref_matmul_bt": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p]),
            "uref_moe_experts_swiglu": (c_int, [c_void_p] * 5 + [c_int64] * 4 + [c_int, c_void_p]),
            "uref_moe_experts_swiglu_mt": (c_int, [c_void_p] * 5 + [c_int64] * 4 + [c_int, c_void_p, c_int]),
            "uref_quant_gemm": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_int, c_int64, c_void_p]),
            "uref_gguf_tensor_raw": (c_int64, [c_char_p, c_char_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p]),
            "uref_gguf_tensor_f32": (c_int64, [c_char_p, c_char_p, c_void_p, c_int64]),
            "uref_rmsnorm": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_float, c_void_p]),
            "uref_rope": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_float, c_int64, c_int, c_void_p]),
            "uref_attention_kv": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int, c_void_p,
                                          c_void_p, c_int64, c_void_p]),
            "uref_embedding": (c_int, [c_void_p, c_int64, c_void_p, c_int, c_int64, c_int64, c_void_p]),
            "uref_softmax": (c_int, [c_void_p, c_int64, c_int64, c_void_p]),
            "uref_moe_experts": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p]),
            "uref_gguf_write_f32": (c_int, [c_char_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
        }
        for n, (r, a) in sig.items():
            f = getattr(L, n)
            f.restype, f.argtypes = r, a
        self.L = L

    def _chk(self, st):
        if st != 0:
            raise ValueError(f"reference status {st}: {self.L.uref_last_error().decode()}")

    def quant_gemm(self, a, b_packed, fmt, N):
        M, K = a.shape
        c = np.empty((M, N), np.float32)
        self._chk(self.L.uref_quant_gemm(_p(a), M, K, _p(b_packed), fmt, N, _p(c)))
        return c

    def gguf_tensor_raw(self, path: str, name: str, cap: int):
        """(bytes, shape outermost first, ggml type) of one tensor through the reference loader."""
        out = np.empty(cap, np.uint8)
        shape = np.zeros(8, np.int64)
        rank, typ = ctypes.c_int(), ctypes.c_int()
        n = self.L.uref_gguf_tensor_raw(os.fsencode(path), name.encode(), _p(out), cap, _p(shape),
                                        ctypes.addressof(rank), ctypes.addressof(typ))
        if n < 0:
            raise ValueError(f"reference gguf status {-n}: {self.L.uref_last_error().decode()}")
        return out[:n].copy(), tuple(int(d) for d in shape[:rank.value]), typ.value

    def gguf_tensor_f32(self, path: str, name: str, n: int) -> np.ndarray:
        """One tensor dequantized at load time by the reference loader (gguf_load_tensor_f32),
        as the reference Session does with its default options."""
        out = np.empty(n, np.float32)
        got = self.L.uref_gguf_tensor_f32(os.fsencode(path), name.encode(), _p(out), n)
        if got < 0:
            raise ValueError(f"reference gguf status {-got}: {self.L.uref_last_error().decode()}")
        return out[:got].copy()

    # ---- decode-step kernels (rows are independent sequences)
    def rmsnorm(self, x, w, eps):
        y = np.empty_like(x)
        self._chk(self.L.uref_rmsnorm(_p(x), _p(w), x.shape[0], x.shape[1], eps, _p(y)))
        return y

    def rope(self, x, positions, theta, head_dim, mode):
        y = np.empty_like(x)
        pos = np.ascontiguousarray(positions, np.float32)
        self._chk(self.L.uref_rope(_p(x), _p(pos), x.shape[0], x.shape[1], theta, head_dim, mode, _p(y)))
        return y

    def attention_kv(self, q, k, v, num_heads, past_k, past_v):
        """q [B, q_dim], k/v [B, kv_dim], past_k/v [B, past, kv_dim] (past may be 0)."""
        B, q_dim = q.shape
        out = np.empty_like(q)
        past = past_k.shape[1]
        self._chk(self.L.uref_attention_kv(_p(q), _p(k), _p(v), B, q_dim, k.shape[1], num_heads,
                                           _p(past_k) if past else None, _p(past_v) if past else None, past,
                                           _p(out)))
        return out

    def embedding(self, tokens, table, fmt, vocab, D):
        t = np.ascontiguousarray(tokens, np.float32)
        out = np.empty((t.shape[0], D), np.float32)
        self._chk(self.L.uref_embedding(_p(t), t.shape[0], _p(table), fmt, vocab, D, _p(out)))
        return out

    def softmax(self, x):
        y = np.empty_like(x)
        self._chk(self.L.uref_softmax(_p(x), x.shape[0], x.shape[1], _p(y)))
        return y

    def gguf_write_f32(self, path: str, tensors):
        """tensors: [(name, f32 array)] written by the reference's gguf_write_f32 (dims reversed as GGUF)."""
        n = len(tensors)
        names = (ctypes.c_char_p * n)(*[t[0].encode() for t in tensors])
        ranks = (ctypes.c_int * n)(*[t[1].ndim for t in tensors])
        dims = np.array([d for _, a in tensors for d in reversed(a.shape)], np.uint64)
        arrs = [np.ascontiguousarray(a, np.float32) for _, a in tensors]
        data = (ctypes.c_void_p * n)(*[a.ctypes.data for a in arrs])
        self._chk(self.L.uref_gguf_write_f32(os.fsencode(path), n, names, ranks, _p(dims), data))

    def dequant(self, fmt, packed: np.ndarray, rows: int, cols: int, pitch: int) -> np.ndarray:
        out = np.empty((rows, cols), np.float32)
        base = packed.ctypes.data
        for r in range(rows):
            self._chk(self.L.uref_dequant_row(fmt, base + r * pitch, cols, out.ctypes.data + r * cols * 4))
        return out

    def experts_linear(self, x, W, top):
        B, D = x.shape
        y = np.empty((B, D), np.float32)
        self._chk(self.L.uref_moe_experts(_p(x), _p(W), _p(top), B, D, W.shape[0], _p(y)))
        return y

    def router(self, x, w):
        T, D = x.shape
        E = w.shape[0]
        pr = np.empty((T, E), np.float32)
        top = np.empty((T, 1), np.float32)
        self._chk(self.L.uref_moe_router(_p(x), _p(w), T, D, E, _p(pr), _p(top)))
        return pr, top

    def logits(self, x, w):
        T, D = x.shape
        E = w.shape[0]
        c = np.empty((T, E), np.float32)
        self._chk(self.L.uref_matmul_bt(_p(x), _p(w), T, D, E, _p(c)))
        return c

    def experts(self, x, G, U, Dn, probs, top_k, threads: int = 1):
        T, D = x.shape
        E, I, _ = G.shape
        y = np.empty((T, D), np.float32)
        self._chk(self.L.uref_moe_experts_swiglu_mt(_p(x), _p(G), _p(U), _p(Dn), _p(probs), T, D, E, I, top_k,
                                                    _p(y), threads))
        return y


def reference_available() -> bool:
    return os.path.exists(REF_SO)
