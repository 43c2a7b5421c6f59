"""Seeded synthetic MoE layers in plain numpy -- TEST INFRASTRUCTURE ONLY.

bench.py's reference arm (``--impl reference``) times the reference's own CPU
code; it must not load the product library, not even to make its inputs.  This
module restates, in numpy, the two input utilities the product exports for
that purpose, so the reference process builds the same seeded layer without it:

* ``fill_normal``: the counter-based normal generator of
  ``uaii_moe_fill_normal`` (splitmix64 finaliser keyed by (seed, stream), two
  64-bit draws per pair of outputs, Box-Muller in double precision, rounded to
  f32 once);
* ``quantize_rows``: the round-to-nearest GGUF block quantizer of
  ``uaii_moe_quantize_rows`` for Q4_0, Q8_0, Q4_K and Q6_K (f32 arithmetic in
  the same order; f16 scales rounded to nearest even).

The block byte layouts are GGUF's (the reference's dequantizer,
libs/uaii-quant/src/gguf_dequant.cpp:117-134, :203-217, :308-340, :381-416,
reads them back).  tests/test_oracle.py checks both functions against the
library bit for bit.  The transcendental functions come from numpy rather than
the C library; a last-bit difference in a double there almost never survives
the rounding to f32, and the test bounds how often it does.

``CONFIGS`` restates the benchmark layers (shapes,
formats, routing skew, seeds) so the reference arm needs nothing from the
product package; the same test checks it against ``uaii_moe.synthetic``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

F32, Q4_0, Q8_0, Q4_K, Q6_K = 0, 7, 11, 14, 16
_BLOCK = {Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}

def _mix64(z: np.ndarray) -> np.ndarray:
    """splitmix64 finaliser (wrapping uint64 arithmetic)."""
    with np.errstate(over="ignore"):
        z = z + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def _mix64_scalar(z: int) -> int:
    return int(_mix64(np.array([z & 0xFFFFFFFFFFFFFFFF], np.uint64))[0])


def fill_normal(shape, seed: int, stream: int, mean: float = 0.0, std: float = 1.0,
                chunk: int = 1 << 22) -> np.ndarray:
    """out[i] = mean + std * N(0,1), counter-based: identical to uaii_moe_fill_normal."""
    n = int(np.prod(shape)) if shape != () else 1
    inner = _mix64_scalar((stream * 0xD1B54A32D192ED03 + 0x7F4A7C15) & 0xFFFFFFFFFFFFFFFF)
    key = np.uint64(_mix64_scalar(seed ^ inner))
    out = np.empty(n, np.float32)
    two_pi = 6.283185307179586476925286766559
    m, sd = float(np.float32(mean)), float(np.float32(std))  # the C entry point takes f32 mean and std
    for i0 in range(0, n, chunk):
        i1 = min(n, i0 + chunk)
        p0, p1 = i0 >> 1, (i1 + 1) >> 1
        p = np.arange(p0, p1, dtype=np.uint64)
        with np.errstate(over="ignore"):
            a = _mix64(key + np.uint64(2) * p)
            b = _mix64(key + np.uint64(2) * p + np.uint64(1))
        u1 = ((a >> np.uint64(11)).astype(np.float64) + 1.0) * (1.0 / 9007199254740992.0)
        u2 = (b >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
        r = np.sqrt(-2.0 * np.log(u1))
        ang = two_pi * u2
        z = np.empty(2 * (p1 - p0), np.float64)
        z[0::2] = r * np.cos(ang)
        z[1::2] = r * np.sin(ang)
        z = z[i0 - 2 * p0: i1 - 2 * p0]
        out[i0:i1] = (m + sd * z).astype(np.float32)
    return out.reshape(shape)


def _f16_bits(v: np.ndarray) -> np.ndarray:
    return v.astype(np.float16).view(np.uint16)


def _f16_val(bits: np.ndarray) -> np.ndarray:
    return bits.view(np.float16).astype(np.float32)


def _signed_absmax(x: np.ndarray) -> np.ndarray:
    """Per last-axis group: the value of largest magnitude (first on ties), with its sign."""
    idx = np.argmax(np.abs(x), axis=-1)
    return np.take_along_axis(x, idx[..., None], axis=-1)[..., 0]


def _put16(b: np.ndarray, col: int, bits: np.ndarray):
    b[:, col] = (bits & 0xFF).astype(np.uint8)
    b[:, col + 1] = (bits >> 8).astype(np.uint8)


def _q4_0(x: np.ndarray) -> np.ndarray:  # x [nb, 32] -> [nb, 18]
    f = np.float32
    mx = _signed_absmax(x)
    dh = _f16_bits(mx / f(-8.0))
    d = _f16_val(dh)
    with np.errstate(divide="ignore"):
        idv = np.where(d != 0, f(1.0) / d, f(0.0)).astype(np.float32)
    q = np.clip(np.rint(x * idv[:, None]).astype(np.int32) + 8, 0, 15).astype(np.uint8)
    b = np.empty((x.shape[0], 18), np.uint8)
    _put16(b, 0, dh)
    b[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    return b


def _q8_0(x: np.ndarray) -> np.ndarray:  # [nb, 32] -> [nb, 34]
    f = np.float32
    amax = np.abs(_signed_absmax(x))
    dh = _f16_bits(amax / f(127.0))
    d = _f16_val(dh)
    with np.errstate(divide="ignore"):
        idv = np.where(d != 0, f(1.0) / d, f(0.0)).astype(np.float32)
    q = np.clip(np.rint(x * idv[:, None]).astype(np.int32), -127, 127).astype(np.int8)
    b = np.empty((x.shape[0], 34), np.uint8)
    _put16(b, 0, dh)
    b[:, 2:] = q.view(np.uint8)
    return b


def _q4_k(x: np.ndarray) -> np.ndarray:  # [nb, 256] -> [nb, 144]
    f = np.float32
    g = x.reshape(-1, 8, 32)
    lo = np.minimum(g.min(axis=2), f(0.0))
    hi = np.maximum(g.max(axis=2), lo)
    scale = (hi - lo) / f(15.0)
    negmin = -lo
    smax = scale.max(axis=1)
    mmax = negmin.max(axis=1)
    dh, mh = _f16_bits(smax / f(63.0)), _f16_bits(mmax / f(63.0))
    d, dm = _f16_val(dh), _f16_val(mh)
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d[:, None] > 0, np.clip(np.rint(scale / d[:, None]), 0, 63), 0).astype(np.int32)
        mn = np.where(dm[:, None] > 0, np.clip(np.rint(negmin / dm[:, None]), 0, 63), 0).astype(np.int32)
    b = np.empty((x.shape[0], 144), np.uint8)
    _put16(b, 0, dh)
    _put16(b, 2, mh)
    b[:, 4:8] = ((sc[:, :4] & 63) | ((sc[:, 4:] >> 4) << 6)).astype(np.uint8)
    b[:, 8:12] = ((mn[:, :4] & 63) | ((mn[:, 4:] >> 4) << 6)).astype(np.uint8)
    b[:, 12:16] = ((sc[:, 4:] & 15) | ((mn[:, 4:] & 15) << 4)).astype(np.uint8)
    ed = (d[:, None] * sc.astype(np.float32)).astype(np.float32)
    em = (dm[:, None] * mn.astype(np.float32)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        qv = np.rint((g + em[:, :, None]) / ed[:, :, None])
        q = np.where(ed[:, :, None] > 0, np.clip(qv, 0, 15), 0).astype(np.uint8).reshape(-1, 4, 2, 32)
    b[:, 16:] = (q[:, :, 0, :] | (q[:, :, 1, :] << 4)).reshape(-1, 128)
    return b


def _q6_k(x: np.ndarray) -> np.ndarray:  # [nb, 256] -> [nb, 210]
    f = np.float32
    g = x.reshape(-1, 16, 16)
    scale = _signed_absmax(g) / f(-32.0)
    smax = np.abs(scale).max(axis=1)
    dh = _f16_bits(smax / f(127.0))
    d = _f16_val(dh)
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d[:, None] > 0, np.clip(np.rint(scale / d[:, None]), -128, 127), 0).astype(np.int32)
        e = (d[:, None] * sc.astype(np.float32)).astype(np.float32)
        qv = np.rint(g / e[:, :, None])
        q = np.where(e[:, :, None] != 0, np.clip(qv + 32, 0, 63), 32).astype(np.uint8).reshape(-1, 2, 4, 32)
    b = np.empty((x.shape[0], 210), np.uint8)
    q1, q2, q3, q4 = q[:, :, 0], q[:, :, 1], q[:, :, 2], q[:, :, 3]  # [nb, half, 32]
    ql = np.empty((x.shape[0], 2, 64), np.uint8)
    ql[:, :, :32] = (q1 & 15) | ((q3 & 15) << 4)
    ql[:, :, 32:] = (q2 & 15) | ((q4 & 15) << 4)
    b[:, :128] = ql.reshape(-1, 128)
    b[:, 128:192] = ((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6)).reshape(-1, 64)
    b[:, 192:208] = sc.astype(np.int8).view(np.uint8)
    _put16(b, 208, dh)
    return b


_QUANT = {Q4_0: _q4_0, Q8_0: _q8_0, Q4_K: _q4_k, Q6_K: _q6_k}


def packed_nbytes(fmt: int, n: int) -> int:
    if fmt == F32:
        return 4 * n
    qk, bb = _BLOCK[fmt]
    return n // qk * bb


def quantize_rows(fmt: int, src: np.ndarray, chunk_rows: int = 4096) -> np.ndarray:
    """f32 [rows, cols] -> GGUF blocks [rows, packed_nbytes(cols)], as uaii_moe_quantize_rows."""
    src = np.ascontiguousarray(src, np.float32)
    rows, cols = src.shape
    qk, bb = _BLOCK[fmt]
    if cols % qk:
        raise ValueError("cols must be a multiple of the block size")
    out = np.empty((rows, cols // qk * bb), np.uint8)
    for r0 in range(0, rows, chunk_rows):
        r1 = min(rows, r0 + chunk_rows)
        blocks = src[r0:r1].reshape(-1, qk)
        out[r0:r1] = _QUANT[fmt](blocks).reshape(r1 - r0, -1)
    return out


def _quantized_part(args):
    fmt, rows, cols, seed, stream = args
    w = fill_normal((rows, cols), seed, stream, 0.0, 0.02)
    return w if fmt == F32 else quantize_rows(fmt, w)


def quantized_parts(fmt: int, rows: int, cols: int, parts: int, seed: int, stream0: int, pool=None) -> np.ndarray:
    """`parts` matrices [rows, cols], each generated and quantized on its own (streams stream0 + p)."""
    jobs = [(fmt, rows, cols, seed, stream0 + p) for p in range(parts)]
    res = list(pool.map(_quantized_part, jobs)) if pool is not None else [_quantized_part(j) for j in jobs]
    return np.stack(res)


def router_bias(routing: str, E: int, seed: int):
    """Router bias lane of the skewed configurations (the same draws as the product's generator)."""
    if routing == "natural":
        return None
    rng = np.random.default_rng(seed + 12345)
    if routing == "zipf1.1":
        ranks = rng.permutation(E) + 1
        p = ranks.astype(np.float64) ** -1.1
        return np.log(p / p.sum()).astype(np.float32)
    if routing == "hot4":
        b = np.zeros(E, np.float32)
        b[int(rng.integers(E))] = math.log(4.0)
        return b
    raise ValueError(routing)


@dataclass(frozen=True)
class Config:
    name: str
    D: int
    E: int
    I: int
    top_k: int
    gate_fmt: int
    down_fmt: int
    norm_topk: int = 1
    I_sh: int = 0
    shared_fmt: int = Q8_0
    shared_gate: bool = False
    routing: str = "natural"
    seed: int = 0


CONFIGS = {
    "cfg1_q4_0": Config("cfg1_q4_0", 1024, 8, 2816, 2, Q4_0, Q4_0),
    "mixtral": Config("mixtral", 4096, 8, 14336, 2, Q4_K, Q6_K, seed=1),
    "qwen2moe": Config("qwen2moe", 2048, 60, 1408, 4, Q8_0, Q8_0, norm_topk=0, I_sh=5632, shared_fmt=Q8_0,
                       shared_gate=True, routing="zipf1.1", seed=2),
    "qwen3": Config("qwen3", 2048, 128, 768, 8, Q4_0, Q4_0, seed=3),
    "qwen3_hot": Config("qwen3_hot", 2048, 128, 768, 8, Q4_0, Q4_0, routing="hot4", seed=3),
}


@dataclass
class Layer:
    cfg: Config
    router_w: np.ndarray
    gate: np.ndarray
    up: np.ndarray
    down: np.ndarray
    shared: tuple | None = None  # (gate, up, down, gate_inp or None)


def make_layer(cfg: Config, workers: int = 0) -> Layer:
    """The seeded layer of `cfg`, byte-identical to uaii_moe.synthetic.make_layer_weights.
    `workers` > 1 generates the expert matrices in that many spawned processes."""
    pool = None
    if workers > 1:
        import multiprocessing as mp
        pool = mp.get_context("spawn").Pool(workers)
    try:
        s = cfg.seed
        w = fill_normal((cfg.E, cfg.D), s, 10, 0.0, 0.02)
        b = router_bias(cfg.routing, cfg.E, cfg.seed)
        if b is not None:
            w[:, 0] = b
        gate = quantized_parts(cfg.gate_fmt, cfg.I, cfg.D, cfg.E, s, 1000, pool)
        up = quantized_parts(cfg.gate_fmt, cfg.I, cfg.D, cfg.E, s, 2000, pool)
        down = quantized_parts(cfg.down_fmt, cfg.D, cfg.I, cfg.E, s, 3000, pool)
        shared = None
        if cfg.I_sh > 0:
            g = quantized_parts(cfg.shared_fmt, cfg.I_sh, cfg.D, 1, s, 4000, pool)[0]
            u = quantized_parts(cfg.shared_fmt, cfg.I_sh, cfg.D, 1, s, 4001, pool)[0]
            d = quantized_parts(cfg.shared_fmt, cfg.D, cfg.I_sh, 1, s, 4002, pool)[0]
            gi = fill_normal((cfg.D,), s, 4003, 0.0, 0.02) if cfg.shared_gate else None
            shared = (g, u, d, gi)
    finally:
        if pool is not None:
            pool.close()
            pool.join()
    return Layer(cfg, w, gate, up, down, shared)


def make_tokens(cfg: Config, T: int, stream: int = 0) -> np.ndarray:
    """Seeded N(0,1) activations; the bias lane x[:, 0] = 1 for skewed routing."""
    x = fill_normal((T, cfg.D), cfg.seed, 50 + stream)
    if cfg.routing != "natural":
        x[:, 0] = 1.0
    return x
