"""Regenerate tests/golden/golden.npz from the REFERENCE's own compiled code.

Run where the reference tree exists (oracle/Makefile builds oracle/_ref from it):

    make -C oracle && python tests/golden/make_golden.py

Every expected output here comes from oracle/_ref/libuaii_ref.so, i.e. from
the unmodified reference functions quant::dequant_gguf_row,
kernels::moe_router_f32, kernels::matmul_f32 and kernels::moe_experts_swiglu_f32.
Inputs are either stored (small) or regenerated from a seed recipe with the
library's synthetic-input utilities; for the latter the SHA-256 of the packed
bytes is stored so a test can prove it rebuilt the same inputs.
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "universal-ai-inference_b200"))

import uaii_moe as um  # noqa: E402
from oracle.oracle import Reference  # noqa: E402

# offset of the f16 scale `d` inside one block, per format (gguf_dequant.cpp:12-66)
D_OFFSET = {um.Q4_0: 0, um.Q4_1: 0, um.Q5_0: 0, um.Q5_1: 0, um.Q8_0: 0, um.Q2_K: 80, um.Q3_K: 108,
            um.Q4_K: 0, um.Q5_K: 0, um.Q6_K: 208}
GGUF_FORMATS = [um.Q4_0, um.Q4_1, um.Q5_0, um.Q5_1, um.Q8_0, um.Q2_K, um.Q3_K, um.Q4_K, um.Q5_K, um.Q6_K]

# (name, gate/up format, down format) of the expert-layer cases
EXPERT_CASES = [("q4_0", um.Q4_0, um.Q4_0), ("q8_0", um.Q8_0, um.Q8_0), ("q4k_q6k", um.Q4_K, um.Q6_K)]
EXP_T, EXP_D, EXP_I, EXP_E, EXP_K = 8, 256, 256, 4, 2


def dequant_input(fmt: int, rows: int = 3, cols: int = 512) -> np.ndarray:
    """Random block bytes with special scale values planted: f16 subnormals,
    +inf and NaN in the `d` field of some blocks."""
    qk, bb = um.BLOCK[fmt]
    pitch = um.packed_nbytes(fmt, cols)
    rng = np.random.default_rng(1000 + fmt)
    p = rng.integers(0, 256, size=(rows, pitch), dtype=np.uint8)
    o = D_OFFSET[fmt]
    specials = [(0, 0, 0x0001), (0, 1, 0x83FF), (1, 0, 0x7C00), (2, 0, 0x7E01), (2, 1, 0x0000)]
    for r, b, bits in specials:
        p[r, b * bb + o] = bits & 0xFF
        p[r, b * bb + o + 1] = bits >> 8
    return p


def expert_inputs(gfmt: int, dfmt: int, seed: int):
    """Seeded synthetic layer: x ~ N(0,1), weights ~ N(0, 0.02) quantized."""
    T, D, I, E = EXP_T, EXP_D, EXP_I, EXP_E
    x = um.fill_normal((T, D), seed, 1)
    w = um.fill_normal((E, D), seed, 2, 0.0, 0.02)
    G = um.quantize_rows(gfmt, um.fill_normal((E * I, D), seed, 3, 0.0, 0.02)).reshape(E, I, -1)
    U = um.quantize_rows(gfmt, um.fill_normal((E * I, D), seed, 4, 0.0, 0.02)).reshape(E, I, -1)
    Dn = um.quantize_rows(dfmt, um.fill_normal((E * D, I), seed, 5, 0.0, 0.02)).reshape(E, D, -1)
    return x, w, G, U, Dn


def sha(*arrs) -> np.ndarray:
    h = hashlib.sha256()
    for a in arrs:
        h.update(np.ascontiguousarray(a).tobytes())
    return np.frombuffer(h.digest(), dtype=np.uint8).copy()


def q4_0_kat_block() -> np.ndarray:
    """The one Q4_0 block of the reference's quant test
    (tests/unit/quant_dequant_test.cpp:37-47): d = 0.5 (f16 0x3800),
    low nibble (j+1)%8 and high nibble (j+4)%8 for j in 0..15."""
    b = np.zeros(18, np.uint8)
    b[0], b[1] = 0x00, 0x38
    for j in range(16):
        b[2 + j] = ((j + 1) % 8) | (((j + 4) % 8) << 4)
    return b


def main():
    R = Reference()
    out = {}
    for fmt in GGUF_FORMATS:
        p = dequant_input(fmt)
        rows, cols = p.shape[0], 512
        out[f"dq_{fmt}_packed"] = p
        out[f"dq_{fmt}_out"] = R.dequant(fmt, p, rows, cols, p.shape[1])

    kat = q4_0_kat_block()
    out["kat_q4_0_packed"] = kat
    out["kat_q4_0_out"] = R.dequant(um.Q4_0, kat, 1, 32, 18)

    # router: D not a multiple of 64 exercises the short last k tile
    x = um.fill_normal((16, 320), 7, 1)
    w = um.fill_normal((6, 320), 7, 2, 0.0, 0.02)
    probs, top = R.router(x, w)
    out.update(router_x=x, router_w=w, router_logits=R.logits(x, w), router_probs=probs, router_top=top)

    # expert layers (packed inputs regenerated from seeds; sha256 recorded)
    for i, (name, gf, df) in enumerate(EXPERT_CASES):
        x, w, G, U, Dn = expert_inputs(gf, df, 20 + i)
        pr, top = R.router(x, w)
        Gf = R.dequant(gf, G.reshape(-1, G.shape[-1]), EXP_E * EXP_I, EXP_D, G.shape[-1]).reshape(EXP_E, EXP_I, EXP_D)
        Uf = R.dequant(gf, U.reshape(-1, U.shape[-1]), EXP_E * EXP_I, EXP_D, U.shape[-1]).reshape(EXP_E, EXP_I, EXP_D)
        Df = R.dequant(df, Dn.reshape(-1, Dn.shape[-1]), EXP_E * EXP_D, EXP_I, Dn.shape[-1]).reshape(EXP_E, EXP_D, EXP_I)
        out[f"exp_{name}_sha"] = sha(x, w, G, U, Dn)
        out[f"exp_{name}_probs"] = pr
        out[f"exp_{name}_y"] = R.experts(x, Gf, Uf, Df, pr, EXP_K)

    # ties: probability rows built from a few repeated values
    rng = np.random.default_rng(77)
    T, D, I, E = 12, 32, 16, 8
    tx = rng.standard_normal((T, D)).astype(np.float32)
    tG = (0.1 * rng.standard_normal((E, I, D))).astype(np.float32)
    tU = (0.1 * rng.standard_normal((E, I, D))).astype(np.float32)
    tD = (0.1 * rng.standard_normal((E, D, I))).astype(np.float32)
    tp = rng.choice(np.array([0.05, 0.1, 0.2], np.float32), size=(T, E)).astype(np.float32)
    out.update(ties_x=tx, ties_G=tG, ties_U=tU, ties_D=tD, ties_probs=tp)
    for k in (1, 2, 3, 8):
        out[f"ties_y_k{k}"] = R.experts(tx, tG, tU, tD, tp, k)

    # the reference's own MoE smoke demo (libs/uaii-runtime/src/demos_phase4.cpp:238-275):
    # E=2, D=4, I=3, top_k=2, WeightInit::Sequence (w[i] = i * 0.01), x = (1,0,0,0)
    seq = lambda *shape: (np.arange(int(np.prod(shape)), dtype=np.float32) * np.float32(0.01)).reshape(shape)
    sx = np.array([[1, 0, 0, 0]], np.float32)
    sw, sG, sU, sD = seq(2, 4), seq(2, 3, 4), seq(2, 3, 4), seq(2, 4, 3)
    sp, st = R.router(sx, sw)
    out.update(smoke_x=sx, smoke_w=sw, smoke_G=sG, smoke_U=sU, smoke_D=sD, smoke_probs=sp, smoke_top=st,
               smoke_y=R.experts(sx, sG, sU, sD, sp, 2))

    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
