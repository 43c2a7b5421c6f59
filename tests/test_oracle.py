"""The CPU oracle (oracle/moe_oracle.c) pinned to the reference.

Two anchors: the committed golden vectors (tests/golden/golden.npz, produced by
the reference's own compiled functions) and, where oracle/_ref exists, the
reference build itself on fresh seeded inputs.  Bitwise equality is required
for dequantized values, router logits/probabilities/argmax and the expert
layer (the oracle repeats the reference's f32 operation order exactly).
"""
import numpy as np
import pytest

from golden.make_golden import (D_OFFSET, EXP_D, EXP_E, EXP_I, EXP_K, EXPERT_CASES, GGUF_FORMATS,
                                expert_inputs, q4_0_kat_block, sha)


def bits_equal(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    same = a.view(np.uint32) == b.view(np.uint32)
    return bool(np.all(same | (np.isnan(a) & np.isnan(b))))


@pytest.mark.parametrize("fmt", GGUF_FORMATS)
def test_dequant_matches_golden(oracle, golden, fmt):
    p = golden[f"dq_{fmt}_packed"]
    out = oracle.dequant(fmt, p, p.shape[0], 512)
    assert bits_equal(out, golden[f"dq_{fmt}_out"])


def test_golden_has_special_scales(golden, um):
    # the fixtures really contain subnormal, inf and NaN block scales
    for fmt in GGUF_FORMATS:
        p = golden[f"dq_{fmt}_packed"]
        o = D_OFFSET[fmt]
        assert int(p[0, o]) | (int(p[0, o + 1]) << 8) == 0x0001
        assert int(p[1, o]) | (int(p[1, o + 1]) << 8) == 0x7C00
        out = golden[f"dq_{fmt}_out"]
        assert np.isnan(out).any() and np.isinf(out).any()


def test_reference_q4_0_known_answer(oracle, golden):
    # the reference's quant test block: d = 0.5, low nibble (j+1)%8, high (j+4)%8
    blk = q4_0_kat_block()
    assert np.array_equal(blk, golden["kat_q4_0_packed"])
    expected = np.array([((j + 1) % 8 - 8) * 0.5 for j in range(16)] +
                        [((j + 4) % 8 - 8) * 0.5 for j in range(16)], np.float32)
    out = oracle.dequant(7, blk, 1, 32)[0]
    assert bits_equal(out, expected)
    assert bits_equal(out, golden["kat_q4_0_out"][0])


def test_router_matches_golden(oracle, golden):
    lg, pr, top = oracle.router(golden["router_x"], golden["router_w"])
    assert bits_equal(lg, golden["router_logits"])
    assert bits_equal(pr, golden["router_probs"])
    assert np.array_equal(top, golden["router_top"])


@pytest.mark.parametrize("name,gf,df", EXPERT_CASES)
def test_experts_match_golden(oracle, golden, um, name, gf, df):
    i = [c[0] for c in EXPERT_CASES].index(name)
    x, w, G, U, Dn = expert_inputs(gf, df, 20 + i)
    assert np.array_equal(sha(x, w, G, U, Dn), golden[f"exp_{name}_sha"]), \
        "synthetic inputs changed: regenerate tests/golden with make_golden.py"
    _, pr, _ = oracle.router(x, w)
    assert bits_equal(pr, golden[f"exp_{name}_probs"])
    y, _, _ = oracle.experts_packed(x, G, gf, U, gf, Dn, df, pr, EXP_E, EXP_I, EXP_K)
    assert bits_equal(y, golden[f"exp_{name}_y"])


@pytest.mark.parametrize("k", [1, 2, 3, 8])
def test_tie_order_matches_golden(oracle, golden, k):
    y, _, _ = oracle.experts_f32(golden["ties_x"], golden["ties_G"], golden["ties_U"], golden["ties_D"],
                                 golden["ties_probs"], k)
    assert bits_equal(y, golden[f"ties_y_k{k}"])


def test_reference_moe_smoke_demo(oracle, golden):
    """The reference's only MoE test (demos_phase4.cpp:186-282): probs sum to 1,
    the top id is 0 or 1, y has 4 values -- plus exact golden values."""
    lg, pr, top = oracle.router(golden["smoke_x"], golden["smoke_w"])
    assert abs(float(pr.sum()) - 1.0) <= 1e-3
    assert top[0, 0] in (0.0, 1.0)
    assert bits_equal(pr, golden["smoke_probs"]) and np.array_equal(top, golden["smoke_top"])
    y, _, _ = oracle.experts_f32(golden["smoke_x"], golden["smoke_G"], golden["smoke_U"], golden["smoke_D"], pr, 2)
    assert y.shape == (1, 4)
    assert bits_equal(y, golden["smoke_y"])


def test_topk_renorm_and_raw(oracle):
    p = np.array([0.1, 0.4, 0.2, 0.3], np.float32)
    ids, w = oracle.topk(p, 2, 1)
    assert list(ids) == [1, 3]
    assert np.allclose(w, [0.4 / 0.7, 0.3 / 0.7])
    ids, w = oracle.topk(p, 2, 0)
    assert np.array_equal(w, np.array([0.4, 0.3], np.float32))
    # all-zero mass falls back to 1 (transformer.cpp:574)
    ids, w = oracle.topk(np.zeros(4, np.float32), 2, 1)
    assert np.array_equal(w, np.zeros(2, np.float32))


# ---- against the reference build itself (skipped where oracle/_ref is absent)

@pytest.mark.parametrize("fmt", GGUF_FORMATS)
def test_dequant_vs_reference_random(oracle, reference, fmt):
    rng = np.random.default_rng(5 + fmt)
    cols = 1024
    pitch = oracle.packed_nbytes(fmt, cols)
    p = rng.integers(0, 256, size=(32, pitch), dtype=np.uint8)
    assert bits_equal(oracle.dequant(fmt, p, 32, cols), reference.dequant(fmt, p, 32, cols, pitch))


@pytest.mark.parametrize("T,D,E", [(1, 64, 2), (33, 100, 8), (64, 2048, 60), (7, 4096, 128)])
def test_router_vs_reference(oracle, reference, um, T, D, E):
    x = um.fill_normal((T, D), 3, T)
    w = um.fill_normal((E, D), 3, E + 1000, 0.0, 0.02)
    lg, pr, top = oracle.router(x, w)
    pr2, top2 = reference.router(x, w)
    assert bits_equal(lg, reference.logits(x, w))
    assert bits_equal(pr, pr2)
    assert np.array_equal(top, top2)


def test_tie_order_vs_reference_exhaustive(oracle, reference):
    """The restated std::partial_sort procedure on thousands of tie-heavy rows."""
    rng = np.random.default_rng(11)
    D, I = 32, 16
    for E in (2, 3, 5, 8, 16, 60, 128):
        G = rng.standard_normal((E, I, D)).astype(np.float32)
        U = rng.standard_normal((E, I, D)).astype(np.float32)
        Dn = rng.standard_normal((E, D, I)).astype(np.float32)
        x = rng.standard_normal((64, D)).astype(np.float32)
        vals = np.array([0.05, 0.1, 0.2, 0.3], np.float32)
        p = rng.choice(vals, size=(64, E)).astype(np.float32)
        for k in sorted({1, 2, 3, 4, 8, E}):
            if k > E:
                continue
            y, _, _ = oracle.experts_f32(x, G, U, Dn, p, k)
            assert bits_equal(y, reference.experts(x, G, U, Dn, p, k)), (E, k)


def test_packed_experts_vs_reference_q4k_q6k(oracle, reference, um):
    T, D, I, E, k = 6, 512, 256, 8, 2
    x = um.fill_normal((T, D), 9, 1)
    w = um.fill_normal((E, D), 9, 2, 0.0, 0.02)
    G = um.quantize_rows(um.Q4_K, um.fill_normal((E * I, D), 9, 3, 0.0, 0.02))
    U = um.quantize_rows(um.Q4_K, um.fill_normal((E * I, D), 9, 4, 0.0, 0.02))
    Dn = um.quantize_rows(um.Q6_K, um.fill_normal((E * D, I), 9, 5, 0.0, 0.02))
    _, pr, _ = oracle.router(x, w)
    y, _, _ = oracle.experts_packed(x, G, um.Q4_K, U, um.Q4_K, Dn, um.Q6_K, pr, E, I, k)
    Gf = oracle.dequant(um.Q4_K, G, E * I, D).reshape(E, I, D)
    Uf = oracle.dequant(um.Q4_K, U, E * I, D).reshape(E, I, D)
    Df = oracle.dequant(um.Q6_K, Dn, E * D, I).reshape(E, D, I)
    assert bits_equal(y, reference.experts(x, Gf, Uf, Df, pr, k))


def _tame_rows(um, rng, fmt, rows, cols):
    """GGUF rows: the library quantizer where it has one, else random bytes with small f16 scales."""
    if fmt in (um.Q4_0, um.Q8_0, um.Q4_K, um.Q6_K):
        return um.quantize_rows(fmt, (rng.standard_normal((rows, cols)) * 0.05).astype(np.float32))
    from golden.make_golden import D_OFFSET
    qk, bb = um.BLOCK[fmt]
    p = rng.integers(0, 256, size=(rows, cols // qk, bb), dtype=np.uint8)
    scale = np.float16(0.002).view(np.uint16)
    for o in [D_OFFSET[fmt]] + ([D_OFFSET[fmt] + 2] if fmt in (8, 10, 12, 14, 15) else []):
        p[:, :, o] = scale & 0xFF
        p[:, :, o + 1] = scale >> 8
    return p.reshape(rows, -1)


@pytest.mark.parametrize("fmt", GGUF_FORMATS)
def test_quant_gemm_vs_reference(oracle, reference, um, fmt):
    """MatMul with a packed B: the restatement equals the reference build bit for bit."""
    rng = np.random.default_rng(70 + fmt)
    M, K, N = 5, 512, 24
    a = rng.standard_normal((M, K)).astype(np.float32)
    b = _tame_rows(um, rng, fmt, N, K)
    c = oracle.quant_gemm(a, b, fmt, N)
    assert np.isfinite(c).all()
    assert bits_equal(c, reference.quant_gemm(a, b, fmt, N))
    r = oracle.quant_gemm(a, b, fmt, N, relu=True)
    assert bits_equal(r, np.where(c > 0, c, np.float32(0.0)).astype(np.float32))  # relu_f32: x > 0 ? x : 0


@pytest.mark.parametrize("B,D,E", [(6, 37, 3), (16, 64, 4), (1, 1, 1), (0, 8, 2)])
def test_experts_linear_vs_reference(oracle, reference, B, D, E):
    """MoEExperts (top-1 linear experts): bitwise, including ids the reference maps to expert 0."""
    rng = np.random.default_rng(90 + D)
    x = rng.standard_normal((B, D)).astype(np.float32)
    W = rng.standard_normal((E, D, D)).astype(np.float32)
    top = rng.integers(-2, E + 2, size=(B, 1)).astype(np.float32)
    if B >= 6:
        top[:6, 0] = [np.nan, 1e30, -0.7, E - 0.3, -1e30, E]
    assert bits_equal(oracle.experts_linear(x, W, top), reference.experts_linear(x, W, top))


# ---- the numpy input synthesizer used by bench.py's reference arm (oracle/synth.py)

@pytest.mark.parametrize("shape,seed,stream,mean,std", [
    ((3, 5001), 42, 7, 0.0, 1.0), ((1 << 20,), 1, 1000, 0.0, 0.02), ((77,), 3, 50, 0.5, 2.0)])
def test_synth_fill_normal_matches_library(um, shape, seed, stream, mean, std):
    from oracle import synth
    a = um.fill_normal(shape, seed, stream, mean, std)
    b = synth.fill_normal(shape, seed, stream, mean, std)
    # numpy's double log/sin/cos may differ from the C library's in the last bit; after rounding
    # to f32 that changes (almost) nothing: at most 1 in 1e5 values, by one f32 ulp
    diff = a.view(np.uint32).astype(np.int64) - b.view(np.uint32).astype(np.int64)
    assert np.abs(diff).max() <= 1 and np.count_nonzero(diff) <= max(1, a.size // 100000)


@pytest.mark.parametrize("fmt_name", ["Q4_0", "Q8_0", "Q4_K", "Q6_K"])
def test_synth_quantizer_matches_library(um, fmt_name):
    from oracle import synth
    fmt = getattr(um, fmt_name)
    src = um.fill_normal((300, 1024), 5, 9, 0.0, 0.02)
    src[3, :40] = 0.0                                       # all-zero blocks
    src[4, 256:512] = 1e-9                                  # f16-subnormal scales
    src[5, :] = 70000.0 * (np.arange(1024) % 3 - 1)         # f16-overflowing scales
    src[6, :] = -np.abs(src[6, :])                          # one-signed blocks
    assert np.array_equal(um.quantize_rows(fmt, src), synth.quantize_rows(fmt, src))


def test_synth_configs_and_layer_match_library(um):
    from oracle import synth
    from uaii_moe.synthetic import CONFIGS, make_layer_weights, make_tokens
    assert set(synth.CONFIGS) == set(CONFIGS)
    for name, c in synth.CONFIGS.items():
        p = CONFIGS[name]
        for f in ("D", "E", "I", "top_k", "gate_fmt", "down_fmt", "norm_topk", "I_sh", "shared_fmt",
                  "shared_gate", "routing", "seed"):
            assert getattr(c, f) == getattr(p, f), (name, f)
    # a whole (small) layer with skewed routing and a gated shared expert, byte for byte
    import dataclasses
    small = synth.Config("t", 256, 6, 256, 2, synth.Q8_0, synth.Q4_K, norm_topk=0, I_sh=512,
                         shared_fmt=synth.Q4_0, shared_gate=True, routing="zipf1.1", seed=5)
    ours = make_layer_weights(type(CONFIGS["mixtral"])(**dataclasses.asdict(small)))
    theirs = synth.make_layer(small)
    for a, b in [(ours.router_w, theirs.router_w), (ours.gate, theirs.gate), (ours.up, theirs.up),
                 (ours.down, theirs.down)] + list(zip(ours.shared, theirs.shared)):
        assert np.array_equal(a, b)
    assert np.array_equal(make_tokens(CONFIGS["qwen3_hot"], 9, 2), synth.make_tokens(synth.CONFIGS["qwen3_hot"], 9, 2))
