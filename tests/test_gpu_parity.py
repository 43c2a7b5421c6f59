"""Device path against the oracle and the reference's golden vectors.

Everything goes through the C ABI (libuaii_moe.so).  Bars:
  * dequantized values, router logits and the top-expert id: bitwise;
  * probabilities: within 4 ulp-scale relative error (the reference's expf
    is not correctly rounded: about 0.06 % of inputs differ by one ulp from
    the double-precision exponential the device rounds);
  * layer outputs: max|y - y_ref| / max|y_ref| <= 2e-3 (REL_TOL).
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from golden.make_golden import (EXP_D, EXP_E, EXP_I, EXP_K, EXPERT_CASES, GGUF_FORMATS,  # noqa: E402
                                expert_inputs)

REL_TOL = 2e-3


def rel_err(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


def bits_equal(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    return bool(np.all((a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))))


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


# ---------------------------------------------------------------- dequant

@pytest.mark.parametrize("fmt", GGUF_FORMATS)
def test_dequant_bitexact_golden_device(backend, golden, fmt):
    p = golden[f"dq_{fmt}_packed"]
    out = torch.empty((p.shape[0], 512), dtype=torch.float32, device="cuda")
    backend.dequant_rows(fmt, dev(p), p.shape[0], 512, out)
    backend.synchronize()
    assert bits_equal(out.cpu().numpy(), golden[f"dq_{fmt}_out"])


@pytest.mark.parametrize("fmt", GGUF_FORMATS)
def test_dequant_bitexact_random_host_staged(backend, oracle, um, fmt):
    rng = np.random.default_rng(100 + fmt)
    rows, cols = 96, 2048
    p = rng.integers(0, 256, size=(rows, um.packed_nbytes(fmt, cols)), dtype=np.uint8)
    out = np.empty((rows, cols), np.float32)
    backend.dequant_rows(fmt, p, rows, cols, out)  # host in, host out
    assert bits_equal(out, oracle.dequant(fmt, p, rows, cols))


def test_dequant_reference_known_answer(backend, golden):
    out = np.empty((1, 32), np.float32)
    backend.dequant_rows(7, golden["kat_q4_0_packed"], 1, 32, out)
    assert bits_equal(out, golden["kat_q4_0_out"])


# ---------------------------------------------------------------- router

def test_router_golden(backend, golden):
    x, w = golden["router_x"], golden["router_w"]
    T, D = x.shape
    E = w.shape[0]
    probs, top, logits = (np.empty((T, E), np.float32), np.empty((T, 1), np.float32),
                          np.empty((T, E), np.float32))
    backend.router(x, w, T, D, E, probs, top, logits)
    assert bits_equal(logits, golden["router_logits"])
    assert np.array_equal(top, golden["router_top"])
    assert np.allclose(probs, golden["router_probs"], rtol=4e-7, atol=0)


@pytest.mark.parametrize("T,D,E", [(1, 4096, 8), (32, 4096, 8), (4096, 4096, 8), (257, 2048, 60),
                                   (1000, 2048, 128), (3, 100, 5),
                                   (300, 1000, 40),    # many experts, a partial last k tile
                                   (130, 998, 33),     # many experts, rows not float4-aligned
                                   (200, 512, 256),    # more experts than one block covers
                                   (40, 2048, 128),    # few tokens: rows split across blocks, folded in order
                                   (600, 1000, 60)])   # split rows with a partial last tile
def test_router_vs_oracle(backend, oracle, um, T, D, E):
    x = um.fill_normal((T, D), 5, T)
    w = um.fill_normal((E, D), 5, E + 99, 0.0, 0.02)
    lg_ref, pr_ref, top_ref = oracle.router(x, w)
    xd, wd = dev(x), dev(w)
    probs = torch.empty((T, E), device="cuda")
    top = torch.empty((T, 1), device="cuda")
    logits = torch.empty((T, E), device="cuda")
    backend.router(xd, wd, T, D, E, probs, top, logits)
    backend.synchronize()
    assert bits_equal(logits.cpu().numpy(), lg_ref)
    assert np.allclose(probs.cpu().numpy(), pr_ref, rtol=4e-7, atol=0)
    assert np.array_equal(top.cpu().numpy(), top_ref)


def test_router_dispatch_arity_and_shapes(backend, um):
    x = np.zeros((2, 64), np.float32)
    w = np.zeros((4, 64), np.float32)
    p = np.zeros((2, 4), np.float32)
    with pytest.raises(um.UaiiMoeError) as e:
        backend.dispatch("MoERouter", [um.f32_desc(x)], [um.f32_desc(p)])
    assert e.value.status == 1 and "MoERouter expects" in e.value.message
    with pytest.raises(um.UaiiMoeError) as e:
        backend.dispatch("MoERouter", [um.f32_desc(x), um.f32_desc(w)],
                         [um.f32_desc(p), um.f32_desc(np.zeros((2, 2), np.float32))])
    assert "top_expert shape" in e.value.message
    with pytest.raises(um.UaiiMoeError) as e:
        backend.dispatch("Attention", [um.f32_desc(x)], [um.f32_desc(p)])
    assert e.value.status == 7


# ---------------------------------------------------------------- experts

@pytest.mark.parametrize("name,gf,df", EXPERT_CASES)
def test_experts_dispatch_golden(backend, golden, um, name, gf, df):
    i = [c[0] for c in EXPERT_CASES].index(name)
    x, w, G, U, Dn = expert_inputs(gf, df, 20 + i)
    probs = golden[f"exp_{name}_probs"]
    y = np.empty_like(x)
    backend.dispatch("MoEExpertsSwiGLU",
                     [um.f32_desc(x), um.packed_desc(G, gf, (EXP_E, EXP_I, EXP_D)),
                      um.packed_desc(U, gf, (EXP_E, EXP_I, EXP_D)),
                      um.packed_desc(Dn, df, (EXP_E, EXP_D, EXP_I)), um.f32_desc(probs)],
                     [um.f32_desc(y)], {"num_experts": EXP_E, "top_k": EXP_K})
    assert rel_err(y, golden[f"exp_{name}_y"]) <= REL_TOL


@pytest.mark.parametrize("k", [1, 2, 3, 8])
def test_experts_tie_order_golden(backend, golden, um, k):
    x, G, U, Dn, p = (golden[n] for n in ("ties_x", "ties_G", "ties_U", "ties_D", "ties_probs"))
    T, D = x.shape
    E, I, _ = G.shape
    y = np.empty_like(x)
    backend.experts(x, G, um.F32, U, um.F32, Dn, um.F32, p, T, D, E, I, k, 1, y)
    assert rel_err(y, golden[f"ties_y_k{k}"]) <= 1e-5


@pytest.mark.parametrize("B,D,E,where", [(7, 300, 3, "host"), (64, 1024, 8, "device"), (1, 4096, 2, "host")])
def test_legacy_experts_dispatch_vs_oracle(backend, oracle, um, B, D, E, where):
    """MoEExperts (top-1 linear experts, dense f32 W [E, D, D]) bit for bit, out-of-range ids included."""
    rng = np.random.default_rng(B + D)
    x = rng.standard_normal((B, D)).astype(np.float32)
    W = (rng.standard_normal((E, D, D)) * 0.05).astype(np.float32)
    top = rng.integers(0, E, size=(B, 1)).astype(np.float32)
    if B >= 6:
        top[:6, 0] = [np.nan, 1e30, -0.7, E - 0.3, -1e30, E]
    ref = oracle.experts_linear(x, W, top)
    if where == "host":
        y = np.empty_like(x)
        backend.dispatch("MoEExperts", [um.f32_desc(x), um.f32_desc(W), um.f32_desc(top)], [um.f32_desc(y)],
                         {"num_experts": E})
    else:
        xd, Wd, td = dev(x), dev(W), dev(top)
        yd = torch.empty_like(xd)
        backend.dispatch("MoEExperts", [um.f32_desc(xd), um.f32_desc(Wd), um.f32_desc(td)], [um.f32_desc(yd)],
                         {"num_experts": E})
        backend.synchronize()
        y = yd.cpu().numpy()
    assert bits_equal(y, ref)


def test_legacy_experts_dispatch_checks(backend, um):
    x = np.zeros((2, 8), np.float32)
    W = np.zeros((3, 8, 8), np.float32)
    top = np.zeros((2, 1), np.float32)
    y = np.empty_like(x)
    with pytest.raises(um.UaiiMoeError) as e:
        backend.dispatch("MoEExperts", [um.f32_desc(x), um.f32_desc(W)], [um.f32_desc(y)], {"num_experts": 3})
    assert "MoEExperts expects x,experts_w,top_expert" in e.value.message
    with pytest.raises(um.UaiiMoeError) as e:  # num_experts defaults to 1
        backend.dispatch("MoEExperts", [um.f32_desc(x), um.f32_desc(W), um.f32_desc(top)], [um.f32_desc(y)])
    assert "experts_w shape" in e.value.message


def test_reference_smoke_demo_on_device(backend, golden, um):
    """The reference's MoE smoke demo shapes (E=2, D=4, I=3) through dispatch."""
    x, w = golden["smoke_x"], golden["smoke_w"]
    probs, top = np.empty((1, 2), np.float32), np.empty((1, 1), np.float32)
    backend.dispatch("MoERouter", [um.f32_desc(x), um.f32_desc(w)], [um.f32_desc(probs), um.f32_desc(top)],
                     {"num_experts": 2})
    assert abs(float(probs.sum()) - 1.0) <= 1e-3 and top[0, 0] in (0.0, 1.0)
    assert np.array_equal(top, golden["smoke_top"])
    y = np.empty((1, 4), np.float32)
    backend.dispatch("MoEExpertsSwiGLU",
                     [um.f32_desc(x), um.f32_desc(golden["smoke_G"]), um.f32_desc(golden["smoke_U"]),
                      um.f32_desc(golden["smoke_D"]), um.f32_desc(golden["smoke_probs"])],
                     [um.f32_desc(y)], {"num_experts": 2, "top_k": 2})
    assert rel_err(y, golden["smoke_y"]) <= 1e-5


def layer_case(um, gf, df, T, D, E, I, k, seed, norm=1):
    x = um.fill_normal((T, D), seed, 1)
    w = um.fill_normal((E, D), seed, 2, 0.0, 0.02)
    G = um.quantize_rows(gf, um.fill_normal((E * I, D), seed, 3, 0.0, 0.02)).reshape(E, I, -1)
    U = um.quantize_rows(gf, um.fill_normal((E * I, D), seed, 4, 0.0, 0.02)).reshape(E, I, -1)
    Dn = um.quantize_rows(df, um.fill_normal((E * D, I), seed, 5, 0.0, 0.02)).reshape(E, D, -1)
    return x, w, G, U, Dn


@pytest.mark.parametrize("gf,df,T,D,E,I,k,norm", [
    (7, 7, 64, 1024, 8, 2816, 2, 1),        # config 1 shapes
    (14, 16, 5, 1024, 8, 512, 2, 1),        # Mixtral formats, reduced width
    (11, 11, 40, 512, 12, 384, 4, 0),       # Qwen2 formats, no renormalisation
    (7, 7, 50, 512, 32, 256, 8, 1),         # Qwen3 formats
    (7, 7, 1, 256, 4, 256, 4, 1),           # k == E
    (8, 10, 9, 256, 6, 256, 3, 1),          # Q4_1 gate/up, Q5_1 down
    (12, 15, 7, 256, 4, 512, 2, 1),         # Q2_K gate/up, Q5_K down
    (13, 9, 7, 512, 4, 256, 2, 1),          # Q3_K gate/up, Q5_0 down
])
def test_ffn_vs_oracle(backend, oracle, um, gf, df, T, D, E, I, k, norm):
    if gf in (8, 12, 13):  # formats without a quantizer: random bytes with tame scales
        rng = np.random.default_rng(T * 31 + D)
        x = um.fill_normal((T, D), 4, 1)
        w = um.fill_normal((E, D), 4, 2, 0.0, 0.02)
        G, U, Dn = (random_blocks(um, rng, f, rows, cols) for f, rows, cols in
                    ((gf, E * I, D), (gf, E * I, D), (df, E * D, I)))
    else:
        x, w, G, U, Dn = layer_case(um, gf, df, T, D, E, I, k, 40 + T)
    _, pr, _ = oracle.router(x, w)
    y_ref, ids_ref, _ = oracle.experts_packed(x, G, gf, U, gf, Dn, df, pr, E, I, k, norm)
    L = um.make_layer(D, E, I, k, norm, w, G, gf, U, gf, Dn, df)
    y = np.empty_like(x)
    probs = np.empty((T, E), np.float32)
    backend.ffn(L, x, T, y, probs)
    assert np.allclose(probs, pr, rtol=4e-7, atol=0)
    assert rel_err(y, y_ref) <= REL_TOL


def random_blocks(um, rng, fmt, rows, cols):
    """Random GGUF rows whose f16 scales are set to small finite values."""
    from golden.make_golden import D_OFFSET
    qk, bb = um.BLOCK[fmt]
    p = rng.integers(0, 256, size=(rows, cols // qk, bb), dtype=np.uint8)
    scale = np.float16(0.002).view(np.uint16)
    offs = [D_OFFSET[fmt]]
    if fmt in (8, 10, 12, 14, 15):  # a second f16 (min / dmin) follows or precedes d
        offs.append(D_OFFSET[fmt] + 2)
    for o in offs:
        p[:, :, o] = scale & 0xFF
        p[:, :, o + 1] = scale >> 8
    return p.reshape(rows, -1)


def test_ffn_shared_expert_sigmoid_gate(backend, oracle, um):
    T, D, E, I, Ish, k = 16, 512, 8, 256, 768, 4
    x, w, G, U, Dn = layer_case(um, 11, 11, T, D, E, I, k, 77)
    Gs = um.quantize_rows(11, um.fill_normal((Ish, D), 77, 6, 0.0, 0.02))
    Us = um.quantize_rows(11, um.fill_normal((Ish, D), 77, 7, 0.0, 0.02))
    Ds = um.quantize_rows(11, um.fill_normal((D, Ish), 77, 8, 0.0, 0.02))
    gi = um.fill_normal((D,), 77, 9, 0.0, 0.02)
    _, pr, _ = oracle.router(x, w)
    for gate in (None, gi):
        y_ref, _, _ = oracle.experts_packed(x, G, 11, U, 11, Dn, 11, pr, E, I, k, 0)
        oracle.shared_packed(x, Gs, 11, Us, 11, Ds, 11, gate, Ish, y_ref)
        L = um.make_layer(D, E, I, k, 0, w, G, 11, U, 11, Dn, 11, shared=(Ish, Gs, 11, Us, 11, Ds, 11, gate))
        y = np.empty_like(x)
        backend.ffn(L, x, T, y)
        assert rel_err(y, y_ref) <= REL_TOL


def test_ffn_device_and_host_agree_and_deterministic(backend, um):
    T, D, E, I, k = 33, 512, 8, 512, 2
    x, w, G, U, Dn = layer_case(um, 14, 16, T, D, E, I, k, 5)
    L = um.make_layer(D, E, I, k, 1, w, G, 14, U, 14, Dn, 16)
    y_host = np.empty_like(x)
    backend.ffn(L, x, T, y_host)
    xd, wd, Gd, Ud, Dd = (dev(a) for a in (x, w, G, U, Dn))
    Ld = um.make_layer(D, E, I, k, 1, wd, Gd, 14, Ud, 14, Dd, 16)
    outs = []
    for _ in range(2):
        y = torch.empty((T, D), device="cuda")
        backend.ffn(Ld, xd, T, y)
        backend.synchronize()
        outs.append(y.cpu().numpy())
    assert bits_equal(outs[0], outs[1])
    assert bits_equal(outs[0], y_host)


def test_ffn_token_permutation_equivariance(backend, um):
    T, D, E, I, k = 24, 256, 8, 256, 2
    x, w, G, U, Dn = layer_case(um, 7, 7, T, D, E, I, k, 8)
    L = um.make_layer(D, E, I, k, 1, w, G, 7, U, 7, Dn, 7)
    y = np.empty_like(x)
    backend.ffn(L, x, T, y)
    perm = np.random.default_rng(0).permutation(T)
    xp = np.ascontiguousarray(x[perm])
    yp = np.empty_like(x)
    backend.ffn(L, xp, T, yp)
    assert bits_equal(yp, y[perm])


def test_zero_tokens_is_a_no_op(backend, um):
    D, E, I = 256, 4, 256
    x, w, G, U, Dn = layer_case(um, 7, 7, 1, D, E, I, 2, 9)
    L = um.make_layer(D, E, I, 2, 1, w, G, 7, U, 7, Dn, 7)
    y = np.full((1, D), 7.0, np.float32)
    backend.ffn(L, x, 0, y)
    assert (y == 7.0).all()


def test_bad_arguments_are_reported(backend, um):
    D, E, I = 256, 4, 256
    x, w, G, U, Dn = layer_case(um, 7, 7, 2, D, E, I, 2, 9)
    y = np.empty_like(x)
    with pytest.raises(um.UaiiMoeError) as e:  # gate/up formats differ
        backend.ffn(um.make_layer(D, E, I, 2, 1, w, G, 7, U, 11, Dn, 7), x, 2, y)
    assert e.value.status == 7
    with pytest.raises(um.UaiiMoeError) as e:  # K-quant row length must be a multiple of 256
        backend.ffn(um.make_layer(D, E, 96, 2, 1, w, G, 7, U, 7, Dn, 16), x, 2, y)
    assert e.value.status == 1
    with pytest.raises(um.UaiiMoeError) as e:  # wrong num_experts attribute
        backend.dispatch("MoEExpertsSwiGLU",
                         [um.f32_desc(x), um.packed_desc(G, 7, (E, I, D)), um.packed_desc(U, 7, (E, I, D)),
                          um.packed_desc(Dn, 7, (E, D, I)), um.f32_desc(np.zeros((2, E), np.float32))],
                         [um.f32_desc(y)], {"num_experts": E + 1, "top_k": 2})
    assert "shape mismatch" in e.value.message


def test_registered_weights_are_reused_and_released(backend, um):
    T, D, E, I, k = 4, 256, 4, 256, 2
    x, w, G, U, Dn = layer_case(um, 7, 7, T, D, E, I, k, 12)
    L = um.make_layer(D, E, I, k, 1, w, G, 7, U, 7, Dn, 7)
    y0 = np.empty_like(x)
    backend.ffn(L, x, T, y0)  # unregistered: staged per call
    for a in (w, G, U, Dn):
        backend.register_weights(a)
    y1 = np.empty_like(x)
    backend.ffn(L, x, T, y1)
    assert bits_equal(y0, y1)
    G[...] = 0  # registered buffers are not re-read: the cached copy is used
    y2 = np.empty_like(x)
    backend.ffn(L, x, T, y2)
    assert bits_equal(y0, y2)
    for a in (w, G, U, Dn):
        backend.release_weights(a)
    with pytest.raises(um.UaiiMoeError) as e:
        backend.release_weights(G)
    assert e.value.status == 2
    y3 = np.empty_like(x)
    backend.ffn(L, x, T, y3)  # unregistered again: zero gate weights now take effect
    assert not bits_equal(y0, y3)


# ---------------------------------------------------------------- tensor-core path

@pytest.mark.parametrize("gf,df,T,D,E,I,k", [
    (7, 7, 1, 1024, 8, 2816, 2),       # config 1 shapes, decode (slot tile 16, split-K down)
    (7, 7, 64, 1024, 8, 2816, 2),      # config 1 shapes, 64 tokens
    (14, 16, 1, 1024, 8, 2048, 2),     # Mixtral formats (Q4_K / Q6_K), decode
    (14, 16, 32, 1024, 8, 2048, 2),    # Mixtral formats, 32 tokens
    (14, 16, 700, 512, 4, 2048, 2),    # Mixtral formats, slot tile 256
    (11, 11, 100, 512, 8, 512, 4),     # Q8_0, slot tile 64
    (7, 7, 200, 2048, 16, 768, 8),     # Qwen3 formats, slot tile 128
    (7, 7, 3, 256, 4, 256, 4),         # k == E, tiny
])
def test_tensor_core_path_vs_oracle(backend, oracle, um, gf, df, T, D, E, I, k):
    x, w, G, U, Dn = layer_case(um, gf, df, T, D, E, I, k, 60 + T)
    _, pr, _ = oracle.router(x, w)
    y_ref, _, _ = oracle.experts_packed(x, G, gf, U, gf, Dn, df, pr, E, I, k, 1)
    L = um.make_layer(D, E, I, k, 1, w, G, gf, U, gf, Dn, df)
    y = np.empty_like(x)
    backend.set_expert_path(2)
    try:
        backend.ffn(L, x, T, y)
    finally:
        backend.set_expert_path(0)
    assert rel_err(y, y_ref) <= REL_TOL


@pytest.mark.parametrize("gf,df,T,D,E,I,k", [
    (14, 16, 5, 256, 4, 256, 2),      # Q6_K rows of 256 elements: 210 bytes, not a 16-byte pitch
    (11, 11, 40, 256, 6, 1408, 4),    # Q8_0 rows of 1408 elements (the Qwen2-MoE down projection): 1496 bytes
    (7, 7, 24, 256, 4, 320, 2),       # Q4_0 rows of 320 elements: 180 bytes; last quad of 64 elements
])
def test_tensor_core_path_pads_unaligned_pitch(backend, oracle, um, gf, df, T, D, E, I, k):
    # rows whose byte pitch is not a multiple of 16 cannot be TMA tensor-map rows: the
    # backend stages a copy with padded rows, bytes unchanged
    x, w, G, U, Dn = layer_case(um, gf, df, T, D, E, I, k, 90 + I)
    _, pr, _ = oracle.router(x, w)
    y_ref, _, _ = oracle.experts_packed(x, G, gf, U, gf, Dn, df, pr, E, I, k, 1)
    y = np.empty_like(x)
    backend.set_expert_path(2)
    try:
        backend.ffn(um.make_layer(D, E, I, k, 1, w, G, gf, U, gf, Dn, df), x, T, y)
        assert backend.last_plan()["tensor_cores"]
    finally:
        backend.set_expert_path(0)
    assert rel_err(y, y_ref) <= REL_TOL


def test_tensor_core_path_refuses_unsupported_shapes(backend, um):
    # d_model must be a multiple of 128 (the weight-row tile of the down projection)
    D, E, I = 96, 4, 256
    x, w, G, U, Dn = layer_case(um, 7, 7, 2, D, E, I, 2, 3)
    y = np.empty_like(x)
    backend.set_expert_path(2)
    try:
        with pytest.raises(um.UaiiMoeError) as e:
            backend.ffn(um.make_layer(D, E, I, 2, 1, w, G, 7, U, 7, Dn, 7), x, 2, y)
        assert e.value.status == 7
    finally:
        backend.set_expert_path(0)
    backend.ffn(um.make_layer(D, E, I, 2, 1, w, G, 7, U, 7, Dn, 7), x, 2, y)  # automatic: CUDA cores


def test_tensor_core_shared_expert(backend, oracle, um):
    T, D, E, I, Ish, k = 48, 512, 8, 256, 1024, 4
    x, w, G, U, Dn = layer_case(um, 11, 11, T, D, E, I, k, 78)
    Gs = um.quantize_rows(11, um.fill_normal((Ish, D), 78, 6, 0.0, 0.02))
    Us = um.quantize_rows(11, um.fill_normal((Ish, D), 78, 7, 0.0, 0.02))
    Ds = um.quantize_rows(11, um.fill_normal((D, Ish), 78, 8, 0.0, 0.02))
    gi = um.fill_normal((D,), 78, 9, 0.0, 0.02)
    _, pr, _ = oracle.router(x, w)
    y_ref, _, _ = oracle.experts_packed(x, G, 11, U, 11, Dn, 11, pr, E, I, k, 0)
    oracle.shared_packed(x, Gs, 11, Us, 11, Ds, 11, gi, Ish, y_ref)
    L = um.make_layer(D, E, I, k, 0, w, G, 11, U, 11, Dn, 11, shared=(Ish, Gs, 11, Us, 11, Ds, 11, gi))
    y = np.empty_like(x)
    backend.set_expert_path(2)
    try:
        backend.ffn(L, x, T, y)
    finally:
        backend.set_expert_path(0)
    assert rel_err(y, y_ref) <= REL_TOL


# ---------------------------------------------------------------- warp-MMA schedule (decode widths)

@pytest.mark.parametrize("gf,df,T,D,E,I,k", [
    (14, 16, 1, 1024, 8, 2048, 2),     # Mixtral formats, one token: 8-slot tiles, split-K down
    (14, 16, 32, 1024, 8, 2048, 2),    # Mixtral formats, 8 slots per expert
    (14, 16, 60, 512, 8, 1024, 2),     # 16-slot tiles
    (7, 7, 3, 1024, 8, 2816, 2),       # config 1 shapes (Q4_0)
    (11, 11, 9, 512, 12, 384, 4),      # Q8_0 (two boxes per window); K % 256 == 128 for down
    (7, 7, 5, 384, 4, 640, 2),         # Q4_0 with a half quad at the end of both projections
    (7, 7, 50, 512, 32, 256, 8),       # Qwen3 formats, many experts
    (14, 16, 5, 256, 4, 256, 2),       # Q6_K rows of 210 bytes: padded pitch
    (7, 7, 300, 256, 4, 256, 2),       # forced far above decode widths: many 16-slot tiles per expert
])
def test_warp_mma_path_vs_oracle(backend, oracle, um, gf, df, T, D, E, I, k):
    x, w, G, U, Dn = layer_case(um, gf, df, T, D, E, I, k, 120 + T)
    _, pr, _ = oracle.router(x, w)
    y_ref, _, _ = oracle.experts_packed(x, G, gf, U, gf, Dn, df, pr, E, I, k, 1)
    L = um.make_layer(D, E, I, k, 1, w, G, gf, U, gf, Dn, df)
    y = np.empty_like(x)
    backend.set_expert_path(3)
    try:
        backend.ffn(L, x, T, y)
        plan = backend.last_plan()
    finally:
        backend.set_expert_path(0)
    kquant = gf in (14, 16) and df in (14, 16)
    quad = ("quad_mma_i8" if gf == 14 and plan["slot_tile"] == 8 else "quad_mma") if kquant else "warp_mma"
    assert plan["schedule"] == quad and plan["slot_tile"] in (8, 16)
    assert rel_err(y, y_ref) <= REL_TOL


@pytest.mark.parametrize("gf,df,T,D,E,I,k", [
    (14, 16, 1, 1024, 8, 2048, 2),     # Mixtral formats: Q6_K windows at all eight 16-byte offsets
    (14, 16, 60, 512, 8, 1024, 2),     # 16-slot tiles
    (16, 14, 5, 512, 4, 768, 2),       # Q6_K gate/up, Q4_K down; three quads per down row (odd)
    (14, 14, 9, 768, 6, 512, 3),       # Q4_K only, three quads per gate/up row
    (16, 16, 3, 256, 4, 512, 2),       # one quad per gate/up row: the odd-quad warps idle; padded pitch
    (14, 16, 20, 512, 32, 512, 8),     # many experts, top-8
    (14, 16, 300, 256, 4, 256, 2),     # forced far above decode widths: many 16-slot tiles per expert
])
def test_quad_schedule_vs_oracle_and_unit_schedule(backend, oracle, um, gf, df, T, D, E, I, k):
    """The warp-MMA schedule over whole K-quant super-blocks: against the oracle within the
    layer bar, and against the per-unit warp-MMA schedule (path 4).  Q4_K enters the quad
    schedule's products unrounded (q*sc exact in f16, d and dmin in f32) where the other
    schedules round fp16(d*sc*q - dmin*m); Q6_K operands are the same values."""
    x, w, G, U, Dn = layer_case(um, gf, df, T, D, E, I, k, 300 + T)
    _, pr, _ = oracle.router(x, w)
    y_ref, _, _ = oracle.experts_packed(x, G, gf, U, gf, Dn, df, pr, E, I, k, 1)
    L = um.make_layer(D, E, I, k, 1, w, G, gf, U, gf, Dn, df)
    ys = {}
    for path in (3, 4):
        y = np.empty_like(x)
        backend.set_expert_path(path)
        try:
            backend.ffn(L, x, T, y)
            ys[path] = (y, backend.last_plan())
        finally:
            backend.set_expert_path(0)
    # Q4_K gate/up at 8-slot tiles runs on 16-bit integer activations (test_quad_integer_activations_vs_oracle)
    i8 = gf == 14 and ys[3][1]["slot_tile"] == 8
    assert ys[3][1]["schedule"] == ("quad_mma_i8" if i8 else "quad_mma") and ys[4][1]["schedule"] == "warp_mma"
    err_quad, err_unit = rel_err(ys[3][0], y_ref), rel_err(ys[4][0], y_ref)
    assert err_quad <= REL_TOL
    # no less accurate than the per-unit schedule (Q4_K: more accurate, its weights are unrounded)
    assert err_quad <= 1.25 * max(err_unit, 1e-4), (err_quad, err_unit)
    if gf == 16 and df == 16:  # identical Q6_K operands: only the f32 summation order differs
        assert rel_err(ys[3][0], ys[4][0]) <= 1e-4


@pytest.mark.parametrize("T,I,path", [(1, 1024, 0), (2, 1024, 0), (1, 1024, 5), (2, 1024, 5)])
def test_quad_tail_split_vs_oracle_and_repeatable(backend, oracle, um, T, I, path):
    """Gate/up tiles of a last wave that fills at most half of the GPU are cut into K ranges
    run by different CTAs (2 experts x I/64 tiles here, all in one partial wave); the CTA that
    finishes a tile's last range adds the ranges in order.  Against the oracle, and
    bit-identical over repeated calls (the per-tile counters are left at zero); on integer
    (path 0) and f16 (path 5) activations."""
    gf, df, D, E, k = 14, 16, 4096, 8, 2
    x, w, G, U, Dn = layer_case(um, gf, df, T, D, E, I, k, 900 + T)
    _, pr, _ = oracle.router(x, w)
    y_ref, _, _ = oracle.experts_packed(x, G, gf, U, gf, Dn, df, pr, E, I, k, 1)
    L = um.make_layer(D, E, I, k, 1, w, G, gf, U, gf, Dn, df)
    backend.set_graphs(False)
    backend.set_expert_path(path)
    try:
        ys = []
        for _ in range(3):
            y = np.empty_like(x)
            backend.ffn(L, x, T, y)
            ys.append(y)
        assert backend.last_plan()["schedule"] == ("quad_mma_i8" if path == 0 else "quad_mma")
    finally:
        backend.set_expert_path(0)
        backend.set_graphs(True)
    assert rel_err(ys[0], y_ref) <= REL_TOL
    assert bits_equal(ys[0], ys[1]) and bits_equal(ys[0], ys[2])


@pytest.mark.parametrize("T,D,I,case", [(1, 4096, 1024, "normal"), (5, 4096, 2048, "normal"), (8, 1024, 1024, "normal"),
                                        (16, 4096, 1024, "normal"), (8, 1024, 512, "outliers"),
                                        (8, 1024, 512, "zero_quads"), (3, 256, 256, "normal")])
def test_quad_integer_activations_vs_oracle(backend, oracle, um, T, D, I, case):
    """The Q4_K quad gate/up on 16-bit integer activations (int8 mma.sync over the raw nibbles,
    exact int32 sub-block sums): against the oracle at the layer bar, and no further from it
    than twice the f16-activation path's error (plus 1e-5).  Cases: N(0,1) activations; an
    outlier 100 times the rest in every quad (it sets the scale of the other 255; far larger ones
    overflow the f16 hidden activations of either path);
    whole quads and a whole row of zeros (zero scale)."""
    gf, df, E, k = 14, 16, 8, 2
    x, w, G, U, Dn = layer_case(um, gf, df, T, D, E, I, k, 2100 + T + D)
    if case == "outliers":
        x[:, ::256] *= 100.0
    elif case == "zero_quads":
        x[:, 256:512] = 0.0
        x[T // 2, :] = 0.0
    x = np.ascontiguousarray(x, np.float32)
    _, pr, _ = oracle.router(x, w)
    y_ref, _, _ = oracle.experts_packed(x, G, gf, U, gf, Dn, df, pr, E, I, k, 1)
    L = um.make_layer(D, E, I, k, 1, w, G, gf, U, gf, Dn, df)
    ys = {}
    try:
        for path in (0, 5):
            backend.set_expert_path(path)
            y = np.empty_like(x)
            backend.ffn(L, x, T, y)
            ys[path] = (y, backend.last_plan()["schedule"])
    finally:
        backend.set_expert_path(0)
    assert ys[0][1] == "quad_mma_i8" and ys[5][1] == "quad_mma"
    e_i8, e_f16 = rel_err(ys[0][0], y_ref), rel_err(ys[5][0], y_ref)
    assert e_i8 <= REL_TOL, (e_i8, e_f16)
    assert e_i8 <= 2 * e_f16 + 1e-5, (e_i8, e_f16)


@pytest.mark.parametrize("T,D,I,mode", [(1, 1024, 2048, "1"), (1, 4096, 2048, "1"), (8, 4096, 2048, ""),
                                        (12, 4096, 3072, ""), (32, 4096, 2048, "")])
def test_quad_down_balanced_ranges(oracle, um, monkeypatch, T, D, I, mode):
    """The quad-schedule down projection in balanced ranges (every CTA an equal share of the
    tile-major quad sequence; tiles cut between CTAs finished by the CTA that completes the last
    piece): against the oracle, against whole-unit K splits (UAII_MOE_DOWN_RANGES=0, the same
    partials grouped differently: 1e-5), and bit-identical over repeated calls (the per-CTA
    counters are left at zero).  Automatic mode takes ranges from one tile per SM up (8, 12 and
    32 tokens here; 32 tokens on 16-slot tiles); forced ranges ("1") at 1 token run more CTAs
    than quads, one-quad pieces of a tile spread over several CTAs."""
    gf, df, E, k = 14, 16, 8, 2
    x, w, G, U, Dn = layer_case(um, gf, df, T, D, E, I, k, 2600 + T + D)
    _, pr, _ = oracle.router(x, w)
    y_ref, _, _ = oracle.experts_packed(x, G, gf, U, gf, Dn, df, pr, E, I, k, 1)
    L = um.make_layer(D, E, I, k, 1, w, G, gf, U, gf, Dn, df)

    def run(env, calls):
        if env:
            monkeypatch.setenv("UAII_MOE_DOWN_RANGES", env)
        else:
            monkeypatch.delenv("UAII_MOE_DOWN_RANGES", raising=False)
        b = um.Backend(0)
        try:
            b.set_graphs(False)
            out = []
            for _ in range(calls):
                y = np.empty_like(x)
                b.ffn(L, x, T, y)
                out.append(y)
            return out, b.last_plan()
        finally:
            b.close()

    ys, plan = run(mode, 2)
    assert plan["down_splits"] == 1, plan
    (y2,), plan2 = run("0", 1)
    assert rel_err(ys[0], y_ref) <= REL_TOL
    assert bits_equal(ys[0], ys[1])
    assert rel_err(ys[0], y2) <= 1e-5


@pytest.mark.parametrize("T,D,E,k", [(1, 4096, 8, 2), (7, 2048, 60, 4), (16, 2048, 128, 8), (3, 1024, 5, 5), (32, 4096, 8, 2)])
def test_decode_routing_launch_matches_separate_kernels(backend, oracle, um, T, D, E, k):
    """At decode widths the layer routes in one launch (router, softmax, top-k, slot numbering):
    its probabilities equal the router kernels' bit for bit, its output meets the layer bar
    against the oracle (the top-k path included), and repeated calls give the same bits."""
    I, gf, df = 256, um.Q4_0, um.Q4_0
    x, w, G, U, Dn = layer_case(um, gf, df, T, D, E, I, k, 1500 + T)
    L = um.make_layer(D, E, I, k, 1, w, G, gf, U, gf, Dn, df)
    probs_ffn = np.empty((T, E), np.float32)
    y = np.empty_like(x)
    backend.ffn(L, x, T, y, probs_ffn)
    probs_r, top_r = np.empty((T, E), np.float32), np.empty((T, 1), np.float32)
    backend.router(x, w, T, D, E, probs_r, top_r)
    assert bits_equal(probs_ffn, probs_r)
    _, pr, _ = oracle.router(x, w)
    y_ref = oracle.experts_packed(x, G, gf, U, gf, Dn, df, pr, E, I, k, 1)[0]
    assert rel_err(y, y_ref) <= REL_TOL
    y2 = np.empty_like(x)
    backend.ffn(L, x, T, y2)
    assert bits_equal(y, y2)


@pytest.mark.parametrize("gf,df", [(14, 16), (14, 14)])
def test_mixed_schedule_at_16_slot_tiles(backend, oracle, um, gf, df):
    """16-slot tiles of a K-quant layer: gate/up on tcgen05 (operands in tc_kpos order), the down
    projection on the quad schedule (its h written by the tcgen05 epilogue in the quad order)."""
    T, D, E, I, k = 32, 1024, 8, 1024, 2
    x, w, G, U, Dn = layer_case(um, gf, df, T, D, E, I, k, 77)
    _, pr, _ = oracle.router(x, w)
    y_ref, _, _ = oracle.experts_packed(x, G, gf, U, gf, Dn, df, pr, E, I, k, 1)
    L = um.make_layer(D, E, I, k, 1, w, G, gf, U, gf, Dn, df)
    y = np.empty_like(x)
    backend.ffn(L, x, T, y)
    plan = backend.last_plan()
    assert (plan["schedule"], plan["slot_tile"]) == ("tcgen05", 16), plan
    assert rel_err(y, y_ref) <= REL_TOL
    y2 = np.empty_like(x)
    backend.set_expert_path(2)  # tcgen05 for both projections
    try:
        backend.ffn(L, x, T, y2)
    finally:
        backend.set_expert_path(0)
    assert rel_err(y, y2) <= 1e-3


def test_automatic_schedule_picks_warp_mma_for_decode(backend, um):
    D, E, I, k = 1024, 8, 2048, 2
    # tiles hold the mean slots per expert plus two standard deviations below 32 slots
    for T, sched, tile in ((1, "quad_mma_i8", 8), (8, "quad_mma_i8", 8), (32, "tcgen05", 16), (64, "tcgen05", 32),
                           (512, "tcgen05", 128)):
        x, w, G, U, Dn = layer_case(um, 14, 16, T, D, E, I, k, 5)
        y = np.empty_like(x)
        backend.ffn(um.make_layer(D, E, I, k, 1, w, G, 14, U, 14, Dn, 16), x, T, y)
        plan = backend.last_plan()
        assert (plan["schedule"], plan["slot_tile"]) == (sched, tile), (T, plan)


def test_warp_mma_and_tcgen05_agree(backend, um):
    # same operands, different accumulation order: the two schedules agree to f32 rounding
    T, D, E, I, k = 12, 1024, 8, 1024, 2
    x, w, G, U, Dn = layer_case(um, 14, 16, T, D, E, I, k, 8)
    L = um.make_layer(D, E, I, k, 1, w, G, 14, U, 14, Dn, 16)
    ys = []
    for path in (2, 4):
        y = np.empty_like(x)
        backend.set_expert_path(path)
        try:
            backend.ffn(L, x, T, y)
        finally:
            backend.set_expert_path(0)
        ys.append(y)
    assert rel_err(ys[1], ys[0]) <= 1e-4


def test_warp_mma_refuses_unsupported_shapes(backend, um):
    # d_ff = 320 is a tcgen05 shape (multiple of 64) but not a warp-MMA one (multiple of 128)
    D, E, I = 256, 4, 320
    x, w, G, U, Dn = layer_case(um, 7, 7, 2, D, E, I, 2, 3)
    y = np.empty_like(x)
    backend.set_expert_path(3)
    try:
        with pytest.raises(um.UaiiMoeError) as e:
            backend.ffn(um.make_layer(D, E, I, 2, 1, w, G, 7, U, 7, Dn, 7), x, 2, y)
        assert e.value.status == 7
    finally:
        backend.set_expert_path(0)
    backend.ffn(um.make_layer(D, E, I, 2, 1, w, G, 7, U, 7, Dn, 7), x, 2, y)  # automatic: tcgen05
    assert backend.last_plan()["schedule"] == "tcgen05"


@pytest.mark.parametrize("T", [4, 16])
def test_warp_mma_shared_expert(backend, oracle, um, T):
    D, E, I, Ish, k = 512, 8, 256, 1024, 4
    x, w, G, U, Dn = layer_case(um, 11, 11, T, D, E, I, k, 79)
    Gs = um.quantize_rows(11, um.fill_normal((Ish, D), 79, 6, 0.0, 0.02))
    Us = um.quantize_rows(11, um.fill_normal((Ish, D), 79, 7, 0.0, 0.02))
    Ds = um.quantize_rows(11, um.fill_normal((D, Ish), 79, 8, 0.0, 0.02))
    gi = um.fill_normal((D,), 79, 9, 0.0, 0.02)
    _, pr, _ = oracle.router(x, w)
    y_ref, _, _ = oracle.experts_packed(x, G, 11, U, 11, Dn, 11, pr, E, I, k, 0)
    oracle.shared_packed(x, Gs, 11, Us, 11, Ds, 11, gi, Ish, y_ref)
    L = um.make_layer(D, E, I, k, 0, w, G, 11, U, 11, Dn, 11, shared=(Ish, Gs, 11, Us, 11, Ds, 11, gi))
    y = np.empty_like(x)
    backend.set_expert_path(3)
    try:
        backend.ffn(L, x, T, y)
    finally:
        backend.set_expert_path(0)
    assert rel_err(y, y_ref) <= REL_TOL


def test_registered_device_weights_keep_padded_rows(backend, oracle, um):
    # Q8_0 rows of 1408 elements (1496 bytes) need a 16-byte pitch for the tensor maps: for
    # registered device weights the padded copy is made once, and results do not change
    torch = pytest.importorskip("torch")
    T, D, E, I, k = 8, 256, 6, 1408, 4
    x, w, G, U, Dn = layer_case(um, 11, 11, T, D, E, I, k, 31)
    _, pr, _ = oracle.router(x, w)
    y_ref, _, _ = oracle.experts_packed(x, G, 11, U, 11, Dn, 11, pr, E, I, k, 1)
    dev = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (w, G, U, Dn)]
    L = um.make_layer(D, E, I, k, 1, dev[0], dev[1], 11, dev[2], 11, dev[3], 11)
    y0 = np.empty_like(x)
    backend.ffn(L, x, T, y0)
    for a in dev:
        backend.register_weights(a)
    try:
        ys = []
        for _ in range(2):
            backend.profile_enable(True)
            y = np.empty_like(x)
            backend.ffn(L, x, T, y)
            _, launches = backend.profile_read()
            backend.profile_enable(False)
            ys.append((y, launches))
        assert bits_equal(ys[0][0], y0) and bits_equal(ys[1][0], y0)
        assert ys[1][1] == ys[0][1] - 1  # the second call reuses the padded down rows (one launch fewer)
    finally:
        for a in dev:
            backend.release_weights(a)
    assert rel_err(y0, y_ref) <= REL_TOL
    y2 = np.empty_like(x)
    backend.ffn(L, x, T, y2)  # released: padded per call again
    assert bits_equal(y2, y0)


# ---------------------------------------------------------------- MatMul with a packed B (quant_gemm_f32)

def _qrows(um, fmt, rows, cols, seed):
    if fmt in (um.Q4_0, um.Q8_0, um.Q4_K, um.Q6_K):
        return um.quantize_rows(fmt, um.fill_normal((rows, cols), seed, 3, 0.0, 0.05))
    return random_blocks(um, np.random.default_rng(seed), fmt, rows, cols)


@pytest.mark.parametrize("fmt,M,K,N,path,sched", [
    (14, 1, 1024, 256, 0, "warp_mma"),       # Q4_K decode row: warp-MMA, split K
    (16, 5, 2048, 512, 0, "warp_mma"),       # Q6_K
    (7, 64, 512, 384, 0, "tcgen05"),         # Q4_0, 64-slot tile
    (11, 300, 256, 128, 0, "tcgen05"),       # Q8_0, 256-slot tiles
    (11, 3, 1408, 256, 2, "tcgen05"),        # Q8_0 rows of 1496 bytes (padded pitch), forced tcgen05
    (7, 40, 384, 128, 3, "warp_mma"),        # forced warp-MMA above decode width; K % 256 == 128
])
def test_quant_matmul_tensor_cores_vs_oracle(backend, oracle, um, fmt, M, K, N, path, sched):
    x = um.fill_normal((M, K), 17 + M, 1)
    W = _qrows(um, fmt, N, K, 5 + N)
    y_ref = oracle.quant_gemm(x, W, fmt, N)
    y = np.empty((M, N), np.float32)
    backend.set_expert_path(path)
    try:
        backend.quant_matmul(x, M, K, W, fmt, N, y)
        plan = backend.last_plan()
    finally:
        backend.set_expert_path(0)
    assert plan["schedule"] == sched, plan
    assert rel_err(y, y_ref) <= REL_TOL


@pytest.mark.parametrize("fmt,M,K,N", [
    (15, 7, 512, 128),    # Q5_K: no tensor-core decoder -> CUDA cores, f32
    (7, 9, 256, 100),     # N not a multiple of 128
    (13, 2, 768, 64),     # Q3_K
])
def test_quant_matmul_cuda_cores_vs_oracle(backend, oracle, um, fmt, M, K, N):
    x = um.fill_normal((M, K), 23 + M, 1)
    W = _qrows(um, fmt, N, K, 9 + N)
    y_ref = oracle.quant_gemm(x, W, fmt, N)
    y = np.empty((M, N), np.float32)
    backend.quant_matmul(x, M, K, W, fmt, N, y)
    assert not backend.last_plan()["tensor_cores"]
    assert rel_err(y, y_ref) <= 1e-5


def test_matmul_dispatch_packed_b_and_relu(backend, oracle, um):
    # dispatch_cpu's MatMul / MatMulRelu with a packed B and transpose_b (dispatch.cpp:82-100)
    M, K, N = 6, 512, 256
    x = um.fill_normal((M, K), 31, 1)
    W = _qrows(um, um.Q4_K, N, K, 31)
    y_ref = oracle.quant_gemm(x, W, um.Q4_K, N)
    for op, relu in (("MatMul", False), ("MatMulRelu", True)):
        y = np.full((M, N), np.nan, np.float32)
        backend.dispatch(op, [um.f32_desc(x), um.packed_desc(W, um.Q4_K, (N, K))], [um.f32_desc(y)],
                         {"transpose_b": True})
        ref = np.where(y_ref > 0, y_ref, np.float32(0)) if relu else y_ref
        assert rel_err(y, ref) <= REL_TOL, op
        if relu:
            assert (y >= 0).all()
    with pytest.raises(um.UaiiMoeError) as e:  # f32 B stays with the backend's own MatMul
        backend.dispatch("MatMul", [um.f32_desc(x), um.f32_desc(np.zeros((N, K), np.float32))],
                         [um.f32_desc(np.empty((M, N), np.float32))], {"transpose_b": True})
    assert e.value.status == 7


def test_quant_matmul_device_buffers_and_registered_weights(backend, oracle, um):
    torch = pytest.importorskip("torch")
    M, K, N = 4, 1408, 256  # Q8_0 rows of 1496 bytes: padded once when registered
    x = um.fill_normal((M, K), 41, 1)
    W = _qrows(um, um.Q8_0, N, K, 41)
    y_ref = oracle.quant_gemm(x, W, um.Q8_0, N)
    xd, Wd = torch.from_numpy(x).cuda(), torch.from_numpy(W).cuda()
    yd = torch.empty((M, N), device="cuda")
    backend.quant_matmul(xd, M, K, Wd, um.Q8_0, N, yd)
    backend.synchronize()
    y0 = yd.cpu().numpy()
    assert rel_err(y0, y_ref) <= REL_TOL
    backend.register_weights(Wd)
    try:
        for _ in range(2):
            backend.quant_matmul(xd, M, K, Wd, um.Q8_0, N, yd)
            backend.synchronize()
            assert bits_equal(yd.cpu().numpy(), y0)
    finally:
        backend.release_weights(Wd)


def test_layer_from_gguf_file_matches_arrays(backend, oracle, um, tmp_path):
    # the MoE layer of a GGUF block, mapped (uaii_moe_gguf_moe_layer), gives the same bits as the
    # same bytes passed as arrays; registered mapped weights are uploaded once
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from test_gguf import _block, _write
    w = _block(um, seed=12)
    path = str(tmp_path / "layer.gguf")
    _write(path, w)
    T = 9
    x = um.fill_normal((T, 256), 5, 1)
    ref_layer = um.make_layer(256, 4, 128, 2, 1, w["router"], w["gate"], um.Q4_K, w["up"], um.Q4_K, w["down"],
                              um.Q8_0, shared=(256, w["gs"], um.Q8_0, w["us"], um.Q8_0, w["ds"], um.Q8_0, None))
    y_ref = np.empty_like(x)
    backend.ffn(ref_layer, x, T, y_ref)
    with um.GgufFile(path) as g:
        L = g.moe_layer(0)
        views = [g.tensor(n)[0] for n in ("blk.0.ffn_gate_inp.weight", "blk.0.ffn_gate_exps.weight",
                                         "blk.0.ffn_up_exps.weight", "blk.0.ffn_down_exps.weight",
                                         "blk.0.ffn_gate_shexp.weight", "blk.0.ffn_up_shexp.weight",
                                         "blk.0.ffn_down_shexp.weight")]
        for v in views:
            backend.register_weights(v)
        try:
            for _ in range(2):
                y = np.empty_like(x)
                backend.ffn(L, x, T, y)
                assert bits_equal(y, y_ref)
        finally:
            for v in views:
                backend.release_weights(v)
    _, pr, _ = oracle.router(x, w["router"])
    y_o, _, _ = oracle.experts_packed(x, w["gate"], um.Q4_K, w["up"], um.Q4_K, w["down"], um.Q8_0, pr, 4, 128, 2, 1)
    oracle.shared_packed(x, w["gs"], um.Q8_0, w["us"], um.Q8_0, w["ds"], um.Q8_0, None, 256, y_o)
    assert rel_err(y_ref, y_o) <= REL_TOL


def test_graph_replay_matches_launches(backend, um):
    # repeated device-resident calls are captured into a CUDA graph and replayed; replays read
    # the buffers' current contents and give the same bits as plain launches
    torch = pytest.importorskip("torch")
    T, D, E, I, k = 3, 1024, 8, 2048, 2
    x, w, G, U, Dn = layer_case(um, 14, 16, T, D, E, I, k, 44)
    dev = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (w, G, U, Dn)]
    L = um.make_layer(D, E, I, k, 1, dev[0], dev[1], um.Q4_K, dev[2], um.Q4_K, dev[3], um.Q6_K)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty((T, D), device="cuda")
    backend.set_graphs(False)
    try:
        backend.ffn(L, xd, T, yd)
        backend.synchronize()
        y_plain = yd.cpu().numpy().copy()
        xd2 = torch.from_numpy(um.fill_normal((T, D), 45, 1)).cuda()
        backend.ffn(L, xd2, T, yd)
        backend.synchronize()
        y_plain2 = yd.cpu().numpy().copy()
    finally:
        backend.set_graphs(True)
    xg = torch.empty_like(xd)
    for i in range(5):  # plain, capture, replays
        xg.copy_(xd if i % 2 == 0 else xd2)
        torch.cuda.synchronize()
        backend.ffn(L, xg, T, yd)
        backend.synchronize()
        assert bits_equal(yd.cpu().numpy(), y_plain if i % 2 == 0 else y_plain2), i


@pytest.mark.parametrize("T,D,E,k", [(1, 64, 8, 2), (37, 256, 16, 4), (300, 512, 60, 4), (64, 2048, 128, 8)])
def test_route_assignments_bitwise(backend, oracle, um, T, D, E, k):
    # the fused layer's token -> expert assignment equals the reference procedure on the
    # reference probabilities, including exact ties (duplicated router rows)
    x = um.fill_normal((T, D), 50 + E, 1)
    w = um.fill_normal((E, D), 50 + E, 2, 0.0, 0.05)
    w[E // 2] = w[1]  # experts with identical logits: the heap procedure orders the tie
    w[E - 1] = w[2]
    for norm in (1, 0):
        ids = np.empty((T, k), np.int32)
        wts = np.empty((T, k), np.float32)
        backend.route(x, w, T, D, E, k, norm, ids, wts)
        _, pr, _ = oracle.router(x, w)
        for t in range(T):
            ref_ids, ref_w = oracle.topk(pr[t], k, norm)
            assert np.array_equal(ids[t], ref_ids), (t, ids[t], ref_ids)
            assert rel_err(wts[t], ref_w) <= 4e-7


@pytest.mark.parametrize("T", [4096, 7000])
def test_ffn_host_buffers_in_overlapped_chunks(backend, oracle, um, T):
    """Host x and y with device-resident weights: the batch runs in chunks of at least 2048
    tokens whose host copies overlap the neighbouring chunks' layer work.  Token rows are
    independent, so the probabilities must equal the one-shot device call bit for bit and
    the outputs must agree within f32 regrouping (a chunk's plan may pick other down-
    projection splits, which regroups f32 sums); sampled rows are checked against the oracle."""
    D, E, I, k = 1024, 8, 1024, 2
    x, w, G, U, Dn = layer_case(um, 14, 16, T, D, E, I, k, 21)
    xd, wd, Gd, Ud, Dd = (dev(a) for a in (x, w, G, U, Dn))
    Ld = um.make_layer(D, E, I, k, 1, wd, Gd, 14, Ud, 14, Dd, 16)
    y_dev = torch.empty((T, D), device="cuda")
    p_dev = torch.empty((T, E), device="cuda")
    backend.ffn(Ld, xd, T, y_dev, p_dev)
    backend.synchronize()
    xh = torch.from_numpy(x).pin_memory()
    yh = torch.full((T, D), float("nan")).pin_memory()
    ph = torch.full((T, E), float("nan")).pin_memory()
    for _ in range(2):  # the second call finds the first call's streams and staging in place
        backend.ffn(Ld, xh, T, yh, ph)
        assert bits_equal(ph.numpy(), p_dev.cpu().numpy())
        assert rel_err(yh.numpy(), y_dev.cpu().numpy()) <= 1e-5
    rows = np.sort(np.random.default_rng(T).choice(T, size=6, replace=False))
    _, pr, _ = oracle.router(np.ascontiguousarray(x[rows]), w)
    y_ref, _, _ = oracle.experts_packed(np.ascontiguousarray(x[rows]), G, 14, U, 14, Dn, 16, pr, E, I, k, 1)
    assert rel_err(yh.numpy()[rows], y_ref) <= REL_TOL
