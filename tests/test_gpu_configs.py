"""The benchmark configurations at full size, against the oracle.

Every configuration runs on the device with its full token count (the same
seeded synthetic layer and tokens as bench.py).  The oracle then recomputes a
seeded sample of rows on the host: each row's result depends only on that row
(the reference's GEMMs tile over rows only), so a sampled row must equal the
row of the full-batch device result.  Bars: routing probabilities within
4e-7 relative, the layer output within 2e-3 max relative over the sampled rows
(f16 tensor-core operands, f32 accumulate).

Every row of the batch is then checked too: the same layer is run again on the
CUDA-core schedule (f32 dequant and f32 products, ~1e-6 from the oracle, which
these tests confirm on the sampled rows), and the tensor-core output must be
within the 2e-3 bar of it over the WHOLE batch -- so a fault confined to some
slot tiles (an expert's last partial tile, a 256-slot accumulator drain, one K
split) cannot hide between the sampled rows.  Size-independent properties are
checked on the whole batch as well: outputs finite, and for renormalised top-k
the probabilities of every token sum to one.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

REL_TOL = 2e-3
PROB_TOL = 4e-7
SIMT_TOL = 1e-5  # CUDA-core f32 path against the oracle (same products, different summation order)


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


_CACHE = {}


def _weights(name):
    from uaii_moe.synthetic import CONFIGS, make_layer_weights
    if name not in _CACHE:
        _CACHE.clear()  # one full-size layer on the host at a time
        _CACHE[name] = make_layer_weights(CONFIGS[name])
    return _CACHE[name]


@pytest.mark.parametrize("name,T,n_check", [
    ("cfg1_q4_0", 64, 64),        # configs[0]: every token
    ("mixtral", 1, 1),            # configs[1], decode
    ("mixtral", 32, 8),
    ("mixtral", 4096, 8),         # prefill (256-slot tiles)
    ("qwen2moe", 4096, 16),       # configs[2]: Zipf routing, no renorm, sigmoid-gated shared expert
    ("qwen3", 16384, 24),         # configs[3]: 128 experts, top-8
    ("qwen3_hot", 16384, 24),     # configs[3] skewed: one 4x hot expert
])
def test_config_full_size_vs_oracle(um, oracle, name, T, n_check):
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    from uaii_moe.synthetic import CONFIGS, make_tokens
    cfg = CONFIGS[name]
    lw = _weights(name)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda() if a is not None else None
    arrays = {"router_w": dev(lw.router_w), "gate": dev(lw.gate), "up": dev(lw.up), "down": dev(lw.down),
              "shared": tuple(dev(a) for a in lw.shared) if lw.shared is not None else None}
    L = lw.layer_struct(arrays)
    x = make_tokens(cfg, T, 0)
    xd = dev(x)
    y = torch.empty((T, cfg.D), device="cuda")
    probs = torch.empty((T, cfg.E), device="cuda")
    y32 = torch.empty((T, cfg.D), device="cuda")
    be = um.Backend(0)
    try:
        be.ffn(L, xd, T, y, probs)
        be.synchronize()
        plan = be.last_plan()
        be.set_expert_path(1)  # the CUDA-core f32 schedule of the same layer, for the whole-batch check
        be.ffn(L, xd, T, y32)
        be.synchronize()
        assert be.last_plan()["tensor_cores"] == 0
    finally:
        be.close()
    y = y.cpu().numpy()
    y32 = y32.cpu().numpy()
    probs = probs.cpu().numpy()
    assert np.isfinite(y).all()
    if cfg.norm_topk:
        np.testing.assert_allclose(probs.sum(axis=1), 1.0, rtol=0, atol=1e-5)
    rows = np.sort(np.random.default_rng(1234 + T).choice(T, size=n_check, replace=False))
    xs = np.ascontiguousarray(x[rows])
    _, pr, _ = oracle.router(xs, lw.router_w)
    assert _rel(probs[rows], pr) <= PROB_TOL
    # token -> expert assignments of the whole batch, checked bit for bit on the sampled rows
    ids = np.empty((T, cfg.top_k), np.int32)
    wts = np.empty((T, cfg.top_k), np.float32)
    be2 = um.Backend(0)
    try:
        be2.route(xd, arrays["router_w"], T, cfg.D, cfg.E, cfg.top_k, cfg.norm_topk, ids, wts)
    finally:
        be2.close()
    for j, r in enumerate(rows):
        ref_ids, ref_w = oracle.topk(pr[j], cfg.top_k, cfg.norm_topk)
        assert np.array_equal(ids[r], ref_ids), (r, ids[r], ref_ids)
        assert _rel(wts[r], ref_w) <= PROB_TOL
    y_ref, _, _ = oracle.experts_packed(xs, lw.gate, cfg.gate_fmt, lw.up, cfg.gate_fmt, lw.down, cfg.down_fmt, pr,
                                        cfg.E, cfg.I, cfg.top_k, cfg.norm_topk)
    if lw.shared is not None:
        g, u, d, gi = lw.shared
        oracle.shared_packed(xs, g, cfg.shared_fmt, u, cfg.shared_fmt, d, cfg.shared_fmt, gi, cfg.I_sh, y_ref)
    assert _rel(y[rows], y_ref) <= REL_TOL
    # the whole batch: the f32 schedule is anchored to the oracle on the sampled rows ...
    assert np.isfinite(y32).all()
    assert _rel(y32[rows], y_ref) <= SIMT_TOL
    # ... and every row of the tensor-core output must meet the bar against it
    err = np.abs(y.astype(np.float64) - y32).max(axis=1) / max(np.abs(y32).max(), 1e-30)
    assert float(err.max()) <= REL_TOL, (plan, int(err.argmax()), float(err.max()))
