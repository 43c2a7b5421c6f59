"""Batched greedy decode on the device (uaii_moe_decoder_*) against the reference.

The oracle is the reference's own kernels (oracle/_ref: embedding_f32, rmsnorm_f32,
quant_gemm_f32, rope_f32, attention_kv_f32, moe_router_f32, softmax_f32) composed in the
order of the seq-1 transformer graph its GGUF loader builds
(libs/uaii-loaders/src/gguf.cpp:905-1210), with the MoE experts from the oracle
restatement pinned to moe_experts_swiglu_f32, run for a batch of sequences at one
position per step (rows are independent, so a batch is the reference's batch-1 run
repeated).  The cache is prefilled with the same f16-representable K/V values on both
sides; positions decoded afterwards stay f32 in the reference and f16 on the device.

Bars: logits within 5e-3 of the largest logit per step (f16 tensor-core operands and
an f16 KV cache against f32 throughout); the greedy token equal to the reference's
wherever the reference's top-two margin exceeds twice the observed logit error.
Teacher forcing: both sides consume the reference's tokens, so one close call cannot
derail the rest of the run.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

NL, D, H, HKV, HD, E, TOPK, I, V, B, S0, STEPS = 2, 512, 8, 2, 128, 4, 2, 512, 1024, 3, 5, 3
THETA, EPS = 1e6, 1e-5
LOGIT_TOL = 5e-3


def _weights(um):
    seed = 41
    f = lambda shape, stream, std=0.05, mean=0.0: um.fill_normal(shape, seed, stream, mean, std)
    q = lambda fmt, a: um.quantize_rows(fmt, a)
    W = {"emb": q(um.Q8_0, f((V, D), 1)), "out_norm": f((D,), 2, 0.1, 1.0), "blocks": []}
    for l in range(NL):
        s = 100 * (l + 1)
        W["blocks"].append({
            "attn_norm": f((D,), s + 1, 0.1, 1.0), "ffn_norm": f((D,), s + 2, 0.1, 1.0),
            "wq": q(um.Q8_0, f((H * HD, D), s + 3)), "wk": q(um.Q8_0, f((HKV * HD, D), s + 4)),
            "wv": q(um.Q8_0, f((HKV * HD, D), s + 5)), "wo": q(um.Q8_0, f((D, H * HD), s + 6)),
            "router": f((E, D), s + 7), "gate": q(um.Q4_K, f((E * I, D), s + 8)),
            "up": q(um.Q4_K, f((E * I, D), s + 9)), "down": q(um.Q6_K, f((E * D, I), s + 10))})
    # prefilled cache, f16-representable: [layer] -> [B, HKV, S0, HD]
    kv = [(f((B, HKV, S0, HD), s, 1.0).astype(np.float16).astype(np.float32),
           f((B, HKV, S0, HD), s + 1, 1.0).astype(np.float16).astype(np.float32)) for s in (500, 600)]
    return W, kv


def _device_decoder(um, backend, W, kv, max_seq):
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    blocks, keep = [], []
    for b in W["blocks"]:
        d = {k: dev(v) for k, v in b.items()}
        keep.append(d)
        moe = um.make_layer(D, E, I, TOPK, 1, d["router"], d["gate"], um.Q4_K, d["up"], um.Q4_K, d["down"], um.Q6_K)
        blocks.append({"attn_norm": d["attn_norm"], "ffn_norm": d["ffn_norm"], "wq": d["wq"], "wq_fmt": um.Q8_0,
                       "wk": d["wk"], "wk_fmt": um.Q8_0, "wv": d["wv"], "wv_fmt": um.Q8_0, "wo": d["wo"],
                       "wo_fmt": um.Q8_0, "moe": moe})
    emb, out_norm = dev(W["emb"]), dev(W["out_norm"])
    dec = um.Decoder(backend, NL, D, H, HKV, V, B, max_seq, blocks, out_norm, emb, um.Q8_0, rope_theta=THETA,
                     rms_eps=EPS)
    dec._keep.append(keep)
    for l, (k, v) in enumerate(kv):
        dec.set_kv(l, k, v, S0)
    return dec


def _reference_step(ref, oracle, um, W, tokens, pos, past):
    x = ref.embedding(tokens, W["emb"], um.Q8_0, V, D)
    posv = np.full(B, pos, np.float32)
    for l, b in enumerate(W["blocks"]):
        n = ref.rmsnorm(x, b["attn_norm"], EPS)
        q = ref.rope(ref.quant_gemm(n, b["wq"], um.Q8_0, H * HD), posv, THETA, HD, 0)
        k = ref.rope(ref.quant_gemm(n, b["wk"], um.Q8_0, HKV * HD), posv, THETA, HD, 0)
        v = ref.quant_gemm(n, b["wv"], um.Q8_0, HKV * HD)
        pk, pv = past[l]
        a = ref.attention_kv(q, k, v, H, pk, pv)
        past[l] = (np.ascontiguousarray(np.concatenate([pk, k[:, None, :]], axis=1)),
                   np.ascontiguousarray(np.concatenate([pv, v[:, None, :]], axis=1)))
        x = (x + ref.quant_gemm(a, b["wo"], um.Q8_0, D)).astype(np.float32)
        n2 = ref.rmsnorm(x, b["ffn_norm"], EPS)
        probs, _ = ref.router(n2, b["router"])
        ff, _, _ = oracle.experts_packed(n2, b["gate"], um.Q4_K, b["up"], um.Q4_K, b["down"], um.Q6_K, probs, E, I,
                                         TOPK, 1)
        x = (x + ff).astype(np.float32)
    logits = ref.quant_gemm(ref.rmsnorm(x, W["out_norm"], EPS), W["emb"], um.Q8_0, V)
    return logits, ref.softmax(logits).argmax(axis=1).astype(np.int32)  # first index of the maximum


def test_decoder_matches_reference_graph(um, backend, oracle, reference):
    W, kv = _weights(um)
    dec = _device_decoder(um, backend, W, kv, S0 + STEPS)
    # reference cache layout: [B, positions, n_kv_heads * head_dim]
    past = [tuple(np.ascontiguousarray(a.transpose(0, 2, 1, 3).reshape(B, S0, HKV * HD)) for a in pair)
            for pair in kv]
    tokens = np.random.default_rng(7).integers(0, V, size=B).astype(np.int32)
    try:
        for s in range(STEPS):
            assert dec.position == S0 + s
            logits = np.empty((B, V), np.float32)
            nxt = np.empty(B, np.int32)
            dec.step(tokens, logits, nxt)
            ref_logits, ref_next = _reference_step(reference, oracle, um, W, tokens, S0 + s, past)
            scale = float(np.abs(ref_logits).max())
            err = float(np.abs(logits.astype(np.float64) - ref_logits).max())
            assert err <= LOGIT_TOL * scale, (s, err / scale)
            assert np.array_equal(nxt, logits.argmax(axis=1))
            top2 = np.sort(ref_logits, axis=1)[:, -2:]
            clear = (top2[:, 1] - top2[:, 0]) > 2 * err
            assert np.array_equal(nxt[clear], ref_next[clear]), (s, nxt, ref_next)
            tokens = ref_next  # teacher forcing
    finally:
        dec.close()


def test_decoder_generate_equals_stepping(um, backend):
    W, kv = _weights(um)
    tokens = np.random.default_rng(8).integers(0, V, size=B).astype(np.int32)
    a = _device_decoder(um, backend, W, kv, S0 + 4)
    b = _device_decoder(um, backend, W, kv, S0 + 4)
    try:
        out = np.empty((4, B), np.int32)
        a.generate(tokens, 4, out)
        assert a.position == S0 + 4
        t = tokens
        for s in range(4):
            nxt = np.empty(B, np.int32)
            b.step(t, None, nxt)
            assert np.array_equal(nxt, out[s]), s
            t = nxt
        with pytest.raises(um.UaiiMoeError):  # the cache holds S0 + 4 positions
            a.step(tokens, None, np.empty(B, np.int32))
    finally:
        a.close()
        b.close()


def test_decoder_rejects_bad_tokens_and_config(um, backend):
    W, kv = _weights(um)
    dec = _device_decoder(um, backend, W, kv, S0 + 2)
    try:
        with pytest.raises(um.UaiiMoeError) as e:
            dec.step(np.array([0, V, 1], np.int32), None, np.empty(B, np.int32))
        assert e.value.status == 1 and "token" in e.value.message
    finally:
        dec.close()
    with pytest.raises(um.UaiiMoeError) as e:  # head_dim other than 128
        um.Decoder(backend, 1, D, H, HKV, V, B, 8, [], torch.zeros(D, device="cuda"),
                   torch.zeros(8, device="cuda"), um.Q8_0, head_dim=64)
    assert e.value.status == 1


def test_device_synthetic_inputs_match_host(um, backend):
    n = 1 << 20
    x = torch.empty(n, device="cuda")
    um.fill_normal_device(backend, x, 5, 9, 0.0, 0.02)
    backend.synchronize()
    host = um.fill_normal((n,), 5, 9, 0.0, 0.02)
    diff = x.cpu().numpy().view(np.uint32).astype(np.int64) - host.view(np.uint32).astype(np.int64)
    assert np.abs(diff).max() <= 1 and np.count_nonzero(diff) <= n // 100000
    src = host.reshape(1024, 1024)
    src_d = torch.from_numpy(src).cuda()
    for fmt in (um.Q4_0, um.Q8_0, um.Q4_K, um.Q6_K):
        dst = torch.empty((1024, um.packed_nbytes(fmt, 1024)), dtype=torch.uint8, device="cuda")
        um.quantize_rows_device(backend, fmt, src_d, dst)
        backend.synchronize()
        assert np.array_equal(dst.cpu().numpy(), um.quantize_rows(fmt, src)), fmt


def test_decoder_matches_the_reference_session_generate(um, backend, tmp_path):
    """The f1 oracle of the reference itself: its unmodified Session (oracle/_ref runtime build)
    loads a GGUF file of a 2-layer Mixtral-shaped model, prefills a 4-token prompt one token per
    run and generates greedily (tests/reference_decoder_session.py, a child process, CPU).  The
    device decoder gets the same packed tensors, steps through the same prompt from an empty cache
    (two identical sequences in the batch) and, teacher forced with the reference's tokens, must
    give logits within LOGIT_TOL of the largest logit at every generated position and the same
    greedy token wherever the reference's top-two margin exceeds twice the observed error."""
    so = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                      "libuaii_ref_runtime.so")
    if not os.path.exists(so):
        pytest.skip("reference runtime not built")
    helper = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_decoder_session.py")
    p = subprocess.run([sys.executable, helper, str(tmp_path)], capture_output=True, text=True, timeout=600)
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert p.returncode == 0 and lines, p.stderr[-2000:]
    ref = json.loads(lines[-1])
    W = dict(np.load(tmp_path / "weights.npz"))
    nl, hd, steps = 2, 128, len(ref["tokens"])
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    blocks, keep = [], []
    for l in range(nl):
        g = lambda n: dev(W[f"blk.{l}.{n}.weight"])
        d = {n: g(n) for n in ("attn_norm", "ffn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate_inp",
                               "ffn_gate_exps", "ffn_up_exps", "ffn_down_exps")}
        keep.append(d)
        moe = um.make_layer(D, E, I, TOPK, 1, d["ffn_gate_inp"], d["ffn_gate_exps"], um.Q4_K, d["ffn_up_exps"],
                            um.Q4_K, d["ffn_down_exps"], um.Q6_K)
        blocks.append({"attn_norm": d["attn_norm"], "ffn_norm": d["ffn_norm"], "wq": d["attn_q"], "wq_fmt": um.Q8_0,
                       "wk": d["attn_k"], "wk_fmt": um.Q8_0, "wv": d["attn_v"], "wv_fmt": um.Q8_0,
                       "wo": d["attn_output"], "wo_fmt": um.Q8_0, "moe": moe})
    emb, out_norm = dev(W["token_embd.weight"]), dev(W["output_norm.weight"])
    prompt = ref["prompt"]
    dec = um.Decoder(backend, nl, D, H, HKV, V, 2, len(prompt) + steps, blocks, out_norm, emb, um.Q8_0,
                     rope_theta=THETA, rms_eps=EPS, head_dim=hd)
    dec._keep.append(keep)
    try:
        for t in prompt[:-1]:  # positions 0 .. P-2
            dec.step(np.array([t, t], np.int32), None, np.empty(2, np.int32))
        tok = prompt[-1]
        for j in range(steps):
            logits = np.empty((2, V), np.float32)
            nxt = np.empty(2, np.int32)
            dec.step(np.array([tok, tok], np.int32), logits, nxt)
            r = np.asarray(ref["logits"][j], np.float64)
            scale = float(np.abs(r).max())
            err = float(np.abs(logits.astype(np.float64) - r[None, :]).max())
            assert err <= LOGIT_TOL * scale, (j, err / scale)
            assert np.array_equal(logits[0], logits[1])
            top2 = np.sort(r)[-2:]
            if top2[1] - top2[0] > 2 * err:
                assert int(nxt[0]) == ref["tokens"][j], (j, int(nxt[0]), ref["tokens"][j])
            tok = ref["tokens"][j]  # teacher forcing
    finally:
        dec.close()
