"""The reference's own Session decoding a small Mixtral-shaped GGUF model (the f1 oracle).

    python tests/reference_decoder_session.py OUT_DIR

Writes OUT_DIR/model.gguf (llama architecture, MoE blocks: router f32, experts Q4_K/Q4_K/Q6_K,
attention and the tied embedding Q8_0) and OUT_DIR/weights.npz (the same arrays), then runs the
unmodified reference runtime (oracle/_ref/libuaii_ref_runtime.so): the GGUF loader builds its
seq-1 graph (libs/uaii-loaders/src/gguf.cpp:905-1210) and Session::generate (session.cpp:910-1046)
prefills the prompt one token per run into its batch-1 KV cache and samples greedily.  One
generate call per step, teacher forced: step j generates one token after prompt + the reference's
own tokens so far, and the logits tensor then holds the scores of that last position.  Prints one
JSON line {prompt, tokens, logits}.  CPU only (the reference runs its host kernels; weights are
dequantized to f32 at load, the default options).
"""
from __future__ import annotations

import ctypes
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)

from gguf_writer import (F32 as KV_F32, STRING, U32, GGML_F32, GGML_Q4_K, GGML_Q6_K, GGML_Q8_0,  # noqa: E402
                         write_gguf)
from oracle import synth  # noqa: E402

RUNTIME_SO = os.path.join(REPO, "oracle", "_ref", "libuaii_ref_runtime.so")
NL, D, H, HKV, HD, E, TOPK, I, V = 2, 512, 8, 2, 128, 4, 2, 512, 1024
THETA, EPS, CTX = 1e6, 1e-5, 64
Q8_0, Q4_K, Q6_K = 11, 14, 16
PROMPT = [17, 400, 3, 999]
STEPS = 4


def weights(seed: int = 43):
    f = lambda shape, stream, std=0.05, mean=0.0: synth.fill_normal(shape, seed, stream, mean, std)
    q = synth.quantize_rows
    W = {"token_embd.weight": q(Q8_0, f((V, D), 1)), "output_norm.weight": f((D,), 2, 0.1, 1.0)}
    for l in range(NL):
        s, p = 100 * (l + 1), f"blk.{l}."
        W[p + "attn_norm.weight"] = f((D,), s + 1, 0.1, 1.0)
        W[p + "ffn_norm.weight"] = f((D,), s + 2, 0.1, 1.0)
        W[p + "attn_q.weight"] = q(Q8_0, f((H * HD, D), s + 3))
        W[p + "attn_k.weight"] = q(Q8_0, f((HKV * HD, D), s + 4))
        W[p + "attn_v.weight"] = q(Q8_0, f((HKV * HD, D), s + 5))
        W[p + "attn_output.weight"] = q(Q8_0, f((D, H * HD), s + 6))
        W[p + "ffn_gate_inp.weight"] = f((E, D), s + 7)
        W[p + "ffn_gate_exps.weight"] = q(Q4_K, f((E * I, D), s + 8))
        W[p + "ffn_up_exps.weight"] = q(Q4_K, f((E * I, D), s + 9))
        W[p + "ffn_down_exps.weight"] = q(Q6_K, f((E * D, I), s + 10))
    return W


def write_model(path: str, W) -> None:
    shapes = {"token_embd.weight": (V, D), "output_norm.weight": (D,)}
    types = {"token_embd.weight": GGML_Q8_0, "output_norm.weight": GGML_F32}
    for l in range(NL):
        p = f"blk.{l}."
        shapes.update({p + "attn_norm.weight": (D,), p + "ffn_norm.weight": (D,), p + "attn_q.weight": (H * HD, D),
                       p + "attn_k.weight": (HKV * HD, D), p + "attn_v.weight": (HKV * HD, D),
                       p + "attn_output.weight": (D, H * HD), p + "ffn_gate_inp.weight": (E, D),
                       p + "ffn_gate_exps.weight": (E, I, D), p + "ffn_up_exps.weight": (E, I, D),
                       p + "ffn_down_exps.weight": (E, D, I)})
        types.update({p + "attn_norm.weight": GGML_F32, p + "ffn_norm.weight": GGML_F32,
                      p + "attn_q.weight": GGML_Q8_0, p + "attn_k.weight": GGML_Q8_0, p + "attn_v.weight": GGML_Q8_0,
                      p + "attn_output.weight": GGML_Q8_0, p + "ffn_gate_inp.weight": GGML_F32,
                      p + "ffn_gate_exps.weight": GGML_Q4_K, p + "ffn_up_exps.weight": GGML_Q4_K,
                      p + "ffn_down_exps.weight": GGML_Q6_K})
    kv = [("general.architecture", STRING, "llama"), ("general.name", STRING, "uaii-b200-f1-check"),
          ("llama.block_count", U32, NL), ("llama.context_length", U32, CTX), ("llama.embedding_length", U32, D),
          ("llama.attention.head_count", U32, H), ("llama.attention.head_count_kv", U32, HKV),
          ("llama.attention.key_length", U32, HD), ("llama.attention.value_length", U32, HD),
          ("llama.rope.freq_base", KV_F32, THETA), ("llama.attention.layer_norm_rms_epsilon", KV_F32, EPS),
          ("llama.expert_count", U32, E), ("llama.expert_used_count", U32, TOPK)]
    write_gguf(path, kv, [(n, types[n], shapes[n], np.ascontiguousarray(a).tobytes()) for n, a in W.items()])


def main() -> None:
    out_dir = sys.argv[1]
    W = weights()
    np.savez(os.path.join(out_dir, "weights.npz"), **W)
    model = os.path.join(out_dir, "model.gguf")
    write_model(model, W)
    rt = ctypes.CDLL(RUNTIME_SO, mode=ctypes.RTLD_GLOBAL)
    vp, cp, i32, sz = ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_size_t
    for name, res, args in (("urt_last_error", cp, []), ("urt_session_create", i32, [cp, cp, cp, i32, i32, vp]),
                            ("urt_session_destroy", None, [vp]), ("urt_session_get_f32", i32, [vp, cp, vp, sz, vp]),
                            ("urt_session_generate", i32, [vp, vp, sz, ctypes.c_int64, vp, sz, vp])):
        fn = getattr(rt, name)
        fn.restype, fn.argtypes = res, args
    sess = ctypes.c_void_p()
    st = rt.urt_session_create(model.encode(), b"cpu", None, 1, 1, ctypes.byref(sess))
    assert st == 0, rt.urt_last_error()
    seq = list(PROMPT)
    tokens, logits = [], []
    n = ctypes.c_size_t()
    for _ in range(STEPS):
        p = np.array(seq, np.int64)
        out = np.zeros(len(seq) + 1, np.int64)
        st = rt.urt_session_generate(sess, p.ctypes.data, len(seq), 1, out.ctypes.data, out.size, ctypes.byref(n))
        assert st == 0 and n.value == len(seq) + 1, rt.urt_last_error()
        lg = np.empty(V, np.float32)
        assert rt.urt_session_get_f32(sess, b"logits", lg.ctypes.data, V, ctypes.byref(n)) == 0 and n.value == V
        tokens.append(int(out[-1]))
        logits.append(lg.tolist())
        seq.append(int(out[-1]))
    rt.urt_session_destroy(sess)
    print(json.dumps({"prompt": PROMPT, "tokens": tokens, "logits": logits}))


if __name__ == "__main__":
    main()
