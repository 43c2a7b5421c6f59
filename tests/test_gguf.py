"""GGUF files mapped by the library (uaii_moe_gguf_*): parsing, tensor views, the MoE
layer of a block, corrupt-file handling, and agreement with the reference loader
(gguf_read_header / gguf_load_tensor_raw / gguf_write_f32, compiled in oracle/_ref).
CPU only: nothing here touches a device."""
from __future__ import annotations

import os

import numpy as np
import pytest

from gguf_writer import (ARRAY, F32, GGML_F32, GGML_I32, GGML_Q4_0, GGML_Q4_K, GGML_Q6_K, GGML_Q8_0, STRING, U32,
                         as_bytes,
                         write_gguf)

D, E, I, ISH = 256, 4, 128, 256


def _block(um, seed=3):
    rng = np.random.default_rng(seed)
    router = (rng.standard_normal((E, D)) * 0.1).astype(np.float32)
    gate = um.quantize_rows(um.Q4_K, (rng.standard_normal((E * I, D)) * 0.02).astype(np.float32)).reshape(E, I, -1)
    up = um.quantize_rows(um.Q4_K, (rng.standard_normal((E * I, D)) * 0.02).astype(np.float32)).reshape(E, I, -1)
    down = um.quantize_rows(um.Q8_0, (rng.standard_normal((E * D, I)) * 0.02).astype(np.float32)).reshape(E, D, -1)
    gs = um.quantize_rows(um.Q8_0, (rng.standard_normal((ISH, D)) * 0.02).astype(np.float32))
    us = um.quantize_rows(um.Q8_0, (rng.standard_normal((ISH, D)) * 0.02).astype(np.float32))
    ds = um.quantize_rows(um.Q8_0, (rng.standard_normal((D, ISH)) * 0.02).astype(np.float32))
    gi = (rng.standard_normal(D) * 0.1).astype(np.float32)
    return dict(router=router, gate=gate, up=up, down=down, gs=gs, us=us, ds=ds, gi=gi)


def _write(path, w, alignment=32, align_key=False):
    kv = [("general.architecture", STRING, "qwen2moe"),
          ("qwen2moe.expert_count", U32, E),
          ("qwen2moe.expert_used_count", U32, 2),
          ("qwen2moe.rope.freq_base", F32, 1.0e6),
          ("tokenizer.ggml.tokens", ARRAY, (STRING, ["<s>", "</s>", "hello"]))]
    if align_key:
        kv.append(("general.alignment", U32, alignment))
    tensors = [("blk.0.ffn_gate_inp.weight", GGML_F32, (E, D), as_bytes(w["router"])),
               ("blk.0.ffn_gate_exps.weight", GGML_Q4_K, (E, I, D), as_bytes(w["gate"])),
               ("blk.0.ffn_up_exps.weight", GGML_Q4_K, (E, I, D), as_bytes(w["up"])),
               ("blk.0.ffn_down_exps.weight", GGML_Q8_0, (E, D, I), as_bytes(w["down"])),
               ("blk.0.ffn_gate_shexp.weight", GGML_Q8_0, (ISH, D), as_bytes(w["gs"])),
               ("blk.0.ffn_up_shexp.weight", GGML_Q8_0, (ISH, D), as_bytes(w["us"])),
               ("blk.0.ffn_down_shexp.weight", GGML_Q8_0, (D, ISH), as_bytes(w["ds"])),
               ("blk.0.ffn_gate_inp_shexp.weight", GGML_F32, (D,), as_bytes(w["gi"])),
               ("token_types", GGML_I32, (3,), as_bytes(np.arange(3, dtype=np.int32)))]
    return write_gguf(path, kv, tensors, alignment=alignment), tensors


@pytest.mark.parametrize("alignment,align_key", [(32, False), (64, True)])
def test_gguf_tensors_metadata_and_moe_layer(um, tmp_path, alignment, align_key):
    w = _block(um)
    path = str(tmp_path / "moe.gguf")
    _, tensors = _write(path, w, alignment, align_key)
    with um.GgufFile(path) as g:
        listed = g.tensors()
        assert [t[0] for t in listed] == [t[0] for t in tensors]
        for (name, fmt, shape, nbytes), (_, gt, shp, data) in zip(listed, tensors):
            assert shape == tuple(shp), name
            if gt == GGML_I32:
                assert fmt == -1
                continue
            view, fmt2, _ = g.tensor(name)
            assert fmt2 == fmt and nbytes == len(data) and view.tobytes() == data, name
        assert g.kv_str("general.architecture") == "qwen2moe"
        assert g.kv_int("qwen2moe.expert_count") == E
        assert g.kv_float("qwen2moe.rope.freq_base") == 1.0e6
        with pytest.raises(um.UaiiMoeError) as e:
            g.kv_int("tokenizer.ggml.tokens")  # arrays are skipped, not integers
        assert e.value.status == um.NOT_FOUND
        L = g.moe_layer(0)
        assert (L.d_model, L.n_experts, L.d_ff, L.top_k, L.norm_topk) == (D, E, I, 2, 1)
        assert (L.gate_fmt, L.up_fmt, L.down_fmt) == (um.Q4_K, um.Q4_K, um.Q8_0)
        assert L.router_w == g.tensor("blk.0.ffn_gate_inp.weight")[0].ctypes.data
        assert L.down_exps == g.tensor("blk.0.ffn_down_exps.weight")[0].ctypes.data
        assert L.shared_d_ff == ISH and L.gate_shexp_fmt == um.Q8_0
        assert not L.gate_inp_shexp  # the reference's graph adds the shared expert ungated
        Lg = g.moe_layer(0, shexp_gate=True)
        assert Lg.gate_inp_shexp == g.tensor("blk.0.ffn_gate_inp_shexp.weight")[0].ctypes.data
        with pytest.raises(um.UaiiMoeError) as e:
            g.moe_layer(1)
        assert e.value.status == um.NOT_FOUND


def test_gguf_rejects_corrupt_files(um, tmp_path):
    w = _block(um)
    path = str(tmp_path / "ok.gguf")
    _write(path, w)
    raw = open(path, "rb").read()
    cases = {"magic": b"GGUX" + raw[4:], "version": raw[:4] + b"\x01\0\0\0" + raw[8:]}
    for cut in (10, 24, 40, 200, 800, len(raw) - 100):  # header, metadata, tensor index, data
        cases[f"cut{cut}"] = raw[:cut]
    for name, data in cases.items():
        p = str(tmp_path / f"{name}.gguf")
        open(p, "wb").write(data)
        with pytest.raises(um.UaiiMoeError) as e:
            um.GgufFile(p)
        assert e.value.status == um.INVALID_ARGUMENT, name
    with pytest.raises(um.UaiiMoeError) as e:
        um.GgufFile(str(tmp_path / "missing.gguf"))
    assert e.value.status == um.NOT_FOUND


def test_gguf_matches_reference_loader(um, reference, tmp_path):
    w = _block(um, seed=8)
    path = str(tmp_path / "ref.gguf")
    _, tensors = _write(path, w)  # alignment 32: the reference's fixed data alignment
    with um.GgufFile(path) as g:
        for name, gt, shape, data in tensors:
            if gt == GGML_I32:
                continue  # the reference's type table has no I32 at ggml's number
            rbytes, rshape, rtype = reference.gguf_tensor_raw(path, name, len(data) + 64)
            view, fmt, shp = g.tensor(name)
            assert rtype == gt and rshape == shp and rbytes.tobytes() == view.tobytes(), name


def test_gguf_reads_reference_writer_output(um, reference, tmp_path):
    rng = np.random.default_rng(1)
    a = rng.standard_normal((3, 5)).astype(np.float32)
    b = rng.standard_normal((2, 4, 8)).astype(np.float32)
    path = str(tmp_path / "written_by_reference.gguf")
    reference.gguf_write_f32(path, [("a", a), ("blk.0.b", b)])
    with um.GgufFile(path) as g:
        assert g.kv_int("llama.expert_count") == 4
        for name, arr in (("a", a), ("blk.0.b", b)):
            view, fmt, shape = g.tensor(name)
            assert fmt == um.F32 and shape == arr.shape
            assert np.array_equal(view.view(np.float32).reshape(arr.shape), arr)


def test_reference_session_q4_0_load_order_differs_by_interleave(um, reference, oracle, tmp_path):
    """Pins the reference discrepancy this library records and does not replicate: the
    stock Session dequantizes Q4_0 at load time with gguf_load_tensor_f32, which writes the
    two nibbles of byte j to elements 2j and 2j+1 (libs/uaii-loaders/src/gguf.cpp:514-520),
    while dequant_gguf_row -- the GGUF/ggml order this library and the oracle follow -- puts
    them at j and j+16 (libs/uaii-quant/src/gguf_dequant.cpp:126-131).  Both run here
    through the reference build; they must differ by exactly that permutation.  Q8_0 and
    the K-quants load identically through both routes."""
    rows, cols = 6, 256
    src = um.fill_normal((rows, cols), 3, 1, 0.0, 0.02)
    path = str(tmp_path / "q.gguf")
    tensors = []
    packed = {}
    for fmt, gt in ((um.Q4_0, GGML_Q4_0), (um.Q8_0, GGML_Q8_0), (um.Q4_K, GGML_Q4_K), (um.Q6_K, GGML_Q6_K)):
        packed[fmt] = um.quantize_rows(fmt, src)
        tensors.append((f"t{fmt}", gt, (rows, cols), packed[fmt].tobytes()))
    write_gguf(path, [("general.architecture", STRING, "llama")], tensors)
    for fmt in packed:
        loaded = reference.gguf_tensor_f32(path, f"t{fmt}", rows * cols).reshape(rows, cols)
        row_order = reference.dequant(fmt, packed[fmt], rows, cols, packed[fmt].shape[1])
        assert np.array_equal(row_order, oracle.dequant(fmt, packed[fmt], rows, cols))
        if fmt != um.Q4_0:
            assert np.array_equal(loaded.view(np.uint32), row_order.view(np.uint32)), fmt
            continue
        assert not np.array_equal(loaded, row_order)
        blocks = row_order.reshape(-1, 2, 16)            # [block][lo/hi nibble][byte j]
        interleaved = blocks.transpose(0, 2, 1).reshape(rows, cols)  # element 2j = lo(j), 2j+1 = hi(j)
        assert np.array_equal(loaded.view(np.uint32), interleaved.view(np.uint32))
