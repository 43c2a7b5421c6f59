#!/usr/bin/env python
"""MoE FFN tokens/s on B200 -- one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config mixtral] [--tokens 4096]

A step is one forward of one MoE FFN layer (router -> top-k -> permute ->
gate/up/SwiGLU -> down -> weighted combine) over `--tokens` tokens per GPU,
through the library's C ABI (uaii_moe_ffn_forward).  Weights are the seeded
synthetic GGUF layer of the chosen configuration (random-init, quantized by the
library); activations are seeded N(0,1).  Under torchrun every rank runs its
own replica of the layer on its own tokens (weak scaling, no data-path
collective); the step time is the max over ranks.

`value`: tokens/s with inputs resident in HBM.  `e2e`: the same metric through
the same call with pinned HOST buffers, so every step includes the host->device
copy of x and the device->host copy of y.  `--impl reference` times the
reference's own CPU implementation (oracle/_ref, or the oracle restatement
where that build is absent) on a bounded token sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "universal-ai-inference_b200"))

import numpy as np  # noqa: E402

METRIC = "MoE FFN tokens/s"
UNIT = "tokens/s"
WORKLOAD_NOTE = {
    "mixtral": "Mixtral-8x7B-shaped MoE FFN layer (BASELINE configs[1]): d_model 4096, 8 experts, top-2 "
               "renormalised, d_ff 14336, gate/up Q4_K, down Q6_K",
    "cfg1_q4_0": "config 1 layer: d_model 1024, 8 experts, top-2, d_ff 2816, Q4_0",
    "qwen2moe": "Qwen2-MoE-A2.7B-shaped layer: d_model 2048, 60 experts top-4 (no renorm), d_ff 1408, "
                "shared d_ff 5632 with sigmoid gate, Q8_0, Zipf(1.1) routing",
    "qwen3": "Qwen3-30B-A3B-shaped layer: d_model 2048, 128 experts top-8, d_ff 768, Q4_0",
    "qwen3_hot": "Qwen3-30B-A3B-shaped layer with a 4x hot expert",
}
# DRAM bytes (read + write) per launch of the dominant kernel, from one ncu capture of the same
# command (dram__bytes_read.sum + dram__bytes_write.sum); absent workloads report null.
NCU_TRAFFIC = {
    ("mixtral_T1", "gateup"): 132193536 + 5757184,
    ("mixtral_T1", "down"): 98642688 + 452608,
    ("mixtral_T8", "gateup"): 462690304 + 4268544,
    ("mixtral_T8", "down"): 346857728 + 846592,
    ("mixtral_T32", "gateup"): 529084672 + 5518336,
    ("mixtral_T32", "down"): 398761984 + 4418304,
    ("mixtral_T4096", "gateup"): 601846784 + 218835200,
    ("mixtral_T4096", "down"): 930714112 + 116809728,
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="mixtral")
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"],
                    help="weak: --tokens per GPU; strong: --tokens in total, split across the GPUs")
    ap.add_argument("--path", type=int, default=0,
                    help="0 auto, 1 CUDA-core GEMV, 2 tcgen05 tensor-core GEMM, 3 warp-MMA tensor-core GEMM "
                         "(whole super-blocks for K-quants), 4 warp-MMA with one 32-element unit per lane, "
                         "5 auto with the Q4_K quad gate/up on f16 instead of 16-bit integer activations")
    ap.add_argument("--ep-chunks", type=int, default=1,
                    help="N > 1: token chunks whose exchanges overlap the previous chunk's experts")
    ap.add_argument("--no-graphs", action="store_true", help="plain launches instead of CUDA-graph replay")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--layers", type=int, default=32, help="mixtral_decode: transformer blocks")
    return ap.parse_args()


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained", p["bf16_tflops"]), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


class ClockSampler:
    """SM clock and clock-event (throttle) reasons read through NVML every 2 ms
    while the timed region runs (read-only queries)."""
    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device_index: int):
        self.dev = device_index
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self.err = None
        self._stop = None
        self._thread = None

    def _handle(self, nv):
        try:  # the CUDA device's NVML handle by PCI bus id (CUDA_VISIBLE_DEVICES may remap indices)
            import torch
            pr = torch.cuda.get_device_properties(self.dev)
            bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
            return nv.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:  # noqa: BLE001
            return nv.nvmlDeviceGetHandleByIndex(self.dev)

    def __enter__(self):
        import threading
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = self._handle(nv)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        except Exception as e:  # noqa: BLE001
            self.err = f"NVML unavailable: {type(e).__name__}"
            return self
        self._stop = threading.Event()
        self._nv, self._h = nv, h

        def run():
            while not self._stop.is_set():
                self.sample_now()
                self._stop.wait(0.002)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()
        return self

    def sample_now(self):
        """One reading (also called from the timing thread while queued work runs, so a
        short timed region has at least one sample under load)."""
        if self._stop is None:
            return
        nv, h = self._nv, self._h
        try:
            self.samples.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
            mask = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
            for name, bit in self.REASONS.items():
                if mask & bit:
                    self.reasons.add(name)
        except Exception:  # noqa: BLE001
            pass

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)

    def summary(self):
        if self.err:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err]}
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples), "source": "NVML, 2 ms"}


# ------------------------------------------------------------------ reference / CPU baseline

def cpu_reference_run(cfg, lw, x_sample, steps: int, warmup: int):
    """Time the reference CPU path on `x_sample` tokens: returns (tokens/s, cores, kind)."""
    from oracle.oracle import Oracle, Reference, reference_available
    threads = os.cpu_count() or 1
    T = x_sample.shape[0]
    if reference_available():
        R = Reference()
        kind = "reference"
        # load-time dequant to f32 (excluded from timing), as the reference Session does
        def deq(fmt, packed, rows, cols):
            flat = packed.reshape(-1, packed.shape[-1])
            return R.dequant(fmt, flat, rows, cols, flat.shape[1])
        E, I, D = cfg.E, cfg.I, cfg.D
        G = deq(cfg.gate_fmt, lw.gate, E * I, D).reshape(E, I, D)
        U = deq(cfg.gate_fmt, lw.up, E * I, D).reshape(E, I, D)
        Dn = deq(cfg.down_fmt, lw.down, E * D, I).reshape(E, D, I)

        def step():
            probs, _ = R.router(x_sample, lw.router_w)
            return R.experts(x_sample, G, U, Dn, probs, cfg.top_k, threads)
    else:
        O = Oracle()
        kind = "port"
        threads = 1

        def step():
            _, probs, _ = O.router(x_sample, lw.router_w)
            return O.experts_packed(x_sample, lw.gate, cfg.gate_fmt, lw.up, cfg.gate_fmt, lw.down, cfg.down_fmt,
                                    probs, cfg.E, cfg.I, cfg.top_k, cfg.norm_topk)
    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = time.perf_counter() - t0
    return T * steps / dt, threads, kind


def cpu_sample_tokens(cfg, T: int) -> int:
    threads = os.cpu_count() or 1
    # about 10-30 s of CPU work: the expert loop costs ~2*3*D*I*k flops per token, single-threaded per call
    per_token_s = 2 * 3 * cfg.D * cfg.I * cfg.top_k / 1.5e9
    n = int(min(4 * threads, max(threads, 20.0 / max(per_token_s, 1e-6))))
    return max(1, min(T, n))


PARITY_TOL = 2e-3  # max |y - y_ref| / max |y_ref| over the checked rows (the layer-output bar)


def parity_rows(cfg, probs: np.ndarray, seed: int) -> np.ndarray:
    """A seeded sample of this rank's tokens whose top-k choices cover every expert the
    tokens reach (greedy over a seeded permutation), plus four random rows; bounded to about
    20 s of oracle work."""
    T = probs.shape[0]
    per_row_s = 2 * 3 * cfg.D * (cfg.I * cfg.top_k + cfg.I_sh) / 1.0e9
    cap = int(max(4, min(64, 20.0 / per_row_s)))
    ids = np.argsort(-probs, axis=1, kind="stable")[:, :cfg.top_k]
    reach = set(np.unique(ids).tolist())
    rng = np.random.default_rng(seed)
    order = rng.permutation(T)
    rows, covered = [], set()
    for t in order:
        new = set(ids[t].tolist()) - covered
        if new:
            rows.append(int(t))
            covered |= new
        if covered == reach or len(rows) >= cap - 4:
            break
    extra = [int(t) for t in order[-4:] if int(t) not in rows]
    return np.array(sorted(rows + extra[: max(0, cap - len(rows))]), np.int64)


def parity_check(cfg, lw, x: np.ndarray, y: np.ndarray, probs: np.ndarray, seed: int) -> dict:
    """The device layer output on sampled rows against the oracle (the C restatement pinned to
    the reference build), run on the same seeded inputs: a check, never part of the timing."""
    from oracle.oracle import Oracle
    O = Oracle()
    rows = parity_rows(cfg, probs, seed)
    xs = np.ascontiguousarray(x[rows])
    _, pr, _ = O.router(xs, lw.router_w)
    y_ref, ids, _ = O.experts_packed(xs, lw.gate, cfg.gate_fmt, lw.up, cfg.gate_fmt, lw.down, cfg.down_fmt, pr,
                                     cfg.E, cfg.I, cfg.top_k, cfg.norm_topk)
    if lw.shared is not None:
        g, u, d, gi = lw.shared
        O.shared_packed(xs, g, cfg.shared_fmt, u, cfg.shared_fmt, d, cfg.shared_fmt, gi, cfg.I_sh, y_ref)
    err = float(np.abs(y[rows].astype(np.float64) - y_ref).max() / max(float(np.abs(y_ref).max()), 1e-30))
    return {"rows": int(len(rows)), "experts_covered": int(len(np.unique(ids))), "max_rel": err,
            "bar": PARITY_TOL, "oracle": "oracle/moe_oracle.c (pinned to the reference build)",
            "_experts": np.unique(ids)}


# ------------------------------------------------------------------ main

DECODE_NOTE = ("BASELINE configs[4]: greedy decode of a random-init 32-layer Mixtral-shaped model, d_model 4096, "
               "32 query / 8 KV heads of 128, RoPE theta 1e6, RMSNorm, attention Q8_0, experts 8 x top-2 d_ff 14336 "
               "Q4_K/Q4_K/Q6_K, vocab 32000 tied Q8_0, batch 32, KV cache prefilled to 4096 positions")


def run_decode_model(args) -> int:
    """The end-to-end decode configuration on one GPU: weights drawn N(0, 0.02) and quantized on
    the device, the KV cache prefilled with seeded N(0, 1) values at positions 0..4095 (synthetic:
    no prompt is run), then `--steps` greedy steps for the whole batch through
    uaii_moe_decoder_generate.  A step here is one decode step of the batch (32 tokens)."""
    import torch
    import uaii_moe as um
    n_layers, D, H, HKV, HD, V, Bt, E, I, K = args.layers, 4096, 32, 8, 128, 32000, 32, 8, 14336, 2
    S0, steps, warm = 4096, args.steps, args.warmup
    torch.cuda.set_device(0)
    stream = torch.cuda.Stream()
    be = um.Backend(0, stream.cuda_stream)
    keep = []

    def packed(fmt, rows, cols, seed_stream, std=0.02):
        out = torch.empty((rows, um.packed_nbytes(fmt, cols)), dtype=torch.uint8, device="cuda")
        chunk = max(256, (1 << 26) // cols)  # ~256 MB of f32 at a time
        tmp = torch.empty((min(rows, chunk), cols), device="cuda")
        for r0 in range(0, rows, chunk):
            r1 = min(rows, r0 + chunk)
            um.fill_normal_device(be, tmp[: r1 - r0], 7, seed_stream * 4096 + r0 // chunk, 0.0, std)
            um.quantize_rows_device(be, fmt, tmp[: r1 - r0], out[r0:r1])
        be.synchronize()
        keep.append(out)
        return out

    def dense(n, seed_stream, std=0.02):
        t = torch.empty(n, device="cuda")
        um.fill_normal_device(be, t, 7, seed_stream * 4096, 0.0, std)
        keep.append(t)
        return t

    t0 = time.perf_counter()
    emb = packed(um.Q8_0, V, D, 1)
    out_norm = dense(D, 2)
    blocks = []
    for l in range(n_layers):
        s0 = 100 + 20 * l
        router = dense(E * D, s0).view(E, D)
        gate, up = packed(um.Q4_K, E * I, D, s0 + 1), packed(um.Q4_K, E * I, D, s0 + 2)
        down = packed(um.Q6_K, E * D, I, s0 + 3)
        blocks.append({"attn_norm": dense(D, s0 + 4), "ffn_norm": dense(D, s0 + 5),
                       "wq": packed(um.Q8_0, H * HD, D, s0 + 6), "wq_fmt": um.Q8_0,
                       "wk": packed(um.Q8_0, HKV * HD, D, s0 + 7), "wk_fmt": um.Q8_0,
                       "wv": packed(um.Q8_0, HKV * HD, D, s0 + 8), "wv_fmt": um.Q8_0,
                       "wo": packed(um.Q8_0, D, H * HD, s0 + 9), "wo_fmt": um.Q8_0,
                       "moe": um.make_layer(D, E, I, K, 1, router, gate, um.Q4_K, up, um.Q4_K, down, um.Q6_K)})
    be.synchronize()
    synth_s = time.perf_counter() - t0
    dec = um.Decoder(be, n_layers, D, H, HKV, V, Bt, S0 + warm + steps + 1, blocks, out_norm, emb, um.Q8_0,
                     rope_theta=1e6, rms_eps=1e-5)
    dec.fill_kv(S0, 11)
    tok0 = torch.from_numpy(np.random.default_rng(0).integers(0, V, size=Bt).astype(np.int32))
    out = torch.empty((max(warm, 1), Bt), dtype=torch.int32, device="cuda")
    if warm:
        dec.generate(tok0.cuda(), warm, out)
    be.synchronize()
    tokens = out[warm - 1].clone() if warm else tok0.cuda()
    gen = torch.empty((steps, Bt), dtype=torch.int32, device="cuda")
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        torch.cuda.synchronize()
        be.profile_enable(False)  # resets the launch count; no phase events (MoE layers replay their graphs)
        ev0.record(stream)
        dec.generate(tokens, steps, gen)
        ev1.record(stream)
        clk.sample_now()
        torch.cuda.synchronize()
        phases, launches = be.profile_read()
    ms = ev0.elapsed_time(ev1)
    # end to end through the same entry point from a fresh prefill: host token ids in (once) and out
    e2e = None
    if not args.no_e2e:
        host_out = np.empty((steps, Bt), np.int32)
        host_tok = gen[-1].cpu().numpy()
        dec.fill_kv(S0, 11)
        torch.cuda.synchronize()
        ev0.record(stream)
        dec.generate(host_tok, steps, host_out)
        ev1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = ev0.elapsed_time(ev1)
        e2e = {"value": Bt * steps / (e2e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": 4 * Bt / steps,
               "d2h_bytes_per_step": 4 * Bt, "ms_per_step": e2e_ms / steps}
    peaks = load_peaks()
    from uaii_moe import packed_nbytes
    len_avg = S0 + warm + steps / 2.0
    expert_b = E * (2 * I * packed_nbytes(um.Q4_K, D) + D * packed_nbytes(um.Q6_K, I))
    attn_b = (2 * H * HD + 2 * HKV * HD) * packed_nbytes(um.Q8_0, D)
    kv_b = Bt * HKV * len_avg * HD * 2 * 2
    step_bytes = n_layers * (expert_b + attn_b + kv_b) + V * packed_nbytes(um.Q8_0, D)
    achieved = step_bytes / (ms / steps / 1e3) / 1e9
    line = {"metric": "MoE decode tokens/s", "value": Bt * steps / (ms / 1e3), "unit": UNIT, "n_gpus": 1,
            "steps": steps, "warmup": warm, "ms_per_step": ms / steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16",
            "dtype_note": "GGUF blocks dequantized to f16 tensor-core operands, f32 accumulation; KV cache f16; "
                          "norms, RoPE, softmax and residuals in f32",
            "data": "synthetic (random-init weights drawn and quantized on the device, seeded N(0,1) KV prefill)",
            "config": {"workload": f"mixtral_decode_L{n_layers}_B{Bt}_S{S0}", "note": DECODE_NOTE,
                       "layers": n_layers, "batch": Bt, "prefill": S0, "tokens_per_step": Bt,
                       "l2": "inputs larger than L2 (every layer's weights and KV cache re-read each step)"},
            "e2e": e2e, "gpu_launches": launches,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / peaks["hbm_gbs"], "traffic": None,
                         "kernel": "whole decode step (expert GEMMs, attention over the KV cache, projections)",
                         "algorithmic_per_step": step_bytes, "algorithmic_unit": "bytes",
                         "note": "all 8 experts of every layer counted as touched (64 routed slots per layer)"},
            "cpu_baseline": None, "clocks": clk.summary(),
            "synthesis_s": synth_s}
    print(json.dumps(line), flush=True)
    dec.close()
    be.close()
    return 0


def main():
    args = parse()
    if args.config == "mixtral_decode":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the decode configuration is timed by the repo arm "
                                                                  "only (its CPU cost is hours per step)"}))
            return 0
        return run_decode_model(args)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    T = args.tokens if args.scaling == "weak" else args.tokens // max(1, int(os.environ.get("WORLD_SIZE", "1")))
    workload = f"{args.config}_T{args.tokens}" + ("" if args.scaling == "weak" else "_total")

    if args.impl == "reference":
        if rank != 0:
            return 0
        # Inputs from the numpy restatement of the library's seeded generator and quantizer
        # (byte-identical, pinned by tests/test_oracle.py): this process loads the reference
        # build only, never the product library.
        from oracle.synth import CONFIGS as SYNTH_CONFIGS, make_layer, make_tokens as synth_tokens
        cfg = SYNTH_CONFIGS[args.config]
        lw = make_layer(cfg, workers=min(16, os.cpu_count() or 1))
        n = cpu_sample_tokens(cfg, T)
        xs = synth_tokens(cfg, n, 0)
        tps, cores, kind = cpu_reference_run(cfg, lw, xs, args.steps, args.warmup)
        line = {"impl": "reference", "metric": METRIC, "value": tps, "unit": UNIT, "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": args.scaling,
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random-init GGUF layer)",
                "config": {"workload": workload, "note": WORKLOAD_NOTE.get(args.config, ""),
                           "tokens_per_step": n},
                "cpu_baseline": {"value": tps, "unit": UNIT, "cores": cores, "kind": kind,
                                 "sample": f"{n} of {T} tokens per step, all experts dequantized to f32 "
                                           f"before timing (reference load-time dequant)"},
                "e2e": {"value": tps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    import torch
    import uaii_moe as um
    from uaii_moe.synthetic import CONFIGS, make_layer_weights, make_tokens
    cfg = CONFIGS[args.config]
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    lw = make_layer_weights(cfg)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda() if a is not None else None
    # N > 1: expert parallelism (rank r holds experts [r*E/N, (r+1)*E/N) and its own tokens; NCCL
    # all-to-all dispatch and combine every step).  Layers whose expert count N does not divide,
    # or with a shared expert, run as independent replicas.
    ep_mode = world > 1 and cfg.E % world == 0 and lw.shared is None
    if ep_mode:
        from uaii_moe.ep import ExpertParallelFFN
        epr = cfg.E // world
        part = slice(rank * epr, (rank + 1) * epr)
        arrays = {"router_w": dev(lw.router_w), "gate": dev(lw.gate[part]), "up": dev(lw.up[part]),
                  "down": dev(lw.down[part])}
        local_layer = um.make_layer(cfg.D, epr, cfg.I, cfg.top_k, cfg.norm_topk, arrays["router_w"], arrays["gate"],
                                    cfg.gate_fmt, arrays["up"], cfg.gate_fmt, arrays["down"], cfg.down_fmt)
        router_layer = um.make_layer(cfg.D, cfg.E, cfg.I, cfg.top_k, cfg.norm_topk, arrays["router_w"],
                                     arrays["gate"], cfg.gate_fmt, arrays["up"], cfg.gate_fmt, arrays["down"],
                                     cfg.down_fmt)  # only the router fields are read by the dispatch
    else:
        arrays = {"router_w": dev(lw.router_w), "gate": dev(lw.gate), "up": dev(lw.up), "down": dev(lw.down),
                  "shared": tuple(dev(a) for a in lw.shared) if lw.shared is not None else None}
        L = lw.layer_struct(arrays)
    x_host = torch.from_numpy(make_tokens(cfg, T, rank)).pin_memory()
    y_host = torch.empty((T, cfg.D), dtype=torch.float32).pin_memory()
    x = x_host.cuda()
    y = torch.empty((T, cfg.D), dtype=torch.float32, device="cuda")
    probs = torch.empty((T, cfg.E), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()  # inputs were written on the default stream
    stream = torch.cuda.Stream()
    be = um.Backend(local, stream.cuda_stream)
    if args.path:
        be.set_expert_path(args.path)
    if args.no_graphs:
        be.set_graphs(False)
    # a serving process registers its (constant) weights once: layouts derived from them, such as
    # 16-byte-pitch copies of rows the tensor maps cannot address, are then made once, not per call
    for a in arrays.values():
        for t in (a if isinstance(a, tuple) else (a,)):
            if t is not None:
                be.register_weights(t)

    if ep_mode:
        ep = ExpertParallelFFN(be, router_layer, local_layer, cfg.D, cfg.E, cfg.top_k, rank, world,
                               chunks=args.ep_chunks)

        def forward(xin, yout, pr=None):
            with torch.cuda.stream(stream):  # collectives order against the backend's stream
                ep.forward(xin, yout, pr)
    else:
        def forward(xin, yout, pr=None):
            be.ffn(L, xin, T, yout, pr)

    # routing statistics for the roofline (outside any timed region)
    forward(x, y, probs)
    be.synchronize()
    ids = torch.topk(probs, cfg.top_k, dim=1).indices
    touched = int(torch.unique(ids).numel())
    local_entries = ep.last_exchange[2] if ep_mode else T * cfg.top_k
    # correctness of this rank's output before anything is timed (every rank, every N): sampled
    # rows covering every expert its tokens reach, against the oracle; a miss fails the run
    parity = parity_check(cfg, lw, x_host.numpy(), y.cpu().numpy(), probs.cpu().numpy(), 777 + rank)
    covered = torch.zeros(cfg.E, dtype=torch.float64, device="cuda")
    covered[torch.from_numpy(parity.pop("_experts").astype(np.int64)).cuda()] = 1.0
    if dist is not None:  # worst error, all checked rows and the experts they reach, over all ranks
        worst = torch.tensor([parity["max_rel"]], dtype=torch.float64, device="cuda")
        nrows = torch.tensor([float(parity["rows"])], dtype=torch.float64, device="cuda")
        dist.all_reduce(worst, op=dist.ReduceOp.MAX)
        dist.all_reduce(nrows, op=dist.ReduceOp.SUM)
        dist.all_reduce(covered, op=dist.ReduceOp.MAX)
        parity["max_rel"] = float(worst.item())
        parity["rows"] = int(nrows.item())
        parity["ranks"] = world
    parity["experts_covered"] = int(covered.sum().item())

    for _ in range(args.warmup):
        forward(x, y)
    be.synchronize()

    def barrier():
        if dist is not None:
            dist.barrier()

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        torch.cuda.synchronize()
        be.profile_enable(True)  # per-phase CUDA events inside the timed region (plain launches)
        ev0.record(stream)
        for _ in range(args.steps):
            forward(x, y)
        ev1.record(stream)
        clk.sample_now()
        torch.cuda.synchronize()
        barrier()
        phases, launches = be.profile_read()
        be.profile_enable(False)
    ms = ev0.elapsed_time(ev1)
    # Decode widths are launch-bound: the same steps replayed from the CUDA graph the library
    # captures for repeated device-resident calls (phase events off), reported beside the value.
    graph_replay = None
    if not ep_mode and not args.no_graphs and T <= 64:
        for _ in range(3):
            forward(x, y)
        torch.cuda.synchronize()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for _ in range(args.steps):
            forward(x, y)
        g1.record(stream)
        torch.cuda.synchronize()
        gms = g0.elapsed_time(g1)
        graph_replay = {"value": T * args.steps / (gms / 1e3), "unit": UNIT, "ms_per_step": gms / args.steps}
    plan = be.last_plan()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ms = max_over_ranks(ms)
    value = world * T * args.steps / (ms / 1e3)

    e2e = None
    if not args.no_e2e:
        if ep_mode:
            # explicit copies, pinned host x in and host y out every step, double-buffered across
            # steps: step i+1's input is copied in (its own stream) while step i computes, and
            # step i's output is copied out (another stream) while step i+1 computes
            x_in = [torch.empty_like(x) for _ in range(2)]
            y_out = [torch.empty_like(y) for _ in range(2)]
            s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
            ev_in = [torch.cuda.Event() for _ in range(2)]
            ev_done = [torch.cuda.Event() for _ in range(2)]
            ev_out = [torch.cuda.Event() for _ in range(2)]
            for e in ev_done + ev_out:
                e.record(stream)

            def e2e_run(n):
                with torch.cuda.stream(s_in):
                    s_in.wait_event(ev_done[0])
                    x_in[0].copy_(x_host, non_blocking=True)
                    ev_in[0].record(s_in)
                for i in range(n):
                    b = i % 2
                    stream.wait_event(ev_in[b])
                    stream.wait_event(ev_out[b])  # y_out[b] was copied out two steps ago
                    with torch.cuda.stream(stream):
                        ep.forward(x_in[b], y_out[b])
                        ev_done[b].record(stream)
                    if i + 1 < n:
                        with torch.cuda.stream(s_in):
                            s_in.wait_event(ev_done[1 - b])  # x_in[1-b] read by step i-1
                            x_in[1 - b].copy_(x_host, non_blocking=True)
                            ev_in[1 - b].record(s_in)
                    with torch.cuda.stream(s_out):
                        s_out.wait_event(ev_done[b])
                        y_host.copy_(y_out[b], non_blocking=True)
                        ev_out[b].record(s_out)
                stream.wait_stream(s_out)
        else:
            def e2e_run(n):
                for _ in range(n):
                    be.ffn(L, x_host, T, y_host)
        e2e_run(2)
        barrier()
        torch.cuda.synchronize()
        ev0.record(stream)
        e2e_run(args.steps)
        ev1.record(stream)
        torch.cuda.synchronize()
        barrier()
        e2e_ms = max_over_ranks(ev0.elapsed_time(ev1))
        e2e = {"value": world * T * args.steps / (e2e_ms / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": T * cfg.D * 4, "d2h_bytes_per_step": T * cfg.D * 4,
               "ms_per_step": e2e_ms / args.steps}

    # roofline of the dominant phase
    peaks = load_peaks()
    dom = max(("gateup", "down"), key=lambda p: phases[p][0])
    dom_ms, dom_calls = phases[dom]
    avg_s = dom_ms / max(dom_calls, 1) / 1e3
    # this rank's expert work: all its experts' packed rows and the (token, expert) pairs it served
    S = local_entries
    if ep_mode:
        touched = cfg.E // world
    from uaii_moe import packed_nbytes
    act = 2 if plan["tensor_cores"] else 4  # bytes per activation element the kernel reads / writes
    if dom == "gateup":  # packed gate+up rows of the touched experts, x in, h out
        byts = touched * 2 * cfg.I * packed_nbytes(cfg.gate_fmt, cfg.D) + S * cfg.D * act + S * cfg.I * act
        fl = 2 * S * 2 * cfg.D * cfg.I
    else:  # packed down rows, h in, f32 partial sums out
        byts = touched * cfg.D * packed_nbytes(cfg.down_fmt, cfg.I) + S * cfg.I * act + S * cfg.D * 4
        fl = 2 * S * cfg.D * cfg.I
    tokens_per_expert = S / max(touched, 1)
    if tokens_per_expert < 64:
        roof = {"bound": "hbm", "achieved": byts / avg_s / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s"}
    else:
        roof = {"bound": "tensor", "achieved": fl / avg_s / 1e12, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "peak_sustained": peaks["bf16_tflops_sustained"]}
        roof["frac_sustained"] = roof["achieved"] / roof["peak_sustained"]
    roof["frac"] = roof["achieved"] / roof["peak"]
    roof["traffic"] = NCU_TRAFFIC.get((workload, dom))
    sched = {"tcgen05": "tcgen05", "warp_mma": "warp-level mma.sync m16n8k16",
             "quad_mma": "warp-level mma.sync m16n8k16 over whole K-quant super-blocks",
             "quad_mma_i8": "warp-level mma.sync over whole K-quant super-blocks"}.get(plan.get("schedule"), "tcgen05")
    operands = ("gate/up: m16n8k32 int8 on Q4_K nibbles x 16-bit integer activations (two byte planes), exact "
                "int32 per sub-block; down: m16n8k16 f16 operands, f32 accumulate"
                if plan.get("schedule") == "quad_mma_i8" else "f16 operands, f32 accumulate")
    path = (f"tensor-core grouped dequant-GEMM ({sched}, {operands}), "
            f"{plan['slot_tile']}-slot tiles") if plan["tensor_cores"] else "CUDA-core f32 grouped GEMV"
    roof["kernel"] = f"{dom} phase: {path}"
    roof["peak_src"] = f"{peaks['src']} ({'hbm_gbs' if roof['bound'] == 'hbm' else 'bf16_tflops burst'})"
    roof["algorithmic_per_launch"] = byts if roof["bound"] == "hbm" else fl
    roof["algorithmic_unit"] = "bytes" if roof["bound"] == "hbm" else "flops"
    roof["avg_launch_ms"] = avg_s * 1e3

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        n = cpu_sample_tokens(cfg, T)
        xs = make_tokens(cfg, n, 0)
        tps, cores, kind = cpu_reference_run(cfg, lw, xs, 1, 0)
        cpu = {"value": tps, "unit": UNIT, "cores": cores, "kind": kind,
               "sample": f"{n} of the {T} tokens, one pass (router + experts), f32 weights dequantized "
                         f"before timing"}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
                "scaling": args.scaling, "vs_baseline": None, "dtype": "f16" if plan["tensor_cores"] else "f32",
                "dtype_note": ("Q4_K gate/up: raw nibbles (int8) x activations quantized per 256 elements to 16-bit "
                               "integers, exact int32 sub-block sums, f32 scale; down: GGUF blocks dequantized to f16 "
                               "tensor-core operands, f32 accumulation; router, softmax and combine in f32"
                               if plan.get("schedule") == "quad_mma_i8" else
                               "GGUF blocks dequantized to f16 tensor-core operands, f32 accumulation; router, "
                               "softmax and combine in f32") if plan["tensor_cores"] else "f32 throughout",
                "data": "synthetic (seeded random-init GGUF layer, N(0,1) activations)",
                "config": {"workload": workload, "note": WORKLOAD_NOTE.get(args.config, ""),
                           "tokens_per_gpu": T,
                           "parallelism": (f"expert parallel x{world} (NCCL all-to-all dispatch/combine, f16 return rows)" if ep_mode
                                           else f"replicas x{world}" if world > 1 else "1 GPU"),
                           "l2": "inputs larger than L2 (packed expert weights re-read every step)",
                           "experts_touched": touched},
                "e2e": e2e, "gpu_launches": launches, "graph_replay": graph_replay, "roofline": roof,
                "cpu_baseline": cpu,
                "clocks": clk.summary(),
                "phases_ms_per_step": {p: v[0] / args.steps for p, v in phases.items()},
                "parity": parity}
        print(json.dumps(line), flush=True)
    be.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if not parity["max_rel"] <= PARITY_TOL:
        print(f"bench: parity check failed: max_rel {parity['max_rel']:.3e} > {PARITY_TOL}", file=sys.stderr)
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
