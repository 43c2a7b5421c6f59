"""Seeded synthetic MoE layers with the shapes of the benchmark configurations.

All values come from the library's counter-based generator (uaii_moe_fill_normal)
and GGUF quantizer (uaii_moe_quantize_rows), so the same seed gives the same
bytes on every host.  Weights are N(0, 0.02) before quantization; activations
are N(0, 1).  Router bias, where a configuration asks for skewed routing, uses a
constant-1 activation lane: x[:, 0] = 1 and router_w[e, 0] = b_e, so the
reference router (which has no bias input) sees exactly the same logits.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

from . import F32, Q4_0, Q4_K, Q6_K, Q8_0, fill_normal, make_layer, quantize_rows


@dataclass
class LayerConfig:
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
    routing: str = "natural"  # natural | zipf1.1 | hot4
    seed: int = 0


CONFIGS = {
    "cfg1_q4_0": LayerConfig("cfg1_q4_0", 1024, 8, 2816, 2, Q4_0, Q4_0),
    "mixtral": LayerConfig("mixtral", 4096, 8, 14336, 2, Q4_K, Q6_K, seed=1),
    "qwen2moe": LayerConfig("qwen2moe", 2048, 60, 1408, 4, Q8_0, Q8_0, norm_topk=0, I_sh=5632,
                            shared_fmt=Q8_0, shared_gate=True, routing="zipf1.1", seed=2),
    "qwen3": LayerConfig("qwen3", 2048, 128, 768, 8, Q4_0, Q4_0, seed=3),
    "qwen3_hot": LayerConfig("qwen3_hot", 2048, 128, 768, 8, Q4_0, Q4_0, routing="hot4", seed=3),
}


@dataclass
class SyntheticLayer:
    cfg: LayerConfig
    router_w: np.ndarray
    gate: np.ndarray
    up: np.ndarray
    down: np.ndarray
    shared: tuple | None = None  # (gate, up, down, gate_inp or None)
    keep: list = field(default_factory=list)

    def layer_struct(self, arrays=None):
        """uaii_moe_layer pointing at `arrays` (defaults to the host arrays)."""
        a = arrays or {"router_w": self.router_w, "gate": self.gate, "up": self.up, "down": self.down,
                       "shared": self.shared}
        c = self.cfg
        sh = None
        if a["shared"] is not None:
            g, u, d, gi = a["shared"]
            sh = (c.I_sh, g, c.shared_fmt, u, c.shared_fmt, d, c.shared_fmt, gi)
        return make_layer(c.D, c.E, c.I, c.top_k, c.norm_topk, a["router_w"], a["gate"], c.gate_fmt, a["up"],
                          c.gate_fmt, a["down"], c.down_fmt, sh)


def _quantized(fmt: int, rows_per_part: int, cols: int, parts: int, seed: int, stream0: int) -> np.ndarray:
    """`parts` matrices [rows_per_part, cols], each generated and quantized on its own."""
    out = []
    for p in range(parts):
        w = fill_normal((rows_per_part, cols), seed, stream0 + p, 0.0, 0.02)
        out.append(w if fmt == F32 else quantize_rows(fmt, w))
    return np.stack(out)


def router_bias(cfg: LayerConfig) -> np.ndarray | None:
    if cfg.routing == "natural":
        return None
    rng = np.random.default_rng(cfg.seed + 12345)
    if cfg.routing == "zipf1.1":
        ranks = rng.permutation(cfg.E) + 1
        p = ranks.astype(np.float64) ** -1.1
        return np.log(p / p.sum()).astype(np.float32)
    if cfg.routing == "hot4":
        b = np.zeros(cfg.E, np.float32)
        b[int(rng.integers(cfg.E))] = math.log(4.0)
        return b
    raise ValueError(cfg.routing)


def make_layer_weights(cfg: LayerConfig) -> SyntheticLayer:
    s = cfg.seed
    w = fill_normal((cfg.E, cfg.D), s, 10, 0.0, 0.02)
    b = router_bias(cfg)
    if b is not None:
        w[:, 0] = b
    gate = _quantized(cfg.gate_fmt, cfg.I, cfg.D, cfg.E, s, 1000)
    up = _quantized(cfg.gate_fmt, cfg.I, cfg.D, cfg.E, s, 2000)
    down = _quantized(cfg.down_fmt, cfg.D, cfg.I, cfg.E, s, 3000)
    shared = None
    if cfg.I_sh > 0:
        g = _quantized(cfg.shared_fmt, cfg.I_sh, cfg.D, 1, s, 4000)[0]
        u = _quantized(cfg.shared_fmt, cfg.I_sh, cfg.D, 1, s, 4001)[0]
        d = _quantized(cfg.shared_fmt, cfg.D, cfg.I_sh, 1, s, 4002)[0]
        gi = fill_normal((cfg.D,), s, 4003, 0.0, 0.02) if cfg.shared_gate else None
        shared = (g, u, d, gi)
    return SyntheticLayer(cfg, w, gate, up, down, shared)


def make_tokens(cfg: LayerConfig, T: int, stream: int = 0) -> np.ndarray:
    x = fill_normal((T, cfg.D), cfg.seed, 50 + stream)
    if cfg.routing != "natural":
        x[:, 0] = 1.0
    return x


def algorithmic_bytes(cfg: LayerConfig, T: int, touched_experts: int) -> int:
    """Bytes a layer forward must move at least: packed weights of the experts
    that received tokens, the shared expert, the router weight, x and y."""
    from . import packed_nbytes
    per_expert = 2 * cfg.I * packed_nbytes(cfg.gate_fmt, cfg.D) + cfg.D * packed_nbytes(cfg.down_fmt, cfg.I)
    b = touched_experts * per_expert + cfg.E * cfg.D * 4 + 2 * T * cfg.D * 4
    if cfg.I_sh:
        b += 2 * cfg.I_sh * packed_nbytes(cfg.shared_fmt, cfg.D) + cfg.D * packed_nbytes(cfg.shared_fmt, cfg.I_sh)
    return b


def flops(cfg: LayerConfig, T: int) -> int:
    return 2 * T * cfg.top_k * 3 * cfg.D * cfg.I + 2 * T * 3 * cfg.D * cfg.I_sh + 2 * T * cfg.E * cfg.D
