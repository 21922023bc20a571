"""Seeded synthetic models of the benchmark configurations.

Weights are N(0, std) values (a counter-based splitmix64 stream, Box-Muller
in float64) quantized to Q4_0 with the reference's quantizer
(src/quant/blocks.rs:50-82), restated here in vectorised numpy with the same
f32 operations: block min/max, d = max(-min/8, max/7) or -(max(max/8,
-min/7)), id = 1/d, q = clamp(round_half_away(x*id) + 8, 0, 15), f16 scale
rounded to nearest even.  RMSNorm scales are 1.0.

The same host bytes feed the GPU path and, in the tests and the CPU
baseline, the oracle, so both sides always see identical inputs.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from ._lib import Config

GOLDEN = np.uint64(0x9E3779B97F4A7C15)


def _mix64(z: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def normal_f32(n: int, seed: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    """n values of N(mean, std); value i depends only on (seed, i)."""
    pairs = (n + 1) // 2
    k = np.arange(pairs, dtype=np.uint64)
    s = np.uint64(seed & 0xFFFFFFFFFFFFFFFF)
    with np.errstate(over="ignore"):
        r1 = _mix64(s + (np.uint64(2) * k + np.uint64(1)) * GOLDEN)
        r2 = _mix64(s + (np.uint64(2) * k + np.uint64(2)) * GOLDEN)
    u1 = ((r1 >> np.uint64(11)).astype(np.float64) + 1.0) * (1.0 / 9007199254740992.0)
    u2 = (r2 >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
    rad = np.sqrt(-2.0 * np.log(u1))
    ang = 2.0 * np.pi * u2
    z = np.empty(2 * pairs, dtype=np.float64)
    z[0::2] = rad * np.cos(ang)
    z[1::2] = rad * np.sin(ang)
    return (mean + std * z[:n]).astype(np.float32)


def _round_half_away(v: np.ndarray) -> np.ndarray:
    t = np.trunc(v)
    frac = v - t  # exact
    return t + np.where(np.abs(frac) >= 0.5, np.sign(v), 0).astype(np.float32)


def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    """BlockQ4_0 bytes (n/32 * 18) of f32 values x (len multiple of 32)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, 32)
    f8, f7 = np.float32(8.0), np.float32(7.0)
    mn = np.minimum(x.min(axis=1), np.float32(0.0))
    mx = np.maximum(x.max(axis=1), np.float32(0.0))
    d_pos = np.maximum(-mn / f8, mx / f7)
    d_neg = np.maximum(mx / f8, -mn / f7)
    d = np.where(d_pos <= d_neg, d_pos, -d_neg).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(d != 0, np.float32(1.0) / np.where(d != 0, d, 1), 0).astype(np.float32)
    q = _round_half_away(x * idv[:, None]) + np.float32(8.0)
    q = np.clip(q, 0, 15).astype(np.uint8)
    out = np.empty((x.shape[0], 18), dtype=np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:18] = q[:, :16] | (q[:, 16:] << 4)
    return out.reshape(-1)


def synth_q4(rows: int, cols: int, seed: int, std: float = 0.02, chunk_rows: int = 8192) -> np.ndarray:
    """rows x cols Q4_0 matrix of N(0, std) values; row-chunked to bound memory."""
    out = np.empty(rows * cols // 32 * 18, dtype=np.uint8)
    per_row = cols // 32 * 18
    for r0 in range(0, rows, chunk_rows):
        r1 = min(rows, r0 + chunk_rows)
        vals = normal_f32((r1 - r0) * cols, _sub_seed(seed, r0), 0.0, std)
        out[r0 * per_row:r1 * per_row] = quantize_q4_0(vals)
    return out


def _sub_seed(seed: int, i: int) -> int:
    return (seed * 0x100000001B3 + (i + 1) * 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF


@dataclass
class HostWeights:
    """Host copies of a Llama-shaped Q4_0 model in the reference's formats
    (TransformerWeights / ModelWeights, transformer.rs:35-57)."""
    token_embd: np.ndarray
    layers: list
    output_norm: np.ndarray
    lm_head: np.ndarray | None
    vocab: int
    meta: dict = field(default_factory=dict)

    @property
    def num_layers(self) -> int:
        return len(self.layers)

    def q4_bytes(self) -> int:
        keys = ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down")
        n = sum(lw[k].nbytes for lw in self.layers for k in keys)
        return n + (self.lm_head.nbytes if self.lm_head is not None else self.token_embd.nbytes)


def synth_model(cfg: Config, num_layers: int, vocab: int, seed: int = 1234,
                std: float = 0.02) -> HostWeights:
    d, h = cfg.dim, cfg.hidden_dim
    kvd = d // cfg.num_heads * cfg.num_kv_heads
    ones = np.ones(d, dtype=np.float32)
    layers = []
    for l in range(num_layers):
        b = 100 + 16 * l
        layers.append({
            "rms_att_weight": ones,
            "wq": synth_q4(d, d, _sub_seed(seed, b + 1), std),
            "wk": synth_q4(kvd, d, _sub_seed(seed, b + 2), std),
            "wv": synth_q4(kvd, d, _sub_seed(seed, b + 3), std),
            "wo": synth_q4(d, d, _sub_seed(seed, b + 4), std),
            "rms_ffn_weight": ones,
            "w_gate": synth_q4(h, d, _sub_seed(seed, b + 6), std),
            "w_up": synth_q4(h, d, _sub_seed(seed, b + 7), std),
            "w_down": synth_q4(d, h, _sub_seed(seed, b + 8), std),
        })
    return HostWeights(synth_q4(vocab, d, _sub_seed(seed, 1), std), layers, ones,
                       synth_q4(vocab, d, _sub_seed(seed, 2), std), vocab,
                       {"seed": seed, "std": std})


# The BASELINE configurations (shapes only; weights are synthetic).
CONFIGS = {
    "cfg1": dict(cfg=Config(256, 512, 4, 4, 512, 1e-5), layers=2, vocab=1024),
    "cfg2": dict(cfg=Config(288, 768, 6, 6, 256, 1e-5), layers=6, vocab=32000),
    # SmolLM2-135M shape; max_seq_len 2048 + room for the decode steps
    "cfg3": dict(cfg=Config(576, 1536, 9, 3, 2048 + 64, 1e-5), layers=30, vocab=49152),
    # cfg4: one Llama-3-8B-shaped layer (dim 4096, hidden 14336, 32/8 heads,
    # head_dim 128) for the attention and GEMV kernel sweeps; small vocab
    "cfg4": dict(cfg=Config(4096, 14336, 32, 8, 8192 + 64, 1e-5), layers=1, vocab=2048),
    # cfg5: SmolLM2 shape with a 4096-token prompt and 128 decode steps
    "cfg5": dict(cfg=Config(576, 1536, 9, 3, 4096 + 128, 1e-5), layers=30, vocab=49152),
}


def config(name: str, max_seq_len: int | None = None) -> tuple[Config, int, int]:
    c = CONFIGS[name]
    cfg = Config(c["cfg"].dim, c["cfg"].hidden_dim, c["cfg"].num_heads, c["cfg"].num_kv_heads,
                 max_seq_len or c["cfg"].max_seq_len, c["cfg"].rms_eps)
    return cfg, c["layers"], c["vocab"]
