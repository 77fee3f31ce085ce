"""Seeded synthetic inputs for the sampling benchmarks and parity tests.

The reference publishes no dataset for this path; these generators produce the
shapes and value distributions of the five sampling configurations the
benchmark is quoted on (logit rows of a Qwen2.5-sized vocabulary, greedy,
heterogeneous top-k/top-p, grammar-constrained and vocab-sharded).  They use
numpy's PCG64 so that the same seed gives the same rows on every machine, and
the per-row uniform is ``random.Random(seed_b).random()`` -- the exact draw
miniserve's ``Sampler.sample(..., seed=seed_b)`` makes (miniserve/sampler.py:32,62).
"""
from __future__ import annotations

import random
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

QWEN_VOCAB = 151936


@dataclass
class Batch:
    name: str
    logits: np.ndarray            # [B, V] float32 (or uint16 bf16 bits when bf16=True)
    temperature: np.ndarray       # [B] float64
    top_k: np.ndarray             # [B] int32
    top_p: np.ndarray             # [B] float64
    uniforms: np.ndarray          # [B] float64
    seeds: np.ndarray             # [B] int64, uniforms[b] == Random(seeds[b]).random()
    bf16: bool = False
    mask: Optional[np.ndarray] = None   # [B, ceil(V/32)] uint32, bit set = allowed
    extra: dict = field(default_factory=dict)

    @property
    def B(self) -> int:
        return self.logits.shape[0]

    @property
    def V(self) -> int:
        return self.logits.shape[1]


def row_seeds(seed: int, B: int) -> np.ndarray:
    return np.array([seed * 1_000_003 + b for b in range(B)], dtype=np.int64)


def uniforms_for(seeds) -> np.ndarray:
    return np.array([random.Random(int(s)).random() for s in seeds], dtype=np.float64)


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns, round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def zipf_rows(rng: np.random.Generator, B: int, V: int, noise: float = 0.5) -> np.ndarray:
    """logit_i = -1.1 ln(rank_i) + N(0, noise^2), ranks a seeded permutation of 1..V."""
    out = np.empty((B, V), dtype=np.float32)
    base = -1.1 * np.log(np.arange(1, V + 1, dtype=np.float64))
    for b in range(B):
        perm = rng.permutation(V)
        out[b] = (base[perm] + rng.normal(0.0, noise, V)).astype(np.float32)
    return out


def config1(seed: int = 1, B: int = 8, V: int = QWEN_VOCAB, greedy: bool = False) -> Batch:
    """Qwen2.5-0.5B-shaped step: N(0, 2^2) + 8.0 at 5 seeded indices; T=0.7, k=50, p=0.9."""
    rng = np.random.default_rng(seed)
    x = rng.normal(0.0, 2.0, (B, V)).astype(np.float32)
    for b in range(B):
        idx = rng.choice(V, size=min(5, V), replace=False)
        x[b, idx] += np.float32(8.0)
    seeds = row_seeds(seed, B)
    T = np.full(B, 0.0 if greedy else 0.7)
    return Batch("config1" + ("_greedy" if greedy else ""), x, T, np.full(B, 50, np.int32),
                 np.full(B, 0.9), uniforms_for(seeds), seeds)


def config2(seed: int = 2, B: int = 256, V: int = QWEN_VOCAB, bf16: bool = False) -> Batch:
    """Greedy + temperature-only: N(0, 3^2) with one +10 spike; T in {0, 1.0}; k=0, p=1."""
    rng = np.random.default_rng(seed)
    x = rng.normal(0.0, 3.0, (B, V)).astype(np.float32)
    spike = rng.integers(0, V, B)
    x[np.arange(B), spike] += np.float32(10.0)
    T = np.where(rng.random(B) < 0.5, 0.0, 1.0)
    seeds = row_seeds(seed, B)
    logits = to_bf16_bits(x) if bf16 else x
    return Batch("config2_" + ("bf16" if bf16 else "fp32"), logits, T, np.zeros(B, np.int32),
                 np.ones(B), uniforms_for(seeds), seeds, bf16=bf16)


def config3(seed: int = 3, B: int = 512, V: int = QWEN_VOCAB) -> Batch:
    """Heterogeneous: Zipf logits; k in {0,1,20,50,200}, p ~ U(0.5, 1], T ~ U(0.2, 1.5)."""
    rng = np.random.default_rng(seed)
    x = zipf_rows(rng, B, V)
    k = rng.choice(np.array([0, 1, 20, 50, 200], np.int32), B)
    p = 1.0 - 0.5 * rng.random(B)
    T = 0.2 + 1.3 * rng.random(B)
    seeds = row_seeds(seed, B)
    return Batch("config3", x, T, k.astype(np.int32), p, uniforms_for(seeds), seeds)


_JSON_HEAVY = '{}[]:,"\\0123456789' + "truefalsn"  # structural characters, digits, literal letters


def json_vocab(seed: int = 4, V: int = QWEN_VOCAB):
    """Synthetic vocabulary: V printable-ASCII strings of 1-8 characters, JSON
    structural characters, digits and true/false/null letters 4x as likely."""
    rng = random.Random(seed)
    chars = [chr(c) for c in range(0x20, 0x7F)]
    weights = [4 if c in _JSON_HEAVY else 1 for c in chars]
    return ["".join(rng.choices(chars, weights, k=rng.randint(1, 8))) for _ in range(V)]


def _json_value(rng: random.Random, depth: int):
    r = rng.random()
    if depth < 4 and r < 0.3:
        return {f"k{rng.randint(0, 99)}": _json_value(rng, depth + 1) for _ in range(rng.randint(0, 16))}
    if depth < 4 and r < 0.55:
        return [_json_value(rng, depth + 1) for _ in range(rng.randint(0, 16))]
    if r < 0.7:
        return "".join(rng.choice('abc xyz_"\\/\n\t') for _ in range(rng.randint(0, 6)))
    if r < 0.85:
        return rng.choice([rng.randint(-1000, 1000), round(rng.uniform(-100, 100), rng.randint(0, 4)), 1e21, -0.5])
    return rng.choice([True, False, None])


def json_prefixes(seed: int = 4, B: int = 128):
    """B seeded prefixes of seeded random JSON values (nesting depth <= 4,
    <= 16 items per level), cut at a random length."""
    import json
    rng = random.Random(seed * 7919 + 1)
    out = []
    for _ in range(B):
        text = json.dumps(_json_value(rng, 0), separators=(",", ":") if rng.random() < 0.5 else (", ", ": "))
        out.append(text[: rng.randint(0, len(text))])
    return out


def config4(seed: int = 4, B: int = 128, V: int = QWEN_VOCAB) -> Batch:
    """JSON-grammar rows: N(0, 2^2) logits, T=0.8, p=0.95, k=0; the synthetic
    vocabulary and prefixes ride in ``extra`` (the mask is built from them)."""
    rng = np.random.default_rng(seed)
    x = rng.normal(0.0, 2.0, (B, V)).astype(np.float32)
    seeds = row_seeds(seed, B)
    return Batch("config4", x, np.full(B, 0.8), np.zeros(B, np.int32), np.full(B, 0.95), uniforms_for(seeds),
                 seeds, extra={"vocab": json_vocab(seed, V), "prefixes": json_prefixes(seed, B)})


def config5(seed: int = 5, B: int = 1024, V: int = 256000) -> Batch:
    """Vocab-sharded large vocab: Zipf logits; k=50, p=0.95, T=0.9."""
    rng = np.random.default_rng(seed)
    x = zipf_rows(rng, B, V)
    seeds = row_seeds(seed, B)
    return Batch("config5", x, np.full(B, 0.9), np.full(B, 50, np.int32), np.full(B, 0.95),
                 uniforms_for(seeds), seeds)
