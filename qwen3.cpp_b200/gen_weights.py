#!/usr/bin/env python3
"""Seeded random-init Qwen3 weights written in the Qwen3.bin layout.

The real Qwen3-0.6B checkpoint is not available offline, so parity tests and benchmarks run on
random weights of the same architecture, written in exactly the format asriva32/Qwen3.cpp's
convert.py produces (convert.py:2-20 documents it; the record writer is convert.py:250-261, the
metadata JSON convert.py:70-111 with sorted keys and compact separators, and the tensor names and
order convert.py:218-243). The reference loader (src/inference.cpp:445-510) and this framework's
loader both read the file.

Values: every matrix (and the embedding) is N(0, std) from numpy's PCG64 generator seeded with
`seed`, drawn in tensor-record order and rounded to bf16 (round to nearest even); every norm
weight is 1.0. No tokenizer records are written.

Usage:  python gen_weights.py OUT.bin [--seed 0] [--std 0.02] [--max-seq-len 40960]
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import struct
from pathlib import Path

import numpy as np

MAGIC = b"QWEN3CP\0"
VERSION = 1
DTYPE_BF16 = 3

# Qwen3-0.6B (the shapes tst/test_loader.cpp:35-47 checks).
QWEN3_0_6B = dict(
    arch="Qwen3ForCausalLM",
    dtype="bf16",
    dim=1024,
    hidden_dim=3072,
    head_dim=128,
    n_layers=28,
    n_heads=16,
    n_kv_heads=8,
    vocab_size=151936,
    max_seq_len=40960,
    bos_token_id=151643,
    eos_token_id=151645,
    rope_theta=1000000.0,
    rotary_dim=128,
    norm_eps=1e-06,
    act_type="silu",
    tie_word_embeddings=True,
    attention_bias=False,
    qk_norm=True,
)

LAYER_TENSORS = (
    # (suffix, shape as a function of the config, is_norm)
    ("attn.norm.weight", lambda c: (c["dim"],), True),
    ("attn.q_norm.weight", lambda c: (c["head_dim"],), True),
    ("attn.k_norm.weight", lambda c: (c["head_dim"],), True),
    ("attn.wq.weight", lambda c: (c["n_heads"] * c["head_dim"], c["dim"]), False),
    ("attn.wk.weight", lambda c: (c["n_kv_heads"] * c["head_dim"], c["dim"]), False),
    ("attn.wv.weight", lambda c: (c["n_kv_heads"] * c["head_dim"], c["dim"]), False),
    ("attn.wo.weight", lambda c: (c["dim"], c["n_heads"] * c["head_dim"]), False),
    ("mlp.norm.weight", lambda c: (c["dim"],), True),
    ("mlp.w1.weight", lambda c: (c["hidden_dim"], c["dim"]), False),
    ("mlp.w2.weight", lambda c: (c["dim"], c["hidden_dim"]), False),
    ("mlp.w3.weight", lambda c: (c["hidden_dim"], c["dim"]), False),
)


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (nearest even) and return the raw uint16 bits."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + (0x7FFF + ((u >> 16) & 1))) >> 16).astype(np.uint16)
    if nan.any():
        r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def tensor_plan(cfg: dict) -> list[tuple[str, tuple[int, ...], bool]]:
    """Record names, shapes and norm flags in convert.py:218-243 order."""
    plan = [("model.embed.weight", (cfg["vocab_size"], cfg["dim"]), False)]
    for layer in range(cfg["n_layers"]):
        for suffix, shape, is_norm in LAYER_TENSORS:
            plan.append((f"model.layers.{layer}.{suffix}", shape(cfg), is_norm))
    plan.append(("model.norm.weight", (cfg["dim"],), True))
    if not cfg["tie_word_embeddings"]:
        plan.append(("model.output.weight", (cfg["vocab_size"], cfg["dim"]), False))
    return plan


def metadata_json(cfg: dict) -> bytes:
    keys = sorted(QWEN3_0_6B.keys())
    return json.dumps({k: cfg[k] for k in keys}, sort_keys=True, separators=(",", ":")).encode()


def random_tensor(rng: np.random.Generator, shape, is_norm: bool, std: float) -> np.ndarray:
    if is_norm:
        return np.full(shape, 0x3F80, dtype=np.uint16)  # 1.0 in bf16
    n = int(np.prod(shape))
    out = np.empty(n, dtype=np.uint16)
    chunk = 1 << 24
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        vals = rng.standard_normal(e - s, dtype=np.float32)
        vals *= np.float32(std)
        out[s:e] = f32_to_bf16_bits(vals)
    return out.reshape(shape)


def write_record(f, name: str, bits: np.ndarray) -> None:
    nb = name.encode()
    f.write(struct.pack("<I", len(nb)))
    f.write(nb)
    f.write(struct.pack("<II", DTYPE_BF16, bits.ndim))
    for d in bits.shape:
        f.write(struct.pack("<Q", int(d)))
    raw = np.ascontiguousarray(bits, dtype=np.uint16).tobytes()
    f.write(struct.pack("<Q", len(raw)))
    f.write(raw)


def write_model(path: str | os.PathLike, cfg: dict | None = None, seed: int = 0,
                std: float = 0.02) -> Path:
    """Write a random-init Qwen3.bin; returns the path. Writes to a temp name, then renames."""
    cfg = dict(QWEN3_0_6B if cfg is None else cfg)
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(path.name + f".tmp{os.getpid()}")
    rng = np.random.default_rng(seed)
    plan = tensor_plan(cfg)
    meta = metadata_json(cfg)
    with open(tmp, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<IQ", VERSION, len(meta)))
        f.write(meta)
        f.write(struct.pack("<Q", len(plan)))
        for name, shape, is_norm in plan:
            write_record(f, name, random_tensor(rng, shape, is_norm, std))
    os.replace(tmp, path)
    return path


def random_block_weights(cfg: dict, seed: int, std: float = 0.02) -> list[np.ndarray]:
    """One decoder block's weights (BlockWeights order, include/inference.h:163-176) as bf16
    bits, drawn like write_model draws a layer."""
    rng = np.random.default_rng(seed)
    return [random_tensor(rng, shape(cfg), is_norm, std) for _, shape, is_norm in LAYER_TENSORS]


def cached_model(seed: int = 0, cfg: dict | None = None, cache_dir: str | None = None) -> Path:
    """Path of a random-init model file, generated on first use. The cache directory is
    $Q3_WEIGHTS_DIR, else /tmp/q3b200_weights."""
    cfg = dict(QWEN3_0_6B if cfg is None else cfg)
    d = Path(cache_dir or os.environ.get("Q3_WEIGHTS_DIR", "/tmp/q3b200_weights"))
    tag = "qwen3_0.6b" if cfg == QWEN3_0_6B else "cfg" + hashlib.sha1(metadata_json(cfg)).hexdigest()[:12]
    p = d / f"{tag}_seed{seed}.bin"
    if not p.exists():
        write_model(p, cfg, seed)
    return p


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("output", type=Path)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--std", type=float, default=0.02)
    ap.add_argument("--max-seq-len", type=int, default=QWEN3_0_6B["max_seq_len"])
    args = ap.parse_args()
    cfg = dict(QWEN3_0_6B, max_seq_len=args.max_seq_len)
    write_model(args.output, cfg, args.seed, args.std)


if __name__ == "__main__":
    main()
