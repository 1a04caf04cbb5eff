#!/usr/bin/env python3
"""Regenerate the golden fixtures of tests/golden/ from the reference engine itself.

    python tests/golden/make_golden.py

Runs the UNMODIFIED reference (asriva32/Qwen3.cpp src/inference.cpp, compiled into
oracle/_ref/libq3ref.so by oracle/Makefile) on seeded random-init weights written by
qwen3.cpp_b200/gen_weights.py, and stores its outputs:

  tiny_model.npz   a 2-layer model (dim 64, 4 Q / 2 KV heads of 16, vocab 256) at context 8, 20
                   tokens, so positions run past the context and the attention-sink ring buffer
                   wraps: logits, per-layer hidden states and every KV-cache row afterwards.
  qwen3_0.6b.npz   Qwen3-0.6B (seed 0), 4 tokens at context 512: top-64 logits, logit sums,
                   per-layer hidden states of the last token, KV rows; plus the weight file's
                   sha256 so a changed generator is caught.
  block.npz        one decoder block (tiny dims, seed 5) over a cache prefilled with N(0,1)
                   bf16 values, several (pos, kv_len) cases.
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(ROOT / "qwen3.cpp_b200"))

import gen_weights  # noqa: E402
import oracle  # noqa: E402

OUT = Path(__file__).resolve().parent

TINY_CFG = dict(gen_weights.QWEN3_0_6B, dim=64, hidden_dim=128, head_dim=16, n_layers=2,
                n_heads=4, n_kv_heads=2, vocab_size=256, max_seq_len=64, rotary_dim=16,
                rope_theta=10000.0, bos_token_id=1, eos_token_id=2)
TINY_SEED = 7
TINY_CTX = 8
TINY_TOKENS = [5, 17, 255, 0, 42, 42, 7, 100, 3, 9, 200, 11, 64, 128, 1, 2, 33, 250, 8, 77]

FULL_TOKENS = [17, 151935, 0, 4242]
FULL_CTX = 512

BLOCK_CFG = dict(dim=64, hidden_dim=96, head_dim=16, n_heads=4, n_kv_heads=2, max_seq_len=48,
                 rotary_dim=16, rope_theta=1000000.0, norm_eps=1e-6)
BLOCK_SEED = 5
BLOCK_CASES = [(0, 1), (5, 6), (31, 32), (47, 48)]  # (pos = kv_pos, kv_len)


def sha256(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            h.update(chunk)
    return h.hexdigest()


def tiny_model(tmp: Path) -> None:
    path = gen_weights.write_model(tmp / "tiny.bin", TINY_CFG, TINY_SEED)
    m = oracle.RefModel(path, TINY_CTX)
    L, D = TINY_CFG["n_layers"], TINY_CFG["dim"]
    logits, hidden, pos_math = [], [], []
    for pos, tok in enumerate(TINY_TOKENS):
        h, lg = m.forward(tok, pos, layers=True)
        logits.append(lg)
        hidden.append(h)
        pos_math.append(oracle.positions(pos, TINY_CTX))
    kvd = TINY_CFG["n_kv_heads"] * TINY_CFG["head_dim"]
    k = np.zeros((L, TINY_CTX, kvd), np.uint16)
    v = np.zeros((L, TINY_CTX, kvd), np.uint16)
    for l in range(L):
        for s in range(TINY_CTX):
            k[l, s], v[l, s] = m.kv_row(l, s)
    np.savez_compressed(OUT / "tiny_model.npz", tokens=np.array(TINY_TOKENS, np.int32),
                        ctx=TINY_CTX, seed=TINY_SEED, logits=np.stack(logits),
                        hidden=np.stack(hidden), k_cache=k, v_cache=v,
                        positions=np.array(pos_math, np.int32),
                        weights_sha256=sha256(path))


def full_model() -> None:
    path = gen_weights.cached_model(0)
    m = oracle.RefModel(path, FULL_CTX)
    tops_i, tops_v, sums, hid = [], [], [], None
    for pos, tok in enumerate(FULL_TOKENS):
        h, lg = m.forward(tok, pos, layers=True)
        order = np.argsort(-lg, kind="stable")[:64]
        tops_i.append(order.astype(np.int32))
        tops_v.append(lg[order])
        sums.append([float(lg.astype(np.float64).sum()), float((lg.astype(np.float64) ** 2).sum())])
        hid = h
    kv = {}
    for l in (0, 13, 27):
        for s in range(len(FULL_TOKENS)):
            kv[f"k_{l}_{s}"], kv[f"v_{l}_{s}"] = m.kv_row(l, s)
    np.savez_compressed(OUT / "qwen3_0.6b.npz", tokens=np.array(FULL_TOKENS, np.int32),
                        ctx=FULL_CTX, top_idx=np.stack(tops_i), top_val=np.stack(tops_v),
                        logit_sums=np.array(sums), hidden_last=hid,
                        weights_sha256=sha256(path), **kv)


def block() -> None:
    cfg = BLOCK_CFG
    w = gen_weights.random_block_weights(dict(cfg, n_layers=1), BLOCK_SEED)
    rng = np.random.default_rng(BLOCK_SEED + 100)
    kvd = cfg["n_kv_heads"] * cfg["head_dim"]
    k0 = gen_weights.f32_to_bf16_bits(rng.standard_normal((cfg["max_seq_len"], kvd), np.float32))
    v0 = gen_weights.f32_to_bf16_bits(rng.standard_normal((cfg["max_seq_len"], kvd), np.float32))
    xs, outs, ks, vs = [], [], [], []
    for pos, kv_len in BLOCK_CASES:
        b = oracle.RefBlock(cfg, w)
        b.set_cache(k0, v0)
        x = rng.standard_normal(cfg["dim"], np.float32)
        xs.append(x.copy())
        b.forward(x, pos, 0, pos, kv_len)
        outs.append(x)
        k, v = b.get_cache()
        ks.append(k[pos])
        vs.append(v[pos])
    np.savez_compressed(OUT / "block.npz", seed=BLOCK_SEED, k0=k0, v0=v0, x_in=np.stack(xs),
                        x_out=np.stack(outs), k_row=np.stack(ks), v_row=np.stack(vs),
                        cases=np.array(BLOCK_CASES, np.int32),
                        weights=np.concatenate([x.ravel() for x in w]))


def main() -> None:
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        tiny_model(Path(d))
    block()
    full_model()
    for p in sorted(OUT.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
