"""The C-ABI library builds for sm_100a, loads without a GPU, exports every symbol its headers
declare, and applies the reference loader's checks (which run before any CUDA call)."""
import ctypes as C
import re
import struct
from pathlib import Path

import numpy as np
import pytest

import gen_weights

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        if 'extern "C"' not in text:
            continue
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        for m in re.finditer(r"\b(q3_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


def test_library_exports_declared_symbols(q3lib):
    L = q3lib.lib()
    syms = declared_symbols()
    assert len(syms) >= 25
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing


def test_version_and_error_plumbing(q3lib):
    assert b"sm_100a" in q3lib.lib().q3_version()
    with pytest.raises(q3lib.InvalidArgument):
        q3lib.check(q3lib.lib().q3_model_load(None, 512, 0, None))


def _write_tiny(path, **over):
    cfg = dict(gen_weights.QWEN3_0_6B, dim=32, hidden_dim=64, head_dim=16, n_layers=1, n_heads=2,
               n_kv_heads=1, vocab_size=50, max_seq_len=64, rotary_dim=16)
    cfg.update(over)
    return gen_weights.write_model(path, cfg, 0)


def _load_error(q3lib, path, ctx=16):
    h = C.c_void_p()
    st = q3lib.lib().q3_model_load(str(path).encode(), ctx, 0, C.byref(h))
    return st, q3lib.lib().q3_last_error().decode()


def test_loader_errors_match_reference_kinds(q3lib, tmp_path):
    p = _write_tiny(tmp_path / "ok.bin")
    raw = bytearray(p.read_bytes())
    # Missing file -> runtime_error "Failed to open model file" (src/inference.cpp:446-449).
    st, msg = _load_error(q3lib, tmp_path / "nope.bin")
    assert st == 1 and "Failed to open model file" in msg
    # Bad magic (:451-455).
    bad = bytearray(raw)
    bad[0:8] = b"QWEN3XX\0"
    (tmp_path / "magic.bin").write_bytes(bad)
    st, msg = _load_error(q3lib, tmp_path / "magic.bin")
    assert st == 1 and "magic" in msg
    # Bad version (:457-460).
    bad = bytearray(raw)
    bad[8:12] = struct.pack("<I", 2)
    (tmp_path / "ver.bin").write_bytes(bad)
    st, msg = _load_error(q3lib, tmp_path / "ver.bin")
    assert st == 1 and "version" in msg
    # Truncated payload.
    (tmp_path / "trunc.bin").write_bytes(raw[: len(raw) - 10])
    st, msg = _load_error(q3lib, tmp_path / "trunc.bin")
    assert st == 1
    # Context outside (0, max_seq_len] -> invalid_argument (:530-532).
    for ctx in (0, -3, 65):
        st, msg = _load_error(q3lib, p, ctx)
        assert st == 2 and "Context length" in msg, (ctx, st, msg)
    # Config validation -> invalid_argument (:145-157).
    p2 = _write_tiny(tmp_path / "heads.bin", n_heads=3, n_kv_heads=2)
    st, msg = _load_error(q3lib, p2)
    assert st == 2 and "divisible" in msg
    # Non-bf16 file dtype -> runtime_error (:465-467).
    p3 = _write_tiny(tmp_path / "dtype.bin", dtype="fp32")
    st, msg = _load_error(q3lib, p3)
    assert st == 1 and "bf16" in msg


def test_block_create_validates_sizes(q3lib):
    import kats
    cfg = kats.block_config()
    w = kats.block_weights()
    w[3] = w[3][:2]  # wrong wq size -> invalid_argument (src/inference.cpp:744-751)
    with pytest.raises(q3lib.InvalidArgument, match="wq"):
        q3lib.Block(cfg, w)


def test_oracle_reader_matches_file_layout(tmp_path):
    import oracle
    p = _write_tiny(tmp_path / "x.bin")
    cfg, recs = oracle.read_qwen3_bin(p)
    assert cfg["dim"] == 32 and cfg["tie_word_embeddings"] is True
    assert len(recs) == 1 + 11 + 1  # embed, one layer, final norm (tied: no output record)
    assert recs["model.embed.weight"].shape == (50, 32)
    assert recs["model.layers.0.attn.wq.weight"].byte_size == 32 * 32 * 2
    wf = oracle.WeightFile(p)
    assert np.all(wf.tensor("model.norm.weight") == 0x3F80)


def test_full_weight_file_layout(full_weights):
    """Shapes and record count the reference's loader test pins (tst/test_loader.cpp:35-68),
    minus the three tokenizer records a random-init file does not carry."""
    import oracle
    cfg, recs = oracle.read_qwen3_bin(full_weights)
    assert (cfg["dim"], cfg["hidden_dim"], cfg["head_dim"], cfg["n_layers"], cfg["n_heads"],
            cfg["n_kv_heads"], cfg["vocab_size"]) == (1024, 3072, 128, 28, 16, 8, 151936)
    assert cfg["tie_word_embeddings"] and cfg["qk_norm"]
    assert len(recs) == 313 - 3
    e = recs["model.embed.weight"]
    assert e.shape == (151936, 1024) and e.byte_size == 311164928 and e.data_offset > 0
    assert recs["model.layers.0.attn.q_norm.weight"].shape == (128,)
