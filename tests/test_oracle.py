"""The oracle pinned against the reference: its own known-answer tests (tst/test_block.cpp), the
golden fixtures generated from the reference engine (tests/golden/make_golden.py), and - where
the reference library is built - bit-exact agreement on seeded random inputs."""
import numpy as np
import pytest

import gen_weights
import kats
import oracle

IMPLS = ["port"] + (["reference"] if oracle.ref_available() else [])


def _ops(kind):
    return oracle.port_ops if kind == "port" else oracle.ref_ops


def _block_cls(kind):
    return oracle.PortBlock if kind == "port" else oracle.RefBlock


@pytest.mark.parametrize("kind", IMPLS)
def test_known_answers_ops(kind):
    ops = _ops(kind)
    kats.check_rope(lambda x, hd, pos, th, rd: ops.rope(x, hd, pos, th, rd))
    kats.check_greedy(ops.greedy)
    kats.check_softmax(ops.softmax)


@pytest.mark.parametrize("kind", IMPLS)
def test_known_answers_block(kind):
    kats.check_blocks(lambda cfg, w: _block_cls(kind)(cfg, w))


def test_positions_ring_buffer():
    """num_sink / kv_pos / kv_len of src/inference.cpp:605-613."""
    for ctx in (1, 2, 5, 8, 512):
        for pos in range(0, 3 * ctx + 7):
            ns, kp, kl = oracle.positions(pos, ctx)
            if pos < ctx:
                assert (ns, kp, kl) == (0, pos, pos + 1)
            else:
                s = min(4, ctx - 1)
                assert ns == s and kl == ctx
                assert kp == s + (pos - s) % (ctx - s)


def test_port_tiny_model_matches_golden(tmp_path, golden):
    g = golden["tiny_model"]
    import make_golden
    path = gen_weights.write_model(tmp_path / "tiny.bin", make_golden.TINY_CFG, int(g["seed"]))
    m = oracle.PortModel(path, int(g["ctx"]))
    for pos, tok in enumerate(g["tokens"]):
        assert oracle.positions(pos, int(g["ctx"])) == tuple(g["positions"][pos])
        h, lg = m.forward(int(tok), pos, layers=True)
        np.testing.assert_array_equal(lg, g["logits"][pos])
        np.testing.assert_array_equal(h, g["hidden"][pos])
    for l in range(g["k_cache"].shape[0]):
        for s in range(g["k_cache"].shape[1]):
            k, v = m.kv_row(l, s)
            np.testing.assert_array_equal(k, g["k_cache"][l, s])
            np.testing.assert_array_equal(v, g["v_cache"][l, s])


def test_port_block_matches_golden(golden):
    g = golden["block"]
    import make_golden
    cfg = make_golden.BLOCK_CFG
    w = gen_weights.random_block_weights(dict(cfg, n_layers=1), int(g["seed"]))
    np.testing.assert_array_equal(np.concatenate([x.ravel() for x in w]), g["weights"])
    for i, (pos, kv_len) in enumerate(g["cases"]):
        b = oracle.PortBlock(cfg, w)
        b.set_cache(g["k0"], g["v0"])
        x = g["x_in"][i].copy()
        b.forward(x, int(pos), 0, int(pos), int(kv_len))
        np.testing.assert_array_equal(x, g["x_out"][i])
        k, v = b.get_cache()
        np.testing.assert_array_equal(k[pos], g["k_row"][i])
        np.testing.assert_array_equal(v[pos], g["v_row"][i])


@pytest.mark.slow
def test_port_full_model_matches_golden(full_weights, golden):
    g = golden["qwen3_0.6b"]
    m = oracle.PortModel(full_weights, int(g["ctx"]))
    for pos, tok in enumerate(g["tokens"]):
        h, lg = m.forward(int(tok), pos, layers=True)
        np.testing.assert_array_equal(lg[g["top_idx"][pos]], g["top_val"][pos])
        order = np.argsort(-lg, kind="stable")[:64]
        np.testing.assert_array_equal(order, g["top_idx"][pos])
        s = lg.astype(np.float64)
        assert s.sum() == g["logit_sums"][pos][0] and (s * s).sum() == g["logit_sums"][pos][1]
    np.testing.assert_array_equal(h, g["hidden_last"])
    for l in (0, 13, 27):
        for s in range(len(g["tokens"])):
            k, v = m.kv_row(l, s)
            np.testing.assert_array_equal(k, g[f"k_{l}_{s}"])
            np.testing.assert_array_equal(v, g[f"v_{l}_{s}"])


@pytest.mark.skipif(not oracle.ref_available(), reason="reference library not built")
def test_port_ops_bit_exact_vs_reference():
    rng = np.random.default_rng(11)
    P, R = oracle.port_ops, oracle.ref_ops
    for n in (1, 7, 16, 33, 1024, 3072):
        x = rng.standard_normal(n).astype(np.float32)
        w = gen_weights.f32_to_bf16_bits(rng.standard_normal(n).astype(np.float32))
        np.testing.assert_array_equal(P.rmsnorm(x, w, 1e-6), R.rmsnorm(x, w, 1e-6))
        np.testing.assert_array_equal(P.softmax(x * 30), R.softmax(x * 30))
        assert P.greedy(x) == R.greedy(x)
    for n, m in ((5, 17), (64, 1024), (3, 3072)):
        x = rng.standard_normal(m).astype(np.float32)
        w = gen_weights.f32_to_bf16_bits(0.02 * rng.standard_normal((n, m)).astype(np.float32))
        np.testing.assert_array_equal(P.matmul(x, w), R.matmul(x, w))
    for pos in (0, 1, 77, 4095, 32767):
        x = rng.standard_normal(2048).astype(np.float32)
        np.testing.assert_array_equal(P.rope(x, 128, pos, 1e6, 128), R.rope(x, 128, pos, 1e6, 128))
    for kv_len in (1, 9, 200):
        q = rng.standard_normal(128).astype(np.float32)
        k = gen_weights.f32_to_bf16_bits(rng.standard_normal((kv_len, 1024)).astype(np.float32))
        v = gen_weights.f32_to_bf16_bits(rng.standard_normal((kv_len, 1024)).astype(np.float32))
        for off in (0, 384):
            np.testing.assert_array_equal(P.attn(q, k, v, 128, 8, kv_len, off),
                                          R.attn(q, k, v, 128, 8, kv_len, off))
    w1 = gen_weights.f32_to_bf16_bits(0.02 * rng.standard_normal((96, 64)).astype(np.float32))
    w2 = gen_weights.f32_to_bf16_bits(0.02 * rng.standard_normal((64, 96)).astype(np.float32))
    w3 = gen_weights.f32_to_bf16_bits(0.02 * rng.standard_normal((96, 64)).astype(np.float32))
    x = rng.standard_normal(64).astype(np.float32)
    np.testing.assert_array_equal(P.ffn(x, w1, w2, w3), R.ffn(x, w1, w2, w3))


@pytest.mark.skipif(not oracle.ref_available(), reason="reference library not built")
def test_port_block_bit_exact_vs_reference_with_wrap():
    """Random block, positions past the context (sink re-rotation active)."""
    cfg = dict(dim=64, hidden_dim=96, head_dim=16, n_heads=4, n_kv_heads=2, max_seq_len=8,
               rotary_dim=16, rope_theta=10000.0, norm_eps=1e-6)
    w = gen_weights.random_block_weights(dict(cfg, n_layers=1), 3, std=0.2)
    bp, br = oracle.PortBlock(cfg, w), oracle.RefBlock(cfg, w)
    rng = np.random.default_rng(4)
    for pos in range(20):
        ns, kp, kl = oracle.positions(pos, cfg["max_seq_len"])
        x = rng.standard_normal(cfg["dim"]).astype(np.float32)
        xp, xr = x.copy(), x.copy()
        bp.forward(xp, pos, ns, kp, kl)
        br.forward(xr, pos, ns, kp, kl)
        np.testing.assert_array_equal(xp, xr)
        for a, b in zip(bp.get_cache(), br.get_cache()):
            np.testing.assert_array_equal(a, b)


def test_port_rejects_bad_ranges():
    cfg = kats.block_config()
    b = oracle.PortBlock(cfg, kats.block_weights())
    x = np.zeros(4, np.float32)
    for args in ((-1, 0, 0, 1), (0, 0, 0, 0), (0, 0, 0, 5), (0, 0, 1, 1), (0, 2, 0, 1),
                 (0, 4, 0, 4), (4, 1, 0, 4)):
        with pytest.raises(oracle.OracleError) as e:
            b.forward(x, *args)
        assert e.value.code == 3


def test_port_forward_many_is_tokenwise_bit_exact(tmp_path):
    """The layer-by-layer many-token oracle (used for long prompts) equals token-by-token
    ForwardToken calls bit for bit: logits, argmax, per-layer hidden states of the last token,
    KV rows, and a token-wise step afterwards; and rejects a range that would wrap the ring."""
    cfg = dict(gen_weights.QWEN3_0_6B, n_layers=2, vocab_size=4096)
    path = gen_weights.write_model(tmp_path / "m.bin", cfg, seed=3)
    toks = np.random.default_rng(1).integers(0, 4096, 71).astype(np.int32)
    a, b = oracle.PortModel(path, 128), oracle.PortModel(path, 128)
    for pos in range(10):
        a.forward(int(toks[pos]), pos)
        b.forward(int(toks[pos]), pos)
    lgs = []
    for pos in range(10, 71):
        h, lg = a.forward(int(toks[pos]), pos, layers=True)
        lgs.append(lg)
    want = np.ones(61, bool)
    want[5:20] = False
    r = b.forward_many(toks[10:], 10, want=want, logits=True, layers=True)
    np.testing.assert_array_equal(r["logits"], np.stack(lgs)[want])
    assert np.array_equal(r["argmax"][want], np.stack(lgs)[want].argmax(axis=1))
    assert np.all(r["argmax"][~want] == -1)
    np.testing.assert_array_equal(r["hidden_last"], h)
    for l in range(2):
        for s in (0, 9, 10, 42, 70):
            for x, y in zip(a.kv_row(l, s), b.kv_row(l, s)):
                np.testing.assert_array_equal(x, y)
    np.testing.assert_array_equal(a.forward(5, 71), b.forward(5, 71))
    with pytest.raises(oracle.OracleError):
        b.forward_many(toks[:60], 100)
