"""GPU parity of the free kernels and of one decoder block against the oracle (C restatement of
the reference, bit-exact with it), through the C ABI."""
import numpy as np
import pytest

import gen_weights
import kats
import oracle

pytestmark = pytest.mark.gpu

P = oracle.port_ops


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


def _dev(torch, a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).cuda()
    return torch.from_numpy(a.copy()).cuda()


def _host(t, dtype=np.float32):
    a = t.cpu().numpy()
    return a.view(np.uint16) if dtype == np.uint16 else a


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


class GpuOps:
    def __init__(self, torch, q3):
        self.t = torch
        self.q3 = q3

    def sync(self):
        self.t.cuda.synchronize()

    def rope(self, x, head_dim, pos, theta, rotary_dim):
        d = _dev(self.t, np.asarray(x, np.float32))
        self.q3.rope(d.data_ptr(), d.numel(), head_dim, pos, theta, rotary_dim)
        self.sync()
        return _host(d)

    def greedy(self, x):
        d = _dev(self.t, np.asarray(x, np.float32))
        out = self.t.zeros(1, dtype=self.t.int32, device="cuda")
        self.q3.greedy(d.data_ptr(), d.numel(), out.data_ptr())
        self.sync()
        return int(out.item())

    def softmax(self, x):
        d = _dev(self.t, np.asarray(x, np.float32))
        self.q3.softmax(d.data_ptr(), d.data_ptr(), d.numel())
        self.sync()
        return _host(d)

    def rmsnorm(self, x, w, eps):
        dx, dw = _dev(self.t, x), _dev(self.t, w)
        out = self.t.empty_like(dx)
        self.q3.rmsnorm(out.data_ptr(), dx.data_ptr(), dw.data_ptr(), eps, dx.numel())
        self.sync()
        return _host(out)

    def matmul(self, x, w):
        dx, dw = _dev(self.t, x), _dev(self.t, w)
        out = self.t.empty(w.shape[0], dtype=self.t.float32, device="cuda")
        self.q3.matmul(out.data_ptr(), dx.data_ptr(), dw.data_ptr(), w.shape[0], w.shape[1])
        self.sync()
        return _host(out)

    def ffn(self, x, w1, w2, w3):
        hidden, dim = w1.shape
        dx = _dev(self.t, x)
        d1, d2, d3 = _dev(self.t, w1), _dev(self.t, w2), _dev(self.t, w3)
        out = self.t.empty(dim, dtype=self.t.float32, device="cuda")
        l1 = self.t.empty(hidden, dtype=self.t.float32, device="cuda")
        l2 = self.t.empty(hidden, dtype=self.t.float32, device="cuda")
        self.q3.ffn(out.data_ptr(), l1.data_ptr(), l2.data_ptr(), dx.data_ptr(), d1.data_ptr(),
                    d2.data_ptr(), d3.data_ptr(), hidden, dim)
        self.sync()
        return _host(out)

    def attn(self, q, k, v, head_dim, n_kv_heads, kv_len, head_offset=0):
        dq, dk, dv = _dev(self.t, q), _dev(self.t, k), _dev(self.t, v)
        out = self.t.empty(head_dim, dtype=self.t.float32, device="cuda")
        ws = self.t.empty(self.q3.attn_workspace_size(head_dim, kv_len), dtype=self.t.uint8,
                          device="cuda")
        self.q3.attn(out.data_ptr(), ws.data_ptr(), dq.data_ptr(), dk.data_ptr() + 2 * head_offset,
                     dv.data_ptr() + 2 * head_offset, head_dim, n_kv_heads, kv_len)
        self.sync()
        return _host(out)


@pytest.fixture(scope="module")
def gops(torch_cuda, q3lib):
    return GpuOps(torch_cuda, q3lib)


def test_known_answers_gpu_ops(gops):
    kats.check_rope(gops.rope)
    kats.check_greedy(gops.greedy)
    kats.check_softmax(gops.softmax)


def test_known_answers_gpu_block(q3lib):
    kats.check_blocks(lambda cfg, w: q3lib.Block(cfg, w))


def test_greedy_ties_and_sizes(gops):
    rng = np.random.default_rng(0)
    for n in (1, 2, 31, 1000, 151936):
        x = rng.standard_normal(n).astype(np.float32)
        assert gops.greedy(x) == P.greedy(x)
        if n > 3:
            x[n // 3] = x[n - 1] = x.max() + 1.0  # tie: the lowest index wins
            assert gops.greedy(x) == n // 3
    with pytest.raises(gops.q3.InvalidArgument):
        gops.q3.greedy(0, 0, 0)


def test_free_kernels_vs_oracle(gops):
    rng = np.random.default_rng(1)
    for n in (1, 7, 128, 1024, 3072):
        x = rng.standard_normal(n).astype(np.float32)
        w = gen_weights.f32_to_bf16_bits(rng.standard_normal(n).astype(np.float32))
        np.testing.assert_allclose(gops.rmsnorm(x, w, 1e-6), P.rmsnorm(x, w, 1e-6), rtol=2e-6,
                                   atol=1e-6)
        np.testing.assert_allclose(gops.softmax(x * 20), P.softmax(x * 20), rtol=1e-5, atol=1e-7)
    for n, m in ((5, 17), (2048, 1024), (1024, 3072), (151936, 1024), (3, 9)):
        x = rng.standard_normal(m).astype(np.float32)
        w = gen_weights.f32_to_bf16_bits(0.02 * rng.standard_normal((n, m)).astype(np.float32))
        np.testing.assert_allclose(gops.matmul(x, w), P.matmul(x, w), rtol=1e-4, atol=2e-5)
    for pos in (0, 1, 511, 32767):
        x = rng.standard_normal(2048).astype(np.float32)
        np.testing.assert_allclose(gops.rope(x, 128, pos, 1e6, 128), P.rope(x, 128, pos, 1e6, 128),
                                   rtol=1e-6, atol=1e-6)
    w1 = gen_weights.f32_to_bf16_bits(0.02 * rng.standard_normal((3072, 1024)).astype(np.float32))
    w2 = gen_weights.f32_to_bf16_bits(0.02 * rng.standard_normal((1024, 3072)).astype(np.float32))
    w3 = gen_weights.f32_to_bf16_bits(0.02 * rng.standard_normal((3072, 1024)).astype(np.float32))
    x = rng.standard_normal(1024).astype(np.float32)
    assert rel_l2(gops.ffn(x, w1, w2, w3), P.ffn(x, w1, w2, w3)) < 1e-5
    for kv_len in (1, 9, 300, 5000):
        q = rng.standard_normal(128).astype(np.float32)
        k = gen_weights.f32_to_bf16_bits(rng.standard_normal((kv_len, 1024)).astype(np.float32))
        v = gen_weights.f32_to_bf16_bits(rng.standard_normal((kv_len, 1024)).astype(np.float32))
        for off in (0, 896):
            got = gops.attn(q, k, v, 128, 8, kv_len, off)
            want = P.attn(q, k, v, 128, 8, kv_len, off)
            np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-5)


def _block_cfg(max_seq_len):
    c = gen_weights.QWEN3_0_6B
    return dict(dim=c["dim"], hidden_dim=c["hidden_dim"], head_dim=c["head_dim"],
                n_heads=c["n_heads"], n_kv_heads=c["n_kv_heads"], max_seq_len=max_seq_len,
                rotary_dim=c["rotary_dim"], rope_theta=c["rope_theta"], norm_eps=c["norm_eps"])


@pytest.mark.parametrize("length", [1, 128, 2048, 8192])
def test_block_parity_qwen3_shapes(q3lib, length):
    """A Qwen3-0.6B decoder block (weights N(0,0.02) from seed 1) over a KV cache prefilled with
    N(0,1) bf16 values to `length` rows, input hidden state N(0,1) at position `length`."""
    cfg = _block_cfg(length + 1)
    w = gen_weights.random_block_weights(dict(cfg, n_layers=1), 1)
    rng = np.random.default_rng(1000 + length)
    kvd = cfg["n_kv_heads"] * cfg["head_dim"]
    k0 = gen_weights.f32_to_bf16_bits(rng.standard_normal((length + 1, kvd)).astype(np.float32))
    v0 = gen_weights.f32_to_bf16_bits(rng.standard_normal((length + 1, kvd)).astype(np.float32))
    x = rng.standard_normal(cfg["dim"]).astype(np.float32)
    ob = oracle.PortBlock(cfg, w)
    ob.set_cache(k0, v0)
    gb = q3lib.Block(cfg, w)
    gb.set_cache(k0, v0)
    xo, xg = x.copy(), x.copy()
    ob.forward(xo, length, 0, length, length + 1)
    gb.forward(xg, length, 0, length, length + 1)
    assert rel_l2(xg, xo) <= 1e-5, rel_l2(xg, xo)
    ko, vo = ob.get_cache()
    kg, vg = gb.get_cache()
    # Rows other than the written slot are untouched, bit for bit.
    np.testing.assert_array_equal(np.delete(kg, length, 0), np.delete(k0, length, 0))
    np.testing.assert_array_equal(np.delete(vg, length, 0), np.delete(v0, length, 0))
    # The written row agrees to within one bf16 ulp (fp32 summation order differs).
    for a, b in ((kg[length], ko[length]), (vg[length], vo[length])):
        d = np.abs(a.astype(np.int32) - b.astype(np.int32))
        assert d.max() <= 1 and (d > 0).mean() < 0.02


def test_block_golden_through_gpu(q3lib, golden):
    import make_golden
    g = golden["block"]
    cfg = make_golden.BLOCK_CFG
    w = gen_weights.random_block_weights(dict(cfg, n_layers=1), int(g["seed"]))
    for i, (pos, kv_len) in enumerate(g["cases"]):
        b = q3lib.Block(cfg, w)
        b.set_cache(g["k0"], g["v0"])
        x = g["x_in"][i].copy()
        b.forward(x, int(pos), 0, int(pos), int(kv_len))
        assert rel_l2(x, g["x_out"][i]) < 1e-5


def test_block_wrap_matches_oracle(q3lib):
    """Positions past the context: ring-buffer slots and sink re-rotation on the GPU."""
    cfg = dict(dim=64, hidden_dim=96, head_dim=16, n_heads=4, n_kv_heads=2, max_seq_len=8,
               rotary_dim=16, rope_theta=10000.0, norm_eps=1e-6)
    w = gen_weights.random_block_weights(dict(cfg, n_layers=1), 3, std=0.2)
    ob, gb = oracle.PortBlock(cfg, w), q3lib.Block(cfg, w)
    rng = np.random.default_rng(4)
    for pos in range(24):
        ns, kp, kl = oracle.positions(pos, cfg["max_seq_len"])
        x = rng.standard_normal(cfg["dim"]).astype(np.float32)
        xo, xg = x.copy(), x.copy()
        ob.forward(xo, pos, ns, kp, kl)
        gb.forward(xg, pos, ns, kp, kl)
        assert rel_l2(xg, xo) < 1e-4, pos
        for a, b in zip(gb.get_cache(), ob.get_cache()):
            np.testing.assert_allclose(gen_weights.bf16_bits_to_f32(a),
                                       gen_weights.bf16_bits_to_f32(b), rtol=2e-2, atol=1e-3)
