"""Known-answer tests of the reference's tst/test_block.cpp (lines 90-192), restated so that the
same checks run against the reference itself, the C oracle and the GPU path.

Each implementation supplies ``ops`` (rope, greedy, softmax) and ``make_block(cfg, weights)``
returning an object with ``forward(x, pos, num_sink, kv_pos, kv_len)``, ``reset()`` /
``reset_cache()`` and ``get_cache()``; range errors must raise an exception whose class name or
code marks it as out_of_range.
"""
from __future__ import annotations

import math

import numpy as np

import gen_weights

TOL = 1e-5  # CheckNear, tst/test_block.cpp:19-25


def bf16(x: float) -> np.uint16:
    return gen_weights.f32_to_bf16_bits(np.array([x], np.float32))[0]


def round_bf16(x: float) -> float:
    return float(gen_weights.bf16_bits_to_f32(np.array([bf16(x)]))[0])


def _w(vals, shape=None):
    a = gen_weights.f32_to_bf16_bits(np.array(vals, np.float32))
    return a.reshape(shape) if shape else a


def near(actual, expected, what):
    assert abs(float(actual) - float(expected)) <= TOL, f"{what}: expected {expected}, got {actual}"


def check_rope(rope_fn):
    """tst/test_block.cpp:90-97: ApplyRotaryEmb(rotary, 4, 4, 1, 10000, 4)."""
    r = rope_fn(np.array([1.0, 2.0, 3.0, 4.0], np.float32), 4, 1, 10000.0, 4)
    near(r[0], math.cos(1.0) - 3.0 * math.sin(1.0), "rotary first half 0")
    near(r[2], 3.0 * math.cos(1.0) + math.sin(1.0), "rotary second half 0")
    near(r[1], 2.0 * math.cos(0.01) - 4.0 * math.sin(0.01), "rotary first half 1")
    near(r[3], 4.0 * math.cos(0.01) + 2.0 * math.sin(0.01), "rotary second half 1")


def check_greedy(greedy_fn):
    """tst/test_block.cpp:99-100."""
    assert greedy_fn(np.array([-2.0, 0.5, 0.25], np.float32)) == 1


def check_softmax(softmax_fn):
    """tst/test_block.cpp:102-115: stability with large negative inputs."""
    s = softmax_fn(np.array([-10000.0, -10001.0, -10002.0], np.float32))
    tot = 1.0 + math.exp(-1.0) + math.exp(-2.0)
    near(s[0], 1.0 / tot, "softmax large-negative value 0")
    near(s[1], math.exp(-1.0) / tot, "softmax large-negative value 1")
    near(s[2], math.exp(-2.0) / tot, "softmax large-negative value 2")


def expanded_config():
    return dict(dim=2, hidden_dim=2, head_dim=2, n_heads=2, n_kv_heads=1, max_seq_len=2,
                rotary_dim=2, rope_theta=10000.0, norm_eps=1e-5)


def expanded_weights():
    """MakeExpandedQueryWeights, tst/test_block.cpp:70-84."""
    return [_w([1, 1]), _w([1, 1]), _w([1, 1]), _w([0] * 8, (4, 2)), _w([0] * 4, (2, 2)),
            _w([0] * 4, (2, 2)), _w([0] * 8, (2, 4)), _w([1, 1]), _w([0] * 4, (2, 2)),
            _w([0] * 4, (2, 2)), _w([0] * 4, (2, 2))]


def block_config():
    return dict(dim=4, hidden_dim=2, head_dim=2, n_heads=2, n_kv_heads=1, max_seq_len=4,
                rotary_dim=2, rope_theta=10000.0, norm_eps=1e-5)


def block_weights():
    """MakeWeights, tst/test_block.cpp:48-68."""
    eye = np.eye(4, dtype=np.float32)
    return [_w([1] * 4), _w([1, 1]), _w([1, 1]), _w([0] * 16, (4, 4)),
            _w([1, 0, 0, 0, 0, 1, 0, 0], (2, 4)), _w([0, 0, 1, 0, 0, 0, 0, 1], (2, 4)),
            _w(eye.ravel(), (4, 4)), _w([1] * 4), _w([0] * 8, (2, 4)), _w([0] * 8, (4, 2)),
            _w([0] * 8, (2, 4))]


def is_out_of_range(exc: BaseException) -> bool:
    return (getattr(exc, "code", None) == 3 or "OutOfRange" in type(exc).__name__
            or isinstance(exc, IndexError))


def check_blocks(make_block):
    """tst/test_block.cpp:117-192."""
    # Expanded-query GQA block: zero projections leave the residual stream unchanged.
    b = make_block(expanded_config(), expanded_weights())
    x = np.array([1.0, -1.0], np.float32)
    b.forward(x, 0, 0, 0, 1)
    near(x[0], 1.0, "expanded-query residual 0")
    near(x[1], -1.0, "expanded-query residual 1")

    cfg = block_config()
    b = make_block(cfg, block_weights())
    x = np.array([1.0, 2.0, 3.0, 4.0], np.float32)
    rms = math.sqrt(7.5 + cfg["norm_eps"])
    b.forward(x, 0, 0, 0, 1)
    # Both query heads share the only KV head, so both receive the same value.
    cv0, cv1 = round_bf16(3.0 / rms), round_bf16(4.0 / rms)
    near(x[0], 1.0 + cv0, "first attention residual")
    near(x[1], 2.0 + cv1, "second attention residual")
    near(x[2], 3.0 + cv0, "GQA first value")
    near(x[3], 4.0 + cv1, "GQA second value")
    k, v = b.get_cache()
    key_rms = math.sqrt(((1.0 / rms) ** 2 + (2.0 / rms) ** 2) / 2.0 + cfg["norm_eps"])
    f = gen_weights.bf16_bits_to_f32
    near(f(k[0, 0:1])[0], round_bf16((1.0 / rms) / key_rms), "cached normalized key 0")
    near(f(k[0, 1:2])[0], round_bf16((2.0 / rms) / key_rms), "cached normalized key 1")
    near(f(v[0, 0:1])[0], cv0, "cached value 0")
    near(f(v[0, 1:2])[0], cv1, "cached value 1")

    (b.reset_cache if hasattr(b, "reset_cache") else b.reset)()
    k, v = b.get_cache()
    assert not k.any(), "ResetCache did not clear keys"
    assert not v.any(), "ResetCache did not clear values"

    try:
        b.forward(x, 4, 1, 0, 4)
    except Exception as e:  # noqa: BLE001 - the reference throws std::out_of_range
        assert is_out_of_range(e), f"wrong error kind: {e!r}"
    else:
        raise AssertionError("Block accepted a write into the sink region")
