"""Tensor-parallel decode (q3_tp_*) against the oracle.

world = 1 runs the shard/all-reduce code paths with a single rank on one GPU; world = 2 runs two
ranks on two GPUs (child processes through torch.distributed.run; skipped with fewer GPUs).
Teacher-forced top-1 agreement with the oracle >= 99%, and every rank returns the same tokens.
"""
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
TOP1_AGREEMENT = 0.99
PROMPT, STEPS, CTX = 40, 24, 512


def _gpu_count():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.fixture(scope="module")
def case(full_weights):
    rng = np.random.default_rng(41)
    prompt = rng.integers(0, 151936, PROMPT).astype(np.int32)
    cont = rng.integers(0, 151936, STEPS).astype(np.int32)
    cpu = oracle.PortModel(full_weights, CTX)
    am = []
    for pos, t in enumerate(np.concatenate([prompt, cont])):
        am.append(int(np.argmax(cpu.forward(int(t), pos))))
    return prompt, cont, np.array(am)


@pytest.mark.parametrize("solo_allreduce", [False, True])
def test_tp_single_rank(q3lib, full_weights, case, solo_allreduce):
    """World 1; with solo_allreduce the o_proj / down_proj partials go through the all-reduce
    kernel (this rank its only member), so the exchange-buffer code runs on one GPU."""
    prompt, cont, ref = case
    m = q3lib.Qwen3(full_weights, CTX)
    try:
        _, nxt = m.prefill(prompt, 0)
        assert nxt == ref[PROMPT - 1]
        tp = q3lib.TpDecoder(m, 0, 1)
        tp.connect([tp.ipc_handle()])
        tp.configure(solo_allreduce=solo_allreduce)
        am = tp.decode_forced(cont, PROMPT)
        assert float((am == ref[PROMPT:PROMPT + STEPS]).mean()) >= TOP1_AGREEMENT
        free = tp.decode(int(am[-1]), PROMPT + STEPS, 8)
        assert free.shape == (8,) and np.all((free >= 0) & (free < 151936))
        with pytest.raises(q3lib.OutOfRange):
            tp.decode(0, CTX - 2, 4)  # past the context
        tp.close()
    finally:
        m.close()


def test_tp_wait_timeout_refuses_then_resets(q3lib, full_weights):
    """A peer that never answers: a world-2 decoder whose peer slot is its own buffer (nothing
    raises that peer's flag). Every bounded wait runs out after a short budget; decode reports
    DeviceTimeout promptly (later all-reduces of the step see the error and skip their waits),
    then refuses to decode until reset; reset clears the refusal."""
    import time
    m = q3lib.Qwen3(full_weights, 64)
    try:
        tp = q3lib.TpDecoder(m, 0, 2)
        h = tp.ipc_handle()
        tp.connect([h, h])
        tp.configure(wait_cycles=20_000_000)  # ~10 ms at the boost clock
        _, nxt = m.prefill(np.arange(8, dtype=np.int32), 0)
        t0 = time.perf_counter()
        with pytest.raises(q3lib.DeviceTimeout):
            tp.decode(nxt, 8, 4)
        assert time.perf_counter() - t0 < 20.0
        with pytest.raises(q3lib.Q3RuntimeError) as e:
            tp.decode(nxt, 8, 1)
        assert not isinstance(e.value, q3lib.DeviceTimeout)
        tp.reset()
        with pytest.raises(q3lib.DeviceTimeout):  # still no peer: times out again, not refused
            tp.decode(nxt, 8, 1)
        tp.close()
    finally:
        m.close()


def _run_workers(full_weights, case, tmp_path, mode):
    prompt, cont, ref = case
    inputs = tmp_path / "inputs.npz"
    np.savez(inputs, prompt=prompt, cont=cont, ctx=CTX)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = tmp_path / "res"
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1",
           f"--master-port={port}", str(ROOT / "tests" / "tp_worker.py"), str(full_weights),
           str(inputs), str(out), mode]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    return [np.load(f"{out}.rank{k}.npz") for k in range(2)]


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
def test_tp_peer_leaves_between_steps(full_weights, case, tmp_path):
    """Rank 1 stops taking part after a first decode call (it leaves between steps, with nothing
    of its own in flight); rank 0's next decode ends with DeviceTimeout within its short wait
    budget and then refuses further steps."""
    res = _run_workers(full_weights, case, tmp_path, "leave")
    assert int(res[0]["timed_out"]) == 1 and int(res[0]["refused"]) == 1
    assert float(res[0]["seconds"]) < 20.0


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
def test_tp_two_ranks(full_weights, case, tmp_path):
    prompt, cont, ref = case
    res = _run_workers(full_weights, case, tmp_path, "decode")
    for k in range(2):
        assert int(res[k]["next"]) == ref[PROMPT - 1]
        assert float((res[k]["argmax"] == ref[PROMPT:PROMPT + STEPS]).mean()) >= TOP1_AGREEMENT
    assert np.array_equal(res[0]["argmax"], res[1]["argmax"])
    assert np.array_equal(res[0]["free"], res[1]["free"])
