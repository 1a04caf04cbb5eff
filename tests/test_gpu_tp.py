"""Tensor-parallel decode (q3_tp_*) against the oracle, on every step path (the fused persistent
kernel with its in-kernel exchange, the per-step graph with this library's all-reduce kernels, and
the graph with NCCL collectives, the comparison arm).

world = 1 runs the shard/exchange code paths with a single rank on one GPU; world = 2 runs two
ranks on two GPUs (child processes through torch.distributed.run; skipped with fewer GPUs).
Teacher-forced top-1 agreement with the oracle >= 99% over 256 decode positions (positions 40 to
295: the fused kernel's attention from the ring up to 128 cached positions, split over CTAs past
them), and every rank returns the same tokens.
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
PROMPT, STEPS, CTX = 40, 256, 512
PATHS = ["fused", "graph"]  # the paths with bounded waits (failure tests)
ALL_PATHS = PATHS + ["graph_nccl"]


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
    am = cpu.forward_many(np.concatenate([prompt, cont]), 0)["argmax"]
    return prompt, cont, np.asarray(am)


def _set_path(q3lib, tp, path):
    want = {"fused": q3lib.TpDecoder.FUSED, "graph": q3lib.TpDecoder.GRAPH,
            "graph_nccl": q3lib.TpDecoder.GRAPH_NCCL}[path]
    if path == "graph_nccl":
        with pytest.raises(q3lib.InvalidArgument):
            tp.path = want  # no communicator yet
        tp.nccl_connect(q3lib.TpDecoder.nccl_unique_id())  # world 1: this rank alone
    tp.path = want
    assert tp.path == want


@pytest.mark.parametrize("path", ALL_PATHS)
@pytest.mark.parametrize("solo_allreduce", [False, True])
def test_tp_single_rank(q3lib, full_weights, case, solo_allreduce, path):
    """World 1; with solo_allreduce the o_proj / down_proj partials (graph) or the
    down-projection sums and greedy candidates (fused) go through the exchange words with this
    rank as the only member, so the exchange code runs on one GPU."""
    prompt, cont, ref = case
    m = q3lib.Qwen3(full_weights, CTX)
    try:
        _, nxt = m.prefill(prompt, 0)
        assert nxt == ref[PROMPT - 1]
        if path == "graph_nccl" and solo_allreduce:
            pytest.skip("the NCCL path always goes through its collectives")
        tp = q3lib.TpDecoder(m, 0, 1)
        assert tp.path == q3lib.TpDecoder.FUSED  # the default on B200
        _set_path(q3lib, tp, path)
        tp.connect([tp.ipc_handle()])
        tp.configure(solo_allreduce=solo_allreduce)
        am = tp.decode_forced(cont, PROMPT)
        agree = float((am == ref[PROMPT:PROMPT + STEPS]).mean())
        print(f"\n[parity] tp world 1 {path} solo={solo_allreduce}: positions={STEPS}, "
              f"agree={agree}, flips={int((am != ref[PROMPT:PROMPT + STEPS]).sum())}")
        assert agree >= TOP1_AGREEMENT
        free = tp.decode(int(am[-1]), PROMPT + STEPS, 8)
        assert free.shape == (8,) and np.all((free >= 0) & (free < 151936))
        with pytest.raises(q3lib.OutOfRange):
            tp.decode(0, CTX - 2, 4)  # past the context
        tp.close()
    finally:
        m.close()


@pytest.mark.parametrize("path", PATHS)
def test_tp_wait_timeout_refuses_then_resets(q3lib, full_weights, path):
    """A peer that never answers: a world-2 decoder whose peer slot is its own buffer (nothing
    raises that peer's flag or writes its exchange words). Every bounded wait runs out after a
    short budget; decode reports DeviceTimeout promptly (later waits see the error and skip),
    then refuses to decode until reset; reset clears the refusal."""
    import time
    m = q3lib.Qwen3(full_weights, 64)
    try:
        tp = q3lib.TpDecoder(m, 0, 2)
        _set_path(q3lib, tp, path)
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


def _run_workers(full_weights, case, tmp_path, mode, path="fused"):
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
           str(inputs), str(out), mode, path]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    return [np.load(f"{out}.rank{k}.npz") for k in range(2)]


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("path", PATHS)
def test_tp_peer_leaves_between_steps(full_weights, case, tmp_path, path):
    """Rank 1 stops taking part after a first decode call (it leaves between steps, with nothing
    of its own in flight); rank 0's next decode ends with DeviceTimeout within its short wait
    budget and then refuses further steps."""
    res = _run_workers(full_weights, case, tmp_path, "leave", path)
    assert int(res[0]["timed_out"]) == 1 and int(res[0]["refused"]) == 1
    assert float(res[0]["seconds"]) < 20.0


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("path", ALL_PATHS)
def test_tp_two_ranks(full_weights, case, tmp_path, path):
    prompt, cont, ref = case
    res = _run_workers(full_weights, case, tmp_path, "decode", path)
    for k in range(2):
        assert int(res[k]["next"]) == ref[PROMPT - 1]
        agree = float((res[k]["argmax"] == ref[PROMPT:PROMPT + STEPS]).mean())
        print(f"\n[parity] tp world 2 {path} rank {k}: positions={STEPS}, agree={agree}")
        assert agree >= TOP1_AGREEMENT
    assert np.array_equal(res[0]["argmax"], res[1]["argmax"])
    assert np.array_equal(res[0]["free"], res[1]["free"])
