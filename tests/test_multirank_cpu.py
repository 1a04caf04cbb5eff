"""Host logic of bench.py on CPU. Two gloo ranks (spawned processes) take the slowest rank's time,
split the data-parallel sequences without overlap, and exchange the tensor-parallel handles in rank
order - the steps `bench.py --gpus N` takes under torchrun; and the summary of the nvidia-smi clock
samples that goes into the bench line."""
import multiprocessing as mp
import os
import socket
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, port: int, out) -> None:
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(WORLD))
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist

    import bench

    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60))
    try:
        world, r, _ = bench.dist_info()
        slowest = bench.max_over_ranks(10.0 + 5.0 * r, world, device="cpu")
        share = bench.dp_share(64, r, world)
        handles = bench.gather_handles(bytes([r]) * 64, world)
        out.put((r, slowest, share, handles))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, port, out)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(WORLD):
            r, slowest, share, handles = out.get(timeout=120)
            results[r] = (slowest, share, handles)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert sorted(results) == list(range(WORLD))
    for slowest, _, handles in results.values():
        assert slowest == 15.0  # every rank reports the slowest rank's time
        assert handles == [bytes([0]) * 64, bytes([1]) * 64]  # rank order
    shares = [set(results[r][1]) for r in range(WORLD)]
    assert not (shares[0] & shares[1]) and shares[0] | shares[1] == set(range(64))


def test_single_rank_needs_no_process_group():
    sys.path.insert(0, str(ROOT))
    import bench

    assert bench.max_over_ranks(3.5, 1) == 3.5
    assert bench.dp_share(5, 0, 1) == [0, 1, 2, 3, 4]
    assert bench.gather_handles(b"h", 1) == [b"h"]


def test_clock_samples_summary():
    """bench.py's reading of nvidia-smi samples: median SM clock, maximum, reasons seen Active."""
    sys.path.insert(0, str(ROOT))
    import bench

    text = "\n".join([
        "0, 1965, 1965, 700.1, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
        "0, 1950, 1965, 990.5, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "0, 1800, 1965, 1000.0, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "0, [N/A], [N/A], [N/A], [N/A], [N/A], [N/A], [N/A], [N/A]",
        "",
    ])
    got = bench.Clocks.summarize(text)
    assert got == {"sm_mhz": 1950.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"],
                   "samples": 4}
    assert bench.Clocks.summarize("") == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [],
                                          "samples": 0}
