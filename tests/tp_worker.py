"""One rank of the tensor-parallel decode test (launched by tests/test_gpu_tp.py through
torch.distributed.run). Prefills the prompt on this rank's own model, connects the ranks' exchange
buffers, runs teacher-forced and free-running decode, and writes its results to <out>.rank<r>.npz.

    python -m torch.distributed.run --nproc-per-node N tests/tp_worker.py <weights> <inputs.npz> <out> [mode] [path]

mode "decode" (default): the parity run. Mode "leave": after one decode call together, every rank
but 0 stops taking part (leaves between steps, nothing of its own in flight); rank 0 decodes once
more with a short wait budget and records whether it timed out, how long that took, and whether
the decoder then refused another step. path: "fused" (default), "graph" or "graph_nccl".
"""
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "qwen3.cpp_b200"))


def main():
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import q3b200

    weights, inputs, out = sys.argv[1], sys.argv[2], sys.argv[3]
    mode = sys.argv[4] if len(sys.argv) > 4 else "decode"
    path = sys.argv[5] if len(sys.argv) > 5 else "fused"
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    d = np.load(inputs)
    prompt, cont = d["prompt"], d["cont"]
    m = q3b200.Qwen3(weights, int(d["ctx"]), device=local)
    _, nxt = m.prefill(prompt, 0)
    tp = q3b200.TpDecoder(m, rank, world)
    if path == "graph_nccl":
        uid = [q3b200.TpDecoder.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        tp.nccl_connect(uid[0])
    tp.path = {"fused": q3b200.TpDecoder.FUSED, "graph": q3b200.TpDecoder.GRAPH,
               "graph_nccl": q3b200.TpDecoder.GRAPH_NCCL}[path]
    handles = [None] * world
    dist.all_gather_object(handles, tp.ipc_handle())
    tp.connect(handles)
    dist.barrier()
    if mode == "leave":
        import time
        tp.configure(wait_cycles=20_000_000)  # ~10 ms at the boost clock
        tp.decode_forced(cont[:2], len(prompt))
        dist.barrier()  # every rank's first call has finished; rank 1 now leaves
        res = {"timed_out": 0, "refused": 0, "seconds": 0.0}
        if rank == 0:
            t0 = time.perf_counter()
            try:
                tp.decode_forced(cont[2:4], len(prompt) + 2)
            except q3b200.DeviceTimeout:
                res["timed_out"] = 1
            res["seconds"] = time.perf_counter() - t0
            try:
                tp.decode_forced(cont[4:5], len(prompt) + 4)
            except q3b200.Q3RuntimeError as e:
                res["refused"] = int(not isinstance(e, q3b200.DeviceTimeout))
        np.savez(f"{out}.rank{rank}.npz", **res)
        dist.barrier()
        tp.close()
        m.close()
        dist.destroy_process_group()
        return
    am = tp.decode_forced(cont, len(prompt))
    free = tp.decode(int(am[-1]), len(prompt) + len(cont), 8)
    dist.barrier()
    np.savez(f"{out}.rank{rank}.npz", next=nxt, argmax=am, free=free)
    tp.close()
    m.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
