"""One rank of the tensor-parallel decode test (launched by tests/test_gpu_tp.py through
torch.distributed.run). Prefills the prompt on this rank's own model, connects the ranks' exchange
buffers, runs teacher-forced and free-running decode, and writes its results to <out>.rank<r>.npz.

    python -m torch.distributed.run --nproc-per-node N tests/tp_worker.py <weights> <inputs.npz> <out>
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
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    d = np.load(inputs)
    prompt, cont = d["prompt"], d["cont"]
    m = q3b200.Qwen3(weights, int(d["ctx"]), device=local)
    _, nxt = m.prefill(prompt, 0)
    tp = q3b200.TpDecoder(m, rank, world)
    handles = [None] * world
    dist.all_gather_object(handles, tp.ipc_handle())
    tp.connect(handles)
    dist.barrier()
    am = tp.decode_forced(cont, len(prompt))
    free = tp.decode(int(am[-1]), len(prompt) + len(cont), 8)
    dist.barrier()
    np.savez(f"{out}.rank{rank}.npz", next=nxt, argmax=am, free=free)
    tp.close()
    m.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
