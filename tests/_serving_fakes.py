"""CPU stand-ins for the serving tests: executors that record what they ran, one of which kills its own
process on a chosen request (a worker dying on the host, never a GPU fault)."""

import os
import time


class RecordingExecutor:
    def __init__(self, worker_id: int, die_on: int | None = None, log_dir: str | None = None):
        self.worker_id, self.die_on, self.log_dir = worker_id, die_on, log_dir

    def run(self, r):
        if self.die_on is not None and r.rid == self.die_on:
            os._exit(3)  # the worker process disappears in the middle of a request
        time.sleep(0.001 * (1 + r.size % 5))
        if self.log_dir:
            with open(os.path.join(self.log_dir, f"w{self.worker_id}.log"), "a") as f:
                f.write(f"{r.rid}\n")


def make_recording(worker_id: int):
    return RecordingExecutor(worker_id)


class DieOnFactory:
    """Picklable factory: worker `victim` dies when it starts request `rid`."""

    def __init__(self, victim: int, rid: int):
        self.victim, self.rid = victim, rid

    def __call__(self, worker_id: int):
        return RecordingExecutor(worker_id, die_on=self.rid if worker_id == self.victim else None)


def gloo_rank(rank: int, world: int, port: int, out_dir: str):
    """One rank of a gloo process group running its share of the c4 plan (bench.py's serving path)."""
    import json

    import torch.distributed as dist

    from sokutou_b200 import serving as SV

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    reqs = SV.requests_c4(0)
    done = SV.run_sharded(reqs, RecordingExecutor(rank), rank, world)
    gathered = [None] * world
    dist.all_gather_object(gathered, [rid for rid, _ in done])
    t = max(sec for _, sec in done) if done else 0.0
    import torch
    tt = torch.tensor([t], dtype=torch.float64)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    if rank == 0:
        with open(os.path.join(out_dir, "gloo.json"), "w") as f:
            json.dump({"per_rank": gathered, "max_request_s": float(tt.item())}, f)
    dist.barrier()
    dist.destroy_process_group()
