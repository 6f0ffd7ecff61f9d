"""Request-parallel serving on the host: planning, a world-size-2 gloo run of the
sharded path bench.py uses under torchrun, the host queue, and failure detection — a worker process that
dies mid-request has its claimed requests re-queued to the survivors. No GPU is involved."""

import json
import os
import socket

import pytest
import torch.multiprocessing as mp

import _serving_fakes as F
from sokutou_b200 import serving as SV


def test_plan_lpt_assigns_every_request_once_and_balances():
    reqs = SV.requests_c4(0)
    for n in (1, 2, 4, 8):
        plan = SV.plan_lpt(reqs, n)
        ids = sorted(r.rid for part in plan for r in part)
        assert ids == list(range(64))
        loads = [sum(SV.cost_estimate(r) for r in part) for part in plan]
        biggest = max(SV.cost_estimate(r) for r in reqs)
        # LPT: no worker exceeds the mean load by more than the largest single request
        assert max(loads) <= sum(loads) / n + biggest + 1e-12
    assert SV.plan_lpt(reqs, 4) == SV.plan_lpt(reqs, 4)  # every rank computes the same plan


def test_cost_model_orders_work():
    small, large = SV.Request(0, "dit", 96), SV.Request(1, "dit", 384)
    short, long_ = SV.Request(2, "decode", 200), SV.Request(3, "decode", 1500)
    assert SV.cost_estimate(small) < SV.cost_estimate(large)
    assert SV.cost_estimate(short) < SV.cost_estimate(long_)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_run_over_gloo_world_size_2(tmp_path):
    port = _free_port()
    mp.start_processes(F.gloo_rank, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn", join=True)
    res = json.load(open(tmp_path / "gloo.json"))
    per_rank = res["per_rank"]
    assert sorted(per_rank[0] + per_rank[1]) == list(range(64))
    assert not set(per_rank[0]) & set(per_rank[1])
    plan = SV.plan_lpt(SV.requests_c4(0), 2)
    assert per_rank == [[r.rid for r in part] for part in plan]


def test_host_queue_runs_everything():
    reqs = SV.requests_c4(0)[:24]
    out = SV.serve_local(reqs, 2, F.make_recording, timeout_s=120)
    assert sorted(out["done"]) == sorted(r.rid for r in reqs)
    assert out["dead"] == [] and out["requeued"] == []
    assert {w for w, _ in out["done"].values()} <= {0, 1}


def test_dead_worker_requests_are_requeued():
    reqs = SV.requests_c4(0)[:24]
    victim_rid = sorted(reqs, key=lambda r: (-SV.cost_estimate(r), r.rid))[0].rid  # the first one handed out
    out = SV.serve_local(reqs, 2, F.DieOnFactory(victim=0, rid=victim_rid), timeout_s=120)
    assert sorted(out["done"]) == sorted(r.rid for r in reqs)  # nothing lost
    if out["dead"]:  # worker 0 took the victim request and died
        assert out["dead"] == [0]
        assert victim_rid in out["requeued"]
        assert out["done"][victim_rid][0] == 1  # finished by the survivor
    else:  # worker 1 took it first; it runs normally there
        assert out["done"][victim_rid][0] == 1


def test_all_workers_dead_raises():
    reqs = [SV.Request(0, "dit", 100)]
    with pytest.raises(RuntimeError):
        SV.serve_local(reqs, 1, F.DieOnFactory(victim=0, rid=0), timeout_s=60)
