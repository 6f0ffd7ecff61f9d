"""Request-parallel serving across GPUs, with no collectives.

The reference serves one request at a time per process, one GPU per process
(scripts/run_in_image.sh:24-33, README.md:186). Batch-1 TTS attention does not shard, so scaling
to 1/2/4/8 B200 means independent requests pinned to GPUs:

  * `plan_lpt`     longest-first greedy assignment of requests to workers (static, deterministic:
                   every rank computes the same plan, nothing is exchanged);
  * `run_sharded`  one rank's share, for a torchrun launch (used by bench.py);
  * `serve_local`  a host-side queue feeding one worker process per GPU (CUDA_VISIBLE_DEVICES
                   pinning); workers pull requests, and the requests of a worker that dies are
                   put back on the queue for the survivors;
  * `GpuExecutor`  runs one request's attention workload on a GPU: a DiT request is every
                   attention call of one c2-shaped synthesis (24 layers x 20 steps, CFG on the
                   first 10) at its latent length; a decode request is every talker-layer decode
                   attention of one c3-shaped decode from the 96-token prompt to its final length.
"""

from __future__ import annotations

import multiprocessing as mp
import os
import time
from dataclasses import dataclass


@dataclass(frozen=True)
class Request:
    rid: int
    kind: str      # "dit" or "decode"
    size: int      # latent length L (dit) or final KV length T (decode)


def requests_c4(seed: int = 0) -> list[Request]:
    from .workloads import serving_requests
    return [Request(i, k, s) for i, (k, s) in enumerate(serving_requests(seed))]


def cost_estimate(r: Request) -> float:
    """Rough device seconds: per call, the work at B200 rates plus a launch floor."""
    if r.kind == "dit":
        K = r.size + 512
        calls = [3] * 240 + [1] * 240
        return sum(4 * B * 16 * r.size * K * 128 / 5e14 + 5e-6 for B in calls)
    steps = max(r.size - 96, 0)
    # decodes share grouped launches (GpuExecutor.SLOTS talkers per launch): ~2 TB/s, ~2.5 us per layer each
    return sum(28 * (2 * 8 * (96 + i) * 128 * 2 / 2e12 + 2.5e-6) for i in range(1, steps + 1))


def plan_lpt(reqs: list[Request], n: int) -> list[list[Request]]:
    """Longest processing time first: each request, largest first, goes to the least-loaded worker
    (ties to the lowest index). Deterministic."""
    loads = [0.0] * n
    plan: list[list[Request]] = [[] for _ in range(n)]
    for r in sorted(reqs, key=lambda r: (-cost_estimate(r), r.rid)):
        i = min(range(n), key=lambda j: (loads[j], j))
        plan[i].append(r)
        loads[i] += cost_estimate(r)
    return plan


def run_sharded(reqs: list[Request], executor, rank: int, world: int) -> list[tuple[int, float]]:
    """This rank's share of the plan; returns (rid, seconds) per request run."""
    out = []
    for r in plan_lpt(reqs, world)[rank]:
        t0 = time.perf_counter()
        executor.run(r)
        out.append((r.rid, time.perf_counter() - t0))
    return out


# ---- host queue with worker processes ---------------------------------------------------------------

def _worker(wid: int, device_env: str | None, make_executor, conn):
    if device_env is not None:
        os.environ["CUDA_VISIBLE_DEVICES"] = device_env
    ex = make_executor(wid)
    while True:
        r = conn.recv()
        if r is None:
            return
        t0 = time.perf_counter()
        ex.run(r)
        conn.send((r.rid, time.perf_counter() - t0))


def serve_local(reqs: list[Request], n_workers: int, make_executor, devices: list[str] | None = None,
                timeout_s: float = 600.0) -> dict:
    """Run every request once on `n_workers` spawned worker processes fed from one host queue.

    The coordinator hands each idle worker the next request (longest first) over that worker's own pipe,
    so it always knows what every worker holds. make_executor(worker_id) builds the worker's executor
    inside the worker (a picklable callable); devices[i] becomes worker i's CUDA_VISIBLE_DEVICES. When
    a worker process dies, the request it held goes back to the front of the queue for the survivors.
    Returns {"done": {rid: (worker, seconds)}, "requeued": [...], "dead": [...], "wall_s": ...}.
    """
    from collections import deque
    from multiprocessing.connection import wait

    ctx = mp.get_context("spawn")
    pending = deque(sorted(reqs, key=lambda r: (-cost_estimate(r), r.rid)))
    procs, conns, inflight = {}, {}, {}
    for w in range(n_workers):
        parent, child = ctx.Pipe()
        env = devices[w] if devices else None
        p = ctx.Process(target=_worker, args=(w, env, make_executor, child), daemon=True)
        p.start()
        child.close()
        procs[w], conns[w], inflight[w] = p, parent, None

    def dispatch(w):
        # an idle worker keeps waiting (no stop message yet): it may still take a re-queued request
        inflight[w] = None
        if pending:
            r = pending.popleft()
            inflight[w] = r
            conns[w].send(r)

    done: dict[int, tuple[int, float]] = {}
    requeued, dead = [], []
    t0 = time.perf_counter()
    alive = set(procs)
    for w in list(alive):
        dispatch(w)
    while len(done) < len(reqs):
        if time.perf_counter() - t0 > timeout_s:
            for w in alive:
                procs[w].kill()
            raise TimeoutError("serving did not finish")
        if not alive:
            raise RuntimeError(f"all workers died with {len(reqs) - len(done)} requests left")
        handles = {conns[w]: ("msg", w) for w in alive}
        handles.update({procs[w].sentinel: ("exit", w) for w in alive})
        for h in wait(list(handles), timeout=0.5):
            kind, w = handles[h]
            if w not in alive:
                continue
            if kind == "msg":
                try:
                    rid, sec = conns[w].recv()
                except (EOFError, OSError):
                    continue  # the process is exiting; its sentinel reports it
                done[rid] = (w, sec)
                dispatch(w)
            elif not procs[w].is_alive():  # gone before being told to stop: dead
                alive.discard(w)
                dead.append(w)
                r = inflight[w]
                if r is not None and r.rid not in done:
                    requeued.append(r.rid)
                    pending.appendleft(r)
                    idle = [v for v in alive if inflight[v] is None]
                    if idle:
                        dispatch(idle[0])
    for w in alive:
        try:
            conns[w].send(None)
        except (BrokenPipeError, OSError):
            pass
    for p in procs.values():
        p.join(timeout=5)
        if p.is_alive():
            p.kill()
    return {"done": done, "requeued": requeued, "dead": dead, "wall_s": time.perf_counter() - t0}


# ---- GPU executor --------------------------------------------------------------------------------------

class GpuExecutor:
    """Runs a request's attention workload on one GPU from CUDA graphs captured in `warm`."""

    def __init__(self, device, max_cache: int = 1536):
        import torch
        self.torch = torch
        self.device = torch.device(device)
        self.max_cache = max_cache
        self.dit = {}       # L -> (graph, buffers)
        self.dec = None     # (graph, TalkerAttention, buffers)
        self.slots = None   # (graph, talkers, buffers) of the continuous-batching decode slots

    # Distinct q/k/v per attention call, as in the engine (each layer and step reads new projections):
    # a pool of flat buffers larger than L2, rotated over the calls of every request, so no request
    # replays from a warm L2. One pool serves every latent length (a call views a prefix).
    POOL_BYTES = 384 << 20

    def _pool(self):
        import torch

        from . import ops, workloads as W
        if getattr(self, "_dit_pool", None) is None:
            sh = W.c4_dit(W.C4_L_MAX)
            per = 3 * sh.H * sh.L * sh.hd  # elements of one (B = 3, L max) q, k or v
            n = max(8, -(-self.POOL_BYTES // (3 * per * 2)))
            g = torch.Generator(device=self.device).manual_seed(17)
            qk_w = W.dit_qk_weights(sh, self.device)
            freqs = W.dit_freqs(sh.L, sh.hd, device=self.device)
            sets = []
            for _ in range(n):
                o4 = (torch.randn(3 * sh.L, 4 * sh.H * sh.hd, device=self.device, generator=g) * sh.sigma).bfloat16()
                q, k, v = ops.dit_qkv_prologue(o4, qk_w, freqs, 3, sh.L, sh.H, sh.hd, 1e-6)
                sets.append((q.view(-1), k.view(-1), v.view(-1)))
            self._dit_pool = sets
            self._dit_y = torch.empty(per, device=self.device, dtype=torch.bfloat16)
        return self._dit_pool, self._dit_y

    def _dit_graph(self, L: int):
        import torch

        from . import dit, ops, workloads as W
        sh = W.c4_dit(L)
        sets, yflat = self._pool()
        g = torch.Generator(device=self.device).manual_seed(L)
        ctx = []
        for _ in range(sh.n_layers):
            kc = torch.randn(sh.S, sh.H, sh.hd, device=self.device, generator=g)
            kc = (kc * torch.rsqrt(kc.pow(2).mean(-1, keepdim=True))).bfloat16()
            vc = (torch.randn(sh.S, sh.H, sh.hd, device=self.device, generator=g) * sh.sigma).bfloat16()
            ctx.append((kc, vc))
        bias = dit.cfg_bias(L, sh.Tb, sh.Sp, L, 64, device=self.device)

        def run():
            for i, B in enumerate(sh.synthesis_calls()):
                n = B * sh.H * L * sh.hd
                q, k, v = (t[:n].view(B, sh.H, L, sh.hd) for t in sets[i % len(sets)])
                kc, vc = ctx[i % sh.n_layers]
                ops.dit_attention(q, k, v, kc, vc, bias[:B], out=yflat[:n].view(B, L, sh.H, sh.hd))

        return self._capture(run), (ctx, bias)

    def _decode_graph(self):
        import torch

        from . import qwen3, workloads as W
        s = W.C3
        ta = qwen3.TalkerAttention(s.n_layers, s.nq, s.nkv, self.max_cache, s.theta, s.eps, self.device, torch.bfloat16)
        g = torch.Generator(device=self.device).manual_seed(3)
        ta.k.copy_(torch.randn(ta.k.shape, device=self.device, generator=g))
        ta.v.copy_(torch.randn(ta.v.shape, device=self.device, generator=g))
        qkv = torch.randn(s.n_layers, (s.nq + 2 * s.nkv) * s.hd, device=self.device, generator=g)
        qn = 1 + 0.02 * torch.randn(s.n_layers, s.hd, device=self.device, generator=g)
        kn = 1 + 0.02 * torch.randn(s.n_layers, s.hd, device=self.device, generator=g)
        out = torch.empty(s.n_layers, s.nq * s.hd, device=self.device)

        def run():
            for li in range(s.n_layers):
                ta.attn(li, qkv[li], qn[li], kn[li], out[li], kv_stable=li > 0)
            ta.pos.add_(1)

        ta.pos.fill_(s.prompt)
        gr = self._capture(run)
        return gr, ta, (qkv, qn, kn, out)

    def _capture(self, fn):
        torch = self.torch
        st = torch.cuda.Stream(self.device)
        st.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(st):
            fn()
        torch.cuda.current_stream(self.device).wait_stream(st)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            fn()
        return gr

    def warm(self, reqs: list[Request]):
        for r in reqs:
            if r.kind == "dit" and r.size not in self.dit:
                self.dit[r.size] = self._dit_graph(r.size)
            elif r.kind == "decode" and self.dec is None:
                self.dec = self._decode_graph()
        if any(r.kind == "decode" for r in reqs) and self.slots is None:
            self.slots = self._decode_slots()

    def run(self, r: Request):
        self.warm([r])
        if r.kind == "dit":
            self.dit[r.size][0].replay()
        else:
            gr, ta, _ = self.dec
            ta.pos.fill_(96)
            for _ in range(96, min(r.size, self.max_cache)):
                gr.replay()

    # ---- continuous batching of decode requests -------------------------------------------------
    # SLOTS talkers decode side by side, one grouped launch per layer for all of them
    # (sk_decode_attention_grouped): every step advances every slot by one position; a slot whose
    # request has reached its final length takes the next waiting request (its position reset to the
    # prompt length). Requests are handed out longest first, so the slots finish close together.
    # 16 slots measured best for c4 on one B200: 55.3 sentences/s against 50.2 with 8, 52.0 with 12,
    # 51.8 with 20, 43.8 with 24 and 33.2 with 32 (idle slots keep launching through the tail).
    SLOTS = 16

    def _decode_slots(self):
        import torch

        from . import ops, qwen3, workloads as W
        s, R = W.C3, self.SLOTS
        g = torch.Generator(device=self.device).manual_seed(5)
        tas = []
        for _ in range(R):
            ta = qwen3.TalkerAttention(s.n_layers, s.nq, s.nkv, self.max_cache, s.theta, s.eps, self.device,
                                       torch.bfloat16)
            ta.k.normal_(generator=g)
            ta.v.normal_(generator=g)
            tas.append(ta)
        qkv = torch.randn(R, s.n_layers, (s.nq + 2 * s.nkv) * s.hd, device=self.device, generator=g)
        qn = 1 + 0.02 * torch.randn(s.n_layers, s.hd, device=self.device, generator=g)
        out = torch.empty(R, s.n_layers, s.nq * s.hd, device=self.device)
        descs = [ops.decode_requests([{"qkv": qkv[r, li], "qn": qn[li], "kn": qn[li], "rope": tas[r].rope,
                                       "Kc": tas[r].k[li], "Vc": tas[r].v[li], "pos_ptr": tas[r].pos,
                                       "out": out[r, li], "pos_add": 0, "eps": s.eps} for r in range(R)], self.device)
                 for li in range(s.n_layers)]

        def step():
            for li in range(s.n_layers):
                ops.decode_attention_grouped(descs[li], R, self.max_cache, s.nq, s.nkv, torch.bfloat16,
                                             kv_stable=li > 0)
            for ta in tas:
                ta.pos.add_(1)

        for ta in tas:
            ta.pos.fill_(96)
        gr = self._capture(step)
        return gr, tas, (qkv, qn, out, descs)

    def run_decodes(self, reqs: list[Request]) -> int:
        """Every decode request of `reqs` through the slots; returns the number of steps replayed."""
        self.warm(reqs)
        gr, tas, _ = self.slots
        queue = sorted(reqs, key=lambda r: -r.size)
        left = [0] * self.SLOTS  # steps the slot's current request still needs
        for i, ta in enumerate(tas):
            if queue:
                r = queue.pop(0)
                left[i] = max(0, min(r.size, self.max_cache) - 96)
                ta.pos.fill_(96)
        steps = 0
        while any(left):
            n = min(x for x in left if x > 0)  # replays until the next slot finishes
            for _ in range(n):
                gr.replay()
            steps += n
            for i, ta in enumerate(tas):
                if left[i] > 0:
                    left[i] -= n
                    if left[i] == 0 and queue:
                        r = queue.pop(0)
                        left[i] = max(0, min(r.size, self.max_cache) - 96)
                        ta.pos.fill_(96)
        return steps

    def run_all(self, reqs: list[Request]) -> None:
        """A rank's share of the sweep: its DiT syntheses one after another, its decodes through the slots."""
        for r in reqs:
            if r.kind == "dit":
                self.run(r)
        dec = [r for r in reqs if r.kind == "decode"]
        if dec:
            self.run_decodes(dec)
