"""Benchmark of the B200 attention path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline (`metric`, `value`): DiT attention TFLOP/s over BASELINE config 1 — one full synthesis
(12 layers x 20 flow steps, CFG batch 3 on the first 10 steps, batch 1 on the rest) for each latent
length L in {128, 256, 512}, bf16 in / fp32 accumulate, on the tcgen05 kernel. A step is those
3 x 240 = 720 attention calls, replayed from a CUDA graph; every call reads its own q/k/v
(3 GB of distinct inputs per step, far larger than the 126 MB L2). FLOPs = 4·B·H·L·K·hd per call.
`e2e`: the same calls through the public op with pinned host buffers — each call's q/k/v copied
host->device and y copied back inside the timed region.
Extra keys: `c2` (v4-Large-class DiT attention), `c3` (Qwen3 talker decode attention GB/s over a
full 96 -> 1120 decode, four cache sets rotated so the 129 MB working set misses L2), `serving`
(64 requests sharded request-parallel across the ranks, sentences/s),
`cpu_baseline` (the reference's torch SDPA on the host CPU, float32), `roofline`, `clocks`.
Multi-GPU: one process per GPU under torchrun; the DiT and decode numbers are replicas (weak
scaling, value = sum over ranks), timed as the max over ranks between barriers.
`--impl reference` times the reference arithmetic (torch SDPA on the host CPU, all threads) on a
bounded sample of the same workload and prints the same line with "impl": "reference".
"""

from __future__ import annotations

import argparse
import contextlib
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "dit_attn_tflops"
UNIT = "TFLOP/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "sm_max_mhz": 1965.0}
SPEC = {"hbm_gbs": 8000.0, "bf16_tflops": 2250.0}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {k: float(d[k]) for k in FALLBACK_PEAKS if k in d}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


WORKLOAD = ("BASELINE config 1: DiT attention, full synthesis (12 layers x 20 steps, CFG B=3 on 10 steps, "
            "B=1 on 10) for L in 128/256/512")


def c1_config(world: int, calls: int, flops: int) -> dict:
    """The headline workload, identical in both arms' JSON lines."""
    return {"workload": WORKLOAD, "heads": 12, "head_dim": 64, "text_keys": 64, "speaker_keys": 192,
            "calls_per_step": calls, "flops_per_step": flops, "parallelism": f"replicas x{world}",
            "l2": "inputs larger than L2 (distinct q/k/v per call, ~3 GB per step)"}


def profile_traffic_mix(name: str, shapes):
    """DRAM bytes per launch averaged over the step's call mix, from the per-shape lines
    'traffic_bytes_per_launch <shape>_b<B>: N' of an ncu summary in profiles/<name> (one launch of each
    shape captured with dram__bytes_read.sum and dram__bytes_write.sum). None if a shape is missing."""
    p = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(p):
        return None
    per = {}
    for line in open(p):
        t = line.strip()
        if t.startswith("traffic_bytes_per_launch ") and ":" in t:
            key, val = t[len("traffic_bytes_per_launch "):].split(":", 1)
            try:
                per[key.strip()] = float(val.split()[0])
            except ValueError:
                pass
    tot = n = 0
    for sh in shapes:
        for B in sh.synthesis_calls():
            key = f"{sh.name}_b{B}"
            if key not in per:
                return None
            tot += per[key]
            n += 1
    return round(tot / n) if n else None


# ---------------------------------------------------------------------------------------------- dist
class Dist:
    """One process per GPU under torchrun. The ranks share no data (request-parallel, no collectives on
    the data path); the process group exists only to line the ranks up around the timed region and to
    take the max / sum of the timing scalars, so it is gloo over host scalars, not NCCL."""

    def __init__(self, gpus: int):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist
            torch.cuda.set_device(self.local)
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
            self.pg = dist
        self.device = torch.device("cuda", self.local)

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def _reduce(self, x: float, op) -> float:
        t = torch.tensor([x], dtype=torch.float64)
        self.pg.all_reduce(t, op=op)
        return float(t.item())

    def max(self, x: float) -> float:
        return self._reduce(x, self.pg.ReduceOp.MAX) if self.pg else x

    def sum(self, x: float) -> float:
        return self._reduce(x, self.pg.ReduceOp.SUM) if self.pg else x

    def close(self):
        if self.pg:
            self.pg.barrier()
            self.pg.destroy_process_group()


# ---------------------------------------------------------------------------------------------- clocks
class ClockSampler:
    """This GPU's SM clock and clock-event reasons, read through NVML every `period_s` on a host
    thread (nvidia-smi -lms as a fallback), and summarised over the timed window only: the code
    being timed calls `window(True)` right before its first timed launch and `window(False)` after
    the final synchronize. Reading only; no GPU setting is changed."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}

    def __init__(self, device: torch.device, period_s: float = 0.002):
        self.uuid = None
        try:
            self.uuid = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
        except Exception:
            pass
        self.period = period_s
        self.samples: list[tuple[float, float, int]] = []  # (host time, sm MHz, reason bits)
        self.windows: list[tuple[float, float]] = []
        self._open = None
        self.max_mhz = None
        self.source = None
        self._stop = threading.Event()
        self.proc = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = (pynvml.nvmlDeviceGetHandleByUUID(self.uuid) if self.uuid else pynvml.nvmlDeviceGetHandleByIndex(0))
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            self.source = "nvml"
            started = threading.Event()

            def run():
                while not self._stop.is_set():
                    try:
                        mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                        bits = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.samples.append((time.perf_counter(), float(mhz), int(bits)))
                    except Exception:
                        pass
                    started.set()
                    time.sleep(self.period)

            self.th = threading.Thread(target=run, daemon=True)
            self.th.start()
            started.wait(timeout=2)
        except Exception:
            self._nvidia_smi()
        return self

    def _nvidia_smi(self):
        try:
            cmd = ["nvidia-smi", "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active",
                   "--format=csv,noheader,nounits", "-lms", "25"]
            if self.uuid:
                cmd += ["-i", self.uuid]
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.source = "nvidia-smi"

            def read():
                for line in self.proc.stdout:
                    parts = [x.strip() for x in line.split(",")]
                    try:
                        self.max_mhz = float(parts[1])
                        self.samples.append((time.perf_counter(), float(parts[0]), int(parts[2], 16)))
                    except (ValueError, IndexError):
                        continue

            self.th = threading.Thread(target=read, daemon=True)
            self.th.start()
            time.sleep(0.5)  # nvidia-smi start-up
        except Exception:
            self.source = None

    def window(self, start: bool):
        if start:
            self._open = time.perf_counter()
        elif self._open is not None:
            self.windows.append((self._open, time.perf_counter()))
            self._open = None

    def __exit__(self, *a):
        self._stop.set()
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if getattr(self, "th", None):
            self.th.join(timeout=2)

    def summary(self):
        inside = [x for x in self.samples if any(t0 <= x[0] <= t1 for t0, t1 in self.windows)]
        reasons = sorted(n for n, bit in self.REASONS.items() if any(x[2] & bit for x in inside))
        return {"sm_mhz": statistics.median(x[1] for x in inside) if inside else None, "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(inside), "source": self.source,
                "window_ms": round(sum(t1 - t0 for t0, t1 in self.windows) * 1e3, 2)}


# ---------------------------------------------------------------------------------------------- DiT
class DitSynthesis:
    """All attention calls of one synthesis for one DiT shape, with distinct inputs per call, and a CUDA
    graph that replays them."""

    def __init__(self, shape, device, seed: int):
        from sokutou_b200 import dit, ops, workloads as W
        self.shape = shape
        self.calls = shape.synthesis_calls()
        H, hd, L, S = shape.H, shape.hd, shape.L, shape.S
        g = torch.Generator(device=device).manual_seed(seed)
        qk_w = W.dit_qk_weights(shape, device)
        freqs = W.dit_freqs(L, hd, device=device)
        # per-layer conditioning K/V (unit-RMS keys), shared by every step and CFG row
        self.ctx = []
        for _ in range(shape.n_layers):
            k = torch.randn(S, H, hd, device=device, generator=g)
            k = k * torch.rsqrt(k.pow(2).mean(-1, keepdim=True) + 1e-6)
            v = torch.randn(S, H, hd, device=device, generator=g) * shape.sigma
            self.ctx.append((k.bfloat16().contiguous(), v.bfloat16().contiguous()))
        n_text = int(torch.randint(shape.text_lo, shape.text_hi + 1, (1,), generator=torch.Generator().manual_seed(seed)))
        self.bias = dit.cfg_bias(L, shape.Tb, shape.Sp, L, n_text, device=device)
        # q/k/v pool: one set per call, produced by the q/k producer from seeded projections
        self.q, self.k, self.v, self.y = [], [], [], []
        D = H * hd
        for B in self.calls:
            o4 = (torch.randn(B * L, 4 * D, device=device, generator=g) * shape.sigma).bfloat16()
            q, k, v = ops.dit_qkv_prologue(o4, qk_w, freqs, B, L, H, hd, 1e-6)
            self.q.append(q)
            self.k.append(k)
            self.v.append(v)
            self.y.append(torch.empty((B, L, H, hd), device=device, dtype=torch.bfloat16))
        self.flops = shape.synthesis_flops()
        self.graph = None

    def run(self):
        from sokutou_b200 import ops
        nl = self.shape.n_layers
        for i, B in enumerate(self.calls):
            kc, vc = self.ctx[i % nl]
            ops.dit_attention(self.q[i], self.k[i], self.v[i], kc, vc, self.bias[:B], out=self.y[i])

    def capture(self):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self.run()
        torch.cuda.current_stream().wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.run()

    def input_bytes(self) -> tuple[int, int]:
        h2d = sum(t.numel() * 2 for t in self.q + self.k + self.v)
        h2d += sum(k.numel() * 2 + v.numel() * 2 for k, v in self.ctx) + self.bias.numel() * 2
        d2h = sum(t.numel() * 2 for t in self.y)
        return h2d, d2h


def time_graphs(graphs, steps: int, warmup: int, dist: Dist, label: str = "timed", clk=None):
    """Device time (ms) of `steps` replays of all graphs, after `warmup`; max over ranks. The timed
    replays sit in an NVTX range named `label`, so a profiler can select exactly them
    (ncu --nvtx --nvtx-include "<label>/")."""
    for _ in range(warmup):
        for g in graphs:
            g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if clk is not None:
        clk.window(True)
    torch.cuda.nvtx.range_push(label)
    e0.record()
    for _ in range(steps):
        for g in graphs:
            g.replay()
    e1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    if clk is not None:
        clk.window(False)
    dist.barrier()
    torch.cuda.synchronize()
    return dist.max(e0.elapsed_time(e1))


def dit_e2e(syn: list, steps: int, warmup: int, dist: Dist, device, depth: int = 3):
    """Every call through the public op (ops.dit_attention, C ABI) with inputs and outputs in pinned host
    memory: per flow step, one host->device copy of the q/k/v of all its layers' calls, the calls, and
    one device->host copy of their outputs, all inside the timed region. Three streams pipeline the flow
    steps through a ring of `depth` device slots guarded by events: the inputs of step t+1 go up
    (copy-in stream) and the outputs of step t-1 come back (copy-out stream) while step t computes —
    H2D and D2H use separate copy engines and overlap the kernels."""
    from sokutou_b200 import ops
    s_in, s_cmp, s_out = (torch.cuda.Stream(device) for _ in range(3))
    plans = []
    for s in syn:
        sh, nl = s.shape, s.shape.n_layers
        per = {B: B * sh.H * sh.L * sh.hd for B in (1, 3)}  # elements of one call's q (or k, or v, or y)
        host_in, host_out = {}, {}
        for B in (1, 3):
            # [layer][q | k | v] of one flow step's calls, from the first flow step with this batch size
            first = s.calls.index(B)
            blk = torch.empty(nl, 3, per[B], dtype=torch.bfloat16).pin_memory()
            for li in range(nl):
                for r, t in enumerate((s.q, s.k, s.v)):
                    blk[li, r].copy_(t[first + li].reshape(-1))
            host_in[B] = blk
            host_out[B] = torch.empty(nl, per[B], dtype=torch.bfloat16).pin_memory()
        ring = [(torch.empty(nl * 3 * per[3], dtype=torch.bfloat16, device=device),
                 torch.empty(nl * per[3], dtype=torch.bfloat16, device=device)) for _ in range(depth)]
        hctx = [(k.cpu().pin_memory(), v.cpu().pin_memory()) for k, v in s.ctx]
        dctx = [(torch.empty_like(k), torch.empty_like(v)) for k, v in s.ctx]
        hb = s.bias.cpu().pin_memory()
        plans.append((s, per, host_in, host_out, ring, hctx, dctx, hb, torch.empty_like(s.bias)))
    h2d = d2h = 0

    def one_step(count):
        nonlocal h2d, d2h
        for s, per, host_in, host_out, ring, hctx, dctx, hb, dbias in plans:
            sh, nl = s.shape, s.shape.n_layers
            with torch.cuda.stream(s_in):  # the synthesis' conditioning keys and mask, once
                dbias.copy_(hb, non_blocking=True)
                for (dk, dv), (k, v) in zip(dctx, hctx):
                    dk.copy_(k, non_blocking=True)
                    dv.copy_(v, non_blocking=True)
            if count:
                h2d += hb.numel() * 2 + sum(k.numel() * 2 + v.numel() * 2 for k, v in hctx)
            free_in = [None] * depth   # the kernels that last read slot r's inputs
            free_out = [None] * depth  # the copy that last read slot r's outputs
            n_steps = len(s.calls) // nl
            for t in range(n_steps):
                B = s.calls[t * nl]
                r = t % depth
                din, dout = ring[r]
                n_in, n_out = nl * 3 * per[B], nl * per[B]
                with torch.cuda.stream(s_in):
                    if free_in[r] is not None:
                        s_in.wait_event(free_in[r])
                    din[:n_in].copy_(host_in[B].view(-1), non_blocking=True)
                    landed = torch.cuda.Event()
                    landed.record(s_in)
                with torch.cuda.stream(s_cmp):
                    s_cmp.wait_event(landed)
                    if free_out[r] is not None:
                        s_cmp.wait_event(free_out[r])
                    x = din[:n_in].view(nl, 3, B, sh.H, sh.L, sh.hd)
                    y = dout[:n_out].view(nl, B, sh.L, sh.H, sh.hd)
                    for li in range(nl):
                        kc, vc = dctx[li]
                        ops.dit_attention(x[li, 0], x[li, 1], x[li, 2], kc, vc, dbias[:B], out=y[li])
                    done = torch.cuda.Event()
                    done.record(s_cmp)
                    free_in[r] = done
                with torch.cuda.stream(s_out):
                    s_out.wait_event(done)
                    host_out[B].view(-1).copy_(dout[:n_out], non_blocking=True)
                    back = torch.cuda.Event()
                    back.record(s_out)
                    free_out[r] = back
                if count:
                    h2d += n_in * 2
                    d2h += n_out * 2
            cur = torch.cuda.current_stream(device)  # the next synthesis reuses the ring and ctx buffers
            for st in (s_in, s_cmp, s_out):
                cur.wait_stream(st)
            for st in (s_in, s_cmp, s_out):
                st.wait_stream(cur)

    for _ in range(warmup):
        one_step(False)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream(device)
    e0.record(cur)
    for st in (s_in, s_cmp, s_out):
        st.wait_stream(cur)
    for _ in range(steps):
        one_step(True)
    for st in (s_in, s_cmp, s_out):
        cur.wait_stream(st)
    e1.record(cur)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    return dist.max(e0.elapsed_time(e1)), h2d // max(steps, 1), d2h // max(steps, 1)


# ---------------------------------------------------------------------------------------------- decode
class DecodeBench:
    """c3: 28 layers, prompt 96, decode to T=1120; n_sets independent caches rotated per step."""

    def __init__(self, device, n_sets: int = 4, seed: int = 0):
        from sokutou_b200 import ops, qwen3, workloads as W
        s = W.C3
        self.s, self.n_sets = s, n_sets
        g = torch.Generator(device=device).manual_seed(seed)
        self.ta = []
        for _ in range(n_sets):
            ta = qwen3.TalkerAttention(s.n_layers, s.nq, s.nkv, s.T_final, s.theta, s.eps, device, torch.bfloat16)
            ta.k[:, :, :s.prompt].copy_(torch.randn(ta.k[:, :, :s.prompt].shape, device=device, generator=g))
            ta.v[:, :, :s.prompt].copy_(torch.randn(ta.v[:, :, :s.prompt].shape, device=device, generator=g))
            self.ta.append(ta)
        D = (s.nq + 2 * s.nkv) * s.hd
        self.qkv = torch.randn(s.n_layers, D, device=device, generator=g)
        self.qn = 1 + 0.02 * torch.randn(s.n_layers, s.hd, device=device, generator=g)
        self.kn = 1 + 0.02 * torch.randn(s.n_layers, s.hd, device=device, generator=g)
        self.out = torch.empty(s.n_layers, s.nq * s.hd, device=device)
        self.graph = None

    def step(self):
        for ta in self.ta:
            for li in range(self.s.n_layers):
                # layer 0 follows the position advance; the others follow a kernel that writes neither
                # the position nor their cache (the layer's qkv projection, at the reference call site)
                ta.attn(li, self.qkv[li], self.qn[li], self.kn[li], self.out[li], kv_stable=li > 0)
            ta.pos.add_(1)

    def reset(self):
        for ta in self.ta:
            ta.pos.fill_(self.s.prompt)

    def capture(self):
        self.reset()
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            self.step()
        torch.cuda.current_stream().wait_stream(st)
        self.reset()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.step()
        self.reset()

    def run_decode(self, lo: int, hi: int):
        """Replays decode steps for positions [lo, hi) on every set; returns device ms."""
        for ta in self.ta:
            ta.pos.fill_(lo)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(lo, hi):
            self.graph.replay()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)

    def bytes(self, lo: int, hi: int) -> int:
        return sum(self.s.layer_bytes(p + 1) * self.s.n_layers for p in range(lo, hi)) * self.n_sets


# ---------------------------------------------------------------------------------------------- CPU baseline
def cpu_dit_sample(shapes, seconds: float = 12.0, threads: int | None = None):
    """Torch SDPA on the host CPU (the reference's own op, float32) over one B=3 and one B=1 call per shape,
    repeated for about `seconds`; returns TFLOP/s for the synthesis mix and a description."""
    from oracle.dit_attn_ref import dit_attention_torch_cpu
    from sokutou_b200 import workloads as W
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    per_call = {}
    for sh in shapes:
        for B in (3, 1):
            x = W.dit_call_inputs(sh, B, seed=1)
            D = sh.H * sh.hd
            o = x["o4"].reshape(B, sh.L, 4, sh.H, sh.hd)
            q, k, v = (o[:, :, i].transpose(1, 2).contiguous() for i in range(3))
            args = (q, k, v, x["ctx_k"][None], x["ctx_v"][None], x["bias3"][:B])
            dit_attention_torch_cpu(*args)
            per_call[(sh.name, B)] = (args, sh.flops(B))
    budget = seconds / len(per_call)
    t_call = {}
    for key, (args, _) in per_call.items():
        n, t0 = 0, time.perf_counter()
        while True:
            dit_attention_torch_cpu(*args)
            n += 1
            if time.perf_counter() - t0 > budget:
                break
        t_call[key] = (time.perf_counter() - t0) / n
    tot_flops = sum(sh.synthesis_flops() for sh in shapes)
    tot_time = sum(t_call[(sh.name, B)] for sh in shapes for B in sh.synthesis_calls())
    return tot_flops / tot_time / 1e12, threads, f"one B=3 and one B=1 call per L in {[s.L for s in shapes]}, " \
        f"timed ~{seconds:.0f}s total, scaled to the synthesis call mix"


# ------------------------------------------------------------------------------- fused attention block
def layer_block(device, dist: Dist, calls: int = 120, sets: int = 4) -> dict:
    """One DiT layer's attention block — Q/K/V producer, attention, gate (engine/fused.py:293-298) — as
    one fused launch and as the three separate launches, each timed over `calls` graph-replayed calls
    rotating `sets` input sets (o4 and ctx K/V distinct per set). Reports microseconds per block."""
    from sokutou_b200 import dit, workloads as W
    out = {}
    for name, shape, B in (("c1_L512_b3", W.c1(512), 3), ("c1_L128_b1", W.c1(128), 1), ("c2_b3", W.C2, 3)):
        g = torch.Generator(device=device).manual_seed(5)
        H, hd, L, S = shape.H, shape.hd, shape.L, shape.S
        qk_w = W.dit_qk_weights(shape, device)
        freqs = W.dit_freqs(L, hd, device=device)
        bias = dit.cfg_bias(L, shape.Tb, shape.Sp, L, 40, device=device)[:B].contiguous()
        ins = []
        for _ in range(sets):
            o4 = (torch.randn(B * L, 4 * H * hd, device=device, generator=g) * shape.sigma).bfloat16()
            kc = torch.randn(S, H, hd, device=device, generator=g)
            kc = (kc * torch.rsqrt(kc.pow(2).mean(-1, keepdim=True))).bfloat16()
            vc = (torch.randn(S, H, hd, device=device, generator=g) * shape.sigma).bfloat16()
            ins.append((o4, kc, vc))
        res = {}
        for mode in ("fused", "separate"):
            layers = [dit.DitLayerAttention(B, L, H, hd, S, torch.bfloat16, device, fused=(mode == "fused"))
                      for _ in range(sets)]
            run = lambda: [layers[i % sets](ins[i % sets][0], qk_w, freqs, ins[i % sets][1], ins[i % sets][2], bias)
                           for i in range(calls)]
            st = torch.cuda.Stream(device)
            st.wait_stream(torch.cuda.current_stream(device))
            with torch.cuda.stream(st):
                run()
            torch.cuda.current_stream(device).wait_stream(st)
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                run()
            ms = time_graphs([gr], 3, 3, dist)
            res[f"{mode}_us"] = round(ms * 1e3 / (3 * calls), 3)
            del gr
        res["flops_per_block"] = shape.flops(B)
        res["fused_tflops"] = round(shape.flops(B) / (res["fused_us"] * 1e-6) / 1e12, 2)
        res["speedup"] = round(res["separate_us"] / res["fused_us"], 3)
        out[name] = res
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------------------ reference op on the GPU
def sdpa_gpu(device, dist: Dist, calls: int = 96, min_pool_bytes: int = 384 << 20) -> dict:
    """The op the reference engine runs at engine/fused.py:295 on this GPU — torch's
    F.scaled_dot_product_attention(q, k, v, attn_mask=bias) in bf16 with q (B, H, L, hd), k/v (B, H, K, hd)
    holding the conditioning keys copied into every CFG row (engine/fused.py:127-136) and an additive bf16
    bias (B, 1, 1, K), torch's own backend choice — beside sk_dit_attention on the same values, per c1 L x
    {B3, B1} and c2 B3/B1. Both are graph-replayed over a pool of distinct input sets larger than L2.
    Also times torch's cuDNN and memory-efficient backends forced one at a time (the flash backend takes
    no additive mask). Reports microseconds per call, the ratio sdpa / ours, and the rel. L2 between them."""
    from torch.nn.attention import SDPBackend, sdpa_kernel
    import torch.nn.functional as F

    from sokutou_b200 import dit, ops, workloads as W
    out = {}
    shapes = [(f"c1_L{L}", W.c1(L)) for L in W.C1_SWEEP] + [("c2", W.C2)]
    for name, sh in shapes:
        for B in (3, 1):
            H, hd, L, S = sh.H, sh.hd, sh.L, sh.S
            K = L + S
            g = torch.Generator(device=device).manual_seed(11 + B)
            per_set = 2 * (B * H * L * hd * 2 + 2 * B * H * K * hd) + 2 * S * H * hd * 2
            sets = max(4, -(-min_pool_bytes // per_set))
            bias4 = dit.cfg_bias(L, sh.Tb, sh.Sp, L, 40, device=device)[:B].contiguous()  # (B, K) bf16
            pool = []
            for _ in range(sets):
                q = (torch.randn(B, H, L, hd, device=device, generator=g) * 0.5).bfloat16()
                kl = (torch.randn(B, H, L, hd, device=device, generator=g) * 0.5).bfloat16()
                vl = (torch.randn(B, H, L, hd, device=device, generator=g) * sh.sigma).bfloat16()
                kc = (torch.randn(S, H, hd, device=device, generator=g) * 0.5).bfloat16()
                vc = (torch.randn(S, H, hd, device=device, generator=g) * sh.sigma).bfloat16()
                kf = torch.cat([kl, kc.permute(1, 0, 2).unsqueeze(0).expand(B, H, S, hd)], dim=2).contiguous()
                vf = torch.cat([vl, vc.permute(1, 0, 2).unsqueeze(0).expand(B, H, S, hd)], dim=2).contiguous()
                y_sk = torch.empty(B, L, H, hd, device=device, dtype=torch.bfloat16)
                pool.append((q, kl, vl, kc, vc, kf, vf, y_sk))
            mask = bias4.view(B, 1, 1, K)
            res = {"B": B, "H": H, "hd": hd, "L": L, "K": K, "flops": sh.flops(B), "input_sets": sets}
            try:
                res["torch_backend"] = SDPBackend(int(torch._fused_sdp_choice(pool[0][0], pool[0][5], pool[0][6],
                                                                              attn_mask=mask))).name
            except Exception as e:  # a private helper: report what failed, the timing does not depend on it
                res["torch_backend"] = f"unknown ({type(e).__name__})"

            def run_sk():
                for i in range(calls):
                    q, kl, vl, kc, vc, kf, vf, y_sk = pool[i % sets]
                    ops.dit_attention(q, kl, vl, kc, vc, bias4, out=y_sk)

            def run_sdpa(backend=None):
                def f():
                    ctx = sdpa_kernel([backend]) if backend is not None else contextlib.nullcontext()
                    with ctx:
                        for i in range(calls):
                            q, kl, vl, kc, vc, kf, vf, y_sk = pool[i % sets]
                            F.scaled_dot_product_attention(q, kf, vf, attn_mask=mask)  # the engine's call, as is
                return f

            variants = [("sk", run_sk), ("sdpa", run_sdpa()), ("sdpa_cudnn", run_sdpa(SDPBackend.CUDNN_ATTENTION)),
                        ("sdpa_efficient", run_sdpa(SDPBackend.EFFICIENT_ATTENTION))]
            for key, fn in variants:
                st = torch.cuda.Stream(device)
                st.wait_stream(torch.cuda.current_stream(device))
                try:
                    with torch.cuda.stream(st):
                        fn()
                    torch.cuda.current_stream(device).wait_stream(st)
                    gr = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(gr):
                        fn()
                except RuntimeError as e:  # a forced backend that refuses these inputs (same on every rank)
                    torch.cuda.current_stream(device).wait_stream(st)
                    torch.cuda.synchronize()
                    res[f"{key}_us"] = None
                    res[f"{key}_error"] = str(e).splitlines()[0][:160]
                    continue
                ms = time_graphs([gr], 3, 3, dist)
                res[f"{key}_us"] = round(ms * 1e3 / (3 * calls), 3)
                del gr
            # the same call computed both ways (set 0): SDPA's (B, H, L, hd) against ours (B, L, H, hd)
            q, kl, vl, kc, vc, kf, vf, y_sk = pool[0]
            ops.dit_attention(q, kl, vl, kc, vc, bias4, out=y_sk)
            y_t = F.scaled_dot_product_attention(q, kf, vf, attn_mask=mask).transpose(1, 2).float()
            res["rel_l2_vs_sdpa"] = float((y_sk.float() - y_t).norm() / y_t.norm())
            for key in ("sk", "sdpa", "sdpa_cudnn", "sdpa_efficient"):
                if res.get(f"{key}_us"):
                    res[f"{key}_tflops"] = round(sh.flops(B) / (res[f"{key}_us"] * 1e-6) / 1e12, 1)
            if res.get("sk_us") and res.get("sdpa_us"):
                res["speedup_vs_sdpa"] = round(res["sdpa_us"] / res["sk_us"], 3)
            best = min((res[f"{k}_us"] for k in ("sdpa", "sdpa_cudnn", "sdpa_efficient") if res.get(f"{k}_us")),
                       default=None)
            if best and res.get("sk_us"):
                res["speedup_vs_best_sdpa"] = round(best / res["sk_us"], 3)
            out[f"{name}_b{B}"] = res
            del pool
            torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------------------------------- DiT GEMMs
GEMM_SHAPES = (  # name, M (= B·L rows), N, K, fp8: the attention block's projections at B = 3, L = 512
    ("c1_w_qkvg_b3", 1536, 4 * 768, 768, False), ("c1_w_o_b3", 1536, 768, 768, False),
    ("c2_w_qkvg_b3", 1536, 4 * 2048, 2048, False), ("c2_w_o_b3", 1536, 2048, 2048, False),
    ("c2_w_qkvg_b3_fp8", 1536, 4 * 2048, 2048, True), ("c2_w_o_b3_fp8", 1536, 2048, 2048, True),
    # the MLP around the SwiGLU (engine/fused.py:305-310), hidden = 2.875·D as in the Small model's
    # 1280 -> 3680 (ref/gemm_bench.py:26)
    ("c1_w_13_b3", 1536, 2 * 2208, 768, False), ("c1_w_2_b3", 1536, 768, 2208, False),
    ("c2_w_13_b3", 1536, 2 * 5888, 2048, False), ("c2_w_2_b3", 1536, 2048, 5888, False),
    ("c2_w_13_b3_fp8", 1536, 2 * 5888, 2048, True), ("c2_w_2_b3_fp8", 1536, 2048, 5888, True),
)


def dit_gemm(device, dist: Dist, calls: int = 60, sets: int = 4) -> dict:
    """The DiT projections y = x·wᵀ (engine/fused.py:262-264) on the tcgen05 GEMM (sk_dit_linear; the FP8
    rows: sk_dit_linear_fp8, engine/fp8.py:87-89) and, beside it, torch's own GEMM on the same inputs
    (F.linear / cuBLAS; torch._scaled_mm / cuBLASLt for FP8); `sets` distinct (x, w) pairs rotated over
    `calls` graph-replayed calls. Reports microseconds per call and TFLOP/s (2·M·N·K per call)."""
    from sokutou_b200 import ops
    out = {}
    for name, M, N, K, fp8 in GEMM_SHAPES:
        g = torch.Generator(device=device).manual_seed(9)
        if fp8:
            e4 = torch.float8_e4m3fn
            ins = [((torch.randn(M, K, device=device, generator=g) * 8).to(e4),
                    (torch.randn(N, K, device=device, generator=g) * 32).to(e4),
                    torch.empty(M, N, device=device, dtype=torch.bfloat16)) for _ in range(sets)]
            inv_x = torch.tensor([1 / 16], device=device)
            inv_w = torch.tensor([1 / 64], device=device)
        else:
            ins = [((torch.randn(M, K, device=device, generator=g)).bfloat16(),
                    (torch.randn(N, K, device=device, generator=g) * K ** -0.5).bfloat16(),
                    torch.empty(M, N, device=device, dtype=torch.bfloat16)) for _ in range(sets)]
        res = {"M": M, "N": N, "K": K, "dtype": "e4m3" if fp8 else "bf16"}
        for impl in ("sk", "cublas"):
            if impl == "sk" and fp8:
                run = lambda: [ops.dit_linear_fp8(ins[i % sets][0], ins[i % sets][1], inv_x, inv_w, out=ins[i % sets][2])
                               for i in range(calls)]
            elif impl == "sk":
                run = lambda: [ops.dit_linear(ins[i % sets][0], ins[i % sets][1], out=ins[i % sets][2])
                               for i in range(calls)]
            elif fp8:
                run = lambda: [torch._scaled_mm(ins[i % sets][0], ins[i % sets][1].t(), inv_x, inv_w,
                                                out_dtype=torch.bfloat16, out=ins[i % sets][2]) for i in range(calls)]
            else:
                run = lambda: [torch.matmul(ins[i % sets][0], ins[i % sets][1].t(), out=ins[i % sets][2])
                               for i in range(calls)]
            st = torch.cuda.Stream(device)
            st.wait_stream(torch.cuda.current_stream(device))
            with torch.cuda.stream(st):
                try:
                    run()
                except RuntimeError as e:  # torch's FP8 GEMM may not take this shape or build (same on every rank)
                    if impl == "sk":
                        raise
                    res["cublas_us"] = None
                    res["cublas_error"] = str(e).splitlines()[0][:160]
                    torch.cuda.current_stream(device).wait_stream(st)
                    continue
            torch.cuda.current_stream(device).wait_stream(st)
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                run()
            ms = time_graphs([gr], 3, 3, dist)
            us = ms * 1e3 / (3 * calls)
            key = "us" if impl == "sk" else "cublas_us"
            res[key] = round(us, 3)
            res["tflops" if impl == "sk" else "cublas_tflops"] = round(2 * M * N * K / (us * 1e-6) / 1e12, 1)
            del gr
        out[name] = res
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------------------- grouped decode requests
def c3_grouped(device, dist: Dist, Rs=(8, 32), lo: int = 1023, hi: int = 1120) -> dict:
    """c3-shaped decode attention for R independent talkers in one launch per layer
    (sk_decode_attention_grouped): R requests x 28 layers, positions lo..hi-1 (T >= 1024), each request with
    its own caches (R x 176 MB, far past L2), graph-replayed one decode step (28 grouped launches and the
    position advances) at a time. Bytes per launch: R times the one-request algorithmic bytes."""
    from sokutou_b200 import ops, qwen3, workloads as W
    s = W.C3
    out = {}
    for R in Rs:
        g = torch.Generator(device=device).manual_seed(R)
        tas = []
        for _ in range(R):
            ta = qwen3.TalkerAttention(s.n_layers, s.nq, s.nkv, 1152, s.theta, s.eps, device, torch.bfloat16)
            ta.k.normal_(generator=g)
            ta.v.normal_(generator=g)
            tas.append(ta)
        qkv = torch.randn(R, s.n_layers, (s.nq + 2 * s.nkv) * s.hd, device=device, generator=g)
        qn = 1 + 0.02 * torch.randn(s.n_layers, s.hd, device=device, generator=g)
        att = torch.empty(R, s.n_layers, s.nq * s.hd, device=device)
        descs = [ops.decode_requests([{"qkv": qkv[r, li], "qn": qn[li], "kn": qn[li], "rope": tas[r].rope,
                                       "Kc": tas[r].k[li], "Vc": tas[r].v[li], "pos_ptr": tas[r].pos,
                                       "out": att[r, li], "pos_add": 0, "eps": s.eps} for r in range(R)], device)
                 for li in range(s.n_layers)]

        def step():
            for li in range(s.n_layers):
                ops.decode_attention_grouped(descs[li], R, 1152, s.nq, s.nkv, torch.bfloat16, kv_stable=li > 0)
            for ta in tas:
                ta.pos.add_(1)

        st = torch.cuda.Stream(device)
        st.wait_stream(torch.cuda.current_stream(device))
        for ta in tas:
            ta.pos.fill_(lo)
        with torch.cuda.stream(st):
            step()
        torch.cuda.current_stream(device).wait_stream(st)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            step()
        for ta in tas:
            ta.pos.fill_(lo)
        gr.replay()
        torch.cuda.synchronize()
        dist.barrier()
        for ta in tas:
            ta.pos.fill_(lo)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(lo, hi):
            gr.replay()
        e1.record()
        torch.cuda.synchronize()
        ms = dist.max(e0.elapsed_time(e1))
        del gr
        tot = R * s.n_layers * sum(s.layer_bytes(p + 1) for p in range(lo, hi))
        out[f"R{R}"] = {"us_per_launch": round(ms * 1e3 / ((hi - lo) * s.n_layers), 3),
                        "gbs": round(tot / (ms / 1e3) / 1e9, 1), "requests": R, "T_range": [lo + 1, hi]}
        del tas, descs
        torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------------------- fused decode layer block
def decode_block_bench(device, dist: Dist, hidden: int = 2048, lo: int = 1023, hi: int = 1120) -> dict:
    """One talker layer's attention block — rms_gemv(qkv) -> attention -> gemv(o), the three launches of
    qwen3/kernels.py:619-624 — at the 1.7B talker's width (hidden 2048, bf16 weights, bf16 cache), decoding
    positions lo..hi-1 (T >= 1024) through all 28 layers with distinct weights per layer (0.7 GB, far past
    L2), graph-replayed: the one-launch kernel (sk_decode_attention_block) against the same block as three
    launches (torch's bf16 GEMVs around sk_decode_attention). Bytes per layer: both weight matrices, the
    K/V read and append, qkv/att/h traffic."""
    from sokutou_b200 import ops, qwen3, workloads as W
    s = W.C3
    nl, nq, nkv, hd = s.n_layers, s.nq, s.nkv, s.hd
    g = torch.Generator(device=device).manual_seed(21)
    Dq = (nq + 2 * nkv) * hd
    wq = (torch.randn(nl, Dq, hidden, device=device, generator=g) / hidden ** 0.5).bfloat16()
    wo = (torch.randn(nl, hidden, nq * hd, device=device, generator=g) / (nq * hd) ** 0.5).bfloat16()
    nw = 1 + 0.1 * torch.randn(nl, hidden, device=device, generator=g)
    qn = 1 + 0.02 * torch.randn(nl, hd, device=device, generator=g)
    kn = 1 + 0.02 * torch.randn(nl, hd, device=device, generator=g)
    ta = qwen3.TalkerAttention(nl, nq, nkv, 1536, s.theta, s.eps, device, torch.bfloat16)
    ta.k.copy_(torch.randn(ta.k.shape, device=device, generator=g))
    ta.v.copy_(torch.randn(ta.v.shape, device=device, generator=g))
    h = torch.randn(hidden, device=device, generator=g)
    qkv = torch.empty(Dq, device=device)
    att = torch.empty(nq * hd, device=device)

    def fused():
        for li in range(nl):
            ta.block(li, h, nw[li], s.eps, wq[li], qn[li], kn[li], wo[li], kv_stable=li > 0)
        ta.pos.add_(1)

    def separate():
        for li in range(nl):
            x = (h * nw[li] * torch.rsqrt((h * h).mean() + s.eps)).bfloat16()
            qkv.copy_(torch.mv(wq[li], x))
            ta.attn(li, qkv, qn[li], kn[li], att, kv_stable=li > 0)
            h.add_(torch.mv(wo[li], att.bfloat16()))
        ta.pos.add_(1)

    res = {"hidden": hidden, "layers": nl, "weights": "bf16", "cache": "bf16", "T_range": [lo + 1, hi]}
    w_bytes = (Dq + hidden) * hidden * 2
    tot = sum(w_bytes + s.layer_bytes(p + 1) + 2 * hidden * 4 for p in range(lo, hi)) * nl
    for name, fn in (("fused", fused), ("separate", separate)):
        st = torch.cuda.Stream(device)
        st.wait_stream(torch.cuda.current_stream(device))
        ta.pos.fill_(lo)
        with torch.cuda.stream(st):
            fn()
        torch.cuda.current_stream(device).wait_stream(st)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            fn()
        ta.pos.fill_(lo)
        gr.replay()  # warm-up
        torch.cuda.synchronize()
        dist.barrier()
        ta.pos.fill_(lo)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(lo, hi):
            gr.replay()
        e1.record()
        torch.cuda.synchronize()
        ms = dist.max(e0.elapsed_time(e1))
        del gr
        res[f"{name}_us_per_layer"] = round(ms * 1e3 / ((hi - lo) * nl), 3)
        res[f"{name}_gbs"] = round(tot / (ms / 1e3) / 1e9, 1)
    res["bytes_per_layer_at_T1120"] = w_bytes + s.layer_bytes(hi) + 2 * hidden * 4
    res["speedup"] = round(res["separate_us_per_layer"] / res["fused_us_per_layer"], 3)
    del wq, wo, ta
    torch.cuda.empty_cache()
    return res


# ------------------------------------------------------------------------------------------- prefill
def prefill_bench(device, dist: Dist) -> dict:
    """The c3 prompt (and a 160-token one) through all 28 talker layers' prefill attention, graph-replayed,
    against the same tokens as decode steps (what the cache fill costs without a prefill kernel)."""
    from sokutou_b200 import ops, qwen3, workloads as W
    s = W.C3
    out = {}
    for T in (s.prompt, 160):
        g = torch.Generator(device=device).manual_seed(T)
        ta = qwen3.TalkerAttention(s.n_layers, s.nq, s.nkv, 1536, s.theta, s.eps, device, torch.bfloat16)
        rows = torch.randn(s.n_layers, T, (s.nq + 2 * s.nkv) * s.hd, device=device, generator=g)
        qn = 1 + 0.02 * torch.randn(s.n_layers, s.hd, device=device, generator=g)
        yo = torch.empty(T, s.nq * s.hd, device=device, dtype=torch.bfloat16)
        qb = torch.empty(s.nq, T, s.hd, device=device, dtype=torch.bfloat16)
        od = torch.empty(s.nq * s.hd, device=device)

        def run_prefill():
            for li in range(s.n_layers):
                ops.prefill_attention(rows[li], qn[li], qn[li], s.eps, ta.rope, ta.k[li], ta.v[li], 0, 1536, s.nq,
                                      s.nkv, out=yo, q_buf=qb)

        def run_decode():
            for t in range(T):
                for li in range(s.n_layers):
                    ta.attn(li, rows[li, t], qn[li], qn[li], od, pos_add=t)

        res = {}
        for name, fn in (("prefill", run_prefill), ("decode_steps", run_decode)):
            st = torch.cuda.Stream(device)
            st.wait_stream(torch.cuda.current_stream(device))
            with torch.cuda.stream(st):
                fn()
            torch.cuda.current_stream(device).wait_stream(st)
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                fn()
            ms = time_graphs([gr], 3, 3, dist)
            res[f"{name}_us_per_prompt"] = round(ms * 1e3 / 3, 2)
            del gr
        res["layers"] = s.n_layers
        res["speedup"] = round(res["decode_steps_us_per_prompt"] / res["prefill_us_per_prompt"], 2)
        out[f"T{T}"] = res
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------------------------- serving
def serving(dist: Dist, device):
    """64 requests, longest-first static sharding over the ranks; sentences/s."""
    from sokutou_b200 import serving as SV
    reqs = SV.requests_c4(0)
    plan = SV.plan_lpt(reqs, dist.world)
    mine = plan[dist.rank]
    ex = SV.GpuExecutor(device)
    ex.warm(mine)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    ex.run_all(mine)
    e1.record()
    torch.cuda.synchronize()
    dt = dist.max(e0.elapsed_time(e1) / 1e3)
    dist.barrier()
    return {"requests": len(reqs), "sentences_per_s": len(reqs) / dt, "makespan_s": dt,
            "per_rank_requests": [len(p) for p in plan], "sharding": "longest-first static, no collectives",
            "decode": f"continuous batching over {SV.GpuExecutor.SLOTS} slots, one grouped launch per layer",
            "dit_inputs": "distinct q/k/v per call from a pool larger than L2"}


# ---------------------------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-serving", action="store_true")
    ap.add_argument("--only-c1", action="store_true", help="headline workload only (for launch-list captures)")
    ap.add_argument("--skip", default="", help="comma list of extra sections to leave out: sdpa,layer,gemm,prefill,block,grouped,serving")
    ap.add_argument("--cpu-seconds", type=float, default=20.0, help="CPU time budget of the reference arm")
    a = ap.parse_args()
    if a.impl == "reference":
        return reference_arm(a)
    dist = Dist(a.gpus)
    dev = dist.device
    torch.cuda.set_device(dev)
    from sokutou_b200 import build
    if dist.rank == 0:
        build.build()
    dist.barrier()
    from sokutou_b200 import ops, workloads as W
    pk, pk_kind = peaks()

    # ---- headline: c1 sweep
    shapes = [W.c1(L) for L in W.C1_SWEEP]
    syn = [DitSynthesis(sh, dev, seed=100 + i + 1000 * dist.rank) for i, sh in enumerate(shapes)]
    for s in syn:
        s.capture()
    torch.cuda.synchronize()
    flops_step = sum(s.flops for s in syn)
    launches_step = sum(len(s.calls) for s in syn)
    with ClockSampler(dev) as clk:
        ms = time_graphs([s.graph for s in syn], a.steps, max(a.warmup, 3), dist, label="c1_step", clk=clk)
    ms_step = ms / a.steps
    value = dist.sum(flops_step) / (ms_step / 1e3) / 1e12
    per_gpu = flops_step / (ms_step / 1e3) / 1e12
    per_L = {}
    for s in syn:
        t = time_graphs([s.graph], a.steps, 1, dist) / a.steps
        per_L[f"L{s.shape.L}"] = {"tflops": round(s.flops / (t / 1e3) / 1e12, 2), "ms_per_synthesis": round(t, 4),
                                  "us_per_call": round(t * 1e3 / len(s.calls), 3)}
    if a.only_c1:
        if dist.rank == 0:
            print(json.dumps({"metric": METRIC, "value": round(value, 3), "unit": UNIT, "ms_per_step": round(ms_step, 4),
                              "per_L": per_L, "note": "--only-c1: headline timing only"}), flush=True)
        dist.close()
        return
    e2e_ms, h2d, d2h = dit_e2e(syn, max(1, a.steps // 5), 1, dist, dev)
    e2e_steps = max(1, a.steps // 5)
    e2e_val = dist.sum(flops_step) / (e2e_ms / e2e_steps / 1e3) / 1e12
    for s in syn:
        s.graph = None
    del syn
    torch.cuda.empty_cache()

    # ---- c2 (v4-Large-class)
    c2 = DitSynthesis(W.C2, dev, seed=7 + 1000 * dist.rank)
    c2.capture()
    t2 = time_graphs([c2.graph], max(2, a.steps // 2), 2, dist) / max(2, a.steps // 2)
    c2_res = {"tflops_per_gpu": round(c2.flops / (t2 / 1e3) / 1e12, 2), "ms_per_synthesis": round(t2, 3),
              "us_per_call": round(t2 * 1e3 / len(c2.calls), 3),
              "frac_of_measured_bf16": round(c2.flops / (t2 / 1e3) / 1e12 / pk["bf16_tflops"], 4),
              "frac_of_spec_bf16": round(c2.flops / (t2 / 1e3) / 1e12 / SPEC["bf16_tflops"], 4)}
    c2.graph = None
    del c2
    torch.cuda.empty_cache()

    # ---- c3 decode
    dec = DecodeBench(dev)
    dec.capture()
    s3 = W.C3
    dec.run_decode(s3.prompt, s3.prompt + 32)  # warm-up
    dist.barrier()
    t_full = dist.max(dec.run_decode(s3.prompt, s3.T_final))
    b_full = dec.bytes(s3.prompt, s3.T_final)
    t_hi = dist.max(dec.run_decode(1023, s3.T_final))
    b_hi = dec.bytes(1023, s3.T_final)
    n_calls_full = (s3.T_final - s3.prompt) * s3.n_layers * dec.n_sets
    c3_res = {"gbs_per_gpu": round(b_full / (t_full / 1e3) / 1e9, 1),
              "ms_per_decode": round(t_full / dec.n_sets, 3), "us_per_call": round(t_full * 1e3 / n_calls_full, 3),
              "gbs_at_T_ge_1024": round(b_hi / (t_hi / 1e3) / 1e9, 1),
              "frac_of_measured_hbm_at_T_ge_1024": round(b_hi / (t_hi / 1e3) / 1e9 / pk["hbm_gbs"], 4),
              "frac_of_spec_hbm_at_T_ge_1024": round(b_hi / (t_hi / 1e3) / 1e9 / SPEC["hbm_gbs"], 4),
              "cache_sets_rotated": dec.n_sets, "bytes_per_decode": s3.decode_bytes()}
    del dec
    torch.cuda.empty_cache()

    # ---- the reference's own op on this GPU (torch SDPA) beside ours; fused attention block vs its three
    # launches; projection GEMMs beside cuBLAS; Qwen3 prompt prefill
    skip = set(a.skip.split(",")) if a.skip else set()
    sdpa = None if "sdpa" in skip else sdpa_gpu(dev, dist)
    blocks = None if "layer" in skip else layer_block(dev, dist)
    gemm = None if "gemm" in skip else dit_gemm(dev, dist)
    prefill = None if "prefill" in skip else prefill_bench(dev, dist)
    dblock = None if "block" in skip else decode_block_bench(dev, dist)
    grouped = None if "grouped" in skip else c3_grouped(dev, dist)
    if grouped:
        for v in grouped.values():
            v["frac_of_measured_hbm"] = round(v["gbs"] / pk["hbm_gbs"], 4)
    if dblock:
        dblock["fused_frac_of_measured_hbm"] = round(dblock["fused_gbs"] / pk["hbm_gbs"], 4)

    # ---- c4 serving
    serv = None if (a.no_serving or "serving" in skip) else serving(dist, dev)
    err = ops.device_error()

    # ---- CPU baseline (rank 0, N=1 only)
    cpu = None
    if dist.rank == 0 and dist.world == 1:
        v, cores, sample = cpu_dit_sample(shapes)
        cpu = {"value": round(v, 4), "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}

    if dist.rank == 0:
        traffic = profile_traffic_mix("dit_attn_tc_c1.md", shapes)
        achieved = per_gpu  # every launch in the step is the DiT attention kernel: FLOPs/launch ÷ avg launch time
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": dist.world, "steps": a.steps,
            "warmup": max(a.warmup, 3), "ms_per_step": round(ms_step, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
            "config": c1_config(dist.world, launches_step, flops_step),
            "per_L": per_L,
            "e2e": {"value": round(e2e_val, 4), "unit": UNIT, "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h), "path": "sokutou_b200.ops.dit_attention (C ABI); per flow step one H2D of its calls' q/k/v from pinned host memory and one D2H of their outputs, pipelined over three streams"},
            "gpu_launches": launches_step * a.steps,
            "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": pk["bf16_tflops"], "unit": UNIT,
                         "frac": round(achieved / pk["bf16_tflops"], 4), "peak_kind": f"{pk_kind} bf16 burst",
                         "frac_of_spec": round(achieved / SPEC["bf16_tflops"], 4), "traffic": traffic},
            "c2": c2_res, "c3": c3_res, "sdpa_gpu": sdpa, "layer_block": blocks, "dit_gemm": gemm, "prefill": prefill, "decode_block": dblock, "c3_grouped": grouped, "serving": serv, "cpu_baseline": cpu,
            "clocks": clk.summary(), "device_error": err,
        }
        print(json.dumps(line), flush=True)
    dist.close()


def reference_arm(a):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from sokutou_b200 import workloads as W
    shapes = [W.c1(L) for L in W.C1_SWEEP]
    per_step = max(min(4.0, a.cpu_seconds), a.cpu_seconds / max(a.steps + a.warmup, 1))
    for _ in range(a.warmup):
        cpu_dit_sample(shapes, seconds=per_step / 2)
    vals = []
    t0 = time.perf_counter()
    for _ in range(a.steps):
        v, cores, sample = cpu_dit_sample(shapes, seconds=per_step)
        vals.append(v)
    el = time.perf_counter() - t0
    v = statistics.mean(vals)
    line = {"metric": METRIC, "value": round(v, 5), "unit": UNIT, "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(el * 1e3 / max(a.steps, 1), 1), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)", "impl": "reference",
            "config": c1_config(world, sum(len(sh.synthesis_calls()) for sh in shapes),
                                sum(sh.synthesis_flops() for sh in shapes)),
            "cpu_baseline": {"value": round(v, 5), "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": sample + "; torch F.scaled_dot_product_attention float32 with the ctx keys "
                                                "copied per batch row, as the reference engine runs it"},
            "e2e": {"value": round(v, 5), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
