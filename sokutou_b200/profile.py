"""Small, self-contained runs of one kernel for timing and for ncu captures.

    python -m sokutou_b200.profile --case dit_c1_L512_b3 [--reps 50] [--graph]
    python -m sokutou_b200.profile --case decode_T1120 [--reps 50] [--graph]
    python -m sokutou_b200.profile --case block_T1120 [--reps 50] [--graph]

Prints one JSON record: the case's shape, average microseconds per call from CUDA events over `reps`
back-to-back calls (eager launches, or one CUDA graph holding them with --graph), the algorithmic work
per call, the rate and its fraction of the measured peak (MEASURED_PEAKS.json: bf16 tensor TFLOP/s
for contractions, HBM GB/s for the rest) and, with --cpu, the same call timed on the host cores with
torch's fp32 SDPA (the reference's own op) beside it.
Inputs: distinct buffers per call, rotated over `--sets` copies so that a run can exceed L2.
"""

from __future__ import annotations

import argparse
import json

import torch

from . import dit, ops, qwen3, workloads as W

CASES = {
    # name: (kind, shape args)
    "dit_c1_L128_b3": ("dit", W.c1(128), 3), "dit_c1_L128_b1": ("dit", W.c1(128), 1),
    "dit_c1_L256_b3": ("dit", W.c1(256), 3), "dit_c1_L256_b1": ("dit", W.c1(256), 1),
    "dit_c1_L512_b3": ("dit", W.c1(512), 3), "dit_c1_L512_b1": ("dit", W.c1(512), 1),
    "dit_c2_b3": ("dit", W.C2, 3), "dit_c2_b1": ("dit", W.C2, 1),
    # one DiT layer's attention block: fused launch vs producer + attention + gate launches
    "layer_c1_L128_b1_fused": ("layer", W.c1(128), 1), "layer_c1_L128_b1_sep": ("layer_sep", W.c1(128), 1),
    "layer_c1_L512_b3_fused": ("layer", W.c1(512), 3), "layer_c1_L512_b3_sep": ("layer_sep", W.c1(512), 3),
    "layer_c2_b3_fused": ("layer", W.C2, 3), "layer_c2_b3_sep": ("layer_sep", W.C2, 3),
    # the block's two HBM-bound kernels alone
    "prologue_c1_L512_b3": ("prologue", W.c1(512), 3), "prologue_c2_b3": ("prologue", W.C2, 3),
    "gate_c1_L512_b3": ("gate", W.c1(512), 3), "gate_c2_b3": ("gate", W.C2, 3),
    "prefill_T96": ("prefill", 96, None), "prefill_T160": ("prefill", 160, None),
    "decode_T128": ("decode", 128, None), "decode_T512": ("decode", 512, None),
    "decode_T1120": ("decode", 1120, None), "decode_T1500": ("decode", 1500, None),
    "decode_T1120_kvstable": ("decode", 1120, "kv_stable"), "decode_T128_kvstable": ("decode", 128, "kv_stable"),
    # the projections around the block (M = B·L rows, N, K), tcgen05 GEMM and torch's cuBLAS F.linear
    "linear_c1_qkvg_b3": ("linear", (1536, 3072, 768), "sk"), "cublas_c1_qkvg_b3": ("linear", (1536, 3072, 768), "cublas"),
    "linear_c2_qkvg_b3": ("linear", (1536, 8192, 2048), "sk"), "cublas_c2_qkvg_b3": ("linear", (1536, 8192, 2048), "cublas"),
    "linear_c2_o_b3": ("linear", (1536, 2048, 2048), "sk"), "cublas_c2_o_b3": ("linear", (1536, 2048, 2048), "cublas"),
    "linear_fp8_c2_qkvg_b3": ("linear", (1536, 8192, 2048), "sk_fp8"),
    "scaledmm_c2_qkvg_b3": ("linear", (1536, 8192, 2048), "cublas_fp8"),
    # one talker layer's attention block in one launch (rms_gemv(qkv) -> attention -> gemv(o)), 1.7B width
    "block_T1120": ("block", 1120, 2048), "block_T128": ("block", 128, 2048),
    # R independent decode requests in one launch
    "grouped_R8_T1120": ("grouped", 1120, 8), "grouped_R32_T1120": ("grouped", 1120, 32),
    # calibration: what a chain of dependent kernels costs on this GPU without any attention work
    "calib_tiny": ("calib", 0, None), "calib_copy_4.6MB": ("calib", 4616192, None),
}


def dit_case(shape, B, sets, dev):
    g = torch.Generator(device=dev).manual_seed(0)
    H, hd, L, S = shape.H, shape.hd, shape.L, shape.S
    calls = []
    for _ in range(sets):
        q, k, v = (torch.randn(B, H, L, hd, device=dev, generator=g).bfloat16() for _ in range(3))
        kc = torch.randn(S, H, hd, device=dev, generator=g).bfloat16()
        vc = torch.randn(S, H, hd, device=dev, generator=g).bfloat16()
        y = torch.empty(B, L, H, hd, device=dev, dtype=torch.bfloat16)
        calls.append((q, k, v, kc, vc, y))
    bias = dit.cfg_bias(L, shape.Tb, shape.Sp, L, 40, device=dev)[:B].contiguous()
    fns = [lambda c=c: ops.dit_attention(c[0], c[1], c[2], c[3], c[4], bias, out=c[5]) for c in calls]
    return fns, shape.flops(B), "flop"


def layer_case(shape, B, sets, dev, fused: bool):
    g = torch.Generator(device=dev).manual_seed(0)
    H, hd, L, S = shape.H, shape.hd, shape.L, shape.S
    qk_w = W.dit_qk_weights(shape, dev)
    freqs = W.dit_freqs(L, hd, device=dev)
    bias = dit.cfg_bias(L, shape.Tb, shape.Sp, L, 40, device=dev)[:B].contiguous()
    fns = []
    for _ in range(sets):
        o4 = (torch.randn(B * L, 4 * H * hd, device=dev, generator=g) * 0.5).bfloat16()
        kc = torch.randn(S, H, hd, device=dev, generator=g).bfloat16()
        vc = torch.randn(S, H, hd, device=dev, generator=g).bfloat16()
        layer = dit.DitLayerAttention(B, L, H, hd, S, torch.bfloat16, dev, fused=fused)
        fns.append(lambda o4=o4, kc=kc, vc=vc, layer=layer: layer(o4, qk_w, freqs, kc, vc, bias))
    return fns, shape.flops(B), "flop"


def elementwise_case(kind, shape, B, sets, dev):
    """The producer (q, k, v from o4) or the gate (y · sigmoid(gate)) of one block; work = bytes moved."""
    g = torch.Generator(device=dev).manual_seed(0)
    H, hd, L = shape.H, shape.hd, shape.L
    qk_w = W.dit_qk_weights(shape, dev)
    freqs = W.dit_freqs(L, hd, device=dev)
    fns = []
    for _ in range(sets):
        o4 = (torch.randn(B * L, 4 * H * hd, device=dev, generator=g) * 0.5).bfloat16()
        if kind == "prologue":
            bufs = tuple(torch.empty(B, H, L, hd, device=dev, dtype=torch.bfloat16) for _ in range(3))
            fns.append(lambda o4=o4, bufs=bufs: ops.dit_qkv_prologue(o4, qk_w, freqs, B, L, H, hd, 1e-6, out=bufs))
        else:
            y = torch.randn(B * L, H * hd, device=dev, generator=g).bfloat16()
            out = torch.empty_like(y)
            fns.append(lambda o4=o4, y=y, out=out: ops.dit_gate(y, o4, out=out))
    moved = B * L * H * hd * 2 * (6 if kind == "prologue" else 3)
    return fns, moved, "byte"


def prefill_case(T, sets, dev):
    """One talker layer's prompt prefill (T tokens from position 0); work = the causal FLOPs."""
    s = W.C3
    max_len = 1536
    g = torch.Generator(device=dev).manual_seed(0)
    fns = []
    for _ in range(sets):
        ta = qwen3.TalkerAttention(1, s.nq, s.nkv, max_len, s.theta, s.eps, dev, torch.bfloat16)
        rows = torch.randn(T, (s.nq + 2 * s.nkv) * s.hd, device=dev, generator=g)
        qn = torch.ones(s.hd, device=dev)
        out = torch.empty(T, s.nq * s.hd, device=dev, dtype=torch.bfloat16)
        qb = torch.empty(s.nq, T, s.hd, device=dev, dtype=torch.bfloat16)
        fns.append(lambda ta=ta, rows=rows, qn=qn, out=out, qb=qb: ops.prefill_attention(
            rows, qn, qn, s.eps, ta.rope, ta.k[0], ta.v[0], 0, max_len, s.nq, s.nkv, out=out, q_buf=qb))
    return fns, 4 * s.nq * s.hd * T * (T + 1) // 2, "flop"


def decode_case(T, sets, dev, kv_stable=False):
    s = W.C3
    max_len = 1536
    g = torch.Generator(device=dev).manual_seed(0)
    fns = []
    for _ in range(sets):
        ta = qwen3.TalkerAttention(1, s.nq, s.nkv, max_len, s.theta, s.eps, dev, torch.bfloat16)
        ta.k.copy_(torch.randn(ta.k.shape, device=dev, generator=g))
        ta.v.copy_(torch.randn(ta.v.shape, device=dev, generator=g))
        ta.pos.fill_(T - 1)
        qkv = torch.randn((s.nq + 2 * s.nkv) * s.hd, device=dev, generator=g)
        qn = torch.ones(s.hd, device=dev)
        out = torch.empty(s.nq * s.hd, device=dev)
        fns.append(lambda ta=ta, qkv=qkv, qn=qn, out=out: ta.attn(0, qkv, qn, qn, out, kv_stable=kv_stable))
    return fns, s.layer_bytes(T), "byte"


def block_case(T, hidden, sets, dev):
    """One talker layer's attention block (sk_decode_attention_block) at T keys, bf16 weights and cache;
    work = both weight matrices + the decode attention's bytes + the h / qkv / att traffic."""
    s = W.C3
    max_len = 1536
    g = torch.Generator(device=dev).manual_seed(0)
    Dq = (s.nq + 2 * s.nkv) * s.hd
    fns = []
    for _ in range(sets):
        ta = qwen3.TalkerAttention(1, s.nq, s.nkv, max_len, s.theta, s.eps, dev, torch.bfloat16)
        ta.k.normal_(generator=g)
        ta.v.normal_(generator=g)
        ta.pos.fill_(T - 1)
        wq = (torch.randn(Dq, hidden, device=dev, generator=g) / hidden ** 0.5).bfloat16()
        wo = (torch.randn(hidden, s.nq * s.hd, device=dev, generator=g) / (s.nq * s.hd) ** 0.5).bfloat16()
        h = torch.randn(hidden, device=dev, generator=g)
        nw = torch.ones(hidden, device=dev)
        qn = torch.ones(s.hd, device=dev)
        # the position stays at T - 1: every call re-appends the same row and attends over T keys
        fns.append(lambda ta=ta, wq=wq, wo=wo, h=h, nw=nw, qn=qn: ta.block(0, h, nw, s.eps, wq, qn, qn, wo))
    return fns, (Dq + hidden) * hidden * 2 + s.layer_bytes(T) + 2 * hidden * 4, "byte"


def grouped_case(T, R, sets, dev):
    """R independent decode requests at T keys in one launch (sk_decode_attention_grouped); work = R times
    the one-request bytes."""
    s = W.C3
    max_len = 1152
    g = torch.Generator(device=dev).manual_seed(0)
    fns = []
    for _ in range(sets):
        tas = []
        for _ in range(R):
            ta = qwen3.TalkerAttention(1, s.nq, s.nkv, max_len, s.theta, s.eps, dev, torch.bfloat16)
            ta.k.normal_(generator=g)
            ta.v.normal_(generator=g)
            ta.pos.fill_(T - 1)
            tas.append(ta)
        qkv = torch.randn(R, (s.nq + 2 * s.nkv) * s.hd, device=dev, generator=g)
        qn = torch.ones(s.hd, device=dev)
        out = torch.empty(R, s.nq * s.hd, device=dev)
        descs = ops.decode_requests([{"qkv": qkv[r], "qn": qn, "kn": qn, "rope": tas[r].rope, "Kc": tas[r].k[0],
                                      "Vc": tas[r].v[0], "pos_ptr": tas[r].pos, "out": out[r], "eps": s.eps}
                                     for r in range(R)], dev)
        keep = (tas, qkv, qn, out)
        fns.append(lambda descs=descs, keep=keep: ops.decode_attention_grouped(descs, R, max_len, s.nq, s.nkv))
    return fns, R * s.layer_bytes(T), "byte"


def linear_case(mnk, impl, sets, dev):
    """y = x·wᵀ (engine/fused.py:262-264) on sk_dit_linear or on torch's F.linear (cuBLAS); work = 2·M·N·K."""
    M, N, K = mnk
    g = torch.Generator(device=dev).manual_seed(0)
    fns = []
    inv_x = torch.tensor([1 / 16], device=dev)
    inv_w = torch.tensor([1 / 64], device=dev)
    for _ in range(sets):
        y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        if impl.endswith("fp8"):  # the FP8 path (engine/fp8.py:87-89): e4m3 operands, per-tensor inverse scales
            x = (torch.randn(M, K, device=dev, generator=g) * 8).to(torch.float8_e4m3fn)
            w = (torch.randn(N, K, device=dev, generator=g) * 32).to(torch.float8_e4m3fn)
            if impl == "sk_fp8":
                fns.append(lambda x=x, w=w, y=y: ops.dit_linear_fp8(x, w, inv_x, inv_w, out=y))
            else:
                fns.append(lambda x=x, w=w, y=y: torch._scaled_mm(x, w.t(), inv_x, inv_w, out_dtype=torch.bfloat16,
                                                                  out=y))
            continue
        x = torch.randn(M, K, device=dev, generator=g).bfloat16()
        w = (torch.randn(N, K, device=dev, generator=g) * K ** -0.5).bfloat16()
        if impl == "sk":
            fns.append(lambda x=x, w=w, y=y: ops.dit_linear(x, w, out=y))
        else:
            fns.append(lambda x=x, w=w, y=y: torch.matmul(x, w.t(), out=y))
    return fns, 2 * M * N * K, "flop"


def calib_case(nbytes, sets, dev):
    """A dependent chain of torch kernels: a one-element add (launch floor), or a device copy of
    `nbytes` (twice that moved) over 16 rotating buffer pairs so the copies miss L2."""
    if nbytes == 0:
        x = torch.zeros(1, device=dev)
        return [lambda: x.add_(1.0)], 1, "byte"
    n = nbytes // 2
    bufs = [(torch.randn(n, device=dev).bfloat16(), torch.empty(n, device=dev, dtype=torch.bfloat16))
            for _ in range(16)]
    return [lambda a=a, b=b: b.copy_(a) for a, b in bufs], 2 * nbytes, "byte"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", required=True, choices=sorted(CASES))
    ap.add_argument("--reps", type=int, default=50)
    ap.add_argument("--sets", type=int, default=4)
    ap.add_argument("--graph", action="store_true")
    ap.add_argument("--warm-ms", type=float, default=300.0, help="busy time before timing (clock ramp-up)")
    ap.add_argument("--cpu", action="store_true", help="also time the call on the host CPU (DiT cases)")
    a = ap.parse_args()
    dev = torch.device("cuda:0")
    kind, x, B = CASES[a.case]
    if kind == "dit":
        fns, work, unit = dit_case(x, B, a.sets, dev)
    elif kind in ("prologue", "gate"):
        fns, work, unit = elementwise_case(kind, x, B, a.sets, dev)
    elif kind in ("layer", "layer_sep"):
        fns, work, unit = layer_case(x, B, a.sets, dev, fused=(kind == "layer"))
    elif kind == "prefill":
        fns, work, unit = prefill_case(x, a.sets, dev)
    elif kind == "linear":
        fns, work, unit = linear_case(x, B, a.sets, dev)
    elif kind == "decode":
        fns, work, unit = decode_case(x, a.sets, dev, kv_stable=(B == "kv_stable"))
    elif kind == "block":
        fns, work, unit = block_case(x, B, a.sets, dev)
    elif kind == "grouped":
        fns, work, unit = grouped_case(x, B, a.sets, dev)
    else:
        fns, work, unit = calib_case(x, a.sets, dev)
    for f in fns:
        f()
    torch.cuda.synchronize()
    seq = [fns[i % len(fns)] for i in range(a.reps)]
    run = lambda: [f() for f in seq]
    if a.graph:
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            run()
        torch.cuda.current_stream().wait_stream(st)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            run()
        run = gr.replay
        run()
    torch.cuda.synchronize()
    import time
    t_end = time.perf_counter() + a.warm_ms / 1e3
    while time.perf_counter() < t_end:
        run()
        torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    run()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / a.reps
    rate = work / (us * 1e-6) / (1e12 if unit == "flop" else 1e9)
    rec = {"case": a.case, "kind": kind, "shape": _shape(kind, x, B), "graph": a.graph, "reps": a.reps,
           "us_per_call": round(us, 3), f"{unit}s_per_call": work,
           ("TFLOP/s" if unit == "flop" else "GB/s"): round(rate, 2)}
    peak_key = "bf16_tflops" if unit == "flop" else "hbm_gbs"
    peak = _peaks().get(peak_key)
    if peak:
        rec["frac_of_measured_peak"] = round(rate / peak, 4)
    if a.cpu and kind in ("dit", "layer", "layer_sep"):
        rec["cpu"] = _cpu_dit(x, B)
    rec["device_error"] = ops.device_error()
    print(json.dumps(rec))


def _shape(kind, x, B):
    if kind in ("dit", "layer", "layer_sep", "prologue", "gate"):
        return {"B": B, "H": x.H, "hd": x.hd, "L": x.L, "text_keys": x.Tb, "speaker_keys": x.Sp}
    if kind == "linear":
        return {"M": x[0], "N": x[1], "K": x[2], "impl": B}
    if kind in ("decode", "prefill", "block", "grouped"):
        s = W.C3
        d = {"T": x, "nq": s.nq, "nkv": s.nkv, "hd": s.hd}
        if kind == "block":
            d["hidden"] = B
        if kind == "grouped":
            d["requests"] = B
        return d
    return {"bytes": x}


def _peaks() -> dict:
    import os
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return {k: float(d[k]) for k in ("bf16_tflops", "hbm_gbs") if k in d}
    except (OSError, ValueError, KeyError):
        return {}


def _cpu_dit(shape, B) -> dict:
    """The same attention call on the host CPU: torch's scaled_dot_product_attention in fp32 with all host
    threads (the reference's own op, engine/fused.py:295, ctx keys copied per CFG row as the reference
    does), median of 3 runs."""
    import os
    import time

    torch.set_num_threads(os.cpu_count())
    g = torch.Generator().manual_seed(0)
    H, hd, L, S = shape.H, shape.hd, shape.L, shape.S
    q = torch.randn(B, H, L, hd, generator=g)
    k = torch.randn(B, H, L + S, hd, generator=g)
    v = torch.randn(B, H, L + S, hd, generator=g)
    mask = torch.zeros(B, 1, 1, L + S)
    times = []
    for _ in range(3):
        t0 = time.perf_counter()
        torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=mask)
        times.append(time.perf_counter() - t0)
    t = sorted(times)[1]
    return {"us_per_call": round(t * 1e6, 1), "TFLOP/s": round(shape.flops(B) / t / 1e12, 4), "cores": os.cpu_count()}


if __name__ == "__main__":
    main()
