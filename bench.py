"""Benchmark: Llama-3-8B-shaped decoder layer, all linear projections, GGUF-quantized.

Workload (the headline: the 8B-shaped layer at decode batch M): q/k/v fused 4096->6144, o 4096->4096, gate and up
4096->14336 each (Q4_K), down 14336->4096 (Q6_K); decode batch M (default 1),
f32 activations N(0,1), seeded random-init weights (synthetic data generated on
the device).  One step = one pass of the five projections, each its own
ocl_q_linear call (activation split + fused dequant-GEMV), in the order a
decoder layer runs them.  The step is captured once per weight copy in a CUDA
graph; weights rotate over enough distinct copies (>= 4x the 126 MB L2) that
every step streams its weights from HBM.

metric: algorithmic bytes (quantized weights + f32 activations in + outputs out)
of the layer / time, GB/s.  With --gpus N (torchrun), by default the layer is
split over the N GPUs (tensor parallel, strong scaling: the total work is fixed):
q/k/v, gate, up by output rows, o and down by input columns with their outputs
summed over ranks inside the GEMV (NVLink peer memory; NCCL with --nccl).
--mode replicas instead runs the whole layer on every GPU on its own decode
batch (no exchange step; weak scaling); at N > 1 the replica figure is also
reported beside the headline.  The 70B-shaped layer is always timed tensor
parallel over the N GPUs.

--impl reference times the reference's CPU algorithm (the C restatement in
oracle/: GGUF dequant + sequential-k f32 linear_out_by_in) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

HIDDEN, QKV, FFN = 4096, 6144, 14336
Q4_K, Q6_K = 12, 14
# (name, ggml type, out_features, in_features, split): "col" = split rows, "row" = split K
LAYER = [
    ("qkv", Q4_K, QKV, HIDDEN, "col"),
    ("o", Q4_K, HIDDEN, HIDDEN, "row"),
    ("gate", Q4_K, FFN, HIDDEN, "col"),
    ("up", Q4_K, FFN, HIDDEN, "col"),
    ("down", Q6_K, HIDDEN, FFN, "row"),
]
BLOCK = {Q4_K: (256, 144), Q6_K: (256, 210), 8: (32, 34)}
L2_BYTES = 126 * 2**20
METRIC = "Q4_K/Q6_K GEMV HBM GB/s (% of 8 TB/s); 8B-shape decode tok/s @1/2/4/8"
WORKLOAD = "llama3-8b-shape decoder layer, all linear projections (qkv/o/gate/up Q4_K, down Q6_K)"
KERNELS_PER_CALL = 2  # activation split + GEMV


def wbytes(t, n, k):
    e, b = BLOCK[t]
    return n * (k // e) * b


def proj_bytes(t, n, k, m):
    return wbytes(t, n, k) + 4 * m * k + 4 * m * n


def layer_alg_bytes(m):
    """Algorithmic bytes of one layer pass (whole job): weights + x in + y out."""
    return sum(proj_bytes(t, n, k, m) for _, t, n, k, _ in LAYER)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profile_traffic(kernel_key):
    """Per-launch DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of a
    committed ncu capture, from profiles/dram_traffic.json (None if absent)."""
    f = ROOT / "profiles" / "dram_traffic.json"
    if not f.exists():
        return None
    entry = json.loads(f.read_text()).get(kernel_key)
    return None if entry is None else int(entry["dram_bytes_per_launch"])


class Clocks:
    """nvidia-smi sampler running across the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.1)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        rows = [r.split(", ") for r in out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        mx = float(rows[-1][2])

        def pw(r):
            try:
                return float(r[3])
            except ValueError:
                return 0.0
        loaded = [s for s, r in zip(sm, rows) if pw(r) > 250.0] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.strip() == "Active"})
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# reference arm / CPU baseline (oracle/ -- the reference's CPU algorithm)
# ---------------------------------------------------------------------------
def cpu_inputs(m, seed):
    from ocelotl_b200 import synth
    weights = [synth.quant_blocks(t, n, k, seed, f"cpu.{name}").numpy() for name, t, n, k, _ in LAYER]
    xs = {name: synth.activations(m, k, seed, f"cpu.x.{name}").numpy() for name, t, n, k, _ in LAYER}
    return weights, xs


def cpu_layer_pass(oracle, weights, xs, m, threads, avx2=False):
    t0 = time.perf_counter()
    for (name, t, n, k, _), blocks in zip(LAYER, weights):
        oracle.q_linear(t, blocks, xs[name], m, k, n, threads=threads, avx2=avx2)
    return time.perf_counter() - t0


def has_avx2():
    import oracle
    return bool(oracle.lib().orc_has_avx2())


def host_info():
    model = ""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"nproc": os.cpu_count(), "cpu": model}


def cpu_baseline(m, seed, budget_s=10.0):
    """Reference CPU path, one thread (the reference's dispatch is serial for rows < 32),
    in both of its forms: the scalar linear_out_by_in and the AVX2 tile
    (crates/kernels/src/cpu_avx2.rs:58-253), the reference's fastest CPU mode."""
    import oracle
    oracle.build()
    weights, xs = cpu_inputs(m, seed)

    def timed(avx2):
        passes, spent = 0, 0.0
        while spent < budget_s / 2 and passes < 50:
            spent += cpu_layer_pass(oracle, weights, xs, m, 1, avx2=avx2)
            passes += 1
        return layer_alg_bytes(m) * passes / spent / 1e9, passes, spent
    scalar, sp, ss = timed(False)
    avx = has_avx2()
    fast, fp, fs = timed(True) if avx else (None, 0, 0.0)
    best = fast if fast is not None else scalar
    return {"value": round(best, 3), "unit": "GB/s", "cores": 1, "kind": "port", "host": host_info(),
            "isa": "avx2+fma" if avx else "scalar",
            "scalar_GBs": round(scalar, 3), "avx2_GBs": None if fast is None else round(fast, 3),
            "sample": f"full layer passes (5 projections, M={m}), 1 thread: GGUF dequant + linear_out_by_in restated "
                      f"in C (oracle/oracle.c); scalar sequential-k: {sp} passes in {ss:.1f}s; AVX2 tile: "
                      f"{fp} passes in {fs:.1f}s; value = the faster (AVX2 when the host has it)"}


def run_reference(args):
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    import oracle
    oracle.build()
    threads = os.cpu_count() or 1
    avx = has_avx2()
    weights, xs = cpu_inputs(args.rows, args.seed)
    for _ in range(args.warmup):
        cpu_layer_pass(oracle, weights, xs, args.rows, threads, avx2=avx)
    total = sum(cpu_layer_pass(oracle, weights, xs, args.rows, threads, avx2=avx) for _ in range(args.steps))
    gbs = layer_alg_bytes(args.rows) * args.steps / total / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * total / args.steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random-init GGUF blocks, N(0,1) activations)",
        "config": {"workload": WORKLOAD, "rows": args.rows, "host_threads": threads},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port", "host": host_info(),
                         "isa": "avx2+fma" if avx else "scalar",
                         "sample": f"each step = one full layer pass (M={args.rows}): GGUF dequant + "
                                   f"linear_out_by_in ({'AVX2 tile, cpu_avx2.rs' if avx else 'scalar sequential-k'}) "
                                   f"restated in C (oracle/), output features split over {threads} threads"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def graph_of(fn, be, torch):
    """Capture fn() into a CUDA graph on a side stream with the backend launching on it."""
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        be.use_current_stream()
        fn()  # warm: grows the context's scratch outside capture
        torch.cuda.current_stream().synchronize()
        with torch.cuda.graph(g, stream=s):
            be.use_current_stream()
            fn()
    be.set_stream(None)
    torch.cuda.synchronize()
    return g


def bf16_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["bf16_tflops"]), "measured burst cuBLAS bf16"
    return 1590.0, "fallback"


def run_prefill(be, ws, sh, args, torch):
    """Prefill: the 8B layer's five projections as bf16 tcgen05 GEMMs, M = 512 and 2048 tokens."""
    from ocelotl_b200 import synth
    out = {}
    peak, src = bf16_peak()
    for M in (512, 2048):
        xs = {nm: synth.activations(M, sh[nm][2], args.seed, f"px.{nm}", device="cuda",
                                    dtype=torch.bfloat16).contiguous() for nm in sh}
        ys = {nm: torch.empty(M, sh[nm][1], device="cuda", dtype=torch.bfloat16) for nm in sh}
        xin = {"qkv": "qkv", "o": "o", "gate": "gate", "up": "gate", "down": "down"}

        def layer():
            for nm in sh:
                be.gemm_bf16(xs[xin[nm]], ws[nm].weight, ys[nm])
        g = graph_of(layer, be, torch)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 20
        a.record()
        for _ in range(reps):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        us = 1e3 * a.elapsed_time(b) / reps
        flops = 2 * M * sum(n * k for _, n, k, _ in sh.values())
        tf = flops / (us * 1e-6) / 1e12
        out[str(M)] = {"layer_us": round(us, 1), "TFLOP/s": round(tf, 1), "frac": round(tf / peak, 4),
                       "flops": flops}
        del g
    out["peak"] = {"TFLOP/s": peak, "source": src}
    out["kernel"] = "qgemm_kernel: tcgen05.mma kind::f16, 256x128 CTA tile, weights dequantized to bf16 in smem"
    return out


def run_stack(be, args, torch, synth, dev, rank=0, tp=1, comm=None, group=None):
    """8B linear stack: 32 decoder layers' projections + Q6_K output head + Q8_0 embedding rows,
    per decode token.  Under TP (tp > 1): q/k/v and the gate/up pair split by output rows
    (the pair stays local: act is split the same way), o and down by input columns with
    the cross-rank sum fused into the GEMV, the head split by vocabulary rows with a
    cross-rank greedy pick (TPHead); the embedding table is replicated (one row per token)."""
    from ocelotl_b200.tp import TPHead, TPLinear, _range
    import torch.distributed as dist
    n_layers, vocab = 32, 128256
    shards = [(nm, t, n // tp, k, sp) if sp == "col" else (nm, t, n, k // tp, sp) for nm, t, n, k, sp in LAYER]
    sh = {nm: (t, n, k, sp) for nm, t, n, k, sp in shards}
    layers = []
    for li in range(n_layers):
        ws = {}
        for nm in ("qkv", "o", "down"):
            t, n, k, sp = sh[nm]
            ws[nm] = TPLinear(be, t, synth.quant_blocks(t, n, k, args.seed, f"stack.{li}.{nm}.r{rank}", device=dev),
                              n, k, "out" if (sp == "col" or tp == 1) else "in", comm=comm, group=group)
        # the model path runs gate and up as one gated pass (ocelotl_b200/model.py)
        t, n, k, _ = sh["gate"]
        g = be.upload_quant(t, synth.quant_blocks(t, n, k, args.seed, f"stack.{li}.gate.r{rank}", device=dev), n, k)
        u = be.upload_quant(t, synth.quant_blocks(t, n, k, args.seed, f"stack.{li}.up.r{rank}", device=dev), n, k)
        ws["gate_up"] = be.pair_gated(g, u)
        g.quant.free()
        u.quant.free()
        layers.append(ws)
    v0, v1 = _range(vocab, rank, tp)
    head = TPHead(be, Q6_K, synth.quant_blocks(Q6_K, v1 - v0, HIDDEN, args.seed, f"stack.head.r{rank}", device=dev),
                  v0, v1, HIDDEN, rank, tp, group=group)
    emb = be.upload_quant(8, synth.quant_blocks(8, vocab, HIDDEN, args.seed, "stack.emb", device=dev), vocab, HIDDEN)
    torch.cuda.synchronize()
    res = {"tp": tp}
    wbytes_total = n_layers * sum(wbytes(t, n, k) for _, t, n, k, _ in LAYER) + wbytes(Q6_K, vocab, HIDDEN)
    for m in (1, 8):
        ids = torch.randint(0, vocab, (m,), dtype=torch.int32, device=dev)
        h = torch.empty(m, HIDDEN, device=dev)
        xs = {nm: synth.activations(m, sh[nm][2], args.seed, f"stack.x.{nm}", device=dev) for nm in sh}
        ys = {nm: torch.empty(m, sh[nm][1], device=dev) for nm in sh}
        logits = torch.empty(m, v1 - v0, device=dev)
        next_ids = torch.empty(m, dtype=torch.int64, device=dev)
        act = torch.empty(m, sh["gate"][1], device=dev)

        def token(m=m, ids=ids, h=h, xs=xs, ys=ys, logits=logits, next_ids=next_ids, act=act):
            be.embed_rows(emb, ids, h)
            for ws in layers:
                ws["qkv"].forward(xs["qkv"], m, ys["qkv"])
                ws["o"].forward(xs["o"], m, ys["o"])
                be.linear_gated(ws["gate_up"], xs["gate"], m, act)
                ws["down"].forward(xs["down"], m, ys["down"])
            head.forward(h, m, logits, next_ids)
        token()  # communicators and scratch set up before capture
        torch.cuda.synchronize()
        if tp > 1:
            dist.barrier()
        g = graph_of(token, be, torch)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        if tp > 1:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 10
        a.record()
        for _ in range(reps):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        us = 1e3 * a.elapsed_time(b) / reps
        if tp > 1:
            t_ = torch.tensor([us])
            dist.all_reduce(t_, op=dist.ReduceOp.MAX)
            us = float(t_.item())
        alg = wbytes_total + m * wbytes(8, 1, HIDDEN)
        res[str(m)] = {"token_us": round(us, 1), "tok_s": round(m / (us * 1e-6), 1),
                       "GB/s": round(alg / (us * 1e-6) / 1e9, 1), "alg_bytes": alg}
        del g
    res["note"] = ("per decode step: Q8_0 embedding gather, 32 x (qkv, o, gated gate+up pass, down) quantized GEMVs "
                   "and the Q6_K output head + greedy argmax over the 128256 logits (vocab split over the ranks "
                   "under TP), one CUDA graph; linear layers only (no attention or norms)")
    del layers, head, emb
    torch.cuda.synchronize()
    return res


LAYER_70B = [  # hidden 8192, GQA kv 1024 (q 8192 + k 1024 + v 1024), ffn 28672
    ("qkv", Q4_K, 10240, 8192, "col"),
    ("o", Q4_K, 8192, 8192, "row"),
    ("gate", Q4_K, 28672, 8192, "col"),
    ("up", Q4_K, 28672, 8192, "col"),
    ("down", Q6_K, 8192, 28672, "row"),
]


def run_tp70b(be, args, torch, synth, dev, rank, tp, comm, group):
    """70B-shaped decoder stack's projections under tensor parallelism, per decode token:
    80 distinct layers (43.3 GB of weights over the TP ranks) in one CUDA graph, so every
    token streams every layer's weights from HBM once; nothing is extrapolated."""
    from ocelotl_b200.tp import TPLinear
    import torch.distributed as dist
    n_layers = args.layers_70b
    shards = [(nm, t, n // tp, k, sp) if sp == "col" else (nm, t, n, k // tp, sp) for nm, t, n, k, sp in LAYER_70B]
    per_gpu = sum(wbytes(t, n, k) for _, t, n, k, _ in shards)
    layers = []
    for li in range(n_layers):
        layers.append({nm: TPLinear(be, t, synth.quant_blocks(t, n, k, args.seed, f"70b.{nm}.l{li}.r{rank}",
                                                              device=dev),
                                    n, k, "out" if sp == "col" else "in", comm=comm, group=group)
                       for nm, t, n, k, sp in shards})
    torch.cuda.synchronize()
    total = sum(wbytes(t, n, k) for _, t, n, k, _ in LAYER_70B)
    peak, _ = peaks()
    out = {"layers": n_layers, "per_gpu_weight_bytes_per_layer": per_gpu, "layer_weight_bytes": total,
           "token_weight_bytes": n_layers * total}
    xin = {"qkv": "qkv", "o": "o", "gate": "gate", "up": "gate", "down": "down"}
    for m in (1, 16):
        xs = {nm: synth.activations(m, k, args.seed, f"70b.x.{nm}.r{rank}", device=dev) for nm, t, n, k, _ in shards}
        ys = {nm: torch.empty(m, n, device=dev) for nm, t, n, k, _ in shards}

        def token(m=m, xs=xs, ys=ys):
            for L in layers:
                for nm, *_ in shards:
                    L[nm].forward(xs[xin[nm]], m, ys[nm])
        token()  # communicators and scratch set up before capture
        torch.cuda.synchronize()
        if tp > 1:
            dist.barrier()
        g = graph_of(token, be, torch)
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
        if tp > 1:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 5
        a.record()
        for _ in range(reps):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        us = 1e3 * a.elapsed_time(b) / reps
        if tp > 1:
            t_ = torch.tensor([us])
            dist.all_reduce(t_, op=dist.ReduceOp.MAX)
            us = float(t_.item())
        roof = n_layers * per_gpu / (peak * 1e9) * 1e6
        out[str(m)] = {"token_us": round(us, 1), "tok_s": round(m / (us * 1e-6), 1),
                       "layer_us": round(us / n_layers, 2),
                       "GB/s": round(n_layers * total / (us * 1e-6) / 1e9, 1),
                       "roofline_token_us_per_gpu": round(roof, 1), "frac": round(roof / us, 4)}
        del g
    del layers
    torch.cuda.synchronize()
    return out


def time_graphs(gs, n_it, torch):
    for i in range(3):
        gs[i % len(gs)].replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(n_it):
        gs[i % len(gs)].replay()
    b.record()
    torch.cuda.synchronize()
    return 1e3 * a.elapsed_time(b) / n_it


def run_replicas(be, args, torch, synth, dev, rank, world):
    """Every GPU runs the whole 8B layer on its own decode batch (no exchange
    step): value = all GPUs' algorithmic bytes / max-over-ranks time (weak scaling)."""
    import torch.distributed as dist
    m = args.rows
    layer_w = sum(wbytes(t, n, k) for _, t, n, k, _ in LAYER)
    copies = max(2, -(-4 * L2_BYTES // layer_w))
    weights = [{nm: be.upload_quant(t, synth.quant_blocks(t, n, k, args.seed, f"rep.{nm}.r{rank}.c{c}", device=dev),
                                    n, k) for nm, t, n, k, _ in LAYER} for c in range(copies)]
    xs = {nm: synth.activations(m, k, args.seed, f"rep.x.{nm}.r{rank}", device=dev) for nm, t, n, k, _ in LAYER}
    ys = {nm: torch.empty(m, n, device=dev) for nm, t, n, k, _ in LAYER}
    xin = {"qkv": "qkv", "o": "o", "gate": "gate", "up": "gate", "down": "down"}
    gs = [graph_of(lambda c=c: [be.linear_dev(weights[c][nm], xs[xin[nm]], m, ys[nm]) for nm, *_ in LAYER],
                   be, torch) for c in range(copies)]
    for i in range(3):
        gs[i % copies].replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(args.steps):
        gs[i % copies].replay()
    b.record()
    torch.cuda.synchronize()
    us = 1e3 * a.elapsed_time(b) / args.steps
    if world > 1:
        t_ = torch.tensor([us])
        dist.all_reduce(t_, op=dist.ReduceOp.MAX)
        us = float(t_.item())
    del gs, weights
    torch.cuda.synchronize()
    return {"value": round(world * layer_alg_bytes(m) / (us * 1e-6) / 1e9, 2), "unit": "GB/s", "layer_us": round(us, 3),
            "decode_tok_s": round(world * m / (us * 1e-6), 1), "scaling": "weak",
            "note": f"{world} independent full layers, one per GPU, max-over-ranks time"}


SINGLE_GEMVS = [  # (key, type, out_features, in_features)
    ("q4k_4096x4096", Q4_K, 4096, 4096),     # the single Q4_K dequant + matvec case
    ("q4k_14336x4096", Q4_K, 14336, 4096),   # the 8B gate / up shape
    ("q4k_4096x14336", Q4_K, 4096, 14336),   # Q4_K with the down projection's long K
    ("q6k_4096x14336", Q6_K, 4096, 14336),   # the 8B down projection
]


def run_single_gemvs(be, args, torch, synth, dev, peak):
    """Back-to-back calls of one GEMV shape at M = 1 over distinct weight copies
    (>= 4x L2 together, so every call streams from HBM), in a CUDA graph."""
    out = {}
    for key, t, n, k in SINGLE_GEMVS:
        copies = max(4, -(-4 * L2_BYTES // wbytes(t, n, k)))
        ws = [be.upload_quant(t, synth.quant_blocks(t, n, k, args.seed, f"single.{key}.{c}", device=dev), n, k)
              for c in range(copies)]
        x = synth.activations(1, k, args.seed, f"single.x.{key}", device=dev)
        y = torch.empty(1, n, device=dev)
        g = graph_of(lambda: [be.linear_dev(w, x, 1, y) for w in ws], be, torch)
        us = time_graphs([g], max(10, args.steps // 10), torch) / copies
        b = proj_bytes(t, n, k, 1)
        gbs = b / (us * 1e-6) / 1e9
        out[key] = {"us": round(us, 3), "GB/s": round(gbs, 1), "frac": round(gbs / peak, 4), "bytes": b,
                    "copies": copies}
        del g
        for w in ws:
            w.quant.free()
    torch.cuda.synchronize()
    return out


def run_fused_mlp(be, weights, xs, sh, m, copies, args, torch, dev):
    """The same layer with gate and up as one gated pass over an interleaved
    pair (one GEMV launch streaming both, act = silu(gate) * up)."""
    pairs = [be.pair_gated(weights[c]["gate"].weight, weights[c]["up"].weight) for c in range(copies)]
    n_ffn = sh["gate"][1]
    act = torch.empty(m, n_ffn, device=dev)
    ys = {nm: torch.empty(m, sh[nm][1], device=dev) for nm in ("qkv", "o", "down")}

    def step(c):
        w = weights[c]
        be.linear_dev(w["qkv"].weight, xs["qkv"], m, ys["qkv"])
        be.linear_dev(w["o"].weight, xs["o"], m, ys["o"])
        be.linear_gated(pairs[c], xs["gate"], m, act)
        be.linear_dev(w["down"].weight, xs["down"], m, ys["down"])
    gs = [graph_of(lambda c=c: step(c), be, torch) for c in range(copies)]
    us = time_graphs(gs, max(20, args.steps), torch)
    reps = 2 * copies
    g1 = graph_of(lambda: [be.linear_gated(pairs[r % copies], xs["gate"], m, act) for r in range(reps)], be, torch)
    us_gu = time_graphs([g1], max(3, args.steps // 20), torch) / reps
    t, n, k, _ = sh["gate"]
    gu_bytes = 2 * wbytes(t, n, k) + 4 * m * k + 4 * m * n
    del gs, g1
    for p in pairs:
        p.quant.free()
    return {"layer_us": round(us, 3), "GB/s": round(layer_alg_bytes(m) / (us * 1e-6) / 1e9, 1),
            "decode_tok_s_layer": round(m / (us * 1e-6), 1),
            "gate_up_us": round(us_gu, 3), "gate_up_GB/s": round(gu_bytes / (us_gu * 1e-6) / 1e9, 1),
            "gpu_launches_per_step": KERNELS_PER_CALL * 4,
            "note": "qkv, o, gated(gate+up -> silu(gate)*up), down; GB/s over the same algorithmic bytes as the "
                    "5-projection layer"}


def run_ocelotl(args):
    import torch
    import torch.distributed as dist

    from ocelotl_b200 import synth
    from ocelotl_b200.backend import CudaKernelBackend
    from ocelotl_b200.build import build
    from ocelotl_b200.tp import TPComm, TPLinear

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local if world > 1 else 0)
    dev = torch.device("cuda", torch.cuda.current_device())
    if world > 1:
        import datetime
        # The default group is gloo (host-side barriers and the max-over-ranks
        # timing); an NCCL group is created only for the tensor-parallel steps.
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=180))
    if rank == 0:
        build()
    if world > 1:
        dist.barrier()
    be = CudaKernelBackend(dev.index)
    m = args.rows
    # replicas: every GPU runs the whole layer on its own decode batch (the 8B
    # layer fits one GPU many times over; no exchange step), weak scaling.
    # tp: the layer split over the GPUs (o/down sum over ranks), strong scaling.
    tp = world if args.mode == "tp" else 1
    replicas = world // tp

    shards = [(name, t, n // tp, k, sp) if sp == "col" else (name, t, n, k // tp, sp) for name, t, n, k, sp in LAYER]
    sh = {name: (t, n, k, sp) for name, t, n, k, sp in shards}
    rank_wbytes = sum(wbytes(t, n, k) for _, t, n, k, _ in shards)
    copies = max(2, -(-4 * L2_BYTES // rank_wbytes))
    # row-split layers sum over ranks inside the GEMV (peer memory); NCCL with --nccl
    comm = TPComm(be, rank, world, max_elems=16 * 8192) if (world > 1 and not args.nccl) else None
    layer_comm = comm if tp > 1 else None
    nccl_group = [dist.new_group(backend="nccl")] if tp > 1 else [None]

    def nccl():
        if nccl_group[0] is None:
            nccl_group[0] = dist.new_group(backend="nccl")
        return nccl_group[0]
    weights = []
    for c in range(copies):
        ws = {}
        for name, t, n, k, sp in shards:
            # this rank's shard, generated in place (same distribution as a sharded full weight)
            blocks = synth.quant_blocks(t, n, k, args.seed, f"{name}.r{rank}.c{c}", device=dev)
            # a replica's layer is whole: no split, no cross-rank sum
            ws[name] = TPLinear(be, t, blocks, n, k, "out" if (sp == "col" or tp == 1) else "in", comm=layer_comm,
                                group=nccl_group[0])
            del blocks
        weights.append(ws)
    torch.cuda.synchronize()
    xs = {name: synth.activations(m, k, args.seed, f"x.{name}.r{rank}", device=dev).contiguous()
          for name, t, n, k, _ in shards}
    ys = {name: torch.empty(m, n, device=dev, dtype=torch.float32) for name, t, n, k, _ in shards}
    xin = {"qkv": "qkv", "o": "o", "gate": "gate", "up": "gate", "down": "down"}

    def step(c):
        ws = weights[c]
        for name, t, n, k, sp in shards:
            ws[name].forward(xs[xin[name]], m, ys[name])

    # ---- device-resident timing: one graph per weight copy --------------------
    if tp > 1:
        for c in range(copies):  # NCCL communicators and buffers set up before capture
            step(c)
        torch.cuda.synchronize()
        dist.barrier()
    graphs = [graph_of(lambda c=c: step(c), be, torch) for c in range(copies)]
    run = lambda i: graphs[i % copies].replay()  # noqa: E731
    for i in range(args.warmup):
        run(i)
    torch.cuda.synchronize()
    clocks = Clocks(dev.index)
    clocks.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for i in range(args.steps):
        run(args.warmup + i)
    ev1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t_ = torch.tensor([ms])
        dist.all_reduce(t_, op=dist.ReduceOp.MAX)
        ms = float(t_.item())
    ms_step = ms / args.steps
    # spread of single steps, in a separate pass (an event between steps breaks
    # the overlap of consecutive graphs, so it would slow the timed region)
    n_dist = min(args.steps, 200)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(n_dist + 1)]
    evs[0].record()
    for i in range(n_dist):
        run(i)
        evs[i + 1].record()
    torch.cuda.synchronize()
    step_us = sorted(1e3 * evs[i].elapsed_time(evs[i + 1]) for i in range(n_dist))
    pct = lambda q: round(step_us[min(len(step_us) - 1, int(q * len(step_us)))], 3)  # noqa: E731
    gbs = replicas * layer_alg_bytes(m) / (ms_step * 1e-3) / 1e9

    # ---- per-projection call time (split + GEMV), graphs of back-to-back calls
    proj = {}
    reps = 2 * copies
    for name, t, n, k, sp in shards:
        g = graph_of(lambda name=name: [be.linear_dev(weights[r % copies][name].weight, xs[xin[name]], m, ys[name])
                                        for r in range(reps)], be, torch)
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        it = max(3, args.steps // 20)
        a.record()
        for _ in range(it):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        us = 1e3 * a.elapsed_time(b) / (it * reps)
        pb = proj_bytes(t, n, k, m)
        proj[name] = {"us": round(us, 3), "GB/s": round(pb / (us * 1e-6) / 1e9, 1), "bytes": pb,
                      "type": "Q4_K" if t == Q4_K else "Q6_K"}
    # dominant kernel: the Q4_K GEMV (4 of the 5 calls, ~69% of the bytes); its
    # roofline is quoted on its largest launch, the gate projection
    q4 = [p for p in proj if proj[p]["type"] == "Q4_K"]
    q4_gbs = sum(proj[p]["bytes"] for p in q4) / (sum(proj[p]["us"] for p in q4) * 1e-6) / 1e9
    ach = proj["gate"]["GB/s"]
    peak, peak_kind = peaks()
    roofline = {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4),
                "traffic": profile_traffic("q4k_gate") if (tp == 1 and m == 1) else None,
                "kernel": f"gemv_kernel<Q4_K> (+ its activation split) on gate {sh['gate'][1]}x{sh['gate'][2]}, "
                          f"M={m}; per launch {proj['gate']['bytes']} algorithmic bytes",
                "q4k_all_calls_GBs": round(q4_gbs, 1),
                "peak_source": "measured hbm_gbs (MEASURED_PEAKS.json)" if peak_kind == "measured"
                else "fallback 6.65 TB/s"}

    # ---- end to end through the C ABI with host buffers ----------------------
    pinned_x = {name: xs[name].cpu().pin_memory() for name in xs}
    pinned_y = {name: torch.empty(m * sh[name][1], dtype=torch.float32).pin_memory() for name in ys}
    h2d = replicas * sum(pinned_x[nm].numel() * 4 for nm in ("qkv", "o", "gate", "down"))
    d2h = replicas * sum(pinned_y[nm].numel() * 4 for nm in pinned_y)

    def e2e_step(i):
        ws = weights[i % copies]
        for name, t, n, k, sp in shards:
            be.linear_out_by_in(pinned_x[xin[name]].numpy(), m, k, ws[name].weight, n, None,
                                pinned_y[name].numpy())
            if sp == "row" and tp > 1:
                y = pinned_y[name].to(dev)
                dist.all_reduce(y, group=nccl_group[0])
                pinned_y[name].copy_(y.cpu())

    for i in range(max(3, args.warmup)):
        e2e_step(i)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(args.steps):
        e2e_step(i)
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t_ = torch.tensor([e2e_s])
        dist.all_reduce(t_, op=dist.ReduceOp.MAX)
        e2e_s = float(t_.item())
    e2e_gbs = replicas * layer_alg_bytes(m) * args.steps / e2e_s / 1e9

    # ---- decode batch sweep (M = 1, 2, 4, 8, 16), graphs ----------------------
    sweep = {}
    if args.sweep and tp == 1:
        for mm in (1, 2, 4, 8, 16):
            xm = {nm: synth.activations(mm, sh[nm][2], args.seed, f"sx.{nm}", device=dev) for nm in sh}
            ym = {nm: torch.empty(mm, sh[nm][1], device=dev) for nm in sh}

            def sstep(c, mm=mm, xm=xm, ym=ym):
                for nm in sh:
                    be.linear_dev(weights[c][nm].weight, xm[xin[nm]], mm, ym[nm])
            gs = [graph_of(lambda c=c: sstep(c), be, torch) for c in range(copies)]
            for i in range(3):
                gs[i % copies].replay()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            n_it = max(20, args.steps)
            a.record()
            for i in range(n_it):
                gs[i % copies].replay()
            b.record()
            torch.cuda.synchronize()
            us = 1e3 * a.elapsed_time(b) / n_it
            sweep[str(mm)] = {"layer_us": round(us, 2), "GB/s": round(layer_alg_bytes(mm) / (us * 1e-6) / 1e9, 1),
                              "tok_s_layer": round(mm / (us * 1e-6), 1)}
            del gs

    errs_seen = {"bad_ids": 0, "wait_timeouts": 0}
    bad_sections = []

    def check(section):
        """Device errors of the section just timed; its figures are void if a wait gave up."""
        b, tmo = be.take_device_errors()
        errs_seen["bad_ids"] += b
        errs_seen["wait_timeouts"] += tmo
        if tmo:
            bad_sections.append(section)
        return tmo == 0
    layer_ok = check("layer")
    peak_gbs, _ = peaks()
    single = run_single_gemvs(be, args, torch, synth, dev, peak_gbs) if (args.single and tp == 1) else None
    if single is not None and not check("single_gemvs"):
        single = None
    fused = run_fused_mlp(be, weights, xs, sh, m, copies, args, torch, dev) if (args.fused_mlp and tp == 1) \
        else None
    tp70 = run_tp70b(be, args, torch, synth, dev, rank, world, comm, nccl() if world > 1 else None) \
        if args.tp70b else None
    prefill = run_prefill(be, weights[0], sh, args, torch) if (args.prefill and tp == 1) else None
    if tp70 is not None and not check("tp_70b_stack"):
        tp70 = {"error": "device waits timed out; figures void", "wait_timeouts": errs_seen["wait_timeouts"]}
    stack = run_stack(be, args, torch, synth, dev, rank, tp, layer_comm, nccl() if tp > 1 else None) \
        if args.stack else None
    reps = run_replicas(be, args, torch, synth, dev, rank, world) if (world > 1 and tp > 1 and args.replicas) \
        else None
    check("rest")
    errs = (errs_seen["bad_ids"], errs_seen["wait_timeouts"])
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(m, args.seed, budget_s=args.cpu_budget)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True,
            "scaling": "strong" if args.mode == "tp" else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init GGUF blocks generated on device, N(0,1) activations)",
            "config": {"workload": WORKLOAD, "rows": m,
                       "parallelism": f"tp{world}" if args.mode == "tp" else f"replicas{world}",
                       "l2": f"inputs larger than L2: weights rotate over {copies} distinct copies "
                             f"({copies * rank_wbytes / 1e6:.0f} MB per GPU, >= 4x the 126 MB L2)",
                       "alg_bytes_per_step": replicas * layer_alg_bytes(m),
                       "pct_of_8TBps": round(100 * gbs / 8000.0, 2),
                       "step": "CUDA graph of 5 ocl_q_linear calls" + ("" if tp == 1 else (
                           " + 2 NCCL all-reduces (o, down)" if args.nccl else
                           "; o and down sum over ranks inside the GEMV (ocl_q_linear_allreduce, NVLink peer memory)"))},
            "roofline": roofline,
            "projections": proj,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "path": "CudaKernelBackend.linear_out_by_in -> ocl_q_linear_host per projection (pinned host "
                            "x/y, read and written by the kernels in place over the host link; launches and a "
                            "stream sync inside every call)"},
            "gpu_launches": KERNELS_PER_CALL * len(LAYER) * args.steps,
            "device_errors": {"bad_ids": errs[0], "wait_timeouts": errs[1]},
            "clocks": clk,
            "layer_us": round(ms_step * 1e3, 3),
            "single_step_us_p10_p50_p90": [pct(0.1), pct(0.5), pct(0.9)],
            "decode_tok_s_layer": round(m / (ms_step * 1e-3), 1),
        }
        if sweep:
            line["m_sweep"] = sweep
        if prefill:
            line["prefill_gemm"] = prefill
        if fused:
            line["layer_fused_mlp"] = fused
        if tp70:
            line["tp_70b_stack"] = tp70
        if stack:
            line["linear_stack_8b"] = stack
        if single:
            line["single_gemv_m1"] = single
        if reps:
            line["replicas"] = reps
        if not layer_ok or bad_sections:
            # a bounded device wait gave up: outputs were left unwritten, so the
            # timings do not measure the work; report nothing as a value
            line["error"] = f"device waits timed out in {bad_sections}; values void"
            if not layer_ok:
                line["value"] = None
                line["e2e"]["value"] = None
        print(json.dumps(line), flush=True)
    if world > 1:
        # Leave without tearing the process group down: graphs captured with
        # NCCL work can block destroy_process_group at exit.
        del graphs
        torch.cuda.synchronize()
        dist.barrier()
        sys.stdout.flush()
        sys.stderr.flush()
        os._exit(0 if errs[1] == 0 else 1)
    return 0 if errs[1] == 0 else 1


def run_profile_case(args):
    """Small single-GPU cases for ncu captures (a few launches, a few hundred MB at most).

    gemv: 4 copies of one weight (> L2 together), 8 calls of `rows` activation rows (default 1).
    gemm: one weight, 3 prefill GEMMs of `rows` bf16 activations.
    --case-shape "type:n:k[:rows]" picks the matrix (default the gate projection).
    """
    import torch

    from ocelotl_b200 import synth
    from ocelotl_b200.backend import CudaKernelBackend
    from ocelotl_b200.build import build
    build()
    be = CudaKernelBackend(0)
    dev = torch.device("cuda", 0)
    f = [int(v) for v in args.case_shape.split(":")]
    t, n, k = f[:3]
    if args.case == "gemv":
        rows = f[3] if len(f) > 3 else 1
        ws = [be.upload_quant(t, synth.quant_blocks(t, n, k, 1, f"w{c}", device=dev), n, k) for c in range(4)]
        x = synth.activations(rows, k, 1, "x", device=dev)
        y = torch.empty(rows, n, device=dev)
        for i in range(8):
            be.linear_dev(ws[i % 4], x, rows, y)
    else:
        rows = f[3] if len(f) > 3 else 2048
        w = be.upload_quant(t, synth.quant_blocks(t, n, k, 1, "w", device=dev), n, k)
        x = synth.activations(rows, k, 1, "x", device=dev, dtype=torch.bfloat16).contiguous()
        for _ in range(3):
            be.gemm_bf16(x, w)
    torch.cuda.synchronize()
    errs = be.take_device_errors()
    print(json.dumps({"case": args.case, "shape": args.case_shape, "device_errors": list(errs)}))
    return 0 if errs == (0, 0) else 1


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ocelotl", choices=["ocelotl", "reference"])
    ap.add_argument("--rows", type=int, default=1, help="decode batch M (1..16)")
    ap.add_argument("--seed", type=int, default=0x0CE107)
    ap.add_argument("--sweep", type=int, default=1)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--mode", choices=["replicas", "tp"], default="tp",
                    help="N > 1: one layer split over the GPUs (strong scaling, default) or independent full layers "
                         "per GPU (weak scaling)")
    ap.add_argument("--replicas", type=int, default=1, help="N > 1 in tp mode: also time N independent replicas")
    ap.add_argument("--nccl", action="store_true", help="TP: NCCL all-reduce instead of the fused one")
    ap.add_argument("--tp70b", type=int, default=1, help="also time the 70B-shaped stack (TP = N)")
    ap.add_argument("--layers-70b", type=int, default=80, help="layers of the 70B-shaped stack")
    ap.add_argument("--prefill", type=int, default=1, help="also time the prefill GEMM (bf16 tcgen05, M = 512 / 2048)")
    ap.add_argument("--stack", type=int, default=1, help="also time the 8B linear stack per decode token")
    ap.add_argument("--fused-mlp", type=int, default=1,
                    help="also time the layer with gate+up as one fused gated pass (ocl_q_linear_gated)")
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--single", type=int, default=1, help="also time single GEMV shapes at M = 1")
    ap.add_argument("--case", choices=["gemv", "gemm"], help="run a small profiling case instead of the bench")
    ap.add_argument("--case-shape", default="12:14336:4096")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.case:
        return run_profile_case(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ocelotl(args)


if __name__ == "__main__":
    sys.exit(main())
