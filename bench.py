"""Benchmark of the W8A16 quantized linear layer on B200 (BASELINE.json metric).

Headline: the full Qwen3-0.6B decode-step projection
set -- 28 layers x {fused QKV 4096x1024, o 1024x2048, fused gate_up 6144x1024,
down 1024x3072} + lm_head 151936x1024 = 113 GEMMs, int8 weights with per-row
bf16 scales (~0.6 GB streamed per pass) -- at batch M in {1, 8, 32, 64}.  One
pass = the 113 GEMMs at every M, each M as one grouped persistent launch; one
timed step = ``passes_per_step`` passes back to back in one CUDA graph, sized
so that the timed steps last at least half a second.  Weights: random
N(0, 0.02), seeded, quantised on the GPU; activations N(0, 1) bf16, seeded per
rank (synthetic data -- no checkpoints).

``value``   algorithmic HBM bytes (int8 weights + bf16 scales + bf16 x + bf16 y)
            of all ranks / device time of the timed steps (max over ranks), GB/s.
``per_m``   per batch size: the grouped launch, and the same 113 GEMMs launched
            one by one in model order (``chain``: every launch a dependent one,
            programmatic dependent launch, one CUDA graph) -- the call pattern of
            a model forward through the drop-in op.
``e2e``     the same metric through the public API with host buffers: each step
            copies every GEMM input from pinned host memory and reads the lm_head
            logits back, inside the timed region; ``host_link`` times the same
            copies alone.
The default run also measures the other BASELINE configs, each as its own key:
``config0`` (one gate_proj-shaped linear, M = 1), ``prefill`` (config 2, the
28 layers' GEMMs at M in {512, 2048, 8192}, TFLOP/s, with and without the
SwiGLU epilogue), ``w4`` (config 3, 4-bit asymmetric group-128) and ``llama``
(config 4, Llama-3.2-3B shapes at M in {1, 64, 256}; vocab-sharded lm_head
with an NCCL all-gather when N > 1).  ``--workload`` runs one of them alone.

``--impl reference`` times the reference's CPU path (dequantise-then-matmul,
restated in ``oracle/``) on all host cores for the same metric.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

QWEN_LAYER = [("qkv", 4096, 1024), ("o", 1024, 2048), ("gate_up", 6144, 1024), ("down", 1024, 3072)]
QWEN_HEAD = ("lm_head", 151936, 1024)
LLAMA_LAYER = [("qkv", 5120, 3072), ("o", 3072, 3072), ("gate_up", 16384, 3072), ("down", 3072, 8192)]
LLAMA_HEAD = ("lm_head", 128256, 3072)
LAYERS = 28


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def profiled_traffic(kernel_key: str):
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get(kernel_key)
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ CPU paths
def cpu_path_sample(workload_shapes, m_list, fmt="w8_row", budget_s=10.0, seed=0):
    """The reference's CPU path (dequantise, fp32 matmul, bf16 cast -- restated in
    ``oracle/``) over a bounded sample of the workload: every GEMM shape at every
    batch size, each on a row sample.  Returns (GB/s of algorithmic bytes,
    seconds, description, threads)."""
    import numpy as np
    from threadpoolctl import threadpool_info

    from oracle import quant_oracle as O
    rng = np.random.default_rng(seed)
    done_bytes, t_total, calls = 0, 0.0, 0
    prepared = []
    for name, n, k in workload_shapes:
        rows = min(n, 8192)            # bounded sample of rows per GEMM
        w = (rng.standard_normal((rows, k), dtype=np.float32) * 0.02)
        if fmt == "w4_asym":
            d, sc, z = O.quantize_int4_asym(w, 128)
            deq = (lambda d=d, sc=sc, z=z: O.dequantize_int4_asym(d, sc, z, 128))
            wbytes = rows * k // 2 + 4 * rows * (k // 128)
        else:
            q, sc = O.quantize_int8_rowwise(w)
            deq = (lambda q=q, sc=sc: O.dequantize_int8_rowwise(q, sc))
            wbytes = rows * k + 2 * rows
        for m in m_list:
            x = O.bf16_round(rng.standard_normal((m, k), dtype=np.float32))
            prepared.append((deq, x, wbytes + 2 * m * k + 2 * m * rows))
    start = time.perf_counter()
    while time.perf_counter() - start < budget_s:
        for deq, x, nbytes in prepared:
            t0 = time.perf_counter()
            O.linear(x, deq())
            t_total += time.perf_counter() - t0
            done_bytes += nbytes
            calls += 1
            if time.perf_counter() - start >= budget_s:
                break
    threads = max((i.get("num_threads", 1) for i in threadpool_info()), default=1)
    desc = (f"M in {m_list}: {calls} GEMM calls over row samples (<=8192 rows) of "
            f"{', '.join(name for name, _, _ in workload_shapes)}; {fmt} dequantise + numpy/BLAS fp32 matmul + bf16 cast")
    return done_bytes / t_total / 1e9, t_total, desc, threads


def workload_of(args):
    """(GEMM shapes, batch sizes, weight format, description) of the decode workloads."""
    if args.workload == "llama":
        shapes, ms, fmt = LLAMA_LAYER + [LLAMA_HEAD], [1, 64, 256], "w8_row"
        desc = "llama-3.2-3b decode projection set (BASELINE config 4)"
    elif args.workload == "w4":
        shapes, ms, fmt = QWEN_LAYER + [QWEN_HEAD], [1, 16], "w4_asym"
        desc = "qwen3-0.6b decode projection set, W4A16 asym g128 (BASELINE config 3)"
    else:
        shapes, ms, fmt = QWEN_LAYER + [QWEN_HEAD], [1, 8, 32, 64], "w8_row"
        desc = "qwen3-0.6b decode projection set (BASELINE config 1)"
    if args.batch:
        ms = [int(v) for v in args.batch.split(",")]
    return shapes, ms, fmt, desc


def run_reference(args):
    """--impl reference: the reference's CPU path on the host cores (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    shapes, ms, fmt, wdesc = workload_of(args)
    per_step = max(2.0, min(20.0, 120.0 / max(1, args.steps + args.warmup)))
    vals = []
    # every host core, whatever the launcher set (torchrun exports OMP_NUM_THREADS=1)
    from threadpoolctl import threadpool_limits
    with threadpool_limits(limits=os.cpu_count()):
        for i in range(args.warmup + args.steps):
            v, _, desc, threads = cpu_path_sample(shapes, ms, fmt, budget_s=per_step, seed=i)
            if i >= args.warmup:
                vals.append(v)
    value = statistics.mean(vals)
    gpu_context = reference_gpu_context(args)
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(per_step * 1000, 1), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": wdesc, "batch_m": ms, "gpus_used": 0,
                       "path": "reference CPU path (dequantise + fp32 matmul + bf16 cast), bounded row samples"},
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": desc + f" ({per_step:.1f} s per step)"},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "gpu_context": gpu_context}
    print(json.dumps(line), flush=True)


def reference_gpu_context(args):
    """GPU context, not part of the CPU arm's value: the reference's own CUDA
    decode op (``learning/10_cuda_decode/warp_gemv.cu``, built unmodified by
    ``oracle/build_ref.py``) on this GPU, at config 0 and over the config 1
    projection set at M = 1 (its only batch size), launched one by one in model
    order and captured in a CUDA graph.  Weights are per-row int8 made with
    plain torch (scale = absmax/127 as f32 [N, 1], inverse of ones: the
    reference's calibrated format with group = K)."""
    try:
        import torch
        if not torch.cuda.is_available():
            return None
        from oracle import build_ref
        mod = build_ref.load()
    except Exception as e:            # noqa: BLE001 -- context only, never fatal
        return {"unavailable": f"{type(e).__name__}: {e}"}
    if mod is None:
        return {"unavailable": "the reference extension was not built (oracle/build_ref.py)"}
    device = torch.device("cuda", 0)
    gen = torch.Generator(device=device)

    def quant(n, k, seed):
        gen.manual_seed(seed)
        w = torch.randn(n, k, device=device, generator=gen) * 0.02
        s = w.abs().amax(1, keepdim=True) / 127
        s = torch.where(s == 0, torch.ones_like(s), s)
        q = torch.round(w / s).clamp(-127, 127).to(torch.int8)
        return q, s.float().contiguous()

    def graph_ms(fn, reps):
        fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        for _ in range(3):
            g.replay()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    out = {"kernel": "reference warp_gemv.cu projection<QUANT> (unmodified, sm_100, warps=4)"}
    # config 0: 64 weight copies cycled (larger than L2)
    k = 1024
    ones = torch.ones(k, device=device)
    ws = [quant(3072, k, 1000 + i) for i in range(64)]
    gen.manual_seed(0)
    x = torch.randn(k, device=device, generator=gen).to(torch.bfloat16)
    ms = graph_ms(lambda: [mod.project(x, q, s, ones, k, 4, False, False) for q, s in ws], 10) / 64
    nbytes = 3072 * k + 2 * 3072 + 2 * k + 2 * 3072
    out["config0"] = {"us": round(ms * 1e3, 3), "GB/s": round(nbytes / (ms * 1e-3) / 1e9, 1)}
    del ws
    # config 1 at M = 1: 28 layers + lm_head in model order
    items = []
    for li in range(LAYERS):
        for j, (name, n, kk) in enumerate(QWEN_LAYER):
            q, s = quant(n, kk, 1234 + li * 16 + j)
            items.append((q, s, torch.ones(kk, device=device), kk, name == "gate_up",
                          torch.randn(kk, device=device, generator=gen).to(torch.bfloat16)))
    q, s = quant(QWEN_HEAD[1], QWEN_HEAD[2], 4321)
    items.append((q, s, torch.ones(QWEN_HEAD[2], device=device), QWEN_HEAD[2], False,
                  torch.randn(QWEN_HEAD[2], device=device, generator=gen).to(torch.bfloat16)))
    ms = graph_ms(lambda: [mod.project(xx, qq, ss, inv, kk, 4, False, sw) for qq, ss, inv, kk, sw, xx in items], 5)
    nbytes = sum(qq.numel() + 2 * qq.shape[0] + 2 * kk + 2 * (qq.shape[0] // 2 if sw else qq.shape[0])
                 for qq, ss, inv, kk, sw, xx in items)
    out["config1_m1_chain"] = {"ms": round(ms, 4), "GB/s": round(nbytes / (ms * 1e-3) / 1e9, 1),
                               "gemms": len(items),
                               "bytes_note": "the per-row format's bytes (int8 weights + bf16 scales + x + y), "
                                             "the same count as the headline's"}
    return out


METRIC = "W8A16 GEMM HBM GB/s (decode M<=64) and TFLOP/s (prefill), Qwen3-0.6B shapes"


# ------------------------------------------------------------------ GPU paths
def init_dist(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        # NCCL prints its version banner on stdout when the communicator comes
        # up; send that to stderr so rank 0's stdout stays the one JSON line.
        # Every rank takes the same steps (init, then one barrier).
        import ctypes
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
            dist.barrier()
        finally:
            ctypes.CDLL(None).fflush(None)
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
        pg = dist
    return world, rank, local, pg


def quantize(kl, w, fmt):
    return kl.quantize_int4_asym(w, 128) if fmt == "w4_asym" else kl.quantize_int8_rowwise(w)


def build_weights(kl, shapes, layers, device, seed=1234, fmt="w8_row"):
    import torch
    gen = torch.Generator(device=device)
    weights = []
    for li in range(layers):
        for j, (name, n, k) in enumerate(shapes):
            gen.manual_seed(seed + li * 16 + j)
            w = torch.randn(n, k, device=device, generator=gen) * 0.02
            weights.append((f"{name}{li}", quantize(kl, w, fmt)))
            del w
    return weights


def capture(fn):
    import torch
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


def timed(graph, reps, warm=3):
    """Average device time (ms) of ``reps`` back-to-back replays, after ``warm``."""
    import torch
    for _ in range(warm):
        graph.replay()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        graph.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def max_over_ranks(v, dist, device):
    if dist is None:
        return v
    import torch
    t = torch.tensor([v], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


class DecodeSet:
    """One projection set (GEMMs of every layer + the lm_head) at each batch size:
    per-M activation buffers (views of one contiguous buffer per M), outputs,
    the grouped launch and the dependent chain."""

    def __init__(self, kl, weights, ms_list, device, seed):
        import torch
        self.kl, self.weights, self.ms_list = kl, weights, ms_list
        xg = torch.Generator(device=device)
        xg.manual_seed(seed)
        self.passes, self.x_flat = {}, {}
        for m in ms_list:
            total = sum(m * p.shape[1] for _, p in weights)
            flat = torch.randn(total, device=device, generator=xg).to(torch.bfloat16)
            self.x_flat[m] = flat
            items, off = [], 0
            for name, p in weights:
                n, k = p.shape
                x = flat[off: off + m * k].view(m, k)
                off += m * k
                items.append((name, p, x, torch.empty(m, n, device=device, dtype=torch.bfloat16)))
            self.passes[m] = items
        self.grouped = {m: kl.GroupedLinear([(x, p, y) for _, p, x, y in self.passes[m]]) for m in ms_list}
        for m in ms_list:              # eager warm-up (allocates the workspace before capture)
            self.run_grouped(m)
            self.run_chain(m)
        torch.cuda.synchronize()

    def run_grouped(self, m):
        self.grouped[m].run(pdl=True)

    def run_chain(self, m):
        for name, p, x, y in self.passes[m]:
            self.kl.quant_linear(x, p, out=y, pdl=True)

    def pass_bytes(self, m):
        # weights + their scales (and zeros) + activations in + outputs
        return sum(p.storage_bytes + 2 * x.numel() + 2 * y.numel() for _, p, x, y in self.passes[m])

    def per_m(self, hbm, reps, device, dist):
        out = {}
        for m in self.ms_list:
            gg, gc = capture(lambda m=m: self.run_grouped(m)), capture(lambda m=m: self.run_chain(m))
            t_g = max_over_ranks(timed(gg, reps), dist, device)
            t_c = max_over_ranks(timed(gc, reps), dist, device)
            del gg, gc
            b = self.pass_bytes(m)
            out[str(m)] = {"grouped_ms": round(t_g, 4), "grouped_GB/s": round(b / (t_g * 1e-3) / 1e9, 1),
                           "frac_hbm": round(b / (t_g * 1e-3) / 1e9 / hbm, 3),
                           "chain_ms": round(t_c, 4), "chain_GB/s": round(b / (t_c * 1e-3) / 1e9, 1),
                           "chain_frac_hbm": round(b / (t_c * 1e-3) / 1e9 / hbm, 3),
                           "tokens/s": round(m / (t_c * 1e-3), 1)}
        return out

    def head_alone(self, hbm, device):
        """The largest single GEMM (the lm_head) at the first batch size, graph-timed."""
        import torch
        name, p, x, y = self.passes[self.ms_list[0]][-1]
        g = capture(lambda: [self.kl.quant_linear(x, p, out=y, pdl=True) for _ in range(5)])
        ms = timed(g, 4) / 5
        del g
        m0 = self.ms_list[0]
        n, k = p.shape
        gbs = (p.storage_bytes + 2 * m0 * k + 2 * m0 * n) / (ms * 1e-3) / 1e9
        out = {"ms": round(ms, 4), "GB/s": round(gbs, 1), "frac": round(gbs / hbm, 3), "m": m0}
        # the same head with the top-8 selected in the GEMM's epilogue (no logits written)
        self.kl.lm_head_topk(x, p, 8)
        torch.cuda.synchronize()
        g = capture(lambda: [self.kl.lm_head_topk(x, p, 8) for _ in range(5)])
        out["top8_fused_ms"] = round(timed(g, 4) / 5, 4)
        del g
        return out


def sharded_head_section(kl, full, ms_list, x_of, world, rank, device, dist, steps, fmt="w8_row"):
    """Vocab-sharded lm_head: the shard GEMM + NCCL all-gather of the logits, and
    the top-8 alternative (shard GEMM with the candidates selected in its
    epilogue, all-gather of candidates, merge), each captured once and replayed;
    max over ranks.  Beside them, the same two on the whole head on one GPU
    (every rank runs it alone, no collective), the single-GPU time to beat."""
    import torch
    vocab = full.shape[0]
    lo, hi = kl.sharded_head.shard_bounds(vocab, world, rank)
    if fmt == "w4_asym":
        shard = kl.PackedInt4Asym(full.data[lo:hi].contiguous(), full.scales[lo:hi].contiguous(),
                                  full.zeros[lo:hi].contiguous(), full.group_size)
    else:
        shard = kl.RowwiseInt8(full.data[lo:hi].contiguous(), full.scales[lo:hi].contiguous())
    shead = kl.VocabShardedHead(shard, vocab)
    res = {"vocab": vocab, "ranks": world, "rows_per_rank": hi - lo, "per_m": {}}
    reps = max(5, steps)

    class _One:                          # a single rank without a process group
        @staticmethod
        def barrier():
            torch.cuda.synchronize()
    dist = dist if dist is not None else _One
    for m in ms_list:
        x = x_of(m)
        gathered = torch.empty(vocab, m, dtype=torch.bfloat16, device=device)
        for _ in range(3):
            shead(x, gathered=gathered)
        dist.barrier()
        sg = capture(lambda: shead(x, gathered=gathered))
        dist.barrier()
        t = max_over_ranks(timed(sg, reps), dist if world > 1 else None, device)
        del sg
        for _ in range(3):
            shead.topk(x, 8)
        dist.barrier()
        tg = capture(lambda: shead.topk(x, 8))
        dist.barrier()
        tk = max_over_ranks(timed(tg, reps), dist if world > 1 else None, device)
        del tg
        logits = torch.empty(m, vocab, dtype=torch.bfloat16, device=device)
        for _ in range(3):
            kl.quant_linear(x, full, out=logits)
            kl.lm_head_topk(x, full, 8)
        torch.cuda.synchronize()
        ug = capture(lambda: kl.quant_linear(x, full, out=logits))
        tu = max_over_ranks(timed(ug, reps), dist if world > 1 else None, device)
        del ug
        ugk = capture(lambda: kl.lm_head_topk(x, full, 8))
        tuk = max_over_ranks(timed(ugk, reps), dist if world > 1 else None, device)
        del ugk, logits
        res["per_m"][str(m)] = {"ms": round(t, 4), "allgather_bytes": vocab * m * 2,
                                "shard_weight_GB/s": round(shard.storage_bytes / (t * 1e-3) / 1e9, 1),
                                "top8_ms": round(tk, 4), "top8_gather_bytes": world * m * 8 * 8,
                                "one_gpu_ms": round(tu, 4), "one_gpu_top8_ms": round(tuk, 4)}
    return res


def bench_decode(args, kl, world, rank, local, dist):
    """Config 1 (or 4 with --workload llama, 3 with --workload w4): every
    projection of the decode step at each batch size M, the grouped launch per M
    as the timed step, the dependent chain per M alongside."""
    import torch
    device = torch.device("cuda", local)
    layer, head = (LLAMA_LAYER, LLAMA_HEAD) if args.workload == "llama" else (QWEN_LAYER, QWEN_HEAD)
    _, ms_list, fmt, workload_desc = workload_of(args)
    weights = build_weights(kl, layer, LAYERS, device, fmt=fmt)
    gen = torch.Generator(device=device)
    gen.manual_seed(4321)
    hw = torch.randn(head[1], head[2], device=device, generator=gen) * 0.02
    weights.append(("lm_head", quantize(kl, hw, fmt)))
    del hw
    torch.cuda.empty_cache()
    ds = DecodeSet(kl, weights, ms_list, device, 99 + rank)
    hbm, tf_burst, tf_sus, peak_kind = measured_peaks()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    # one pass = every M once; a timed step = `passes` passes in one graph, so
    # that the timed steps take at least half a second
    one = capture(lambda: [ds.run_grouped(m) for m in ms_list])
    t_pass = max_over_ranks(timed(one, 5), dist, device)
    del one
    passes = max(1, int(-(-500.0 // (args.steps * t_pass))))
    step_graph = capture(lambda: [ds.run_grouped(m) for _ in range(passes) for m in ms_list])
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        step_graph.replay()
    barrier()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        start.record()
        for _ in range(args.steps):
            step_graph.replay()
        stop.record()
        barrier()
    ms_step = max_over_ranks(start.elapsed_time(stop) / args.steps, dist, device)
    del step_graph
    step_bytes = passes * sum(ds.pass_bytes(m) for m in ms_list)
    value = world * step_bytes / (ms_step * 1e-3) / 1e9
    per_m = ds.per_m(hbm, max(5, args.steps // 2), device, dist)

    # ---- e2e through the public API with host buffers
    pinned = {m: torch.empty(ds.x_flat[m].shape, dtype=torch.bfloat16, pin_memory=True).copy_(ds.x_flat[m])
              for m in ms_list}
    head_out = {m: torch.empty(ds.passes[m][-1][3].shape, dtype=torch.bfloat16, pin_memory=True) for m in ms_list}
    h2d = passes * sum(t.numel() * 2 for t in pinned.values())
    d2h = passes * sum(t.numel() * 2 for t in head_out.values())
    per_m_graph = {m: capture(lambda m=m: ds.run_grouped(m)) for m in ms_list}

    # Copies run on their own streams so that the upload of one batch size's
    # activations and the download of another's logits overlap the GEMMs:
    # upload(M) -> step graph(M) -> download(M), with the next upload into a
    # buffer waiting for the graph that last read it, and the next graph
    # waiting for the download of the logits it overwrites.
    main = torch.cuda.current_stream(device)
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    read_done = {m: None for m in ms_list}      # graph(M) finished reading x_flat[M]
    out_done = {m: None for m in ms_list}       # download of M's logits finished

    def e2e_pass():
        for m in ms_list:
            with torch.cuda.stream(s_in):
                if read_done[m] is not None:
                    s_in.wait_event(read_done[m])
                ds.x_flat[m].copy_(pinned[m], non_blocking=True)
                up = torch.cuda.Event()
                up.record(s_in)
            main.wait_event(up)
            if out_done[m] is not None:
                main.wait_event(out_done[m])
            per_m_graph[m].replay()
            ran = torch.cuda.Event()
            ran.record(main)
            read_done[m] = ran
            with torch.cuda.stream(s_out):
                s_out.wait_event(ran)
                head_out[m].copy_(ds.passes[m][-1][3], non_blocking=True)
                down = torch.cuda.Event()
                down.record(s_out)
            out_done[m] = down

    def join():
        main.wait_stream(s_in)
        main.wait_stream(s_out)

    for _ in range(max(1, args.warmup)):
        e2e_pass()
    join()
    barrier()
    s2, t2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    s_in.wait_stream(main)
    s_out.wait_stream(main)
    for _ in range(args.steps * passes):
        e2e_pass()
    join()
    t2.record()
    barrier()
    e2e_ms = max_over_ranks(s2.elapsed_time(t2) / args.steps, dist, device)
    e2e_value = world * step_bytes / (e2e_ms * 1e-3) / 1e9

    # the same host copies alone (every rank at once), one direction at a time
    def copies(direction):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        a.record()
        for _ in range(passes):
            for m in ms_list:
                if direction == "h2d":
                    ds.x_flat[m].copy_(pinned[m], non_blocking=True)
                else:
                    head_out[m].copy_(ds.passes[m][-1][3], non_blocking=True)
        b.record()
        torch.cuda.synchronize()
        return max_over_ranks(a.elapsed_time(b), dist, device)

    copies("h2d")
    t_h2d, t_d2h = copies("h2d"), copies("d2h")
    host_link = {"h2d_ms_per_step": round(t_h2d, 4), "h2d_GB/s_per_rank": round(h2d / (t_h2d * 1e-3) / 1e9, 1),
                 "d2h_ms_per_step": round(t_d2h, 4), "d2h_GB/s_per_rank": round(d2h / (t_d2h * 1e-3) / 1e9, 1),
                 "copies_alone_ms": round(t_h2d + t_d2h, 4),
                 "note": "the step's host copies alone, every rank at once; e2e cannot beat the larger of the "
                         "copy time and the device time"}
    del per_m_graph

    head_alone = ds.head_alone(hbm, device)
    sharded = None
    if world > 1 or args.lm_head_shard:
        sharded = sharded_head_section(kl, ds.passes[ms_list[0]][-1][1], ms_list,
                                       lambda m: ds.passes[m][-1][2], world, rank, device, dist, args.steps, fmt)

    achieved = step_bytes / (ms_step * 1e-3) / 1e9
    result = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": workload_desc,
                   "batch_m": ms_list, "gemms_per_pass": len(ds.passes[ms_list[0]]), "passes_per_step": passes,
                   "bytes_per_step": step_bytes, "weights": ("4-bit asym, bf16 scale/zero per 128-group" if fmt == "w4_asym" else "int8 per-row bf16 scale")
                              + ", N(0,0.02) seeded",
                   "l2": "inputs larger than L2: each pass streams >=0.3 GB of weights, no flush needed",
                   "parallelism": f"replicas x{world}",
                   "launch": "one grouped tcgen05 launch per M (all GEMMs of the pass, independent), "
                             "passes_per_step passes per step in one CUDA graph"},
        "per_m": per_m,
        "roofline": {"bound": "hbm", "kernel": "tc_qgemm_kernel (the step's grouped launches)",
                     "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "peak_source": peak_kind,
                     "traffic": profiled_traffic(f"{args.workload}_step"),
                     "lm_head_alone": head_alone},
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e2e_ms, 4), "host_link": host_link},
        "lm_head_sharded": sharded,
        "gpu_launches": passes * len(ms_list) * args.steps,
        "clocks": clocks.summary(),
    }
    if args.workload == "decode" and not args.only_headline:
        del ds
        torch.cuda.empty_cache()
        qwen_w8 = weights[:-1]
        result["config0"] = section_config0(kl, device, hbm, dist)
        result["prefill"] = section_prefill(kl, qwen_w8, device, tf_burst, peak_kind, args, rank, world, dist)
        del weights, qwen_w8
        torch.cuda.empty_cache()
        result["w4"] = section_decode_other(kl, "w4", device, hbm, args, rank, world, dist)
        result["llama"] = section_decode_other(kl, "llama", device, hbm, args, rank, world, dist)
    return result


def section_config0(kl, device, hbm, dist):
    """one gate_proj-shaped linear (x bf16 [1, 1024], W
    [3072, 1024] ~ N(0, 0.02), per-row int8).  64 differently seeded copies of
    the weights (200 MB, larger than L2) are cycled, each call a dependent launch
    (programmatic dependent launch, one CUDA graph), on each kernel that takes
    the shape."""
    import torch
    n, k, copies = 3072, 1024, 64
    gen = torch.Generator(device=device)
    ws = []
    for i in range(copies):
        gen.manual_seed(1000 + i)
        ws.append(kl.quantize_int8_rowwise(torch.randn(n, k, device=device, generator=gen) * 0.02))
    gen.manual_seed(0)
    x = torch.randn(1, k, device=device, generator=gen).to(torch.bfloat16)
    y = torch.empty(1, n, device=device, dtype=torch.bfloat16)
    nbytes = n * k + 2 * n + 2 * k + 2 * n
    out = {"shape": [1, n, k], "bytes_per_call": nbytes, "l2": f"{copies} weight copies cycled ({copies * n * k >> 20} MiB)"}
    kernel_names = {None: "CUDA-core chain GEMV, full rows per CTA (kl_gemv_chain)",
                    "tc": "single-tile cluster tcgen05 (kl_tc_chain)", "persistent": "stream-K tcgen05 (tc_qgemm)",
                    "simt": "CUDA-core GEMV (gemv_vec)"}
    for path in (None, "tc", "persistent", "simt"):
        def run(path=path):
            for w in ws:
                kl.quant_linear(x, w, out=y, pdl=True, path=path)
        run()
        torch.cuda.synchronize()
        g = capture(run)
        ms = max_over_ranks(timed(g, 10), dist, device) / copies
        del g
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[path or "auto"] = {"us": round(ms * 1e3, 3), "GB/s": round(gbs, 1), "frac_hbm": round(gbs / hbm, 3),
                               "kernel": kernel_names[path]}
    return out


def section_prefill(kl, weights, device, tf_burst, peak_kind, args, rank, world, dist):
    """the 28 layers' four GEMMs (the config 1 weights, 353 MB
    of int8, larger than L2) at M in {512, 2048, 8192}, launched in model order
    with programmatic dependent launch as one CUDA graph per M, without and with
    the SwiGLU epilogue on gate_up.  TFLOP/s = 2*M*N*K summed / device time."""
    import numpy as np
    import torch
    ms_list = [512, 2048, 8192]
    gen = torch.Generator(device=device)
    gen.manual_seed(77 + rank)
    res = {}
    with ClockSampler(device.index or 0) as clocks:
        for m in ms_list:
            xs = {k: torch.randn(m, k, device=device, generator=gen).to(torch.bfloat16) for k in (1024, 2048, 3072)}
            row = {}
            for sw in (False, True):
                ys = {}
                items = []
                for name, p in weights:
                    n, k = p.shape
                    swn = sw and name.startswith("gate_up")
                    key = (n // 2 if swn else n)
                    if key not in ys:
                        ys[key] = torch.empty(m, key, device=device, dtype=torch.bfloat16)
                    items.append((p, xs[k], ys[key], swn))

                def run(items=items):
                    for p, x, y, swn in items:
                        kl.quant_linear(x, p, out=y, swiglu=swn, pdl=True)
                run()
                torch.cuda.synchronize()
                g = capture(run)
                ms = max_over_ranks(timed(g, 3 if m == 8192 else 5), dist, device)
                del g
                flops = sum(2 * m * p.shape[0] * p.shape[1] for p, _, _, _ in items)
                tfs = flops / (ms * 1e-3) / 1e12
                row["swiglu" if sw else "plain"] = {"ms": round(ms, 3), "TFLOP/s": round(tfs, 1),
                                                    "frac": round(tfs / tf_burst, 3)}
            del xs, ys, items
            # the same 112 GEMMs with independent activations and outputs as ONE
            # grouped launch on the CTA-pair kernel (the config 1 treatment)
            probs = [(torch.randn(m, p.shape[1], device=device, generator=gen).to(torch.bfloat16), p,
                      torch.empty(m, p.shape[0], device=device, dtype=torch.bfloat16)) for _, p in weights]
            grp = kl.GroupedLinear(probs)
            grp.run(pdl=True)
            torch.cuda.synchronize()
            g = capture(lambda: grp.run(pdl=True))
            ms = max_over_ranks(timed(g, 3 if m == 8192 else 5), dist, device)
            del g, grp
            flops = sum(2 * m * p.shape[0] * p.shape[1] for _, p in weights)
            tfs = flops / (ms * 1e-3) / 1e12
            row["grouped"] = {"ms": round(ms, 3), "TFLOP/s": round(tfs, 1), "frac": round(tfs / tf_burst, 3)}
            del probs
            res[str(m)] = row
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # the reference's CPU path (dequantise + fp32 matmul + bf16 cast) on a subset:
        # M = 512 tokens against 1024-row slices of each of the four layer shapes
        from oracle import quant_oracle as O
        rng = np.random.default_rng(0)
        t_total, flops = 0.0, 0
        subset = [(1024, 1024), (1024, 2048), (1024, 1024), (1024, 3072)]
        prepared = []
        for n, k in subset:
            q, sc = O.quantize_int8_rowwise(rng.standard_normal((n, k), dtype=np.float32) * 0.02)
            prepared.append((q, sc, O.bf16_round(rng.standard_normal((512, k), dtype=np.float32))))
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < 5.0:
            for q, sc, x in prepared:
                t1 = time.perf_counter()
                O.linear(x, O.dequantize_int8_rowwise(q, sc))
                t_total += time.perf_counter() - t1
                flops += 2 * x.shape[0] * q.shape[0] * q.shape[1]
        from threadpoolctl import threadpool_info
        threads = max((i.get("num_threads", 1) for i in threadpool_info()), default=1)
        cpu = {"value": round(flops / t_total / 1e12, 5), "unit": "TFLOP/s", "cores": threads, "kind": "port",
               "sample": f"M=512 against 1024-row slices of the qkv/o/gate_up/down shapes ({t_total:.1f} s)"}
    return {"unit": "TFLOP/s", "peak": tf_burst, "peak_source": peak_kind, "batch_m": ms_list,
            "launch": ("plain / swiglu: 28 layers x 4 GEMMs per M in model order, programmatic dependent launch, "
                       "one CUDA graph; grouped: the 112 GEMMs with independent activations as one CTA-pair launch"),
            "per_m": res, "cpu_baseline": cpu, "clocks": clocks.summary()}


def section_decode_other(kl, which, device, hbm, args, rank, world, dist):
    """BASELINE config 3 (``w4``: 4-bit asymmetric group-128 weights, Qwen3-0.6B
    decode shapes, M in {1, 16}) or config 4 (``llama``: Llama-3.2-3B shapes,
    int8, M in {1, 64, 256}): the grouped launch and the dependent chain per M,
    the lm_head alone, and at N > 1 the vocab-sharded lm_head."""
    import torch
    if which == "w4":
        layer, head, ms_list, fmt = QWEN_LAYER, QWEN_HEAD, [1, 16], "w4_asym"
    else:
        layer, head, ms_list, fmt = LLAMA_LAYER, LLAMA_HEAD, [1, 64, 256], "w8_row"
    weights = build_weights(kl, layer, LAYERS, device, seed=2024 if which == "w4" else 3030, fmt=fmt)
    gen = torch.Generator(device=device)
    gen.manual_seed(4322)
    hw = torch.randn(head[1], head[2], device=device, generator=gen) * 0.02
    weights.append(("lm_head", quantize(kl, hw, fmt)))
    del hw
    torch.cuda.empty_cache()
    with ClockSampler(device.index or 0) as clocks:
        ds = DecodeSet(kl, weights, ms_list, device, 199 + rank)
        per_m = ds.per_m(hbm, 5, device, dist)
        head_alone = ds.head_alone(hbm, device)
    tf_burst = measured_peaks()[1]
    for m in ms_list:
        flops = sum(2 * m * p.shape[0] * p.shape[1] for _, p, _, _ in ds.passes[m])
        for kind in ("grouped", "chain"):
            t = per_m[str(m)][f"{kind}_ms"]
            per_m[str(m)][f"{kind}_TFLOP/s"] = round(flops / (t * 1e-3) / 1e12, 1)
            per_m[str(m)][f"{kind}_frac_tensor"] = round(flops / (t * 1e-3) / 1e12 / tf_burst, 3)
            per_m[str(m)][f"{kind}_tokens/s_all_ranks"] = round(world * m / (t * 1e-3), 1)
    out = {"workload": ("qwen3-0.6b decode projection set, 4-bit asym g128 (config 3)" if which == "w4"
                        else "llama-3.2-3b projection set, int8 (config 4)"),
           "batch_m": ms_list, "bytes_per_pass": {str(m): ds.pass_bytes(m) for m in ms_list},
           "per_m": per_m, "lm_head_alone": head_alone, "clocks": clocks.summary()}
    if world > 1:
        out["lm_head_sharded"] = sharded_head_section(kl, ds.passes[ms_list[0]][-1][1], ms_list,
                                                      lambda m: ds.passes[m][-1][2], world, rank, device, dist,
                                                      args.steps, fmt)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        shapes = layer + [head]
        v, secs, desc, threads = cpu_path_sample(shapes, [1], fmt, budget_s=5.0)
        out["cpu_baseline"] = {"value": round(v, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                               "sample": desc + f" ({secs:.1f} s, M = 1 only)"}
    del ds, weights
    torch.cuda.empty_cache()
    return out


def bench_prefill(args, kl, world, rank, local, dist):
    import torch
    device = torch.device("cuda", local)
    ms_list = [int(v) for v in args.batch.split(",")] if args.batch else [512, 2048, 8192]
    gen = torch.Generator(device=device)
    gen.manual_seed(77)
    weights = []
    for name, n, k in QWEN_LAYER:
        w = torch.randn(n, k, device=device, generator=gen) * 0.02
        weights.append((name, kl.quantize_int8_rowwise(w), name == "gate_up" and args.swiglu))
    hbm, tf_burst, tf_sus, peak_kind = measured_peaks()
    res = {}
    total_flops, total_ms = 0.0, 0.0
    grouped = {}
    with ClockSampler(local) as clocks:
        for m in ms_list:
            # the 28 layers' GEMMs with independent activations as ONE grouped
            # CTA-pair launch (the first tc_prefill launches of the run: one
            # eager call, then the graph replays)
            probs = []
            for _ in range(LAYERS):
                for name, p, sw in weights:
                    n, k = p.data.shape
                    probs.append((torch.randn(m, k, device=device, generator=gen).to(torch.bfloat16), p,
                                  torch.empty(m, n // 2 if sw else n, device=device, dtype=torch.bfloat16)))
            grp = kl.GroupedLinear(probs, swiglu=bool(args.swiglu))
            grp.run(pdl=True)
            torch.cuda.synchronize()
            gg = capture(lambda: grp.run(pdl=True))
            gms = max_over_ranks(timed(gg, args.steps, warm=args.warmup), dist, device)
            gflops = sum(2 * m * p.data.shape[0] * p.data.shape[1] for _, p, _ in probs)
            grouped[str(m)] = {"ms": round(gms, 4), "TFLOP/s": round(gflops / (gms * 1e-3) / 1e12, 1),
                               "frac": round(gflops / (gms * 1e-3) / 1e12 / tf_burst, 3)}
            del gg, grp, probs
            items = []
            for name, p, sw in weights:
                n, k = p.data.shape
                x = torch.randn(m, k, device=device, generator=gen).to(torch.bfloat16)
                y = torch.empty(m, n // 2 if sw else n, device=device, dtype=torch.bfloat16)
                items.append((name, p, sw, x, y))
            for _ in range(args.warmup):
                for name, p, sw, x, y in items:
                    kl.quant_linear(x, p, out=y, swiglu=sw, pdl=True)
            torch.cuda.synchronize()
            # the layer's four GEMMs as one CUDA graph (no host launch gaps); with
            # programmatic dependent launch each GEMM's set-up and weight stream
            # overlap the previous GEMM's tail
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for name, p, sw, x, y in items:
                    kl.quant_linear(x, p, out=y, swiglu=sw, pdl=True)
            for _ in range(args.warmup):
                graph.replay()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(args.steps):
                graph.replay()
            b.record()
            torch.cuda.synchronize()
            ms = a.elapsed_time(b) / args.steps
            del graph
            flops = sum(2 * m * p.data.shape[0] * p.data.shape[1] for _, p, _, _, _ in items)
            res[str(m)] = {"ms": round(ms, 4), "TFLOP/s": round(flops / (ms * 1e-3) / 1e12, 1),
                           "frac": round(flops / (ms * 1e-3) / 1e12 / tf_burst, 3)}
            total_flops += flops
            total_ms += ms
    value = world * total_flops / (total_ms * 1e-3) / 1e12
    return {"metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(total_ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "qwen3-0.6b prefill layer GEMMs (BASELINE config 2)", "batch_m": ms_list,
                       "swiglu": bool(args.swiglu), "launch": "the 4 layer GEMMs of each M as one CUDA graph, programmatic dependent launch",
                       "l2": "no flush: at M>=2048 each graph replay streams more than the 126 MB L2 in activations and outputs"},
            "per_m": res, "grouped_per_m": grouped,
            "roofline": {"bound": "tensor", "achieved": round(value / world, 1), "peak": tf_burst, "unit": "TFLOP/s",
                         "frac": round(value / world / tf_burst, 4), "peak_source": peak_kind, "traffic": None},
            "gpu_launches": len(weights) * len(ms_list) * args.steps,
            "clocks": clocks.summary()}


def bench_rmsnorm(args, kl, world, rank, local, dist):
    """The fused residual-add + RMSNorm in front of each layer's QKV and gate_up
    (Qwen3-0.6B hidden 1024, bf16).  GB/s = (x, residual, weight read; y and the
    residual stream written) per launch / device time.  Four buffer sets
    (268 MB at M = 8192) rotate so that no launch finds its inputs in L2."""
    import numpy as np
    import torch
    from oracle import quant_oracle as O
    device = torch.device("cuda", local)
    n = QWEN_LAYER[0][2]
    ms_list = [int(v) for v in args.batch.split(",")] if args.batch else [1, 64, 8192]
    hbm, _, _, peak_kind = measured_peaks()
    gen = torch.Generator(device=device)
    gen.manual_seed(5 + rank)
    w = torch.randn(n, device=device, generator=gen).to(torch.bfloat16)
    per_m, total_bytes, total_ms = {}, 0, 0.0
    with ClockSampler(local) as clocks, torch.inference_mode():
        for m in ms_list:
            sets = [tuple(torch.randn(m, n, device=device, generator=gen).to(torch.bfloat16) for _ in range(2))
                    + tuple(torch.empty(m, n, device=device, dtype=torch.bfloat16) for _ in range(2))
                    for _ in range(4)]

            def launch(i):
                x, r, y, c = sets[i % 4]
                N_ = kl._native
                N_.check(N_.lib().kl_rmsnorm(N_.ptr(x), N_.ptr(r), N_.ptr(w), N_.KL_DT_BF16, m, n, 1e-6, 0,
                                             N_.ptr(y), N_.ptr(c), N_.stream_handle(device)))

            reps = 20
            for i in range(args.warmup):
                launch(i)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for i in range(reps):
                    launch(i)
            for _ in range(args.warmup):
                graph.replay()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(args.steps):
                graph.replay()
            b.record()
            torch.cuda.synchronize()
            ms = a.elapsed_time(b) / (args.steps * reps)
            del graph
            nbytes = 5 * m * n * 2 + 2 * n
            per_m[str(m)] = {"us": round(ms * 1e3, 3), "GB/s": round(nbytes / (ms * 1e-3) / 1e9, 1),
                             "frac_hbm": round(nbytes / (ms * 1e-3) / 1e9 / hbm, 3)}
            total_bytes += nbytes
            total_ms += ms
            # spot check against the oracle (first rows of the last set)
            x, r, y, c = sets[(reps - 1) % 4]
            ey, ec = O.qwen_residual_rmsnorm(x[:4].float().cpu().numpy(), r[:4].float().cpu().numpy(),
                                             w.float().cpu().numpy())
            assert np.array_equal(c[:4].float().cpu().numpy(), ec)
            assert np.allclose(y[:4].float().cpu().numpy(), ey, rtol=2e-2, atol=2e-2)
            del sets
    big = str(ms_list[-1])
    value = world * per_m[big]["GB/s"]
    # end to end through the public API: host copies of x and residual in, y and the stream out
    m = ms_list[-1]
    hx = torch.randn(m, n).to(torch.bfloat16).pin_memory()
    hr = torch.randn(m, n).to(torch.bfloat16).pin_memory()
    hy = torch.empty(m, n, dtype=torch.bfloat16).pin_memory()
    hc = torch.empty(m, n, dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        with torch.inference_mode():
            y, c = kl.qwen_residual_rmsnorm(hx.to(device, non_blocking=True), hr.to(device, non_blocking=True),
                                            w)
        hy.copy_(y, non_blocking=True)
        hc.copy_(c, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        e2e_step()
    b.record()
    torch.cuda.synchronize()
    e2e_ms = a.elapsed_time(b) / args.steps
    nbytes = 5 * m * n * 2 + 2 * n
    # CPU: the reference's eager expression as restated in the oracle, numpy on the host
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        xs = np.random.default_rng(0).standard_normal((min(m, 2048), n)).astype(np.float32)
        xs, rs, ws = O.bf16_round(xs), O.bf16_round(xs[::-1].copy()), O.bf16_round(np.ones(n, np.float32))
        t0, reps = time.perf_counter(), 0
        while time.perf_counter() - t0 < 5.0:
            O.qwen_residual_rmsnorm(xs, rs, ws)
            reps += 1
        secs = time.perf_counter() - t0
        cpu = {"value": round(reps * (5 * xs.size * 2 + 2 * n) / secs / 1e9, 3), "unit": "GB/s", "cores": 1,
               "kind": "port", "sample": f"{xs.shape[0]} x {n} bf16 rows, {reps} calls ({secs:.1f} s)"}
    return {"metric": "fused residual-add + RMSNorm HBM GB/s (Qwen3-0.6B hidden 1024, bf16)",
            "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(per_m[big]["us"] * 20 / 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "residual + RMSNorm before QKV / gate_up", "batch_m": ms_list,
                       "n": n, "l2": "4 rotating buffer sets, 268 MB at M=8192 (larger than L2)",
                       "launch": "20 launches per step in a CUDA graph"},
            "per_m": per_m,
            "roofline": {"bound": "hbm", "kernel": "rmsnorm_vec_kernel<bf16, residual>", "achieved": per_m[big]["GB/s"],
                         "peak": hbm, "unit": "GB/s", "frac": per_m[big]["frac_hbm"], "peak_source": peak_kind,
                         "traffic": None},
            "e2e": {"value": round(world * nbytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": 2 * m * n * 2, "d2h_bytes_per_step": 2 * m * n * 2,
                    "ms_per_step": round(e2e_ms, 4)},
            "gpu_launches": 20 * args.steps * len(ms_list),
            "cpu_baseline": cpu,
            "clocks": clocks.summary()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["decode", "prefill", "llama", "w4", "rmsnorm"], default="decode")
    ap.add_argument("--batch", default="", help="comma-separated M values (overrides the workload's)")
    ap.add_argument("--swiglu", action="store_true", help="prefill: fuse SwiGLU into gate_up")
    ap.add_argument("--lm-head-shard", action="store_true", help="llama: vocab-shard the lm_head + NCCL all-gather")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--only-headline", action="store_true", help="decode: skip the config 0/2/3/4 sections")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        run_reference(args)
        return
    kl = importlib.import_module("gpu-kernel-lab_b200")
    world, rank, local, dist = init_dist(args)
    try:
        if args.workload == "prefill":
            result = bench_prefill(args, kl, world, rank, local, dist)
        elif args.workload == "rmsnorm":
            result = bench_rmsnorm(args, kl, world, rank, local, dist)
        else:
            result = bench_decode(args, kl, world, rank, local, dist)
        if rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload not in ("prefill", "rmsnorm"):
            shapes, ms, fmt, _ = workload_of(args)
            v, secs, desc, threads = cpu_path_sample(shapes, ms, fmt, budget_s=10.0)
            result["cpu_baseline"] = {"value": round(v, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                                      "sample": desc + f" ({secs:.1f} s)"}
        elif rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload == "prefill":
            result["cpu_baseline"] = None
        if rank == 0:
            print(json.dumps(result), flush=True)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
