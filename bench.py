"""Benchmark of the quantized-decode hot path on B200.

Headline (BASELINE.json metric "NF4/Q4_0 matvec HBM GB/s"; workload = its
configs[1]): GGUF Q4_0 dequantise-and-matvec at the Llama FFN shapes.  One
step = one up/gate matvec (14336 x 4096) plus one down matvec (4096 x 14336),
batch 1, fp32 activations.  Weights rotate through a pool of independent
matrices larger than twice the L2 cache, so every launch streams from HBM.

  value   = algorithmic bytes (weights + x + y) / device time, whole job
            (N ranks each run the same per-GPU workload: weak scaling)
  e2e     = same metric through the host-buffer C-ABI call
            (aljabr_blackwell_matvec_tb_q4_0: H2D of x, kernel, D2H of y)
  roofline= the Q4_0 kernel's achieved GB/s vs the measured HBM peak

Also reported under "extra": NF4 4096x4096, Q8_0 one Llama-3-8B
layer and GQA decode attention (Hq 32, Hkv 8, D 128, ctx 4096).

`--impl reference` times the CPU implementation of the same path: the C
restatement of the reference's Java row kernels (the Java reference cannot
run on these hosts: no JDK), over all host threads.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

UP_N, UP_K = 14336, 4096
DOWN_N, DOWN_K = 4096, 14336
Q4_BLOCK = 18


def q4_bytes(n, k):
    return n * (k // 32) * Q4_BLOCK


STEP_BYTES = (q4_bytes(UP_N, UP_K) + 4 * UP_K + 4 * UP_N) + (q4_bytes(DOWN_N, DOWN_K) + 4 * DOWN_K + 4 * DOWN_N)
WORKLOAD = "GGUF Q4_0 dequant-matvec, Llama FFN shapes: up/gate 14336x4096 + down 4096x14336, batch 1"
METRIC = "Q4_0 dequant-matvec HBM GB/s (Llama FFN shapes, batch 1)"


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def load_tc_peak():
    """Dense bf16 tensor peak (TFLOP/s, cuBLAS burst) from MEASURED_PEAKS.json."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        if "bf16_tflops" in d:
            return float(d["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def load_traffic(name):
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get(name)
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------- our arm
def run_ours(args, rank, world, local_rank):
    import ctypes

    import torch

    import oracle
    from aljabr_b200 import native

    torch.cuda.set_device(local_rank)
    native.call("aljabr_blackwell_init", local_rank)
    native.call("aljabr_blackwell_set_pdl", 0 if args.no_pdl else 1)   # weights are static here
    dev = torch.device("cuda", local_rank)
    L = native.lib()
    props = torch.cuda.get_device_properties(local_rank)
    l2 = getattr(props, "L2_cache_size", 126 * 2 ** 20) or 126 * 2 ** 20

    # ---- synthetic pool: distinct matrices, total > 2 x L2 -------------------
    g = np.random.default_rng(20260101 + rank)
    base_up = oracle.encode_q4_0(g.normal(0, 0.02, size=(UP_N, UP_K)).astype(np.float32))
    base_dn = oracle.encode_q4_0(g.normal(0, 0.02, size=(DOWN_N, DOWN_K)).astype(np.float32))
    pair_bytes = base_up.nbytes + base_dn.nbytes
    pool = max(3, int(np.ceil(2.5 * l2 / pair_bytes)))
    up_d, dn_d = [], []
    t_up = torch.from_numpy(base_up).to(dev)
    t_dn = torch.from_numpy(base_dn).to(dev)
    for i in range(pool):
        # distinct contents per slot: XOR the code bytes (scales untouched)
        u = t_up.clone()
        d = t_dn.clone()
        if i:
            u.view(-1, 18)[:, 2:] ^= (i * 37) & 0xFF
            d.view(-1, 18)[:, 2:] ^= (i * 53) & 0xFF
        up_d.append(u)
        dn_d.append(d)
    xs_up = [torch.randn(UP_K, device=dev) for _ in range(pool)]
    xs_dn = [torch.randn(DOWN_K, device=dev) for _ in range(pool)]
    ys_up = [torch.empty(UP_N, device=dev) for _ in range(pool)]
    ys_dn = [torch.empty(DOWN_N, device=dev) for _ in range(pool)]
    stream = torch.cuda.Stream(device=dev)
    sh = ctypes.c_void_p(stream.cuda_stream)

    def step(i):
        j = i % pool
        # each launch L2-prefetches the weights of the one after it (a hint;
        # every launch still reads all of its own weights)
        if not args.no_prefetch:
            native.check(L.aljabr_blackwell_prefetch_hint(dn_d[j].data_ptr(), dn_d[j].nbytes))
        native.check(L.aljabr_blackwell_matvec_dev(native.TYPE_Q4_0, ys_up[j].data_ptr(), xs_up[j].data_ptr(),
                                                   up_d[j].data_ptr(), None, UP_K, UP_N, 0, None, sh))
        if not args.no_prefetch:
            nxt = up_d[(j + 1) % pool]
            native.check(L.aljabr_blackwell_prefetch_hint(nxt.data_ptr(), nxt.nbytes))
        native.check(L.aljabr_blackwell_matvec_dev(native.TYPE_Q4_0, ys_dn[j].data_ptr(), xs_dn[j].data_ptr(),
                                                   dn_d[j].data_ptr(), None, DOWN_K, DOWN_N, 0, None, sh))

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    # Launches are recorded into CUDA graphs (chunks of steps replayed back to
    # back) so the host's launch rate does not bound the device timeline.
    chunk = graph_chunk(args.steps)
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i)
    torch.cuda.synchronize(dev)
    graph = capture(torch, stream, lambda: [step(i) for i in range(chunk)])
    replays = args.steps // chunk
    with torch.cuda.stream(stream):     # replay() launches on the current stream
        graph.replay()                  # one untimed replay: graph upload
    torch.cuda.synchronize(dev)

    # ---- timed region: K steps, device time by CUDA events on the stream -----
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local_rank) as clk, torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(replays):
            graph.replay()
        end.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    ms = start.elapsed_time(end)
    ms_max = ms
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms_max = float(t.item())
    per_launch_ms = ms / (2 * args.steps)

    # correctness spot check of the timed kernels (slot 0, oracle as checker)
    y_chk = ys_up[0].cpu().numpy()
    x_chk = xs_up[0].cpu().numpy()
    ref = oracle.matvec_q4_0(up_d[0].cpu().numpy(), x_chk, UP_N, threads=os.cpu_count() or 8)
    err = float(np.max(np.abs(y_chk - ref) / np.maximum(np.abs(ref), 1e-3 * np.abs(ref).max())))

    # ---- e2e: host buffers through the Metal-shaped C-ABI ---------------------
    e2e = None
    if rank == 0 or world > 1:
        host_up = [base_up] + [None]
        model_up = np.ascontiguousarray(base_up)
        model_dn = np.ascontiguousarray(base_dn)
        native.call("aljabr_blackwell_register_model_buffer", ctypes.c_void_p(model_up.ctypes.data), model_up.nbytes)
        native.call("aljabr_blackwell_register_model_buffer", ctypes.c_void_p(model_dn.ctypes.data), model_dn.nbytes)
        hx_up = np.random.default_rng(1).normal(size=UP_K).astype(np.float32)
        hx_dn = np.random.default_rng(2).normal(size=DOWN_K).astype(np.float32)
        hy_up = np.empty(UP_N, np.float32)
        hy_dn = np.empty(DOWN_N, np.float32)

        # buffer addresses taken once, as a Java caller holds its MemorySegments
        # (numpy's .ctypes lookup alone costs microseconds per call)
        a_hy_up, a_hx_up = ctypes.c_void_p(hy_up.ctypes.data), ctypes.c_void_p(hx_up.ctypes.data)
        a_hy_dn, a_hx_dn = ctypes.c_void_p(hy_dn.ctypes.data), ctypes.c_void_p(hx_dn.ctypes.data)
        a_up, a_dn = ctypes.c_void_p(model_up.ctypes.data), ctypes.c_void_p(model_dn.ctypes.data)
        tb = L.aljabr_blackwell_matvec_tb_q4_0

        def e2e_step():
            native.check(tb(a_hy_up, a_hx_up, a_up, UP_K, UP_N))
            native.check(tb(a_hy_dn, a_hx_dn, a_dn, DOWN_K, DOWN_N))

        for _ in range(max(3, args.warmup)):
            e2e_step()
        e2e_steps = min(args.steps, 2000)
        barrier()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            e2e_step()
        t1 = time.perf_counter()
        barrier()
        e2e_s = t1 - t0
        if world > 1:
            t = torch.tensor([e2e_s], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            e2e_s = float(t.item())
        e2e = {"value": round(STEP_BYTES * e2e_steps * world / e2e_s / 1e9, 2), "unit": "GB/s", "steps": e2e_steps,
               "h2d_bytes_per_step": 4 * (UP_K + DOWN_K), "d2h_bytes_per_step": 4 * (UP_N + DOWN_N),
               "timer": "host wall clock around the blocking C-ABI calls (weights registered, HBM-resident)",
               "host_api": "aljabr_blackwell_matvec_tb_q4_0"}
        del host_up
        native.call("aljabr_blackwell_unregister_model_buffer", ctypes.c_void_p(model_up.ctypes.data))
        native.call("aljabr_blackwell_unregister_model_buffer", ctypes.c_void_p(model_dn.ctypes.data))

    extra = {}
    if not args.no_extra:
        if rank == 0 or world == 1:
            extra = run_extra(args, dev, stream, sh, l2)
        del graph                       # it references the pool below; never replayed again
        del up_d, dn_d
        torch.cuda.empty_cache()
        try:
            extra["nf4_decode_llama3_8b"] = run_decode(args, rank, world, dev)
        except Exception as e:  # reported, never hidden: the line says what failed
            extra["nf4_decode_llama3_8b"] = {"error": f"{type(e).__name__}: {e}"}
        if world > 1:   # BASELINE config 5 with the weights sharded over these GPUs
            try:
                extra["c5_nf4_70b_layer_tp"] = run_c5_tp(args, rank, world, dev)
            except Exception as e:
                extra["c5_nf4_70b_layer_tp"] = {"error": f"{type(e).__name__}: {e}"}

    bits = ctypes.c_uint(0)
    native.check(L.aljabr_blackwell_device_status(ctypes.byref(bits)))

    peak, peak_kind = load_peaks()
    achieved = (STEP_BYTES / 2) / (per_launch_ms * 1e-3) / 1e9
    value = STEP_BYTES * args.steps * world / (ms_max * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "q4_0 codes, fp16 scales -> f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "batch": 1, "weights": "N(0,0.02) -> GGUF Q4_0 (GGUFWriter.encodeQ4_0)",
                   "x": "N(0,1) fp32", "pool_matrices": 2 * pool, "pool_bytes": pool * pair_bytes,
                   "l2_bytes": l2, "l2_policy": "inputs larger than L2: weights rotate through a pool > 2x L2",
                   "parallelism": f"independent replicas x{world} (rows of each matrix on one GPU)",
                   "launch": "CUDA graphs of 500 steps" + ("" if args.no_pdl else ", programmatic dependent launch")
                             + ("" if args.no_prefetch else ", each launch L2-prefetches the next launch's first weights")},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                     "traffic": load_traffic("q4_0_matvec"),
                     "kernel": "quant_imma_kernel<Q4_0> (avg of 14336x4096 and 4096x14336 launches)",
                     "algorithmic_bytes_per_launch": STEP_BYTES // 2},
        "gpu_launches": 2 * args.steps,
        "e2e": e2e,
        "parity": {"max_rel_err_vs_oracle": err, "tolerance": 1e-3},
        "device_fault_bits": bits.value,
        "clocks": clk.summary(),
        "extra": extra,
    }
    if rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args, 8.0)
    return line


def graph_chunk(steps: int) -> int:
    """Largest divisor of `steps` that is at most 500 (steps per graph)."""
    for c in range(min(500, steps), 0, -1):
        if steps % c == 0:
            return c
    return 1


def capture(torch, stream, record):
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        record()
    return g


def run_extra(args, dev, stream, sh, l2, which=None, reps=200):
    c5_tokens = [int(v) for v in getattr(args, "c5_tokens", "1,16,64,512").split(",")]
    prefill_tokens = [int(v) for v in getattr(args, "prefill_tokens", "16,64,512").split(",")]
    """Secondary configs, each with its own pool > 2 x L2 and device timing.
    `which` selects a subset of {"nf4", "q8", "attention", "c5", "kquant"} (all if None)."""
    import torch

    import oracle
    from aljabr_b200 import native

    L = native.lib()
    out = {}

    def timed(fn, n):
        """Device ms per call: n calls captured in one graph, replayed 3x."""
        with torch.cuda.stream(stream):
            for i in range(3):
                fn(i)
        torch.cuda.synchronize(dev)
        gr = capture(torch, stream, lambda: [fn(i) for i in range(n)])
        with torch.cuda.stream(stream):
            gr.replay()
        torch.cuda.synchronize(dev)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            s.record(stream)
            for _ in range(3):
                gr.replay()
            e.record(stream)
        torch.cuda.synchronize(dev)
        return s.elapsed_time(e) / (3 * n)

    want = (lambda name: which is None or name in which)
    g = np.random.default_rng(7)

    def nf4_section():
        # NF4 4096 x 4096, block 64
        N = K = 4096
        codes, absmax = oracle.quantize_nf4(g.normal(0, 0.02, size=(N, K)).astype(np.float32), 64)
        per = codes.nbytes + absmax.nbytes
        pool = max(2, int(np.ceil(2.5 * l2 / per)))
        cd = torch.from_numpy(codes).to(dev)
        ad = torch.from_numpy(absmax).to(dev)
        cs = [cd.clone() for _ in range(pool)]
        ams = [ad.clone() for _ in range(pool)]
        xs = [torch.randn(K, device=dev) for _ in range(pool)]
        ys = [torch.empty(N, device=dev) for _ in range(pool)]
        ms = timed(lambda i: native.check(L.aljabr_blackwell_matvec_dev(
            native.TYPE_NF4, ys[i % pool].data_ptr(), xs[i % pool].data_ptr(), cs[i % pool].data_ptr(),
            ctypes_ptr(ams[i % pool]), K, N, 64, None, sh)), reps * 4)
        alg = per + 4 * K + 4 * N
        out["nf4_matvec_4096x4096_b64"] = {"GB/s": round(alg / (ms * 1e-3) / 1e9, 1),
                                           "us_per_launch": round(ms * 1e3, 3), "algorithmic_bytes": alg,
                                           "pool": pool}

    def q8_section():
        # Q8_0: one Llama-3-8B layer's projections
        shapes = [("q", 4096, 4096), ("k", 1024, 4096), ("v", 1024, 4096), ("o", 4096, 4096),
                  ("gate", 14336, 4096), ("up", 14336, 4096), ("down", 4096, 14336)]
        mats = {}
        for name, n, k in shapes:
            mats[name] = torch.from_numpy(
                oracle.encode_q8_0(g.normal(0, 0.02, size=(n, k)).astype(np.float32))).to(dev)
        layer_w = sum(m.numel() for m in mats.values())
        pool8 = max(2, int(np.ceil(2.5 * l2 / layer_w)))
        layers = [{k2: v.clone() for k2, v in mats.items()} for _ in range(pool8)]
        xq = {k: torch.randn(kk, device=dev) for k, _, kk in shapes}
        yq = {k: torch.empty(n, device=dev) for k, n, _ in shapes}

        def q8_layer(i):
            lay = layers[i % pool8]
            for name, n, k in shapes:
                native.check(L.aljabr_blackwell_matvec_dev(native.TYPE_Q8_0, yq[name].data_ptr(),
                                                           xq[name].data_ptr(), lay[name].data_ptr(), None, k, n,
                                                           0, None, sh))
        ms = timed(q8_layer, reps)
        alg = layer_w + sum(4 * (n + k) for _, n, k in shapes)
        out["q8_0_llama3_8b_layer"] = {"GB/s": round(alg / (ms * 1e-3) / 1e9, 1),
                                       "us_per_layer": round(ms * 1e3, 3), "launches_per_layer": len(shapes),
                                       "weight_bytes": layer_w}

    def attention_section():
        # GQA decode attention, Hq 32 / Hkv 8 / D 128, ctx 4096, bf16 KV
        Hq, Hkv, D, ctx = 32, 8, 128, 4096
        kvb = ctx * Hkv * D * 2
        poola = max(2, int(np.ceil(2.5 * l2 / (2 * kvb))))
        ks = [torch.randn(ctx, Hkv * D, device=dev).to(torch.bfloat16) for _ in range(poola)]
        vs = [torch.randn(ctx, Hkv * D, device=dev).to(torch.bfloat16) for _ in range(poola)]
        q = torch.randn(Hq * D, device=dev)
        o = torch.empty(Hq * D, device=dev)
        ms = timed(lambda i: native.check(L.aljabr_blackwell_decode_attention_dev(
            o.data_ptr(), q.data_ptr(), ks[i % poola].data_ptr(), vs[i % poola].data_ptr(), native.KV_BF16,
            Hkv * D, Hkv, Hq, D, ctx, 0, 1.0 / 128 ** 0.5, sh)), reps * 4)
        alg = 2 * kvb + 8 * Hq * D
        out["gqa_decode_attention_ctx4096_bf16"] = {"GB/s": round(alg / (ms * 1e-3) / 1e9, 1),
                                                    "us_per_call": round(ms * 1e3, 3), "algorithmic_bytes": alg,
                                                    "launches_per_call": 1}

    def kquant_section():
        # GGUF Q4_K / Q6_K (GgufQ4RawDot / GgufQ6RawDot) at the Llama FFN shapes of the
        # headline: up 14336x4096 + down 4096x14336 per step.  Synthetic
        # super-blocks: random code / scale bytes with fixed small fp16 super
        # scales (every byte pattern is a valid block).
        g8 = torch.Generator(device=dev).manual_seed(5)
        for name, kind, bb in (("q4_k", native.TYPE_Q4_K, 144), ("q6_k", native.TYPE_Q6_K, 210)):
            shapes = ((14336, 4096), (4096, 14336))
            mats = []
            for n, k in shapes:
                w = torch.randint(0, 256, (n * k // 256 * bb,), dtype=torch.uint8, device=dev, generator=g8)
                v = w.view(-1, bb)
                if kind == native.TYPE_Q4_K:
                    v[:, 0], v[:, 1], v[:, 2], v[:, 3] = 0x00, 0x10, 0x00, 0x0C   # d ~ 6e-5, dmin ~ 2e-4
                else:
                    v[:, 208], v[:, 209] = 0x00, 0x10
                mats.append(w)
            pair = sum(m.numel() for m in mats)
            poolk = max(2, int(np.ceil(2.5 * l2 / pair)))
            ws = [[m.clone() for m in mats] for _ in range(poolk)]
            xk = [[torch.randn(k, device=dev) for _, k in shapes] for _ in range(poolk)]
            yk = [[torch.empty(n, device=dev) for n, _ in shapes] for _ in range(poolk)]
            torch.cuda.synchronize(dev)

            def kstep(i, kind=kind, ws=ws, xk=xk, yk=yk, poolk=poolk, shapes=shapes):
                j = i % poolk
                for m, (n, k) in enumerate(shapes):
                    native.check(L.aljabr_blackwell_matvec_dev(kind, yk[j][m].data_ptr(), xk[j][m].data_ptr(),
                                                               ws[j][m].data_ptr(), None, k, n, 0, None, sh))
            ms = timed(kstep, reps)
            alg = pair + sum(4 * (n + k) for n, k in shapes)
            out[f"{name}_llama_ffn"] = {"GB/s": round(alg / (ms * 1e-3) / 1e9, 1), "us_per_step": round(ms * 1e3, 3),
                                        "launches_per_step": 2, "algorithmic_bytes": alg,
                                        "kernel": f"quant_imma_kernel<{name.upper()}> (integer tensor cores)"}
            del ws, xk, yk

    def c5_section():
        # Batched NF4 on the per-GPU tensor-parallel shard (TP 8) of one
        # Llama-3-70B layer: q 1024x8192, k/v 128x8192, o 1024x8192,
        # gate/up 3584x8192, down 1024x28672 rows of this GPU; bf16 activations,
        # M tokens.  M = 1 runs the batch-1 NF4 matvec on the row-major weights,
        # M > 1 the tcgen05 GEMM on the packed weights (q/k/v and gate/up fused
        # launches).  Weights: uniform random NF4 codes (the NF4 levels are
        # equiprobable for normal weights) and absmax ~ |N(0.05, 0.005)|.
        H, FF, TPW, G = 8192, 28672, 8, 64
        shp = {"q": (H // TPW, H), "k": (1024 // TPW, H), "v": (1024 // TPW, H), "o": (H // TPW, H),
               "gate": (FF // TPW, H), "up": (FF // TPW, H), "down": (H // TPW, FF)}
        nweights = sum(n * k for n, k in shp.values())
        wbytes = sum(n * k // 2 + n * k // G * 4 for n, k in shp.values())
        pool5 = max(2, int(np.ceil(2.5 * l2 / wbytes)))
        gen = torch.Generator(device=dev)
        gen.manual_seed(5)
        raw, packed = [], []
        for _ in range(pool5):
            lr, lp = {}, {}
            for name, (n, k) in shp.items():
                c = torch.randint(0, 256, (n * k // 2,), dtype=torch.uint8, device=dev, generator=gen)
                a = (0.05 + 0.005 * torch.randn(n * k // G, device=dev, generator=gen)).abs()
                pk = torch.empty(native.gemm_nf4_packed_size(n, k, G), dtype=torch.uint8, device=dev)
                torch.cuda.synchronize(dev)
                native.gemm_nf4_pack(pk.data_ptr(), c.data_ptr(), a.data_ptr(), n, k, G, sh.value)
                lr[name], lp[name] = (c, a), pk
            raw.append(lr)
            packed.append(lp)
        torch.cuda.synchronize(dev)
        tc_peak, tc_kind = load_tc_peak()
        hbm_peak, hbm_kind = load_peaks()
        res = {}
        for M in c5_tokens:
            xh = torch.randn(M, H, device=dev).to(torch.bfloat16)
            xf = torch.randn(M, FF, device=dev).to(torch.bfloat16)
            ys = {name: torch.empty(M * n, device=dev) for name, (n, _) in shp.items()}
            if M == 1:
                xh32, xf32 = xh.float().reshape(-1), xf.float().reshape(-1)

                def layer(i):
                    lay = raw[i % pool5]
                    for name, (n, k) in shp.items():
                        c, a = lay[name]
                        native.check(L.aljabr_blackwell_matvec_dev(
                            native.TYPE_NF4, ys[name].data_ptr(), (xf32 if name == "down" else xh32).data_ptr(),
                            c.data_ptr(), ctypes_ptr(a), k, n, G, None, sh))
                launches = len(shp)
            else:
                wsb = max(native.gemm_nf4_workspace_size(M, H, [shp["q"][0], shp["k"][0], shp["v"][0]]),
                          native.gemm_nf4_workspace_size(M, H, [shp["gate"][0], shp["up"][0]]),
                          native.gemm_nf4_workspace_size(M, FF, [shp["down"][0]]))
                ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
                calls = ((("q", "k", "v"), xh, H), (("o",), xh, H), (("gate", "up"), xh, H), (("down",), xf, FF))

                def layer(i):
                    lay = packed[i % pool5]
                    for names, x, k in calls:
                        native.gemm_nf4_dev([ys[nm].data_ptr() for nm in names], [shp[nm][0] for nm in names],
                                            [lay[nm].data_ptr() for nm in names], [shp[nm][0] for nm in names],
                                            x.data_ptr(), M, k, G, ws.data_ptr(), wsb, sh.value)
                launches = 2 * len(calls)          # activation prep + GEMM per call
            torch.cuda.synchronize(dev)
            ms = timed(layer, max(10, reps // 10))
            flops = 2.0 * M * nweights
            hbm_floor_us = wbytes / (hbm_peak * 1e3)
            tc_floor_us = 2.0 * flops / (tc_peak * 1e6)      # two MMAs (Th, Tl) per weight element
            res[f"M{M}"] = {"us_per_layer_shard": round(ms * 1e3, 2), "TFLOP/s": round(flops / (ms * 1e9), 1),
                            "weight_GB/s": round(wbytes / (ms * 1e6), 1), "launches": launches,
                            "floor_us": round(max(hbm_floor_us, tc_floor_us if M > 1 else 0.0), 2),
                            "bound": "hbm" if M == 1 or hbm_floor_us >= tc_floor_us else "tensor"}
            del ys
            torch.cuda.empty_cache()
        out["c5_nf4_batched_70b_layer_tp8_shard"] = {
            "per_gpu_weights": nweights, "weight_bytes": wbytes, "pool_layers": pool5,
            "peaks": {"hbm_GB/s": hbm_peak, "hbm": hbm_kind, "bf16_TFLOP/s": tc_peak, "tensor": tc_kind},
            "tokens": res}

    def prefill_section():
        # Prefill of one Llama-3-8B layer with GGUF Q4_0 weights (the format of
        # configs[1]): the seven projections through the batched tcgen05 GEMM
        # (q/k/v and gate/up as multi-segment calls, fp32 activations) and the
        # causal GQA attention (32 / 8 heads, head_dim 128) over T prompt
        # tokens.  Weights: uniform random Q4_0 codes, block scales
        # |N(0.002, 0.0005)| in fp16; packed once per matrix (not timed).
        H, FF, HQ, HKV, D = 4096, 14336, 32, 8, 128
        shp = {"q": (HQ * D, H), "k": (HKV * D, H), "v": (HKV * D, H), "o": (H, HQ * D),
               "gate": (FF, H), "up": (FF, H), "down": (H, FF)}
        nweights = sum(n * k for n, k in shp.values())
        wbytes = sum(n * k // 32 * 18 for n, k in shp.values())
        poolp = max(2, int(np.ceil(2.5 * l2 / wbytes)))
        gen = torch.Generator(device=dev)
        gen.manual_seed(9)
        packed, raw_o = [], None
        for li in range(poolp):
            lp = {}
            for name, (n, k) in shp.items():
                blk = torch.randint(0, 256, (n * k // 32, 18), dtype=torch.uint8, device=dev, generator=gen)
                d = (0.002 + 0.0005 * torch.randn(n * k // 32, device=dev, generator=gen)).abs().half()
                blk[:, 0:2] = d.view(torch.uint8).reshape(-1, 2)
                pk = torch.empty(native.gemm_q_packed_size(native.TYPE_Q4_0, n, k), dtype=torch.uint8, device=dev)
                torch.cuda.synchronize(dev)
                native.gemm_q_pack(native.TYPE_Q4_0, pk.data_ptr(), blk.data_ptr(), n, k, sh.value)
                lp[name] = pk
                if li == 0 and name == "o":
                    raw_o = blk.cpu().numpy().reshape(-1)
                del blk, d
            packed.append(lp)
        torch.cuda.synchronize(dev)
        tc_peak, tc_kind = load_tc_peak()
        hbm_peak, hbm_kind = load_peaks()
        res = {}
        for T in prefill_tokens:
            xh = torch.randn(T, H, device=dev)
            xf = torch.randn(T, FF, device=dev)
            ys = {name: torch.empty(T * n, device=dev) for name, (n, _) in shp.items()}
            wsb = native.gemm_q_workspace_size(T, FF)
            ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
            calls = ((("q", "k", "v"), xh, H), (("o",), xh, H), (("gate", "up"), xh, H), (("down",), xf, FF))

            def gemm_layer(i):
                lay = packed[i % poolp]
                for names, x, k in calls:
                    native.gemm_q_dev(native.TYPE_Q4_0, [ys[nm].data_ptr() for nm in names],
                                      [shp[nm][0] for nm in names], [lay[nm].data_ptr() for nm in names],
                                      [shp[nm][0] for nm in names], x.data_ptr(), T, k, ws.data_ptr(), wsb, sh.value)
            qa = torch.randn(T, HQ * D, device=dev)
            ka = torch.randn(T, HKV * D, device=dev)
            va = torch.randn(T, HKV * D, device=dev)
            oa = torch.empty(T, HQ * D, device=dev)
            scale = float(1.0 / np.sqrt(D))

            def attention(i):
                native.check(L.aljabr_blackwell_prefill_attention_dev(
                    oa.data_ptr(), qa.data_ptr(), ka.data_ptr(), va.data_ptr(), 1, T, T, HQ, HKV, D, HKV * D,
                    scale, 1, 0, 0.0, sh))
            torch.cuda.synchronize(dev)
            reps_t = max(5, min(50, 20000 // T))
            ms_g = timed(gemm_layer, reps_t)
            ms_a = timed(attention, reps_t)
            # spot checks: token 0 of the o projection (pool slot 0), the attention at T = 64
            gemm_layer(0)
            torch.cuda.synchronize(dev)
            x0 = xh[0].cpu().numpy()
            ref_o = oracle.matvec_q4_0_prepared(raw_o, x0, H, threads=os.cpu_count() or 8)
            err_g = float(np.max(np.abs(ys["o"][:H].cpu().numpy() - ref_o) /
                                 np.maximum(np.abs(ref_o), 1e-3 * np.abs(ref_o).max())))
            err_a = None
            if T == 64:
                attention(0)
                torch.cuda.synchronize(dev)
                ref_a = oracle.prefill_attention(qa.cpu().numpy(), ka.cpu().numpy(), va.cpu().numpy(), T, HQ, HKV,
                                                 D, scale)
                got = oa.cpu().numpy()
                err_a = float(np.max(np.abs(got - ref_a) / np.maximum(np.abs(ref_a), 1e-3 * np.abs(ref_a).max())))
            flops_g = 2.0 * T * nweights
            flops_a = 2.0 * 2.0 * HQ * D * T * (T + 1) / 2
            hbm_floor_us = wbytes / (hbm_peak * 1e3)
            tc_floor_us = 3.0 * flops_g / (tc_peak * 1e6)       # three MMAs per weight x token (hi/lo split)
            us = (ms_g + ms_a) * 1e3
            res[f"T{T}"] = {"layer_us": round(us, 2), "tokens_per_s_per_layer": round(T / (us * 1e-6), 1),
                            "gemm_us": round(ms_g * 1e3, 2), "gemm_TFLOP/s": round(flops_g / (ms_g * 1e9), 1),
                            "gemm_weight_GB/s": round(wbytes / (ms_g * 1e6), 1),
                            "gemm_floor_us": round(max(hbm_floor_us, tc_floor_us), 2),
                            "gemm_bound": "hbm" if hbm_floor_us >= tc_floor_us else "tensor",
                            "gemm_frac_of_floor": round(max(hbm_floor_us, tc_floor_us) / (ms_g * 1e3), 3),
                            "attention_us": round(ms_a * 1e3, 2),
                            "attention_TFLOP/s": round(flops_a / (ms_a * 1e9), 2),
                            "gemm_max_rel_err_token0_o": err_g, "attention_max_rel_err": err_a}
            del ys, ws, xh, xf, qa, ka, va, oa
            torch.cuda.empty_cache()
        out["prefill_q4_0_llama3_8b_layer"] = {
            "weights": nweights, "weight_bytes": wbytes, "pool_layers": poolp,
            "peaks": {"hbm_GB/s": hbm_peak, "hbm": hbm_kind, "bf16_TFLOP/s": tc_peak, "tensor": tc_kind},
            "tokens": res}

    def upload_section():
        # register_model_buffer of a 1 GiB host buffer (the reference's mmap'd
        # model registration): host wall clock, first call in the process (it
        # pins the bounce buffers) and a repeat.
        import ctypes
        import time
        buf = np.random.default_rng(3).integers(0, 256, size=1 << 30, dtype=np.uint8)
        times = []
        for _ in range(3):
            t0 = time.perf_counter()
            native.call("aljabr_blackwell_register_model_buffer", ctypes.c_void_p(buf.ctypes.data), buf.nbytes)
            times.append(time.perf_counter() - t0)
            native.call("aljabr_blackwell_unregister_model_buffer", ctypes.c_void_p(buf.ctypes.data))
        out["model_upload_1gib"] = {"first_GB/s": round(buf.nbytes / times[0] / 1e9, 1),
                                    "repeat_GB/s": round(buf.nbytes / min(times[1:]) / 1e9, 1),
                                    "how": "register_model_buffer: 32 MB chunks via two pinned bounce buffers, "
                                           "host copies on 4 threads overlapping the DMA"}
        del buf

    for name, fn in (("nf4", nf4_section), ("q8", q8_section), ("attention", attention_section),
                     ("kquant", kquant_section), ("c5", c5_section), ("prefill", prefill_section),
                     ("upload", upload_section)):
        if want(name):
            fn()
            torch.cuda.empty_cache()
    return out


def run_c5_tp(args, rank, world, dev, reps=20):
    """BASELINE config 5 at TP = world: one Llama-3-70B layer's NF4 weights
    (block 64) row-sharded over the ranks, each rank's batched NF4 GEMM on
    its rows (the batch-1 matvec at M = 1), and every projection's outputs
    all-gathered in rank order (tp_gemm.gather_token_rows: NCCL over NVLink).
    Device time per layer (CUDA events on the shared stream), max over
    ranks; weights rotate through a pool larger than 2 x L2 per rank."""
    import ctypes

    import torch

    from aljabr_b200 import native
    from aljabr_b200.tp_gemm import gather_token_rows

    L = native.lib()
    H, FF, G = 8192, 28672, 64
    full = {"q": (H, H), "k": (1024, H), "v": (1024, H), "o": (H, H), "gate": (FF, H), "up": (FF, H),
            "down": (H, FF)}
    shp = {n: (r // world, k) for n, (r, k) in full.items()}
    nweights = sum(r * k for r, k in full.values())
    wbytes = sum(n * k // 2 + n * k // G * 4 for n, k in shp.values())
    props = torch.cuda.get_device_properties(dev)
    l2 = getattr(props, "L2_cache_size", 126 * 2 ** 20) or 126 * 2 ** 20
    pool = max(1, int(np.ceil(2.5 * l2 / wbytes)))
    st = torch.cuda.Stream(device=dev)
    sh = ctypes.c_void_p(st.cuda_stream)
    gen = torch.Generator(device=dev)
    gen.manual_seed(50 + rank)
    raw, packed = [], []
    for _ in range(pool):
        lr, lp = {}, {}
        for name, (n, k) in shp.items():
            c = torch.randint(0, 256, (n * k // 2,), dtype=torch.uint8, device=dev, generator=gen)
            a = (0.05 + 0.005 * torch.randn(n * k // G, device=dev, generator=gen)).abs()
            pk = torch.empty(native.gemm_nf4_packed_size(n, k, G), dtype=torch.uint8, device=dev)
            torch.cuda.synchronize(dev)
            native.gemm_nf4_pack(pk.data_ptr(), c.data_ptr(), a.data_ptr(), n, k, G, sh.value)
            lr[name], lp[name] = (c, a), pk
        raw.append(lr)
        packed.append(lp)
    torch.cuda.synchronize(dev)
    groups = (("q", "k", "v"), ("o",), ("gate", "up"), ("down",))
    res = {}
    for M in [int(v) for v in getattr(args, "c5_tokens", "1,16,64,512").split(",")]:
        xh = torch.randn(M, H, device=dev).to(torch.bfloat16)
        xf = torch.randn(M, FF, device=dev).to(torch.bfloat16)
        ys = {name: torch.empty(M * n, device=dev) for name, (n, _) in shp.items()}
        wsb = max(native.gemm_nf4_workspace_size(M, H, [shp["q"][0], shp["k"][0], shp["v"][0]]),
                  native.gemm_nf4_workspace_size(M, H, [shp["gate"][0], shp["up"][0]]),
                  native.gemm_nf4_workspace_size(M, FF, [shp["down"][0]]))
        ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
        xh32, xf32 = xh.float().reshape(-1), xf.float().reshape(-1)

        def layer(i):
            lay = packed[i % pool]
            for names in groups:
                x, k = (xf, FF) if names == ("down",) else (xh, H)
                if M == 1:
                    for nm in names:
                        c, a = raw[i % pool][nm]
                        native.check(L.aljabr_blackwell_matvec_dev(
                            native.TYPE_NF4, ys[nm].data_ptr(), (xf32 if k == FF else xh32).data_ptr(), c.data_ptr(),
                            ctypes.c_void_p(a.data_ptr()), k, shp[nm][0], G, None, sh))
                else:
                    native.gemm_nf4_dev([ys[nm].data_ptr() for nm in names], [shp[nm][0] for nm in names],
                                        [lay[nm].data_ptr() for nm in names], [shp[nm][0] for nm in names],
                                        x.data_ptr(), M, k, G, ws.data_ptr(), wsb, sh.value)
                for nm in names:
                    gather_token_rows(ys[nm].view(M, shp[nm][0]), world)

        with torch.cuda.stream(st):
            for i in range(3):
                layer(i)
        torch.cuda.synchronize(dev)
        # one CUDA graph of `pool` layers (GEMMs and NCCL gathers), replayed;
        # eager launches if this torch / NCCL cannot capture the collectives
        graph, graphed = None, False
        try:
            torch.distributed.barrier()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=st):
                for i in range(pool):
                    layer(i)
            graphed = True
        except Exception:
            graph = None
        torch.cuda.synchronize(dev)
        torch.distributed.barrier()
        n = max(1, reps // pool) if graphed else reps
        with torch.cuda.stream(st):
            if graphed:
                graph.replay()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(st)
            for i in range(n):
                if graphed:
                    graph.replay()
                else:
                    layer(i)
            e.record(st)
        torch.cuda.synchronize(dev)
        layers = n * pool if graphed else n
        t = torch.tensor([s.elapsed_time(e) / layers], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
        res[f"M{M}"] = {"us_per_layer": round(ms * 1e3, 2), "TFLOP/s_whole_job": round(2.0 * M * nweights / (ms * 1e9), 1),
                        "weight_GB/s_per_gpu": round(wbytes / (ms * 1e6), 1), "all_gathers_per_layer": 7,
                        "launch": "CUDA graph" if graphed else "eager (graph capture of the collectives failed)"}
        del graph   # graphs holding NCCL calls go before the process group does
        del ys, ws
        torch.cuda.empty_cache()
    return {"tp": world, "per_gpu_weight_bytes": wbytes, "pool_layers": pool,
            "exchange": "torch.distributed.all_gather (NCCL) of every projection's outputs", "tokens": res}


def ctypes_ptr(t):
    import ctypes
    return ctypes.c_void_p(t.data_ptr())


def run_decode(args, rank, world, dev, tokens_per_run=32, runs=4):
    """Llama-3-8B-shaped NF4 decode tok/s at TP = world.

    Synthetic weights on the device: uniform random NF4 codes (the NF4
    levels are equiprobable for normal weights by construction) and absmax
    ~ |N(0.05, 0.005)|; bf16 KV cache pre-filled with N(0,1) to 4096
    positions; each run greedily decodes `tokens_per_run` tokens at
    positions 4064..4095 entirely on the device (one CUDA graph per token)."""
    import torch

    from aljabr_b200.decode import LLAMA3_8B, LlamaNf4Decoder, nccl_unique_id

    s = LLAMA3_8B
    nid = None
    if world > 1:
        obj = [nccl_unique_id() if rank == 0 else None]
        torch.distributed.broadcast_object_list(obj, src=0)
        nid = obj[0]
    from aljabr_b200 import native
    wkind = getattr(args, "decode_weights", "nf4")
    if wkind != "nf4" and world > 1:
        raise SystemExit("GGUF-typed decode weights run on one GPU (tensor parallel decode is NF4)")
    dec = LlamaNf4Decoder(s, tp_world=world, tp_rank=rank, nccl_id=nid)
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    keep = []
    # GGUF blocks: (bytes, values, [(byte offset of an fp16 scale, its bits)]);
    # random code bytes, fixed small scales (every code pattern is valid).
    gguf_layout = {native.TYPE_Q4_0: (18, 32, [(0, 0x1C00)]), native.TYPE_Q8_0: (34, 32, [(0, 0x1400)]),
                   native.TYPE_Q4_K: (144, 256, [(0, 0x0800), (2, 0x0C00)]),
                   native.TYPE_Q6_K: (210, 256, [(208, 0x0200)])}
    if wkind == "q4_0":
        layer_types = [native.TYPE_Q4_0] * 7
        embd_type = head_type = native.TYPE_Q4_0
    else:   # llama.cpp's Q4_K_M mix: Q4_K, with Q6_K for attn_v, ffn_down and the output matrix
        T4, T6 = native.TYPE_Q4_K, native.TYPE_Q6_K
        layer_types = [T4, T4, T6, T4, T4, T4, T6]
        embd_type, head_type = T4, T6

    def gguf(t, rows, cols):
        bb, per, scales = gguf_layout[t]
        nblk = rows * cols // per
        w = torch.randint(0, 256, (nblk * bb,), dtype=torch.uint8, device=dev, generator=g)
        v = w.view(nblk, bb)
        for off, bits in scales:
            v[:, off], v[:, off + 1] = bits & 0xFF, bits >> 8
        keep.append(w)
        return w.data_ptr(), w.numel()

    def nf4(rows, cols):
        c = torch.randint(0, 256, (rows * cols // 2,), dtype=torch.uint8, device=dev, generator=g)
        a = (0.05 + 0.005 * torch.randn(rows * cols // s.group, device=dev, generator=g)).abs()
        keep.extend([c, a])
        return c.data_ptr(), a.data_ptr()

    H = s.hidden
    weight_bytes = 0
    for layer in range(s.layers if wkind != "nf4" else 0):
        ws = []
        for n, t in zip(("q", "k", "v", "o", "gate", "up", "down"), layer_types):
            p, nb = gguf(t, s.rows(n), s.cols(n))
            ws.append(p)
            weight_bytes += nb
        norm = np.ones(H, np.float32)
        dec.register_layer_typed(layer, ws, layer_types, norm, norm)
    if wkind != "nf4":
        ep, _ = gguf(embd_type, s.vocab, H)
        hp, nb = gguf(head_type, s.vocab, H)
        weight_bytes += nb
        dec.register_output_typed(ep, embd_type, hp, head_type, np.ones(H, np.float32))
    for layer in range(s.layers if wkind == "nf4" else 0):
        cs, As = [], []
        for n in ("q", "k", "v", "o", "gate", "up", "down"):
            rows = s.rows(n) // world
            c, a = nf4(rows, s.cols(n))
            weight_bytes += rows * s.cols(n) // 2 + rows * s.cols(n) // s.group * 4
            cs.append(c)
            As.append(a)
        norm = np.ones(H, np.float32)
        dec.register_layer(layer, cs, As, norm, norm)
    if wkind == "nf4":
        ec, ea = nf4(s.vocab, H)
        hc, ha = nf4(s.vocab // world, H)
        weight_bytes += (s.vocab // world) * H // 2 + (s.vocab // world) * H // s.group * 4
        dec.register_output(ec, ea, hc, ha, np.ones(H, np.float32))
    kvd = s.kv_heads // world * s.head_dim
    for layer in range(s.layers):
        k = torch.randn(s.max_ctx, kvd, device=dev, generator=g).to(torch.bfloat16)
        v = torch.randn(s.max_ctx, kvd, device=dev, generator=g).to(torch.bfloat16)
        dec.sync_kv_cache(layer, s.max_ctx, k, v)
        del k, v
    torch.cuda.synchronize(dev)
    pos0 = s.max_ctx - tokens_per_run
    dec.run(1, pos0, tokens_per_run)            # eager step, graph capture, warm-up
    dec.run(1, pos0, tokens_per_run)
    if world > 1:
        torch.distributed.barrier()
    t0 = time.perf_counter()
    for _ in range(runs):
        dec.run(1, pos0, tokens_per_run)
    dt = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([dt], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        dt = float(t.item())
    n = runs * tokens_per_run
    # e2e: host-driven token loop through decode_step_token (H2D token, D2H argmax per token)
    tok = 1
    t1 = time.perf_counter()
    for i in range(tokens_per_run):
        tok, _ = dec.step(tok, pos0 + i)
    dt_e2e = time.perf_counter() - t1
    if world > 1:
        t = torch.tensor([dt_e2e], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        dt_e2e = float(t.item())
    dec.close()
    kv_bytes = s.layers * (s.max_ctx - tokens_per_run // 2) * kvd * 2 * 2
    per_gpu = weight_bytes + kv_bytes
    tok_s = n / dt
    peak, _ = load_peaks()
    return {"tok_per_s": round(tok_s, 1), "ms_per_token": round(dt * 1e3 / n, 4), "tp": world,
            "bytes_per_token_per_gpu": per_gpu, "achieved_GB/s_per_gpu": round(per_gpu * tok_s / 1e9, 1),
            "hbm_frac_of_measured_peak": round(per_gpu * tok_s / 1e9 / peak, 4),
            "e2e_tok_per_s": round(tokens_per_run / dt_e2e, 1),
            "timer": "host wall clock around decode_run (32-token greedy runs, one sync each); max over ranks",
            "weights": wkind,
            "config": "Llama-3-8B shape, " + {"nf4": "NF4 b64 linear + lm_head + embedding",
                                               "q4_0": "GGUF Q4_0 linear + lm_head + embedding",
                                               "q4_k_m": "GGUF Q4_K linear + embedding, Q6_K attn_v / ffn_down / "
                                                         "lm_head (llama.cpp Q4_K_M mix)"}[wkind]
                      + ", bf16 KV ctx 4096, random weights"}


# ----------------------------------------------------------------- CPU legs
def cpu_baseline(args, seconds: float):
    """The C restatement of the reference's Q4_0 row kernels
    (GgufQ32RawDot.dotRowQ4_0 with GgufRows' 2-chunks-per-thread split) on
    the host cores, over a bounded sample of the same workload."""
    import oracle
    threads = os.cpu_count() or 1
    g = np.random.default_rng(99)
    up = oracle.encode_q4_0(g.normal(0, 0.02, size=(UP_N, UP_K)).astype(np.float32))
    dn = oracle.encode_q4_0(g.normal(0, 0.02, size=(DOWN_N, DOWN_K)).astype(np.float32))
    xu = g.normal(size=UP_K).astype(np.float32)
    xd = g.normal(size=DOWN_K).astype(np.float32)
    oracle.matvec_q4_0(up, xu, UP_N, threads=threads)
    n = 0
    t0 = time.perf_counter()
    while True:
        oracle.matvec_q4_0(up, xu, UP_N, threads=threads)
        oracle.matvec_q4_0(dn, xd, DOWN_N, threads=threads)
        n += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": round(STEP_BYTES * n / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} up+down step(s) of the headline workload in {dt:.1f} s "
                      "(C restatement of GgufQ32RawDot.dotRowQ4_0, rows in 2 chunks per thread)"}


def run_reference(args, rank, world):
    if rank != 0:
        return None
    import oracle
    oracle.build()
    threads = os.cpu_count() or 1
    g = np.random.default_rng(99)
    up = oracle.encode_q4_0(g.normal(0, 0.02, size=(UP_N, UP_K)).astype(np.float32))
    dn = oracle.encode_q4_0(g.normal(0, 0.02, size=(DOWN_N, DOWN_K)).astype(np.float32))
    xu = g.normal(size=UP_K).astype(np.float32)
    xd = g.normal(size=DOWN_K).astype(np.float32)
    for _ in range(args.warmup):
        oracle.matvec_q4_0(up, xu, UP_N, threads=threads)
        oracle.matvec_q4_0(dn, xd, DOWN_N, threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.matvec_q4_0(up, xu, UP_N, threads=threads)
        oracle.matvec_q4_0(dn, xd, DOWN_N, threads=threads)
    dt = time.perf_counter() - t0
    v = STEP_BYTES * args.steps / dt / 1e9
    sample = (f"{args.steps} steps of the headline workload (one up 14336x4096 + one down 4096x14336 Q4_0 "
              f"matvec each) on {threads} host threads")
    return {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3 / args.steps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "q4_0 codes, fp16 scales -> f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "batch": 1},
            "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": sample,
                             "note": "C restatement of the reference's Java CPU kernels; the Java reference "
                                     "itself cannot run here (no JDK on these hosts)"},
            "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_only(args, rank, world, local_rank):
    import ctypes

    import torch

    from aljabr_b200 import native
    torch.cuda.set_device(local_rank)
    native.call("aljabr_blackwell_init", local_rank)
    native.call("aljabr_blackwell_set_pdl", 0 if args.no_pdl else 1)
    dev = torch.device("cuda", local_rank)
    if args.only == "decode":
        return {"only": "decode", **run_decode(args, rank, world, dev, tokens_per_run=args.decode_tokens, runs=1)}
    if args.only == "c5tp":
        if world < 2:
            return {"only": "c5tp", "skipped": "needs torchrun with 2 or more ranks"}
        return {"only": "c5tp", **run_c5_tp(args, rank, world, dev)}
    props = torch.cuda.get_device_properties(local_rank)
    l2 = getattr(props, "L2_cache_size", 126 * 2 ** 20) or 126 * 2 ** 20
    stream = torch.cuda.Stream(device=dev)
    out = run_extra(args, dev, stream, ctypes.c_void_p(stream.cuda_stream), l2, which={args.only},
                    reps=max(1, args.steps))
    return {"only": args.only, **out}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-extra", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-pdl", action="store_true")
    ap.add_argument("--no-prefetch", action="store_true", help="no L2 prefetch hints between the headline launches")
    ap.add_argument("--only", choices=["nf4", "q8", "attention", "decode", "c5", "kquant", "prefill", "upload",
                                       "c5tp"],
                    help="run one secondary workload alone (for profiling); prints its dict")
    ap.add_argument("--decode-tokens", type=int, default=32)
    ap.add_argument("--decode-weights", default="nf4", choices=["nf4", "q4_0", "q4_k_m"],
                    help="weight formats of the --only decode model (GGUF types on one GPU only)")
    ap.add_argument("--c5-tokens", default="1,16,64,512",
                    help="token counts of the batched-NF4 (C5) section, comma separated")
    ap.add_argument("--prefill-tokens", default="16,64,512",
                    help="prompt lengths of the Q4_0 prefill section, comma separated")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    if world > 1:
        import datetime

        import torch
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local_rank))
    if args.only:
        line = run_only(args, rank, world, local_rank)
    else:
        line = run_ours(args, rank, world, local_rank)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
