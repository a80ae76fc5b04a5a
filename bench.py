"""Benchmark of the decode hot path (metric: decode tok/s at batch 1 and
batch 64 on 1/2/4/8 GPUs; Q4_K GEMV HBM GB/s against the measured peak).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl g4|reference]
                    [--workload batch64|batch1|gemv0|kernel-q4|kernel-q6|kernel-gemv|kernel-attn]

Workloads (seeded synthetic data with the shapes of the reference's
configurations; random-init Gemma-4-E4B-shaped Q4_K_M model, no network, no
real GGUF):
  batch64  64 independent sequences with a 4096-token context, then greedy
           decode.  The prompt's KV rows are filled from a seed (--prefill
           fill; a decode step's work does not depend on them) and the last
           prompt token runs through the model; --prefill run decodes the
           whole prompt.  The 64 sequences are sharded over the N ranks (one
           process per GPU, no collective on the data path) -> "scaling":
           "strong".
  batch1   one sequence, 512-token prompt, 128 greedy tokens.
  gemv0    the single Q4_K 10240 x 2560 GEMV alone.
  kernel-* one kernel family on a small case (a few GB on the device), for
           profiler captures: q4 / q6 = the Q4_K gate/up and Q6_K down shapes
           at 64 sequences on the tensor cores, gemv = Q4_K 10240 x 2560 at
           batch 1, attn = a six-layer E4B-shaped model decoding 64 sequences
           at context 2048.
A step is one decode position for all local sequences.  `value` is whole-job
tokens/s with token ids and weights already in HBM (greedy feedback on the
device, CUDA-graph replay); `e2e` is the same metric through the public C-ABI
call g4_decode_batch with host token buffers (H2D + D2H every step).

Extras on rank 0 of the default run: the roofline of the dominant kernel
(batch >= 16: decode attention, timed live with CUDA events on the engine
stream over the engine's own layers; batch 1: the K-quant GEMV over one
layer's matrices), the tensor-core GEMM and whole-step rooflines with the
step's time shares, the single Q4_K GEMV, the `batch1` block (batch-1 decode
of the same model, its step roofline and e2e through g4_forward), GPU and
reference-CPU timings of the single GEMV, one layer's GEMVs and the decode
attention, and the reference CPU path (gemma4-4b/cpu-blas/main.c compiled
unchanged, OpenMP on all host cores) on a bounded sample of the workload.
"""
from __future__ import annotations

import argparse
import ctypes as C
import importlib.util
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "gemma4.c_b200")


def load_pkg():
    if "g4b200" in sys.modules:
        return sys.modules["g4b200"]
    spec = importlib.util.spec_from_file_location("g4b200", os.path.join(PKG, "__init__.py"),
                                                  submodule_search_locations=[PKG])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["g4b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled during a region:
    NVML every 20 ms (read-only queries), else nvidia-smi every 200 ms."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits, in the order of the summary's names
    BITS = (0x8, 0x40, 0x20, 0x4)  # hw_slowdown, hw_thermal_slowdown, sw_thermal_slowdown, sw_power_cap

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.rows = []
        self._stop = threading.Event()
        self._t = None

    def _run_nvml(self) -> bool:
        try:
            import pynvml as N
            N.nvmlInit()
        except Exception:
            return False
        try:
            h = N.nvmlDeviceGetHandleByIndex(self.idx)
            mx = N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM)
            get_reasons = getattr(N, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                N.nvmlDeviceGetCurrentClocksThrottleReasons
            while not self._stop.is_set():
                sm = N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM)
                rs = get_reasons(h)
                self.rows.append([str(self.idx), str(sm), str(mx), "", hex(rs)] +
                                 ["Active" if rs & b else "Not Active" for b in self.BITS])
                self._stop.wait(0.02)
            return True
        except Exception:
            return bool(self.rows)
        finally:
            try:
                N.nvmlShutdown()
            except Exception:
                pass

    def _run(self):
        if self._run_nvml():
            return
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.idx), "--query-gpu=" + self.Q,
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                if out.returncode == 0 and out.stdout.strip():
                    self.rows.append([c.strip() for c in out.stdout.strip().split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4)
                          if len(r) > 5 + i and r[5 + i].strip().lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ---------------------------------------------------------------- distributed plumbing
def shard(seqs: int, world: int, rank: int) -> range:
    """The sequences of `rank`: an even split of `seqs` independent sequences
    over `world` ranks (each rank decodes its share with its own weight
    replica; no collective on the data path)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank %d of world %d" % (rank, world))
    if seqs % world:
        raise ValueError("%d sequences do not divide evenly over %d ranks" % (seqs, world))
    b = seqs // world
    return range(rank * b, (rank + 1) * b)


class Dist:
    """One process per GPU (torchrun env), NCCL for the barrier and the
    max-over-ranks time; backend "gloo" runs the same host logic on CPU."""

    def __init__(self, n_gpus: int, backend: str = "nccl"):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.backend = backend
        self.pg = None
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist
            if backend == "nccl":
                torch.cuda.set_device(self.local)
                dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                        device_id=torch.device("cuda", self.local))
            else:
                dist.init_process_group(backend, timeout=datetime.timedelta(seconds=60))
            self.pg = dist
        if n_gpus != self.world and self.world > 1:
            raise SystemExit("--gpus %d but WORLD_SIZE=%d" % (n_gpus, self.world))

    def barrier(self):
        if self.pg:
            import torch
            if self.backend == "nccl":
                self.pg.barrier(device_ids=[self.local])
                torch.cuda.synchronize()
            else:
                self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device="cuda" if self.backend == "nccl" else "cpu")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


# ---------------------------------------------------------------- reference CPU path
def reference_sample(g4, model, ctx: int, n_steps: int, threads: int, warmup: int = 1):
    """Time the reference forward() (main.c compiled unchanged) for n_steps
    greedy decode positions of one sequence at context `ctx` (KV rows [0, ctx)
    filled with seeded values first), after `warmup` untimed positions (the
    first pages in the weights).  Returns (tok/s, seconds, threads, blas)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    if not oracle.have_reference():
        return None
    warmup = max(1, warmup)
    ref = oracle.Reference(threads=threads)
    rm = ref.model(model.desc(), ctx + warmup + n_steps + 2)
    rm.fill_kv(ctx, seed=7)
    tok = 1
    for i in range(warmup):
        rm.forward(tok, ctx + i, 1)
        tok = ref.sample_greedy(rm.logits())
    t0 = time.perf_counter()
    for i in range(n_steps):
        rm.forward(tok, ctx + warmup + i, 1)
        tok = ref.sample_greedy(rm.logits())
    dt = time.perf_counter() - t0
    rm.close()
    return n_steps / dt, dt, ref.max_threads, ref.blas


# ---------------------------------------------------------------- attention roofline
# DRAM bytes (read + write) per launch over the algorithmic K/V bytes, from
# one ncu capture of each layer kind in the batch-64 E4B case
# (bench.py --workload kernel-attn; profiles/attn_stream_e4b_b64.md):
# sliding (135.39 + 7.69) MB / 134.22 MB (four 64-row splits per CTA),
# global at context 2048 (537.72 + 10.62) MB / 536.87 MB.  The excess is the
# split partials and the new K/V rows.
ATTN_TRAFFIC_RATIO = {"sliding": 1.0661, "global": 1.0214}


def attention_roofline(eng, shape, B: int, pos: int, reps: int = 4):
    """Decode attention (attn_stream_kernel) of the engine's own layers at the
    current position, timed with CUDA events on the engine stream.  Sliding
    and global layers are timed separately (five sliding layers in rotation so
    that their 5 x 134 MB of K/V exceed L2) and combined with the step's mix
    of layer kinds.  Algorithmic bytes per launch = the K and V rows read:
    B * n_kv * nwin * hd * 4 B * 2."""
    S_ = sys.modules["g4b200"].synth
    swa = [l for l in range(shape.n_layers) if S_.is_swa(shape, l)]
    glob = [l for l in range(shape.n_layers) if not S_.is_swa(shape, l)]
    nwin_s = min(pos + 1, shape.sliding_window)
    nwin_g = pos + 1
    by_s = B * shape.n_kv_heads * nwin_s * shape.head_dim_swa * 8
    by_g = B * shape.n_kv_heads * nwin_g * shape.head_dim_full * 8
    ts = eng.time_attention(swa[:5], B, reps) / (reps * min(5, len(swa)))
    tg = eng.time_attention(glob[:2], B, reps) / (reps * min(2, len(glob)))
    step_bytes = len(swa) * by_s + len(glob) * by_g
    step_traffic = ATTN_TRAFFIC_RATIO["sliding"] * len(swa) * by_s + ATTN_TRAFFIC_RATIO["global"] * len(glob) * by_g
    step_ms = len(swa) * ts + len(glob) * tg
    return {"sliding": {"us_per_launch": 1e3 * ts, "bytes_per_launch": by_s, "gbs": by_s / (ts * 1e-3) / 1e9,
                        "launches_per_step": len(swa)},
            "global": {"us_per_launch": 1e3 * tg, "bytes_per_launch": by_g, "gbs": by_g / (tg * 1e-3) / 1e9,
                       "launches_per_step": len(glob)},
            "step_ms": step_ms, "step_bytes": step_bytes, "step_traffic_bytes": step_traffic,
            "gbs": step_bytes / (step_ms * 1e-3) / 1e9}


# ---------------------------------------------------------------- GEMV roofline
def _graph_time(fn, reps: int, stream_holder):
    """Capture fn() (which enqueues kernels on the torch current stream) into a
    CUDA graph and time `reps` replays with CUDA events; returns ms per replay.
    Timing graph replays keeps host launch overhead out of kernel timings."""
    import torch
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        fn(s.cuda_stream)           # warm-up outside capture
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            fn(s.cuda_stream)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(reps):
            g.replay()
        e1.record(s)
        e1.synchronize()
    del g
    return e0.elapsed_time(e1) / reps


def gemv_roofline(g4, B: int, reps: int = 10):
    """The K-quant GEMV kernel over one decoder layer's matrices at the Q4_K_M
    mix (Q 2048x2560, K 512x2560 Q4_K; V 512x2560 Q6_K; O 2560x2048, gate/up
    10240x2560 Q4_K; down 2560x10240 Q6_K) at batch B,
    weights rotated over enough copies to exceed L2, timed as CUDA-graph
    replays with CUDA events."""
    import torch
    S = g4.synth
    rng = np.random.default_rng(1)
    mats = [("q", S.Q4_K, 2048, 2560), ("k", S.Q4_K, 512, 2560), ("v", S.Q6_K, 512, 2560),
            ("o", S.Q4_K, 2560, 2048), ("gate", S.Q4_K, 10240, 2560), ("up", S.Q4_K, 10240, 2560),
            ("down", S.Q6_K, 2560, 10240)]
    layer_bytes = sum(S.row_bytes(t, n) * r for _, t, r, n in mats)
    copies = max(2, int(np.ceil(300e6 / layer_bytes)))
    dev = []
    for c in range(copies):
        dev.append([(nm, t, r, n, g4.weight_upload(S._qmat(rng, t, r, n, 0.02), t, n, r)) for nm, t, r, n in mats])
    nmax = 10240
    x = torch.randn(B, nmax, device="cuda", dtype=torch.float32)
    o = torch.empty(B, 10240, device="cuda", dtype=torch.float32)
    q8 = torch.empty(B * (nmax // 256) * 292, device="cuda", dtype=torch.uint8)
    g4.lib().g4d_quantize_row_q8_K(x.data_ptr(), q8.data_ptr(), 2560, B, None)
    torch.cuda.synchronize()
    res = {}
    for label, filt in (("layer", None), ("q4k_gate_up", ("gate", "up")), ("q6k_down", ("down",))):
        sel = [(nm, t, r, n) for nm, t, r, n in mats if filt is None or nm in filt]

        def run(stream, sel=sel, filt=filt):
            for ci in range(copies):
                for nm, t, r, n, w in dev[ci]:
                    if filt is None or nm in filt:
                        g4.mm_device(o.data_ptr(), x.data_ptr(), w, n, r, t, q8.data_ptr(), 1, B, stream)

        ms = _graph_time(run, reps, None)
        launches = copies * len(sel)
        byts = copies * sum(S.row_bytes(t, n) * r + B * (n * 4 + r * 4) for nm, t, r, n in sel)
        res[label] = {"us_per_launch": 1e3 * ms / launches, "bytes_per_launch": byts / launches,
                      "gbs": byts / (ms * 1e-3) / 1e9}
    for c in dev:
        for *_, w in c:
            g4.free(w)
    return res


def config0_gemv(g4, reps: int = 20, rows: int = 10240):
    """The single Q4_K 10240 x 2560 GEMV at batch 1 (activation
    quantized to Q8_K once), weights rotated over enough copies to exceed L2
    (20 copies = 295 MB), timed as CUDA-graph replays with CUDA events.
    `rows` > 10240 times the same kernel on a taller matrix."""
    import torch
    S = g4.synth
    copies = max(2, 20 * 10240 // rows)
    ws = []
    for c in range(copies):
        w, xh = S.config0_weights(seed=c, rows=rows)
        ws.append(g4.weight_upload(w, S.Q4_K, 2560, rows))
    x = torch.from_numpy(xh).cuda()
    o = torch.empty(rows, device="cuda", dtype=torch.float32)
    q8 = torch.empty(10 * 292, device="cuda", dtype=torch.uint8)
    g4.lib().g4d_quantize_row_q8_K(x.data_ptr(), q8.data_ptr(), 2560, 1, None)
    torch.cuda.synchronize()

    def run(stream):
        for w in ws:
            g4.mm_device(o.data_ptr(), x.data_ptr(), w, 2560, rows, S.Q4_K, q8.data_ptr(), 1, 1, stream)

    ms = _graph_time(run, reps, None) / copies
    byts = 1440 * rows + 2920 + 4 * rows
    for w in ws:
        g4.free(w)
    return {"us_per_gemv": ms * 1e3, "gbs": byts / (ms * 1e-3) / 1e9, "bytes": byts}


# ---------------------------------------------------------------- batch-1 decode
def batch1_decode(g4, model, prompt: int, new: int, dev: int):
    """Batch-1 greedy decode: the first `prompt`-1 positions prefilled in
    batches (g4_prefill, the lm_mode 0 forwards of main.c:2366-2402), the last
    prompt token through the model with the LM head, then `new` greedy tokens
    timed with CUDA events on the engine stream (argmax fed back on the
    device).  e2e: the same tokens through g4_forward with a host token in
    and the host argmax out every position (the drop-in for forward())."""
    import torch
    S = g4.synth
    eng = g4.Engine(model, dev, max_seq=prompt + 2 * new + 8, max_batch=1, prefill_rows=256)
    try:
        toks = np.random.default_rng(4321).integers(0, S.E4B.vocab_size, size=prompt).astype(np.int32)
        td = torch.from_numpy(toks).cuda()
        t0 = time.perf_counter()
        eng.prefill_prompts(toks[None, :], prompt - 1)
        eng.decode_batch_device(1, td.data_ptr() + 4 * (prompt - 1), prompt - 1, 1, None)
        eng.sync()
        prefill_s = time.perf_counter() - t0
        s = torch.cuda.ExternalStream(eng.stream())
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        pos = prompt
        for _ in range(3):  # warm-up (graph capture of the feedback step)
            eng.decode_batch_device(1, None, pos, 1, None)
            pos += 1
        eng.sync()
        e0.record(s)
        for _ in range(new):
            eng.decode_batch_device(1, None, pos, 1, None)
            pos += 1
        e1.record(s)
        e1.synchronize()
        ms = e0.elapsed_time(e1)
        nxt = eng.forward(1, pos, 2)
        pos += 1
        t0 = time.perf_counter()
        for _ in range(new):
            nxt = eng.forward(int(nxt), pos, 2)
            pos += 1
        e2e_s = time.perf_counter() - t0
    finally:
        eng.close()
    ctx = prompt + 3 + new // 2
    kv = sum(2 * model.shape.n_kv_heads * (model.shape.head_dim_swa if S.is_swa(model.shape, l)
                                           else model.shape.head_dim_full) * 4 *
             (min(ctx, model.shape.sliding_window) if S.is_swa(model.shape, l) else ctx)
             for l in range(model.shape.n_layers))
    byts = model.streamed_bytes(1) + kv
    hbm_peak, _, kind = measured_peaks()
    gbs = byts / (ms / new * 1e-3) / 1e9
    return {"workload": "batch-1 greedy decode, %d-token prompt run position by position, %d tokens timed" % (prompt, new),
            "value": new / (ms * 1e-3), "unit": "tok/s", "ms_per_token": ms / new, "prefill_s": prefill_s,
            "prefill_tok_s": prompt / prefill_s, "prefill": "batched (g4_prefill, 256 rows per call)",
            "step_roofline": {"bound": "hbm", "algorithmic_bytes_per_token": byts, "achieved": gbs,
                              "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak, "peak_kind": kind},
            "e2e": {"value": new / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4,
                    "api": "g4_forward (host token in, host argmax out, lm_mode 2), one call per position"}}


def gpu_attention_configs(g4, reps: int = 20):
    """Decode attention of one sequence (8 query / 2 KV heads, head dim 256)
    over a 512-row sliding window and an 8192-row global context, through
    g4d_attn_decode_noalloc on device buffers rotated over > 126 MB (L2)."""
    import ctypes as C_
    import torch
    L = g4.lib()
    res = {}
    for nwin in (512, 8192):
        per = 2 * 2 * nwin * 256 * 4
        copies = max(2, int(np.ceil(300e6 / per)))
        kv = [torch.randn(2, 2, nwin, 256, device="cuda") for _ in range(copies)]
        q = torch.randn(8 * 256, device="cuda") * 0.2
        out = torch.empty(8 * 256, device="cuda")

        def run(i):
            rc = L.g4d_attn_decode_noalloc(C_.c_void_p(out.data_ptr()), C_.c_void_p(q.data_ptr()),
                                           C_.c_void_p(kv[i % copies][0].data_ptr()),
                                           C_.c_void_p(kv[i % copies][1].data_ptr()), nwin, 8, 2, 256, None)
            assert rc == 0, g4.last_error()
        for i in range(3):
            run(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(reps):
            run(i)
        e1.record()
        e1.synchronize()
        us = 1e3 * e0.elapsed_time(e1) / reps
        res["window_%d" % nwin] = {"us": us, "kv_bytes": per, "gbs": per / (us * 1e-6) / 1e9}
        del kv
    return res


def cpu_configs(g4, threads: int):
    """The reference's CPU path on the single-GEMV, one-layer and attention
    shapes: mm() of main.c (Q8_K quantization + AVX2 integer dots for Q4_K,
    fp32 dequant-dot for Q6_K, OpenMP rows) from oracle/_ref, median of 5
    after a warm-up; the decode attention block has no callable function in
    main.c (it is inline in forward, main.c:1909-1950), so it is timed on the
    C restatement (oracle/g4_oracle.c, one thread)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    if not oracle.have_reference():
        return None
    ref = oracle.Reference(threads=threads)
    orc = oracle.Oracle()
    S = g4.synth
    rng = np.random.default_rng(1)

    def med(fn, n=5):
        fn()
        ts = []
        for _ in range(n):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return float(np.median(ts))
    out = {"threads": ref.max_threads, "blas": ref.blas, "kind": "reference"}
    w0, x0 = S.config0_weights(seed=0)
    t = med(lambda: ref.mm(x0, w0, 2560, 10240, S.Q4_K))
    out["q4k_gemv_10240x2560"] = {"ms": 1e3 * t, "gbs": (w0.nbytes + 2920 + 40960) / t / 1e9}
    mats = [(S.Q4_K, 2048, 2560), (S.Q4_K, 512, 2560), (S.Q6_K, 512, 2560), (S.Q4_K, 2560, 2048),
            (S.Q4_K, 10240, 2560), (S.Q4_K, 10240, 2560), (S.Q6_K, 2560, 10240)]
    ws = [(S._qmat(rng, tt, r, n, 0.02), tt, r, n) for tt, r, n in mats]
    xs = {n: rng.standard_normal(n).astype(np.float32) for n in (2048, 2560, 10240)}
    t = med(lambda: [ref.mm(xs[n], w, n, r, tt) for w, tt, r, n in ws])
    lb = sum(w.nbytes for w, *_ in ws)
    out["layer_gemvs_q4km"] = {"ms": 1e3 * t, "weight_bytes": lb, "gbs": lb / t / 1e9}
    for nwin in (512, 8192):
        q = (rng.standard_normal(8 * 256) * 0.2).astype(np.float32)
        k = rng.standard_normal(nwin * 512).astype(np.float32)
        v = rng.standard_normal(nwin * 512).astype(np.float32)
        t = med(lambda: orc.attention(q, k, v, nwin, 512, 8, 2, 256))
        out["attention_window_%d" % nwin] = {"us": 1e6 * t, "kind": "port (C restatement, 1 thread)",
                                             "gbs": 2 * 2 * nwin * 256 * 4 / t / 1e9}
    return out


def kernel_case(g4, which: str, reps: int) -> dict:
    """One kernel family on a small case for profiler captures (see the module doc)."""
    import dataclasses

    import torch
    S = g4.synth
    if which == "attn":
        shape = dataclasses.replace(S.E4B, n_layers=6)
        m = S.make_model(shape, seed=3)
        B, ctx = 64, 2048
        eng = g4.Engine(m, 0, max_seq=ctx + reps + 8, max_batch=B)
        try:
            eng.fill_kv(ctx - 1, seed=5)
            toks = np.arange(B, dtype=np.int32) % shape.vocab_size
            t0 = time.perf_counter()
            for i in range(max(reps, 3)):
                toks = eng.decode_batch(toks, ctx - 1 + i, 1)
            eng.sync()
            dt = time.perf_counter() - t0
        finally:
            eng.close()
        return {"case": "attn", "steps": max(reps, 3), "s": dt}
    t, rows, n, B = {"q4": (S.Q4_K, 10240, 2560, 64), "q6": (S.Q6_K, 2560, 10240, 64),
                     "gemv": (S.Q4_K, 10240, 2560, 1)}[which]
    copies = max(2, int(np.ceil(300e6 / (S.row_bytes(t, n) * rows))))
    rng = np.random.default_rng(1)
    ws = [g4.weight_upload(S.rand_blocks(rng, t, rows, n, 1e-3, 2e-2), t, n, rows) for _ in range(copies)]
    st = torch.cuda.current_stream().cuda_stream
    x = torch.randn(B, n, device="cuda")
    q8 = torch.zeros(B * (n // 256) * 292, dtype=torch.uint8, device="cuda")
    o = torch.zeros(B, rows, device="cuda")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(reps):
        g4.mm_device(o.data_ptr(), x.data_ptr(), ws[i % copies], n, rows, t, q8.data_ptr(), 0, B, st)
    e1.record()
    e1.synchronize()
    for w in ws:
        g4.free(w)
    assert torch.isfinite(o).all().item()
    return {"case": which, "launches": reps, "us_per_call": 1e3 * e0.elapsed_time(e1) / max(reps, 1)}


# ---------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="g4", choices=["g4", "reference"])
    ap.add_argument("--workload", default="batch64",
                    choices=["batch64", "batch1", "gemv0", "kernel-q4", "kernel-q6", "kernel-gemv", "kernel-attn"])
    ap.add_argument("--seqs", type=int, default=None, help="total sequences (default 64 / 1)")
    ap.add_argument("--prompt", type=int, default=None, help="prompt tokens (default 4096 / 512)")
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--prefill", default=None, choices=["run", "fill", "batched"],
                    help="run: decode the prompt position by position; fill: seeded KV rows for the prompt; "
                         "batched: g4_prefill over all sequences (default: fill for batch64, batched for batch1)")
    ap.add_argument("--prefill-sample", type=int, default=512,
                    help="batch64 extras: prompt positions per sequence of the timed batched-prefill sample")
    ap.add_argument("--cpu-steps", type=int, default=6)
    ap.add_argument("--gemv-rows", type=int, default=10240, help="gemv0 workload: matrix rows")
    ap.add_argument("--tc-min", type=int, default=None, help="engine tensor-core batch threshold")
    ap.add_argument("--attn-split", default=None,
                    help="attention rows per CTA 'sliding,global' (multiples of 32; default 128,256)")
    ap.add_argument("--lm-split", action="store_true",
                    help="N > 1: row-split the tied LM head over the ranks (NCCL all-gathers of the hidden "
                         "states and of one argmax key per sequence)")
    a = ap.parse_args()
    if a.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    seqs = a.seqs or (64 if a.workload == "batch64" else 1)
    prompt = a.prompt or (4096 if a.workload == "batch64" else 512)
    g4 = load_pkg()
    S = g4.synth
    metric = "decode tok/s"
    cfg = {"workload": ("batched greedy decode, %d sequences at context %d" % (seqs, prompt)) if a.workload == "batch64"
           else "batch-1 greedy decode after a %d-token prompt" % prompt,
           "model": "Gemma-4-E4B-shaped Q4_K_M (random init, 42 layers, d 2560, ffn 10240, 8:2 GQA, hd 256, "
                    "vocab 262144, tied Q6_K head)",
           "sequences": seqs, "prompt_tokens": prompt, "global_batch": seqs, "seq_len": prompt,
           "parallelism": "sequence shards (dp%d), no collective" % a.gpus,
           "l2": "no flush needed: each step streams 3.2 GB of weights (> 126 MB L2)"}

    if a.workload.startswith("kernel-"):  # profiler cases: one kernel family, small, exits 0
        import torch
        torch.cuda.set_device(0)
        if g4.lib().g4_set_device(0) != 0:
            raise SystemExit("g4_set_device(0) failed: %s" % (g4.last_error(),))
        r = kernel_case(g4, a.workload[len("kernel-"):], max(a.steps, 1))
        print(json.dumps({"kernel_case": r}))
        return
    if a.workload == "gemv0":  # the single Q4_K GEMV alone (used for kernel profiling)
        import torch
        torch.cuda.set_device(0)
        r = config0_gemv(g4, reps=max(a.steps, 1), rows=a.gemv_rows)
        hbm_peak, _, kind = measured_peaks()
        print(json.dumps({"metric": "Q4_K GEMV HBM GB/s", "value": r["gbs"], "unit": "GB/s", "n_gpus": 1,
                          "steps": a.steps, "warmup": a.warmup, "ms_per_step": r["us_per_gemv"] / 1e3,
                          "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8xint4",
                          "data": "synthetic", "config": {"workload": "Q4_K %dx2560 GEMV, batch 1" % a.gemv_rows},
                          "roofline": {"bound": "hbm", "achieved": r["gbs"], "peak": hbm_peak, "unit": "GB/s",
                                       "frac": r["gbs"] / hbm_peak, "peak_kind": kind, "traffic": None}}))
        return
    if a.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return
        threads = os.cpu_count() or 1
        model = S.make_model(S.E4B, seed=3)
        # one step = one greedy decode position of one sequence (the reference decodes the
        # sequences of the batch one after another): K timed steps after W untimed ones
        r = reference_sample(g4, model, prompt, max(1, a.steps), threads, a.warmup)
        if r is None:
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libg4ref.so was not built"}))
            return
        tps, dt, thr, blas = r
        print(json.dumps({"impl": "reference", "metric": metric, "value": tps, "unit": "tok/s", "n_gpus": a.gpus,
                          "steps": max(1, a.steps), "warmup": max(1, a.warmup), "ms_per_step": 1e3 * dt / max(1, a.steps),
                          "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8/fp32",
                          "data": "synthetic", "config": cfg,
                          "cpu_baseline": {"value": tps, "unit": "tok/s", "cores": thr, "kind": "reference",
                                           "sample": "%d greedy decode steps of one sequence at context %d "
                                                     "(reference processes sequences one by one; BLAS: %s)"
                                                     % (max(1, a.steps), prompt, blas)},
                          "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return

    dist = Dist(a.gpus)
    import torch
    torch.cuda.set_device(dist.local)
    try:
        mine_ids = shard(seqs, dist.world, dist.rank)
    except ValueError as ex:
        raise SystemExit(str(ex))
    B = len(mine_ids)
    model = S.make_model(S.E4B, seed=3)
    wbytes = model.weight_bytes()
    max_seq = prompt + a.warmup + a.steps * 2 + 8
    eng = g4.Engine(model, dist.local, max_seq=max_seq, max_batch=B, prefill_rows=256)
    if a.tc_min:
        eng.set_tc_min_batch(a.tc_min)
    if a.attn_split:
        sw, gl = (int(v) for v in a.attn_split.split(","))
        eng.set_attn_split(sw, gl)
        cfg["attn_split"] = [sw, gl]
    if a.lm_split and dist.world > 1:
        import torch.distributed as tdist
        box = [g4.nccl_unique_id() if dist.rank == 0 else None]
        tdist.broadcast_object_list(box, src=0)
        eng.lm_split(box[0], dist.rank, dist.world)
        cfg["lm_head"] = "row-split over %d ranks (NCCL all-gather of hidden states and argmax keys)" % dist.world
    model_keep = model  # host tensors stay alive until the end
    stream = eng.stream()
    # prompts: seeded per global sequence id
    rng = np.random.default_rng(1234)
    allp = rng.integers(0, S.E4B.vocab_size, size=(seqs, prompt), dtype=np.int32)
    mine = allp[mine_ids.start:mine_ids.stop]
    prompts_dev = torch.from_numpy(np.ascontiguousarray(mine.T)).cuda()  # [prompt][B]
    prefill = a.prefill or ("fill" if a.workload == "batch64" else "batched")
    cfg["prefill"] = prefill
    prefill_sample = None
    t0 = time.perf_counter()
    if prefill == "fill":  # KV rows of the prompt from a seed; the last prompt token runs for real
        eng.fill_kv(prompt - 1, seed=1234 + dist.rank)
        if not a.no_extras and dist.world == 1:
            # a timed batched-prefill sample: the first positions of every sequence's prompt through
            # g4_prefill (tensor-core GEMMs over 256 rows per call), over the seeded rows
            n = min(a.prefill_sample, prompt - 1)
            eng.sync()
            t1 = time.perf_counter()
            eng.prefill_prompts(mine, n)
            eng.sync()
            dt = time.perf_counter() - t1
            prefill_sample = {"tokens": n * B, "s": dt, "tok_s": n * B / dt,
                              "sample": "positions 0..%d of %d sequences through g4_prefill, 256 rows per call"
                                        % (n - 1, B)}
        eng.decode_batch_device(B, prompts_dev.data_ptr() + (prompt - 1) * B * 4, prompt - 1, 1, None)
    elif prefill == "batched":
        eng.prefill_prompts(mine, prompt - 1)
        eng.decode_batch_device(B, prompts_dev.data_ptr() + (prompt - 1) * B * 4, prompt - 1, 1, None)
    else:
        for pos in range(prompt):
            lm = 1 if pos == prompt - 1 else 0
            eng.decode_batch_device(B, prompts_dev.data_ptr() + pos * B * 4, pos, lm, None)
    eng.sync()
    prefill_s = time.perf_counter() - t0
    pos = prompt
    for _ in range(a.warmup):
        eng.decode_batch_device(B, None, pos, 1, None)
        pos += 1
    eng.sync()
    dist.barrier()
    s = torch.cuda.ExternalStream(stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dist.local) as clk:
        torch.cuda.synchronize()
        e0.record(s)
        for _ in range(a.steps):
            eng.decode_batch_device(B, None, pos, 1, None)
            pos += 1
        e1.record(s)
        e1.synchronize()
    ms = e0.elapsed_time(e1)
    kernels_per_step = eng.last_step_kernels()
    dist.barrier()
    ms_max = dist.max(ms)
    value = seqs * a.steps / (ms_max / 1e3)

    # e2e: the public C-ABI call with host token buffers, H2D + D2H inside each step
    toks = np.zeros(B, np.int32)
    nxt = eng.decode_batch(toks + 1, pos, 1)
    pos += 1
    dist.barrier()
    t0 = time.perf_counter()
    for _ in range(a.steps):
        nxt = eng.decode_batch(nxt, pos, 1)
        pos += 1
    e2e_s = dist.max(time.perf_counter() - t0)
    e2e = {"value": seqs * a.steps / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 4 * B,
           "d2h_bytes_per_step": 4 * B, "api": "g4_decode_batch (host token ids in, host next ids out)"}

    hbm_peak, tc_peak, peak_kind = measured_peaks()
    if B >= 2:  # the engine's tensor-core threshold (engine.cu tc_min_batch)
        dtype = ("tensor cores: Q4_K as exact fp16 integer products, Q5_K int8 x int8 -> int32, Q6_K int8 x int8 "
                 "-> int32 on 3-piece fixed-point activations; fp32 dense GEMV, attention, KV cache and norms")
    else:
        dtype = ("int8 x int4/int5 dp4a -> int32 (Q4_K/Q5_K x Q8_K), int8 dp4a on 3-piece fixed-point activations "
                 "(Q6_K), fp32 (dense, attention, norms)")
    out = {"metric": metric, "value": value, "unit": "tok/s", "n_gpus": a.gpus, "steps": a.steps,
           "warmup": a.warmup, "ms_per_step": ms_max / a.steps, "higher_is_better": True, "scaling": "strong",
           "vs_baseline": None, "dtype": dtype,
           "data": "synthetic (seeded random-init model and prompts)", "config": cfg,
           "e2e": e2e, "gpu_launches": int(kernels_per_step * a.steps),
           "kernels_per_step": kernels_per_step, "prefill_s": prefill_s, "prefill_sample": prefill_sample,
           "weights_gb": wbytes / 1e9, "clocks": clk.summary()}
    if dist.rank == 0 and not a.no_extras:
        rl = gemv_roofline(g4, B)
        lay = rl["layer"]
        gemm_kernel = ("tensor-core GEMMs gemm_q4tc_kernel / gemm_q6tc_kernel with their operand and merge kernels"
                       if B >= 16 else "gemv_tma_kernel (streaming K-quant GEMV)")
        gemm = {"kernel": gemm_kernel + ", one layer's matrices at batch %d" % B, "bound": "hbm",
                "achieved": lay["gbs"], "peak": hbm_peak, "unit": "GB/s", "frac": lay["gbs"] / hbm_peak,
                "peak_kind": peak_kind, "traffic": None, "algorithmic_bytes_per_launch": lay["bytes_per_launch"],
                "us_per_launch": lay["us_per_launch"], "parts": rl}
        if B >= 16:  # batched decode: attention over 64 x 4096 fp32 K/V rows is the dominant kernel
            at = attention_roofline(eng, S.E4B, B, pos - 1)
            nl = at["sliding"]["launches_per_step"] + at["global"]["launches_per_step"]
            out["roofline"] = {"kernel": "attn_stream_kernel (decode attention, %d sequences, context %d)"
                                         % (B, pos), "bound": "hbm", "achieved": at["gbs"], "peak": hbm_peak,
                               "unit": "GB/s", "frac": at["gbs"] / hbm_peak, "peak_kind": peak_kind,
                               "traffic": at["step_traffic_bytes"] / nl,
                               "algorithmic_bytes_per_launch": at["step_bytes"] / nl,
                               "us_per_launch": 1e3 * at["step_ms"] / nl, "parts": at}
            out["gemm_roofline"] = gemm
            # the whole step against HBM: the streamed weights once + every layer's K/V rows
            sb = model.streamed_bytes(B) + at["step_bytes"]
            out["step_roofline"] = {"bound": "hbm", "algorithmic_bytes_per_step": sb,
                                    "achieved": sb / (ms_max / a.steps * 1e-3) / 1e9, "peak": hbm_peak,
                                    "unit": "GB/s", "frac": sb / (ms_max / a.steps * 1e-3) / 1e9 / hbm_peak}
            # where the step's time goes: attention measured live; the rest is the weight GEMMs and their
            # operand / merge / norm launches (split by kernel in the launch-list summaries under profiles/)
            step_ms = ms_max / a.steps
            out["time_share"] = {"step_ms": step_ms, "attention_ms": at["step_ms"],
                                 "attention": at["step_ms"] / step_ms, "gemms_and_glue": 1.0 - at["step_ms"] / step_ms,
                                 "gemms_and_glue_gbs": model.streamed_bytes(B) / ((step_ms - at["step_ms"]) * 1e-3) / 1e9}
        else:
            out["roofline"] = gemm
        out["q4k_gemv_config0"] = config0_gemv(g4)
        out["q4k_gemv_config0"]["frac"] = out["q4k_gemv_config0"]["gbs"] / hbm_peak
        out["step_hbm_gbs"] = wbytes / (ms_max / a.steps * 1e-3) / 1e9
        if dist.world == 1:
            r = reference_sample(g4, model, prompt, a.cpu_steps, os.cpu_count() or 1)
            if r:
                tps, dt, thr, blas = r
                out["cpu_baseline"] = {"value": tps, "unit": "tok/s", "cores": thr, "kind": "reference",
                                       "sample": "%d greedy decode steps of one sequence at context %d, %.1f s "
                                                 "(BLAS: %s)" % (a.cpu_steps, prompt, dt, blas)}
    eng.close()
    if dist.rank == 0 and dist.world == 1 and not a.no_extras and a.workload == "batch64":
        # the batch-1 half of the metric on the same model, and the per-shape GPU / CPU timings
        b1 = batch1_decode(g4, model, 512, 128, dist.local)
        r = reference_sample(g4, model, 512, a.cpu_steps, os.cpu_count() or 1)
        if r:
            tps, dt, thr, blas = r
            b1["cpu_baseline"] = {"value": tps, "unit": "tok/s", "cores": thr, "kind": "reference",
                                  "sample": "%d greedy decode steps of one sequence at context 512, %.1f s; the "
                                            "reference's own decode formula (generated tokens / decode seconds, "
                                            "main.c:2279-2280) (BLAS: %s)" % (a.cpu_steps, dt, blas)}
        out["batch1"] = b1
        gl = gemv_roofline(g4, 1)["layer"]
        out["shapes_gpu"] = {"q4k_gemv_10240x2560_us": out.get("q4k_gemv_config0", {}).get("us_per_gemv"),
                             "layer_gemvs_batch1": {"us_per_matrix": gl["us_per_launch"], "gbs": gl["gbs"],
                                                    "frac": gl["gbs"] / hbm_peak},
                             "attention_batch1": gpu_attention_configs(g4)}
        out["shapes_cpu"] = cpu_configs(g4, os.cpu_count() or 1)
    del model_keep
    if dist.rank == 0:
        print(json.dumps(out))
    dist.close()


if __name__ == "__main__":
    main()
