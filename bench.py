#!/usr/bin/env python
"""Benchmark of the paged streaming hot path on B200.

Workload: one isolated paged-attention step of the
small model, bf16 - 80 streams x 17 layers, 8 heads of 64, chunk of 2 frames
over 70 cached left-context frames (window 72), 16-frame pages, the free
list a random permutation of the pool (seed 1), Q/K/V and the rel-pos
projection N(0,1)/8.  A step is three launches: step start (page allocator
and window descriptors) together with the rel-pos term of every (layer,
stream, head, query) (each layer's pos rows read once, not once per stream)
-> paged rel-pos attention for all 17 layers with the chunk's K/V append
fused in -> counter update (end).  ``--relpos prepass`` runs the rel-pos
term as its own launch (four launches), ``--relpos in-kernel`` inside the
attention kernel (three).
Streams are
independent, so N GPUs run N replicas with no collective on the data path
(weak scaling): each rank owns its own pool and streams, and the only
collectives are the timing barriers and one max-reduce of the timings.

Metric: paged-attn HBM GB/s = algorithmic bytes of the step / step time.
Algorithmic bytes per stream-layer (bf16): append 8,192 (read new K,V,
write K,V), attention 151,552 (read the 72-row K,V window, read Q, write O).

``--impl reference`` times the reference's algorithm for the same step on
the host cores (dense shift-append, index_select/index_copy_ pack/unpack,
Python mask loop, numpy attention; oracle/baseline.py) - the reference has
no GPU kernels for this path.
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

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "parakeet-streaming_b200"))

SHAPES = {
    "small": dict(layers=17, dim=512, heads=8, att=(70, 1)),
    "large": dict(layers=24, dim=1024, heads=8, att=(70, 13)),
}
PAGE = 16
# K/V page size of the serving engines: pages of 8 frames reserve 80 rows per
# stream for the small model's 72-frame window (16-frame pages: 96) and 96 for
# the large model's 84-frame window (112); the large model then runs the general
# bf16 attention kernel, which time allows at these loads
SERVE_PAGE = {"small": 8, "large": 8}
# share of the free HBM given to stream slots.  Large: 0.90 leaves about 9 GB
# beside the engine's 11 GB (measured).  Small: at 0.93 (60,160 slots) the step
# time, not memory, binds (p99 198 ms), so the cap stays where memory binds first
SLOT_HBM_SHARE = {"small": 0.85, "large": 0.90}


def alg_bytes(shape, es=2):
    """Algorithmic bytes per stream-layer of each op (element size es)."""
    c = SHAPES[shape]
    D, left, T = c["dim"], c["att"][0], c["att"][1] + 1
    W = left + T
    return {
        "append": 2 * (2 * T * D * es),
        "attention": 2 * W * D * es + 2 * T * D * es,
        "gather": 2 * (2 * W * D * es),
        "conv": (2 * 8 + 3 * T) * D * es,   # cache in/out, GLU input [T, 2D], output [T, D]
    }


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--model", choices=list(SHAPES), default="small")
    ap.add_argument("--streams", type=int, default=80)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-breakdown", action="store_true")
    ap.add_argument("--pipeline-streams", type=int, default=None,
                    help="streams of --profile-op streaming (default: the config's 160 / 480)")
    ap.add_argument("--relpos", choices=["fused", "prepass", "in-kernel"], default="fused",
                    help="rel-pos term: all-stream pre-pass in the step-start launch "
                         "(pk_pages_begin_step_relpos), as its own launch (pk_relpos_bd), or "
                         "inside the attention kernel")
    ap.add_argument("--no-serve", action="store_true",
                    help="skip the paced serving search (streams at p99 <= 160 ms)")
    ap.add_argument("--no-graph", action="store_true", help="time eager launches only")
    ap.add_argument("--no-reference-engine", action="store_true",
                    help="skip timing the reference's own engine in the serving search")
    ap.add_argument("--profile", action="store_true",
                    help="prefill + warmup + --steps steps only (for ncu), no report")
    ap.add_argument("--install-reference", metavar="CHECKOUT", default=None,
                    help="install the reference from a source checkout into baseline/_ref and exit")
    ap.add_argument("--wheelhouse", default=None, help="offline wheel directory for pip")
    ap.add_argument("--serve-page-small", type=int, choices=[8, 16], default=None,
                    help="K/V page size of the small model's serving engine (default 8)")
    ap.add_argument("--serve-page-large", type=int, choices=[8, 16], default=None,
                    help="K/V page size of the large model's serving engine (default 8)")
    ap.add_argument("--profile-op", default=None,
                    choices=["append", "attention", "attention+append", "gather",
                             "gather_all_layers", "conv", "features", "streaming", "gemm",
                             "scale_append", "scale_gather", "scale_attention+append",
                             "scale_conv"],
                    help="prefill + warmup, then --steps runs of one breakdown op (for ncu)")
    return ap.parse_args()


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def tensor_peak():
    """Measured dense bf16 TFLOP/s (burst: the GEMMs are timed alone)."""
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self._t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- reference arm
def workload_config(model, streams, world):
    """The ``config`` of both arms' JSON lines (the same workload)."""
    c = SHAPES[model]
    L, D, H, att = c["layers"], c["dim"], c["heads"], c["att"]
    T = att[1] + 1
    per = -(-(att[0] + T - 1) // PAGE) + 1        # pages a stream's window can touch
    pool_mb = streams * per * L * 2 * PAGE * D * 2 / 1e6
    b = alg_bytes(model)
    step_mb = (b["append"] + b["attention"]) * streams * L / 1e6
    return {"workload": f"configs[1] isolated paged-attention step, {model} model",
            "streams_per_gpu": streams, "layers": L, "heads": H, "head_dim": D // H,
            "chunk": T, "left_context": att[0], "page_size": PAGE,
            "page_order": "randperm seed 1",
            "l2": f"inputs > L2: {pool_mb:.0f} MB page pool, {step_mb:.0f} MB read+written "
                  f"per step",
            "parallelism": f"{world} independent replicas (stream sharding)"}


def install_reference(src, wheelhouse=None):
    """Installs the reference into baseline/_ref (git-ignored; it travels with
    the working tree to the GPU box).  pip first, offline; the reference
    builds with hatchling, which no offline wheelhouse here carries, so when
    pip cannot build it the install is what its wheel would hold: the
    reference's pure-Python ``parakeet`` package tree (pyproject's
    ``[tool.hatch.build.targets.wheel] packages = ["parakeet"]``), copied
    unmodified.  Returns the method used."""
    import shutil
    dst = os.path.join(REPO, "baseline", "_ref")
    os.makedirs(dst, exist_ok=True)
    cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
           "--no-deps", "--target", dst, src]
    if wheelhouse:
        cmd[4:4] = ["--find-links", wheelhouse]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode == 0:
        return "pip"
    shutil.copytree(os.path.join(src, "parakeet"), os.path.join(dst, "parakeet"),
                    ignore=shutil.ignore_patterns("__pycache__", "*.pyc"), dirs_exist_ok=True)
    last = (r.stderr or r.stdout).strip().splitlines()[-1:] or [""]
    return f"package tree copied (pip could not build offline: {last[0]})"


class ReferenceTorchStep:
    """configs[1]'s step through the reference's own code on the host cores
    (torch CPU, fp32), from the install under baseline/_ref: its ``Scheduler``
    (pack_states / unpack_states over a ``ModelCache`` slot pool,
    parakeet/engine/scheduler.py:68-201), ``ConformerEncoder._create_streaming_masks``
    (parakeet/modules/encoder.py:167-227), ``ConformerAttention.forward`` per
    layer (parakeet/modules/attention.py:85-125: ``update_attn_cache``,
    ``linear_pos``, ``rel_shift``, the masked fill and SDPA) and the counter
    update of encoder.py:257-260.  The step's Q/K/V are inputs here, so each
    layer's ``qkv`` projection is replaced by a module that hands the forward
    that layer's given rows, and ``linear_out`` by the identity (the metric's
    output is the attention output); everything between runs unmodified."""

    def __init__(self, num_layers, dim, heads, att_context, num_streams, seed=1):
        import torch
        from types import SimpleNamespace
        sys.path.insert(0, os.path.join(REPO, "baseline"))
        import harness
        harness.import_reference()
        from parakeet.engine.scheduler import Scheduler
        from parakeet.modules import ConformerAttention, ModelCache, PositionalEncoding
        from parakeet.modules.cache import StreamingState
        from parakeet.modules.encoder import ConformerEncoder

        self.torch = torch
        self.L, self.D, self.H, self.att, self.B = num_layers, dim, heads, att_context, num_streams
        self.T = att_context[1] + 1

        class Pool:                    # what init_state_pool asks of an encoder
            @staticmethod
            def init_streaming_state(batch_size, device, dtype):
                z = torch.zeros(batch_size, dtype=torch.int64)
                return StreamingState(ModelCache(num_layers, att_context, dim, 9, batch_size,
                                                 device, dtype), z, z.clone())

        self.sched = Scheduler(max_active=num_streams)
        self.sched.init_state_pool(Pool(), torch.device("cpu"), torch.float32, num_streams)
        self.seqs = [SimpleNamespace(encoder_state=self.sched.acquire_state_slot())
                     for _ in range(num_streams)]
        self.masks = lambda *a: ConformerEncoder._create_streaming_masks(
            SimpleNamespace(att_context_size=att_context), *a)
        g = torch.Generator().manual_seed(seed)
        s = (dim // heads) ** -0.5
        self.given = [None] * num_layers

        class Given(torch.nn.Module):   # hands forward() this layer's Q/K/V rows
            def __init__(self, owner, l):
                super().__init__()
                self.owner, self.l = owner, l

            def forward(self, x):
                return self.owner.given[self.l]

        self.attn = []
        for l in range(num_layers):
            a = ConformerAttention(l, heads, dim, use_bias=False)
            with torch.no_grad():
                a.linear_pos.weight.copy_(torch.randn(dim, dim, generator=g) * dim ** -0.5)
                a.pos_bias_u.copy_(torch.randn(heads, dim // heads, generator=g) * s)
                a.pos_bias_v.copy_(torch.randn(heads, dim // heads, generator=g) * s)
            a.qkv, a.linear_out = Given(self, l), torch.nn.Identity()
            self.attn.append(a.eval())
        pe = PositionalEncoding(dim, 0.0, 5000, 0.0)
        pe.extend_pe(5000, torch.device("cpu"))
        self.pos_enc = pe
        self.g = g

    def inputs(self):
        s = (self.D // self.H) ** -0.5
        return self.torch.randn(self.L, self.B, self.T, 3 * self.D, generator=self.g) * s

    def step(self, qkv, lengths=None):
        torch = self.torch
        T = self.T
        length = torch.full((self.B,), T, dtype=torch.int64) if lengths is None else lengths
        with torch.inference_mode():
            st, idx = self.sched.pack_states(self.seqs)
            x = torch.empty(self.B, T, self.D)
            x, pos_emb = self.pos_enc(x, cache_len=self.att[0])
            _, att_mask = self.masks(T, st.cache_lengths, st.processed_frames,
                                     torch.device("cpu"), length)
            out = []
            for l, a in enumerate(self.attn):
                self.given[l] = qkv[l]
                out.append(a(x, pos_emb, att_mask, st.cache))
            st.processed_frames.add_(length)
            st.cache_lengths.add_(length)
            st.cache_lengths.clamp_(max=self.att[0])
            self.sched.unpack_states(st, idx)
        return out


def reference_step_class():
    """The reference's own code (``ReferenceTorchStep``) when baseline/_ref
    holds it, else the float32 numpy restatement (oracle/baseline.py)."""
    sys.path.insert(0, os.path.join(REPO, "baseline"))
    import harness
    if harness.available():
        return ReferenceTorchStep, "reference"
    from oracle.baseline import ReferenceStep
    return ReferenceStep, "port"


def cpu_reference(args, seconds, steps=None):
    """Time the reference's step on the host cores (``reference_step_class``);
    returns (GB/s, steps, seconds, threads, sample, kind)."""
    cls, kind = reference_step_class()
    if kind == "reference":
        import torch
        torch.set_num_threads(os.cpu_count() or 1)
        threads = torch.get_num_threads()
    else:
        try:
            from threadpoolctl import threadpool_info
            threads = max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
        except Exception:
            threads = os.cpu_count() or 1
    c = SHAPES[args.model]
    ref = cls(c["layers"], c["dim"], c["heads"], c["att"], args.streams)
    x = ref.inputs()
    ref.step(x)  # warm (allocations, thread pools)
    done, t0 = 0, time.perf_counter()
    while True:
        ref.step(x)
        done += 1
        el = time.perf_counter() - t0
        if (steps is not None and done >= steps) or (steps is None and el >= seconds):
            break
    b = alg_bytes(args.model, es=2)
    per_step = (b["append"] + b["attention"]) * args.streams * c["layers"]
    what = ("the reference's own Scheduler / ModelCache / masks / ConformerAttention, torch "
            "CPU float32" if kind == "reference" else
            "pack, mask loop, shift-append, attention, unpack; float32 numpy restatement")
    sample = f"{done} steps x {args.streams} streams x {c['layers']} layers ({what})"
    return per_step * done / el / 1e9, done, el, threads, sample, kind


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    K, W = args.steps, args.warmup
    # each step is a bounded sample: at most ~150 s of CPU work for the whole run
    cls, kind = reference_step_class()
    if kind == "reference":
        import torch
        torch.set_num_threads(os.cpu_count() or 1)
    c = SHAPES[args.model]
    streams = args.streams
    probe = cls(c["layers"], c["dim"], c["heads"], c["att"], streams)
    x = probe.inputs()
    probe.step(x)
    t0 = time.perf_counter()
    probe.step(x)
    one = time.perf_counter() - t0
    budget = 150.0 / max(1, K + W)
    sample_streams = streams
    while one * sample_streams / streams > budget and sample_streams > 1:
        sample_streams = max(1, sample_streams // 2)
    del probe
    args2 = argparse.Namespace(**vars(args))
    args2.streams = sample_streams
    gbs, done, el, threads, sample, kind = cpu_reference(args2, 0, steps=K + W)
    b = alg_bytes(args.model)
    print(json.dumps({
        "impl": "reference", "metric": "paged-attn HBM GB/s (append + attention, algorithmic bytes)",
        "value": round(gbs, 4), "unit": "GB/s", "n_gpus": args.gpus, "steps": K, "warmup": W,
        "ms_per_step": round(1e3 * el / done, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args.model, streams, args.gpus),
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": threads,
                         "kind": kind, "sample": sample},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "bytes_per_stream_layer": {"append": b["append"], "attention": b["attention"]},
    }), flush=True)


def ops_at_scale(model, dev, timeit, hbm, streams=2048, layers=2, only=None):
    """One layer's append, gather, attention (+ append) and conv-cache step over
    the 2048 streams of a full serving batch (the serving loop's largest
    step), where a launch moves tens to hundreds of MB; the configs[1]
    breakdown beside it (80 streams) shows the launch- and latency-bound end.
    Full windows (36 steps of prefill), pages a random permutation, bf16."""
    import torch

    from parakeet_b200.ops import PagedKVPool, pages_per_stream
    c = SHAPES[model]
    D, H, att = c["dim"], c["heads"], c["att"]
    left, T = att[0], att[1] + 1
    W, P = left + T, 2 * (left + T) - 1
    dt = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(3)
    rnd = lambda *sh: (torch.randn(*sh, generator=g, device=dev) / 8).to(dt)  # noqa: E731
    n_pages = streams * pages_per_stream(left, T, PAGE)
    order = torch.randperm(n_pages, generator=torch.Generator().manual_seed(1))
    pool = PagedKVPool(layers, D, H, att, streams, dtype=dt, device=dev, page_order=order)
    slots = torch.arange(streams, dtype=torch.int32, device=dev)
    lengths = torch.full((streams,), T, dtype=torch.int32, device=dev)
    qkv = rnd(streams, T, 3 * D)
    q, k, v = qkv[..., :D], qkv[..., D:2 * D], qkv[..., 2 * D:]
    for _ in range(-(-left // T) + 1):
        pool.begin_step(slots, lengths)
        for l in range(layers):
            pool.append(l, k, v, slots)
        pool.end_step(slots, lengths)
    pos, bu, bv = rnd(P, D), rnd(H, D // H), rnd(H, D // H)
    out = torch.empty(streams, T, D, dtype=dt, device=dev)
    kw, vw = (torch.empty(streams, W, D, dtype=dt, device=dev) for _ in range(2))
    x2, wconv = rnd(streams, T, 2 * D), rnd(D, 1, 9)
    lnw, lnb = rnd(D) + 1, rnd(D)
    yconv = torch.empty(streams, T, D, dtype=dt, device=dev)
    nb = alg_bytes(model)
    ops = {
        "append": (lambda: pool.append(0, k, v, slots), nb["append"]),
        "gather": (lambda: pool.gather(0, slots, kw, vw), nb["gather"]),
        "attention+append": (lambda: pool.attention(0, q, pos, bu, bv, slots, lengths, out,
                                                    key=k, value=v),
                             nb["attention"] + nb["append"]),
        "conv": (lambda: pool.conv_step(0, x2, wconv, slots, lengths, lnw, lnb, 1e-5, yconv),
                 nb["conv"]),
    }
    pool.begin_step(slots, lengths)
    res = {"streams": streams}
    for name, (fn, per) in ops.items():
        if only is not None and name != only:
            continue
        t = timeit(fn)
        nbytes = per * streams
        res[name] = {"ms": round(t, 4), "GB/s": round(nbytes / t / 1e6, 1),
                     "frac": round(nbytes / t / 1e6 / hbm, 3), "bytes_per_launch": nbytes}
    torch.cuda.synchronize()
    res["device_error_word"] = pool.read_error()
    del pool
    torch.cuda.empty_cache()
    return res


def encoder_step(model, streams, steps, dev):
    """The drop-in ConformerEncoder (random bf16 weights) stepping `streams`
    slots of one pool: begin step -> 17 layers (cuBLAS GEMMs + this package's
    attention and conv kernels) -> end step, eager and as one CUDA graph."""
    import torch

    from parakeet_b200.modules import ConformerEncoder
    from parakeet_b200.weights import random_encoder_layers
    c = SHAPES[model]
    L, D, H, att = c["layers"], c["dim"], c["heads"], c["att"]
    T = att[1] + 1
    enc = ConformerEncoder(feat_in=128, hidden_size=D, ff_expansion_factor=4, num_layers=L,
                           num_heads=H, subsampling_factor=8, pos_emb_max_len=5000,
                           conv_kernel_size=9, att_context_size=att,
                           subsampling_conv_channels=256, use_bias=False)
    sd = random_encoder_layers(0, L, D, H)
    missing, unexpected = enc.load_state_dict({k: torch.from_numpy(v) for k, v in sd.items()},
                                              strict=False)
    assert not unexpected and all(k.startswith("pre_encode.") for k in missing)
    enc = enc.to(device=dev, dtype=torch.bfloat16).eval()
    state = enc.init_streaming_state(streams, dev, torch.bfloat16)
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(streams, T, D, generator=g, device=dev).to(torch.bfloat16)
    length = torch.full((streams,), T, dtype=torch.int32, device=dev)
    out = {}
    with torch.inference_mode():
        for _ in range(-(-att[0] // T) + 3):   # fill the left context
            y, state = enc(x, state, length=length)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            y, state = enc(x, state, length=length)
        b.record()
        torch.cuda.synchronize()
        out["ms_per_step_eager"] = round(a.elapsed_time(b) / steps, 4)
        try:
            gph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gph):
                y, state = enc(x, state, length=length)
            gph.replay()
            torch.cuda.synchronize()
            a.record()
            for _ in range(steps):
                gph.replay()
            b.record()
            torch.cuda.synchronize()
            out["ms_per_step_graph"] = round(a.elapsed_time(b) / steps, 4)
            del gph
        except Exception as e:   # the measurement is informative; keep the run going
            out["graph_error"] = str(e)[:200]
        out["finite"] = bool(torch.isfinite(y).all().item())
    best = min(v for k, v in out.items() if k.startswith("ms_per_step"))
    audio_ms = T * 80.0   # 8x subsampling of 10 ms frames
    out.update({"model": model, "streams": streams, "layers": L, "chunk_frames": T,
                "audio_ms_per_step": audio_ms,
                "encoder_realtime_factor": round(audio_ms / best, 1),
                "device_error_word": state.cache.pool.read_error()})
    return out


DECODE_CFG = {"small": dict(enc_dim=512, pred_layers=1, vocab=1026, streams=160),
              "large": dict(enc_dim=1024, pred_layers=2, vocab=1024, streams=480)}


def rnnt_decode_step(model, steps, dev, cpu_sample=2):
    """Batched greedy RNNT decode of one chunk for every stream (random bf16
    prediction / joint weights, blank bias set so that about 2.5 tokens are
    emitted per frame): eager and as one CUDA graph; beside it the float64
    restatement of the reference's decode loop (oracle/decode.py) on
    `cpu_sample` streams of the same chunk, scaled to the full batch."""
    import numpy as np
    import torch

    from parakeet_b200.engine.decoding import BatchedGreedyDecoder
    from parakeet_b200.modules import Joiner, Predictor
    from parakeet_b200.weights import random_decoder_state_dict
    c, d = SHAPES[model], DECODE_CFG[model]
    T = c["att"][1] + 1
    B, D, V = d["streams"], d["enc_dim"], d["vocab"]
    sd = random_decoder_state_dict(5, D, 640, 640, V, d["pred_layers"], blank_bias=2.3)
    pred, join = Predictor(640, 640, d["pred_layers"], V), Joiner(D, 640, 640, num_classes=V)
    pred.load_state_dict({k[10:]: torch.from_numpy(v) for k, v in sd.items()
                          if k.startswith("predictor.")})
    join.load_state_dict({k[7:]: torch.from_numpy(v) for k, v in sd.items()
                          if k.startswith("joiner.")})
    pred, join = pred.to(dev, torch.bfloat16).eval(), join.to(dev, torch.bfloat16).eval()
    dec = BatchedGreedyDecoder(pred, join, V, num_slots=B, max_symbols=5)
    slots = torch.arange(B, dtype=torch.int64, device=dev)
    dec.reset_slots(slots)
    g = torch.Generator(device=dev).manual_seed(9)
    enc = torch.randn(B, T, D, generator=g, device=dev).to(torch.bfloat16)
    lengths = torch.full((B,), T, dtype=torch.int32, device=dev)
    out = {"model": model, "streams": B, "frames_per_chunk": T, "max_symbols": 5}
    with torch.inference_mode():
        for _ in range(3):
            tokens, counts = dec.decode(enc, lengths, slots)
        torch.cuda.synchronize()
        out["tokens_per_frame"] = round(float(counts.float().mean()), 2)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            dec.decode(enc, lengths, slots)
        b.record()
        torch.cuda.synchronize()
        out["ms_per_chunk_eager"] = round(a.elapsed_time(b) / steps, 4)
        try:
            gph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gph):
                dec.decode(enc, lengths, slots)
            gph.replay()
            torch.cuda.synchronize()
            a.record()
            for _ in range(steps):
                gph.replay()
            b.record()
            torch.cuda.synchronize()
            out["ms_per_chunk_graph"] = round(a.elapsed_time(b) / steps, 4)
            del gph
        except Exception as e:   # informative; keep the run going
            out["graph_error"] = str(e)[:200]
    from oracle.decode import GreedyDecoderModel
    m = GreedyDecoderModel(sd, d["pred_layers"], V, 5)
    x = enc.float().cpu().numpy().astype(np.float64)
    t0 = time.perf_counter()
    for i in range(cpu_sample):
        m.decode_chunk(x[i].T, *m.new_stream())
    cpu_s = (time.perf_counter() - t0) / cpu_sample * B
    out["cpu_reference_ms_per_chunk"] = round(cpu_s * 1e3, 1)
    out["cpu_reference"] = (f"oracle/decode.py float64 numpy, {cpu_sample} streams timed, "
                            f"scaled to {B}")
    return out


def pre_encode_step(model, steps, dev, cpu_sample=4):
    """Batched streaming pre-encode of one chunk per stream (cache-prefixed
    feature frames -> ConvSubsampling -> drop 2), bf16, eager and as one CUDA
    graph; beside it the reference's per-stream loop (one subsampling call per
    stream, model_runner.py:181-233) run with the drop-in module on the host in
    fp32 on `cpu_sample` streams, scaled to the batch."""
    import torch

    from parakeet_b200.engine.pre_encode import BatchedPreEncoder
    from parakeet_b200.modules import ConvSubsampling
    from parakeet_b200.weights import random_pre_encode_state_dict
    c = SHAPES[model]
    la = c["att"][1]
    B = 160 if model == "small" else 480
    F = 8 + 8 * la
    sd = random_pre_encode_state_dict(6, 128, 256, c["dim"])
    m = ConvSubsampling(c["dim"], 256, 128, 8)
    m.load_state_dict({k: torch.from_numpy(v) for k, v in sd.items()})
    pe = BatchedPreEncoder(m.to(dev, torch.bfloat16).eval(), num_slots=B)
    g = torch.Generator(device=dev).manual_seed(3)
    feats = torch.randn(B, 128, F, generator=g, device=dev).to(torch.bfloat16)
    slots = torch.arange(B, dtype=torch.int32, device=dev)
    out = {"model": model, "streams": B, "feature_frames": F}
    with torch.inference_mode():
        for _ in range(3):
            y = pe.pre_encode(feats, slots, first=False)
        torch.cuda.synchronize()
        out["out_frames"] = int(y.shape[1])
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            pe.pre_encode(feats, slots, first=False)
        b.record()
        torch.cuda.synchronize()
        out["ms_per_chunk_eager"] = round(a.elapsed_time(b) / steps, 4)
        try:
            gph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gph):
                pe.pre_encode(feats, slots, first=False)
            gph.replay()
            torch.cuda.synchronize()
            a.record()
            for _ in range(steps):
                gph.replay()
            b.record()
            torch.cuda.synchronize()
            out["ms_per_chunk_graph"] = round(a.elapsed_time(b) / steps, 4)
            del gph
        except Exception as e:   # informative; keep the run going
            out["graph_error"] = str(e)[:200]
    cpu = ConvSubsampling(c["dim"], 256, 128, 8)
    cpu.load_state_dict({k: torch.from_numpy(v) for k, v in sd.items()})
    cpu.eval()
    x = feats[:cpu_sample].float().cpu()
    cache = torch.zeros(128, 9)
    with torch.inference_mode():
        xi = torch.cat([cache, x[0]], -1)[None]
        cpu(xi.transpose(1, 2), torch.full((1,), xi.size(-1)))   # warm (threads, allocations)
        t0 = time.perf_counter()
        for i in range(cpu_sample):
            xi = torch.cat([cache, x[i]], -1)[None]
            cpu(xi.transpose(1, 2), torch.full((1,), xi.size(-1)))
        el = time.perf_counter() - t0
    out["cpu_reference_ms_per_chunk"] = round(el / cpu_sample * B * 1e3, 1)
    out["cpu_reference"] = (f"per-stream subsampling (model_runner.py:181-233) with the drop-in "
                            f"module, fp32 torch on {torch.get_num_threads()} host threads, "
                            f"{cpu_sample} streams timed, scaled to {B}")
    return out


def synth_audio_batch(streams, n, seed):
    """float32 [streams, n] of configs[2]'s synthetic audio: per stream three
    tones in 100-4000 Hz with random phases plus white noise at 20 dB SNR,
    quantised to pcm16, scaled to [-1, 1)."""
    import numpy as np
    rng = np.random.default_rng(seed)
    t = np.arange(n) / 16000.0
    out = np.empty((streams, n), np.float32)
    for i in range(streams):
        f, ph = rng.uniform(100.0, 4000.0, 3), rng.uniform(0.0, 2 * np.pi, 3)
        tone = sum(np.sin(2 * np.pi * fk * t + p) for fk, p in zip(f, ph)) / 3.0
        x = 0.5 * (tone + rng.standard_normal(n) * np.sqrt(np.mean(tone ** 2)) / 10.0)
        out[i] = np.clip(np.round(x * 32767.0), -32768, 32767) / 32768.0
    return out


def feature_step(model, steps, dev, cpu_sample=8):
    """Batched streaming log-mel extraction of one steady-state chunk per
    stream (pk_features_push: pre-emphasis, window, 512-point FFT, slaney mel,
    log; the reference's defaults, dither included), bf16 output as the
    pre-encoder takes it, eager and as a CUDA graph.  Beside it the reference's
    per-stream push (recompute over the retained buffer, feature_extractor.py:
    97-151) restated in oracle/features.py, timed on `cpu_sample` streams and
    scaled to the batch."""
    import torch

    from parakeet_b200.modules import FeatureExtractor
    la = SHAPES[model]["att"][1]
    B = 160 if model == "small" else 480
    hop = 160
    n0, n = (1 + 8 * la) * hop, (8 + 8 * la) * hop
    F = n // hop
    fe = FeatureExtractor(num_slots=B, device=dev, out_dtype=torch.bfloat16)
    audio = synth_audio_batch(B, n0 + n, seed=21)
    fe.push_batch(audio[:, :n0], list(range(B)), first=True)
    x = torch.from_numpy(audio[:, n0:]).to(dev).contiguous()
    ns = torch.full((B,), n, dtype=torch.int32, device=dev)
    flags = torch.zeros(B, dtype=torch.int32, device=dev)
    slots = torch.arange(B, dtype=torch.int32, device=dev)
    out = torch.empty(B, 128, F, dtype=torch.bfloat16, device=dev)
    nf = torch.empty(B, dtype=torch.int32, device=dev)
    res = {"model": model, "streams": B, "samples_per_push": n, "frames_per_push": F}
    for _ in range(3):
        fe.launch(x, ns, flags, slots, out, F, nf)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        fe.launch(x, ns, flags, slots, out, F, nf)
    b.record()
    torch.cuda.synchronize()
    res["ms_per_push_eager"] = round(a.elapsed_time(b) / steps, 4)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    gph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s), torch.cuda.graph(gph, stream=s):
        for _ in range(10):
            fe.launch(x, ns, flags, slots, out, F, nf)
    torch.cuda.current_stream().wait_stream(s)
    gph.replay()
    torch.cuda.synchronize()
    reps = max(1, steps // 10)
    a.record()
    for _ in range(reps):
        gph.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / (reps * 10)
    del gph
    res["ms_per_push_graph"] = round(ms, 4)
    res["device_error_word"] = fe.error_bits()
    alg = B * n * 4 + B * 512 * 4 * 2 + B * 128 * F * 2
    res["alg_bytes_per_push"] = alg
    res["GB/s"] = round(alg / (ms * 1e-3) / 1e9, 1)
    res["frames_per_s"] = int(B * F / (ms * 1e-3))
    res["l2"] = "inputs L2-resident (back-to-back pushes of one chunk)"
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from oracle.features import FeatureStream, LogMel
    mel = LogMel()
    k = min(cpu_sample, B)
    streams = [FeatureStream(mel) for _ in range(k)]
    for i in range(k):
        streams[i].push(audio[i, :n0])
    t0 = time.perf_counter()
    for i in range(k):
        streams[i].push(audio[i, n0:])
    el = time.perf_counter() - t0
    res["cpu_reference_ms_per_push"] = round(el / k * B * 1e3, 2)
    res["cpu_reference"] = (f"oracle/features.py FeatureStream.push (the reference's recompute "
                            f"over the retained buffer, numpy float64, 1 thread), {k} streams "
                            f"timed, scaled to {B}")
    return res


GEMM_SHAPES = {   # (name, M, N, K, epilogue): the GEMMs of one encoder layer at the streaming batch
    "small": [("ff_linear1+silu", 320, 2048, 512, "silu"),
              ("ff_linear2+residual", 320, 512, 2048, "residual"),
              ("qkv", 320, 1536, 512, "store"),
              ("out_proj+residual", 320, 512, 512, "residual"),
              ("pointwise_conv1", 320, 1024, 512, "store")],
    "large": [("ff_linear1+silu", 6720, 4096, 1024, "silu"),
              ("ff_linear2+residual", 6720, 1024, 4096, "residual"),
              ("qkv", 6720, 3072, 1024, "store"),
              ("out_proj+residual", 6720, 1024, 1024, "residual"),
              ("pointwise_conv1", 6720, 2048, 1024, "store")],
    # a 2048-stream small-model serving step: the encoder layer's at 4096 rows,
    # the greedy decode's per symbol step at 2048 rows
    "serving": [("ff_linear1+silu", 4096, 2048, 512, "silu"),
                ("ff_linear2+residual", 4096, 512, 2048, "residual"),
                ("qkv", 4096, 1536, 512, "store"),
                ("pointwise_conv1", 4096, 1024, 512, "store"),
                ("joint_pred+relu", 2048, 640, 640, "residual_relu"),
                ("joint_out+bias", 2048, 1088, 640, "bias"),
                ("lstm_recurrent", 2048, 2560, 640, "store")],
}


def gemm_step(model, steps, dev):
    """The encoder's projection GEMMs at the streaming batch (160 small / 480
    large streams): pk_gemm_bf16 (tcgen05, epilogue fused) against cuBLAS
    (torch.matmul, epilogue as separate elementwise launches) and, for the
    residual epilogues, cuBLAS with the residual in its own epilogue (addmm),
    each replayed as a CUDA graph of `steps` launches after an L2 flush."""
    import torch

    from parakeet_b200.ops import gemm
    peak, kind = tensor_peak()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    res = {"peak_tflops": peak, "peak_kind": kind, "shapes": []}
    g = torch.Generator(device=dev).manual_seed(5)
    for name, M, N, K, epi in GEMM_SHAPES[model]:
        a = torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16)
        w = (torch.randn(N, K, generator=g, device=dev) / K ** 0.5).to(torch.bfloat16)
        r = torch.randn(M, N, generator=g, device=dev).to(torch.bfloat16)
        bias = torch.randn(N, generator=g, device=dev).to(torch.bfloat16)
        alpha = 1.0 if epi == "residual_relu" else 0.5

        def ours():
            return gemm(a, w, epi, residual=r if epi.startswith("residual") else None,
                        alpha=alpha, bias=bias if epi == "bias" else None)

        def cublas():
            if epi == "bias":
                return torch.addmm(bias, a, w.t())
            y = a @ w.t()
            if epi == "silu":
                return torch.nn.functional.silu(y)
            if epi == "residual":
                return r + 0.5 * y
            if epi == "residual_relu":
                return torch.relu(r + y)
            return y

        def cublas_addmm():   # the residual or bias inside cuBLAS's own epilogue
            if epi == "bias":
                return torch.addmm(bias, a, w.t())
            y = torch.addmm(r, a, w.t(), beta=1, alpha=alpha)
            return y.relu_() if epi == "residual_relu" else y

        row = {"name": name, "M": M, "N": N, "K": K}
        arms = [("tcgen05", ours), ("cublas", cublas)]
        if epi.startswith("residual"):
            arms.append(("cublas_addmm", cublas_addmm))
        for label, fn in arms:
            for _ in range(3):
                fn()
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            gph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(s), torch.cuda.graph(gph, stream=s):
                for _ in range(steps):
                    fn()
            torch.cuda.current_stream().wait_stream(s)
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            gph.replay()
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / steps
            del gph
            tf = 2.0 * M * N * K / (ms * 1e-3) / 1e12
            row[label] = {"us": round(ms * 1e3, 2), "tflops": round(tf, 1),
                          "frac": round(tf / peak, 3)}
        res["shapes"].append(row)
    res["note"] = ("launches back to back in one graph (weights L2-resident after the "
                   "first; the 256 MB flush precedes the replay)")
    return res


def profile_gemm(model, steps, dev):
    """`steps` launches of each GEMM of GEMM_SHAPES[model], nothing else (for ncu)."""
    import torch

    from parakeet_b200.ops import gemm, gemm_error_word
    g = torch.Generator(device=dev).manual_seed(5)
    for name, M, N, K, epi in GEMM_SHAPES[model]:
        a = torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16)
        w = (torch.randn(N, K, generator=g, device=dev) / K ** 0.5).to(torch.bfloat16)
        r = torch.randn(M, N, generator=g, device=dev).to(torch.bfloat16)
        for _ in range(steps):
            gemm(a, w, epi, residual=r if epi == "residual" else None, alpha=0.5)
    torch.cuda.synchronize()
    return {"profile_run": model, "op": "gemm", "steps": steps,
            "device_error_word": gemm_error_word(dev)}


def profile_features(model, steps, dev):
    """First push, then `steps` steady pushes of the log-mel kernel (the
    configuration of feature_step), nothing else: a short launch list for ncu."""
    import torch

    from parakeet_b200.modules import FeatureExtractor
    la = SHAPES[model]["att"][1]
    B = 160 if model == "small" else 480
    n0, n = (1 + 8 * la) * 160, (8 + 8 * la) * 160
    fe = FeatureExtractor(num_slots=B, device=dev, out_dtype=torch.bfloat16)
    audio = synth_audio_batch(B, n0 + n * steps, seed=21)
    fe.push_batch(audio[:, :n0], list(range(B)), first=True)
    for k in range(steps):
        fe.push_batch(audio[:, n0 + k * n:n0 + (k + 1) * n], list(range(B)))
    torch.cuda.synchronize()
    return {"profile_run": model, "op": "features", "steps": steps,
            "device_error_word": fe.error_bits()}


def stage_times(pipe, samples, slots, reps):
    """Device time of each stage of one steady step_audio, each stage captured
    as its own CUDA graph and replayed `reps` times (the stages run in order,
    so every replay sees the state its predecessor left)."""
    import torch

    from parakeet_b200.modules.cache import PagedModelCache, StreamingState
    B, n = samples.shape
    F = pipe.frames_per_push(n, False)
    key = (B, n, False)   # the buffers of this batch size (kept for good once a graph used them)
    ns, flags, feats, nframes = pipe._fe_bufs_graph.get(key) or pipe._fe_bufs[key]
    graphs, res = [], {}
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(name, fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            r = fn()
        graphs.append(g)
        g.replay()
        torch.cuda.synchronize()
        a.record()
        for _ in range(reps):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        res[name] = round(a.elapsed_time(b) / reps, 4)
        return r

    timed("features", lambda: pipe.fe.launch(samples, ns, flags, slots, feats, F, nframes))
    x = timed("pre_encode", lambda: pipe.pre.pre_encode(feats, slots, False))
    y = timed("encoder", lambda: pipe.encoder(x, StreamingState(PagedModelCache(pipe.pool, slots)),
                                              bypass_pre_encode=True)[0])
    T = x.shape[1]
    lengths = torch.full((B,), T, dtype=torch.int32, device=samples.device)
    timed("decode", lambda: pipe.dec.decode(y.transpose(1, 2), lengths, slots))
    del graphs
    return res


def build_streaming_pipeline(model, dev, num_slots, feature_kw=None, page_size=PAGE):
    """StreamingPipeline of configs[2] (small) / configs[3] (large) with random
    bf16 weights over ``num_slots`` stream slots, K/V pages of ``page_size``
    frames."""
    import torch

    from parakeet_b200.engine import StreamingPipeline
    from parakeet_b200.modules import ConformerEncoder, Joiner, Predictor
    from parakeet_b200.weights import (random_decoder_state_dict, random_encoder_layers,
                                       random_pre_encode_state_dict)
    c, d = SHAPES[model], DECODE_CFG[model]
    L, D, H, att = c["layers"], c["dim"], c["heads"], c["att"]
    V = d["vocab"]
    enc = ConformerEncoder(feat_in=128, hidden_size=D, ff_expansion_factor=4, num_layers=L,
                           num_heads=H, subsampling_factor=8, pos_emb_max_len=5000,
                           conv_kernel_size=9, att_context_size=att, subsampling_conv_channels=256,
                           use_bias=False)
    sd = {**random_encoder_layers(0, L, D, H),
          **{f"pre_encode.{k}": v for k, v in random_pre_encode_state_dict(6, 128, 256, D).items()}}
    enc.load_state_dict({k: torch.from_numpy(v) for k, v in sd.items()})
    pre = enc.pre_encode
    sd = random_decoder_state_dict(5, D, 640, 640, V, d["pred_layers"], blank_bias=2.3)
    pred, join = Predictor(640, 640, d["pred_layers"], V), Joiner(D, 640, 640, num_classes=V)
    pred.load_state_dict({k[10:]: torch.from_numpy(v) for k, v in sd.items()
                          if k.startswith("predictor.")})
    join.load_state_dict({k[7:]: torch.from_numpy(v) for k, v in sd.items()
                          if k.startswith("joiner.")})
    mods = [m.to(dev, torch.bfloat16).eval() for m in (enc, pre, pred, join)]
    return StreamingPipeline(*mods, blank_id=V, num_slots=num_slots, feature_kw=feature_kw,
                             page_size=page_size)


def streaming_step(model, steps, dev, profile=False, streams=None):
    """Audio -> tokens for every stream of configs[2] (small, 160 streams) or
    configs[3] on one GPU (large, 480 streams): batched log-mel features ->
    batched pre-encode -> paged encoder -> batched greedy decode
    (engine.pipeline.StreamingPipeline.step_audio), random bf16 weights,
    synthetic audio of configs[2], as one CUDA graph per steady-state step.
    Streams that one GPU sustains in real time at this batch = batch x audio
    per step / step time."""
    import torch

    B = streams or DECODE_CFG[model]["streams"]
    pipe = build_streaming_pipeline(model, dev, B)
    att = SHAPES[model]["att"]
    la = att[1]
    slots = torch.arange(B, dtype=torch.int32, device=dev)
    pipe.start_streams(slots)
    n0, n = (1 + 8 * la) * 160, (8 + 8 * la) * 160
    audio = torch.from_numpy(synth_audio_batch(B, n0 + n, seed=11)).to(dev)
    first, nxt = audio[:, :n0].contiguous(), audio[:, n0:].contiguous()
    out = {"model": model, "streams": B, "audio_ms_per_step": (la + 1) * 80.0,
           "input": "16 kHz float samples, one chunk per stream per step"}
    with torch.inference_mode():
        pipe.step_audio(first, slots, 0)
        for k in range(-(-att[0] // (la + 1)) + 2):   # fill the left context
            tok, cnt = pipe.step_audio(nxt, slots, 1 + k)
        torch.cuda.synchronize()
        if profile:   # eager steps only, bracketed for `ncu --profile-from-start off`
            torch.cuda.cudart().cudaProfilerStart()
            for _ in range(steps):
                pipe.step_audio(nxt, slots, 2)
            torch.cuda.synchronize()
            torch.cuda.cudart().cudaProfilerStop()
            return {"profile_run": model, "op": "streaming", "steps": steps,
                    "device_error_word": pipe.pool.read_error() | pipe.fe.error_bits()}
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            pipe.step_audio(nxt, slots, 2)
        b.record()
        torch.cuda.synchronize()
        out["ms_per_step_eager"] = round(a.elapsed_time(b) / steps, 4)
        try:
            gph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gph):
                tok, cnt = pipe.step_audio(nxt, slots, 2)
            gph.replay()
            torch.cuda.synchronize()
            a.record()
            for _ in range(steps):
                gph.replay()
            b.record()
            torch.cuda.synchronize()
            out["ms_per_step_graph"] = round(a.elapsed_time(b) / steps, 4)
            del gph
        except Exception as e:   # informative; keep the run going
            out["graph_error"] = str(e)[:200]
        out["tokens_per_frame"] = round(float(cnt.float().mean()), 2)
        try:   # chunk k's decode on a second stream under chunk k+1's encoder
            from parakeet_b200.engine import OverlappedStreamingRunner
            runner = OverlappedStreamingRunner(pipe, slots, n)
            for _ in range(3):
                runner.step(nxt)
            runner.drain()
            torch.cuda.synchronize()
            a.record()
            for _ in range(steps):
                runner.step(nxt)
            runner.drain()
            b.record()
            torch.cuda.synchronize()
            out["ms_per_step_overlapped"] = round(a.elapsed_time(b) / steps, 4)
            del runner
        except Exception as e:   # informative; keep the run going
            out["overlap_error"] = str(e)[:200]
        try:
            out["stage_ms_graph"] = stage_times(pipe, nxt, slots, steps)
        except Exception as e:   # informative; keep the run going
            out["stage_error"] = str(e)[:200]
    best = min(v for k, v in out.items() if k.startswith("ms_per_step"))
    out["realtime_streams_at_this_batch"] = int(B * out["audio_ms_per_step"] / best)
    out["device_error_word"] = pipe.pool.read_error() | pipe.fe.error_bits()
    return out


def reference_engine_search(model, dev, limit_ms=160.0, measure_s=3.0, max_trials=8,
                            start=8, pool=1024):
    """The survey's metric 1 for the reference's own engine on this GPU: its
    unmodified ``ModelRunner`` (parakeet/engine/model_runner.py:19-496) in bf16
    with eager CUDA, its three worker threads (``start_workers``), its
    ``Scheduler`` slot pool, its host ``FeatureExtractor`` and per-stream
    pre-encode; random bf16 weights (baseline/harness.py).  One shim: the
    runner moves features to the device but not to the model's dtype
    (model_runner.py:196), which fails in bf16, so the extractor's output is
    cast to bf16.  Streams are paced as ``serve_trial`` paces this package's:
    stream i pushes its chunk k (the engine's first chunk, then its later
    chunks) through ``Sequence.push_samples`` at t0 + phase_i + k * period; a
    chunk's latency is the time from that push to the return of
    ``_decode_batch`` with its tokens (then put on the results queue).  N
    doubles from ``start`` until a trial fails (p99 above the limit, or more
    than one chunk per stream left undecoded at the end; a failing trial is
    repeated once), then bisects."""
    import numpy as np
    import torch

    sys.path.insert(0, os.path.join(REPO, "baseline"))
    import harness
    if not harness.available():
        return {"unavailable": "no reference install under baseline/_ref "
                               "(python bench.py --install-reference <checkout>)"}
    harness.import_reference()
    from parakeet.config import Config
    from parakeet.engine.model_runner import ModelRunner
    from parakeet.engine.scheduler import Scheduler

    c = SHAPES[model]
    la = c["att"][1]
    period = (la + 1) * 0.08
    n0, n = (1 + 8 * la) * 160, (8 + 8 * la) * 160
    net = harness.seeded_parakeet(model, torch.bfloat16)
    fe = net._feature_extractor
    fe_push = fe.push

    def push_bf16(samples, state, final=False):       # the dtype shim (model_runner.py:196)
        f = fe_push(samples, state, final=final)
        return None if f is None else f.to(torch.bfloat16)

    fe.push = push_bf16
    harness.patch_from_pretrained(net)

    class TimedRunner(ModelRunner):
        def _decode_batch(self, seqs, chunks):
            out = super()._decode_batch(seqs, chunks)
            t = time.perf_counter()
            for q in seqs:
                self.done_at[q.request_id].append(t)
            return out

    runner = TimedRunner(Config(size=model, max_num_streams=pool), torch.device(dev),
                         Scheduler(max_active=pool))
    runner.done_at = {}
    audio = synth_audio_batch(64, n0 + 2 * n, seed=11)
    banks = [audio[:, :n0], audio[:, n0:n0 + n], audio[:, n0 + n:]]
    meas = max(3, int(round(measure_s / period)))

    def trial(N, seed, warm=3):
        rng = np.random.default_rng(seed)
        phase = rng.uniform(0.0, period, N)
        seqs = []
        for _ in range(N):
            q = runner.create_sequence()
            runner.add_sequence(q)
            runner.done_at[q.request_id] = []
            seqs.append(q)
        pushed = [[] for _ in range(N)]
        k = np.zeros(N, np.int64)
        if torch.device(dev).type == "cuda":
            torch.cuda.synchronize(dev)
        runner.start_workers()
        t0 = time.perf_counter() + 0.02
        t_meas, t_end = t0 + warm * period, t0 + (warm + meas) * period
        try:
            while True:
                now = time.perf_counter()
                if now >= t_end:
                    break
                due = t0 + phase + k * period
                i = int(np.argmin(due))
                if due[i] > now:
                    time.sleep(min(due[i], t_end) - now)
                    continue
                b = banks[min(int(k[i]), 2)]
                x = b[(i + int(k[i])) % b.shape[0]]
                q = seqs[i]
                with q.lock:
                    q.push_samples(x)
                pushed[i].append(time.perf_counter())
                k[i] += 1
        finally:
            runner.stop_workers()
        lats, backlog = [], 0
        for i, q in enumerate(seqs):
            done = runner.done_at.pop(q.request_id)
            backlog = max(backlog, len(pushed[i]) - len(done))
            lats += [d - p for p, d in zip(pushed[i], done) if p >= t_meas]
            runner._release_sequence(q)
        lat = np.array(lats)
        p99 = float(np.percentile(lat, 99)) * 1e3 if lat.size else float("inf")
        ok = p99 <= limit_ms and backlog <= 1
        return ok, {"streams": N, "ok": ok,
                    "p50_ms": round(float(np.median(lat)) * 1e3, 2) if lat.size else None,
                    "p99_ms": round(p99, 2), "chunks": int(lat.size),
                    "backlog_chunks_at_end": backlog}

    t_start = time.perf_counter()
    trial(min(4, start), seed=0, warm=2)              # module loads, allocator, threads
    trials, ok_n, bad_n, N = [], 0, None, start
    while len(trials) < max_trials:
        ok, rec = trial(N, len(trials) + 1)
        if not ok:
            ok, rec2 = trial(N, 100 + len(trials))
            rec = {**rec2, "first_attempt_p99_ms": rec["p99_ms"]}
        trials.append(rec)
        if ok:
            ok_n = N
        else:
            bad_n = N
        if bad_n is None:
            if 2 * N > pool:
                break
            N *= 2
        else:
            if bad_n - ok_n <= max(2, ok_n // 16):
                break
            N = (ok_n + bad_n) // 2
    best = next((t for t in trials if t["streams"] == ok_n), None)
    del runner, net
    torch.cuda.empty_cache()
    return {"model": model, "limit_ms": limit_ms, "streams_max": ok_n,
            "p99_ms_at_max": best["p99_ms"] if best else None,
            "audio_ms_per_chunk": period * 1e3, "measured_s_per_trial": round(meas * period, 2),
            "search_s": round(time.perf_counter() - t_start, 1), "trials": trials,
            "engine": "reference ModelRunner (unmodified, eager CUDA, bf16, worker threads), "
                      "from baseline/_ref"}


class ServePositions:
    """Stream positions of the paced serving trials on one GPU, one slot each.
    A position always holds a live stream of ``life`` chunks (configs[2]: 30 s
    of audio); when it ends, its slot is released and a new stream starts there
    at the position's next chunk time, so streams join and leave every period
    (about N / life of them).  Positions persist across trials: trial N runs
    positions 0..N-1, whose streams keep their age.  ``age`` is the chunk
    index of each position's current stream; streams start at ages uniform in
    [0, life), and before the first trial every position is stepped through
    min(age, fill) chunks, ``fill`` covering the 70-frame left context and
    then some (36 small, 7 large), so trials run on full windows from their
    first chunk, as steady-state serving does."""

    def __init__(self, cap, period, life, fill, seed):
        import numpy as np
        rng = np.random.default_rng(seed)
        self.cap, self.period, self.life, self.fill = cap, period, life, fill
        self.phase = rng.uniform(0.0, period, cap)
        self.age = rng.integers(0, life, cap).astype(np.int64)
        self.joined = 0


STEP_BUCKETS = (2048, 1024, 512, 256, 128)   # batch sizes of the captured serving steps


class StepGraphs:
    """A CUDA graph of one ``step_audio`` per push class (first, second,
    later chunk) and batch size in ``STEP_BUCKETS``: slots and samples are
    data in each graph's input buffers, so one graph serves any streams of its
    class.  A batch is cut into bucket-sized pieces, largest first; the last
    piece is padded to the smallest bucket with rows of ``dummy`` slots (pool
    slots no served stream uses, started once as streams of their own), so
    every step runs as a graph replay instead of about 300 eager launches
    (about 7.5 ms of host time each)."""

    def __init__(self, pipe, cap, spare, banks, dev):
        import torch
        self.dummy = torch.arange(cap, cap + spare, dtype=torch.int32, device=dev)
        self.g = {}
        pool = torch.cuda.graph_pool_handle()
        for c in (0, 1, 2):
            for Bg in STEP_BUCKETS:
                if Bg > cap:
                    continue
                sl = torch.arange(Bg, dtype=torch.int32)
                gs = sl.to(dev)
                gx = torch.empty(Bg, banks[c].shape[1], dtype=torch.float32, device=dev)
                gx.copy_(banks[c][torch.arange(Bg) % banks[c].shape[0]])
                x0 = banks[0][torch.arange(Bg) % banks[0].shape[0]].to(dev)
                pipe.start_streams(sl)
                # one eager first step: it also applies the releases queued so far,
                # so that the captured step carries none
                pipe.step_audio(x0, gs, 0)
                torch.cuda.synchronize(dev)
                gph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gph, pool=pool):
                    tok, cnt = pipe.step_audio(gx, gs, c)
                pipe.end_streams(sl)
                self.g[(c, Bg)] = (gph, gx, gs, tok, cnt)
        pipe.start_streams(self.dummy.cpu())
        self.sizes = sorted({Bg for _, Bg in self.g}, reverse=True)

    def pieces(self, B):
        """(rows, bucket) of the graph replays that serve a batch of B rows."""
        out, done = [], 0
        while done < B:
            left = B - done
            Bg = next((g for g in self.sizes if g <= left), self.sizes[-1])
            r = min(Bg, left)
            out.append((r, Bg))
            done += r
        return out


def _flush_releases(pipe):
    """Return the pages of streams ended since the last step: a captured step
    carries no releases, so they go in a step start of no rows."""
    import torch
    if pipe.pool.pending_release:
        pipe.pool.begin_step(torch.empty(0, dtype=torch.int32, device=pipe.device))


def _serve_batch(pipe, c, part, k, banks, hbufs, dbufs, hslots, dslots, htok, hcnt, off,
                 graphs):
    """Copies the samples and slots of rows ``part`` (push class c: first,
    second, later) in from pinned host memory, runs their step (replays of
    ``graphs``, a StepGraphs, when given; else eagerly), and queues the tokens'
    copy back to pinned host memory."""
    import torch
    B = part.size
    rs = slice(off, off + B)
    bank = banks[c]
    torch.index_select(bank, 0, torch.from_numpy((part + k[part]) % bank.shape[0]),
                       out=hbufs[c][rs])
    hslots[c][rs].numpy()[:] = part
    if graphs is None:
        dx = dbufs[c][rs]
        dx.copy_(hbufs[c][rs], non_blocking=True)
        ds = dslots[c][rs]
        ds.copy_(hslots[c][rs], non_blocking=True)
        tok, cnt = pipe.step_audio(dx, ds, c)
        htok[c][rs].copy_(tok.view(B, -1), non_blocking=True)
        hcnt[c][rs].copy_(cnt, non_blocking=True)
        return
    _flush_releases(pipe)
    done = 0
    for r, Bg in graphs.pieces(B):
        gph, gx, gs, tok, cnt = graphs.g[(c, Bg)]
        sub = slice(off + done, off + done + r)
        gx[:r].copy_(hbufs[c][sub], non_blocking=True)
        gs[:r].copy_(hslots[c][sub], non_blocking=True)
        if r < Bg:
            gs[r:].copy_(graphs.dummy[:Bg - r])
        gph.replay()
        htok[c][sub].copy_(tok[:r].view(r, -1), non_blocking=True)
        hcnt[c][sub].copy_(cnt[:r], non_blocking=True)
        done += r


def serve_prefill(pipe, pos, bufs, graphs, max_batch=2048):
    """Steps every position through min(age, fill) chunks as fast as the GPU
    runs them (no pacing), so that each stream's pages, conv cache, feature
    history and prediction state are those of a stream of that age."""
    import numpy as np
    import torch
    pipe.start_streams(torch.arange(pos.cap, dtype=torch.int32))
    target = np.minimum(pos.age, pos.fill)
    k = np.zeros(pos.cap, np.int64)
    for c in range(int(target.max(initial=0))):
        sel = np.flatnonzero(target > c)
        cls = min(c, 2)
        for off in range(0, sel.size, max_batch):
            part = sel[off:off + max_batch]
            _serve_batch(pipe, cls, part, k, *bufs, 0, graphs)
        k[sel] += 1
    torch.cuda.synchronize(pipe.device)


def serve_trial(pipe, N, pos, bufs, warm_periods, meas_periods, max_batch=2048,
                graphs=None):
    """Positions 0..N-1 paced in real time: position i's next chunk completes
    at t0 + phase_i + m * period (m = chunks it has pushed in this trial).
    The loop takes every chunk that has completed (one per position per
    iteration), groups them by push class of their stream (first, second,
    later; batches of at most 2048 rows), copies their samples and slots in
    from pinned host memory, runs ``step_audio`` (as replays of the captured
    steps of ``graphs``, a StepGraphs, when given; else eagerly) and copies the
    tokens back to pinned host memory; a chunk's latency is the wall time from
    its completion to its tokens being on the host (the reference's
    push_samples -> DecodeResult, model_runner.py:150-171).  Streams that
    reach their last chunk are released (pages back to the pool at the next
    step) and a new stream starts in their slot.  Returns latencies (s) of
    the chunks completed in the measured periods and the loop's statistics."""
    import numpy as np
    import torch

    period = pos.period
    k = pos.age[:N].copy()
    m = np.zeros(N, np.int64)
    phase = pos.phase[:N]
    t0 = time.perf_counter() + 0.02
    t_meas, t_end = t0 + warm_periods * period, t0 + (warm_periods + meas_periods) * period
    lats, steps, rows, launches, joins = [], 0, 0, 0, 0
    ev = torch.cuda.Event()
    while True:
        now = time.perf_counter()
        if now >= t_end:
            break
        arr = t0 + phase + m * period
        ready = np.flatnonzero(arr <= now)
        if ready.size == 0:
            time.sleep(max(0.0, min(float(arr.min()), t_end) - now))
            continue
        cls = np.minimum(k[ready], 2)
        launched = []
        for c in (0, 1, 2):
            sel = ready[cls == c]
            sel = sel[np.argsort(arr[sel], kind="stable")]
            # batches of at most 2048 rows, oldest first, each in its own rows
            # of the buffers (copies are still in flight)
            for off in range(0, sel.size, max_batch):
                part = sel[off:off + max_batch]
                _serve_batch(pipe, c, part, k, *bufs, off, graphs)
                rows += part.size
                launches += 1
            if sel.size:
                launched.append((sel, arr[sel]))
        ev.record()
        ev.synchronize()
        t_done = time.perf_counter()
        for sel, a in launched:
            lats.append(t_done - a[a >= t_meas])
            k[sel] += 1
            m[sel] += 1
        ended = ready[k[ready] >= pos.life]
        if ended.size:               # streams leave, new ones take their slots
            sl = torch.from_numpy(ended.astype(np.int32))
            pipe.end_streams(sl)
            pipe.start_streams(sl)
            k[ended] = 0
            joins += ended.size
        steps += 1
    pos.age[:N] = k
    pos.joined += joins
    backlog = int(np.max(np.floor((t_end - t0 - phase) / period) + 1 - m))
    lat = np.concatenate(lats) if lats else np.zeros(0)
    return lat, {"iterations": steps, "steps": launches,
                 "mean_batch": round(rows / max(launches, 1), 1),
                 "streams_joined": joins, "backlog_chunks_at_end": backlog}


def reduce_over_ranks(vals, op, world, dev):
    """All-reduce of a few host scalars over the process group (control plane
    of the multi-GPU serving search; identity on one rank)."""
    if world == 1:
        return list(vals)
    import torch
    import torch.distributed as dist
    t = torch.tensor(list(vals), dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=op)
    return t.tolist()


def job_trial(total, world, rank, cap, dev, limit_ms, local_trial):
    """One serving trial of ``total`` streams over the job: ``StreamRouter``
    places them (least loaded; every rank computes the same placement, its
    share is a prefix of its positions), ``local_trial(n)`` serves this rank's
    n and returns (latencies s, stats); the job passes when every rank's p99
    is within the limit and no rank is left behind by more than one chunk."""
    import numpy as np
    import torch.distributed as dist

    from parakeet_b200.engine import StreamRouter
    router = StreamRouter(world, capacity=cap)
    mine = sum(router.place(p) == rank for p in range(total))
    lat, st = local_trial(mine)
    p99 = float(np.percentile(lat, 99)) * 1e3 if lat.size else float("inf")
    p50 = float(np.median(lat)) * 1e3 if lat.size else float("inf")
    mx = dist.ReduceOp.MAX if world > 1 else None
    sm = dist.ReduceOp.SUM if world > 1 else None
    p99, p50m, backlog = reduce_over_ranks([p99, p50, st["backlog_chunks_at_end"]], mx, world, dev)
    chunks, joined, served = reduce_over_ranks(
        [float(lat.size), float(st.get("streams_joined", 0)), float(mine)], sm, world, dev)
    ok = p99 <= limit_ms and backlog <= 1
    return ok, {"streams": total, "streams_per_gpu": round(total / world, 1),
                "streams_served": int(served), "ok": ok, "p50_ms": round(p50m, 2),
                "p99_ms": round(p99, 2), "chunks": int(chunks), "streams_joined": int(joined),
                "backlog_chunks_at_end": int(backlog),
                "iterations": st.get("iterations"), "mean_batch": st.get("mean_batch")}


def serving_search(model, dev, measure_s=3.0, max_trials=9, limit_ms=160.0, use_graph=True,
                   lifetime_s=30.0, start_per_gpu=1024, fixed_total=None, page_size=None):
    """Metric 1 of the survey: the most concurrent streams per GPU served with
    p99 chunk latency <= 160 ms, streams paced in real time (configs[2] /
    configs[3] audio, random bf16 weights), each stream living ``lifetime_s``
    (streams join and leave every period), every window full (positions
    prefilled, ``ServePositions``).  On N GPUs (one process each) the job's
    streams are placed by ``StreamRouter`` (least loaded), each rank serves its
    share, and a trial passes when every rank's p99 and backlog pass (the
    job's p99 is the largest rank p99).  The total doubles from
    ``start_per_gpu`` x N until a trial fails (p99 above the limit, or chunks
    left waiting at the end; a failing trial is repeated once), then
    bisects; slots per GPU are capped by SLOT_HBM_SHARE of its free memory
    (every slot holds its K/V pages).  ``fixed_total``: one trial at that many streams
    (configs[3]: 480 large streams over the job) before the search."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from parakeet_b200.ops import pages_per_stream
    world = dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
    rank = dist.get_rank() if world > 1 else 0

    def reduce(vals, op):
        return reduce_over_ranks(vals, op, world, dev)

    c = SHAPES[model]
    L, D, att = c["layers"], c["dim"], c["att"]
    la = att[1]
    T = la + 1
    period = (la + 1) * 0.08
    n0, n = (1 + 8 * la) * 160, (8 + 8 * la) * 160
    life = int(round(lifetime_s / period))
    fill = -(-att[0] // T) + 1
    ps = page_size or SERVE_PAGE[model]
    per_slot = (pages_per_stream(att[0], T, ps) * L * 2 * ps * D * 2 + L * D * 8 * 2
                + 128 * 9 * 2 + 4096)
    torch.cuda.empty_cache()
    free = torch.cuda.mem_get_info(dev)[0]
    # slots take this share of the free HBM; the rest holds the engine's graphs,
    # activations and sample buffers (measured at the cap: about 3 GB small,
    # 11 GB large, the `hbm` entry of the line)
    cap = int(min(65536, SLOT_HBM_SHARE[model] * free / per_slot)) // 256 * 256
    cap = int(reduce([cap], dist.ReduceOp.MIN if world > 1 else None)[0])
    # the pool holds STEP_BUCKETS[-1] more slots: the rows that pad a step graph
    spare = STEP_BUCKETS[-1] if use_graph else 0
    pipe = build_streaming_pipeline(model, dev, cap + spare, page_size=ps)
    S = pipe.dec.max_symbols
    audio = synth_audio_batch(64, n0 + 2 * n, seed=11)
    banks = [torch.from_numpy(np.ascontiguousarray(a))
             for a in (audio[:, :n0], audio[:, n0:n0 + n], audio[:, n0 + n:])]
    hbufs = [torch.empty(cap, b.shape[1], dtype=torch.float32).pin_memory() for b in banks]
    dbufs = [torch.empty(cap, b.shape[1], dtype=torch.float32, device=dev) for b in banks]
    hslots = [torch.empty(cap, dtype=torch.int32).pin_memory() for _ in range(3)]
    dslots = [torch.empty(cap, dtype=torch.int32, device=dev) for _ in range(3)]
    htok = [torch.empty(cap, T * S, dtype=torch.int32).pin_memory() for _ in range(3)]
    hcnt = [torch.empty(cap, T, dtype=torch.int32).pin_memory() for _ in range(3)]
    bufs = (banks, hbufs, dbufs, hslots, dslots, htok, hcnt)
    meas = max(3, int(round(measure_s / period)))
    warm = 3 if period < 0.5 else 2
    trials, ok_n, bad_n = [], 0, None
    t_start = time.perf_counter()
    with torch.inference_mode():
        # Warm-up: one first, second and later step at batch sizes 1 ... wcap
        # (ratio 1.5), so that every kernel the trials' batch sizes select is
        # loaded (modules load at first launch) and the allocator holds blocks.
        wcap = min(cap, 2048)
        sizes = sorted({min(wcap, int(1.5 ** i)) for i in range(64) if 1.5 ** (i - 1) < wcap})
        for B in sizes:
            sl = torch.arange(B, dtype=torch.int32)
            pipe.start_streams(sl)
            for cc in range(3):
                dbufs[cc][:B].copy_(banks[cc][torch.arange(B) % banks[cc].shape[0]])
                dslots[cc][:B].copy_(sl)
                pipe.step_audio(dbufs[cc][:B], dslots[cc][:B], cc)
            pipe.end_streams(sl)
        torch.cuda.synchronize(dev)
        # Every step as a CUDA graph replay (StepGraphs): the eager step
        # launches about 300 kernels, whose host cost (about 7.5 ms) exceeds
        # their GPU time even at 2048 streams.
        graphs = StepGraphs(pipe, cap, spare, banks, dev) if use_graph else None
        pos = ServePositions(cap, period, life, fill, seed=1000 + rank)
        t_pf = time.perf_counter()
        serve_prefill(pipe, pos, bufs, graphs)
        prefill_s = time.perf_counter() - t_pf
        serve_trial(pipe, min(64, cap), pos, bufs, 2, 1, graphs=graphs)

        def run(total):
            return job_trial(total, world, rank, cap, dev, limit_ms,
                             lambda mine: serve_trial(pipe, mine, pos, bufs, warm, meas,
                                                      graphs=graphs))

        fixed = None
        if fixed_total:
            _, fixed = run(min(fixed_total, cap * world))
        N = min(start_per_gpu, cap) * world
        while len(trials) < max_trials:
            ok, rec = run(N)
            if not ok:   # a trial fails only if its repeat fails too
                ok, rec2 = run(N)
                rec = {**rec2, "first_attempt_p99_ms": rec["p99_ms"]}
            trials.append(rec)
            if ok:
                ok_n = N
            else:
                bad_n = N
            if bad_n is None:
                if N >= cap * world:
                    break
                N = min(2 * N, cap * world)
            else:
                if bad_n - ok_n <= max(64 * world, ok_n // 16):
                    break
                N = (ok_n + bad_n) // 2 // (32 * world) * (32 * world)
    err = pipe.pool.read_error() | pipe.fe.error_bits()
    err = int(reduce([float(err)], dist.ReduceOp.MAX if world > 1 else None)[0])
    # HBM at the end of the search, the engine still resident: how much of the
    # share left beside the slots the rest of the engine used
    free_end, total = torch.cuda.mem_get_info(dev)
    hbm = {"total_gb": round(total / 1e9, 1), "free_before_gb": round(free / 1e9, 1),
           "slots_gb": round((cap + spare) * per_slot / 1e9, 1),
           "peak_allocated_gb": round(torch.cuda.max_memory_allocated(dev) / 1e9, 1),
           "free_at_end_gb": round(free_end / 1e9, 1)}
    del pipe
    torch.cuda.empty_cache()
    best = next((t for t in trials if t["streams"] == ok_n), None)
    out = {"model": model, "limit_ms": limit_ms, "n_gpus": world,
           "streams_max": ok_n, "streams_per_gpu": round(ok_n / world, 1),
           "capped_by_memory": bad_n is None and ok_n == cap * world, "slot_cap_per_gpu": cap,
           "page_size": ps, "hbm": hbm,
           "p99_ms_at_max": best["p99_ms"] if best else None,
           "audio_ms_per_chunk": period * 1e3, "measured_s_per_trial": round(meas * period, 2),
           "stream_life_s": lifetime_s, "prefill_chunks": fill,
           "prefill_s": round(prefill_s, 1), "search_s": round(time.perf_counter() - t_start, 1),
           "trials": trials, "device_error_word": err,
           "step_graphs": sorted(graphs.sizes) if graphs is not None else None,
           "method": "streams paced in real time, full windows (prefilled), 30 s lifetimes "
                     "(streams leave and new ones join), batched steps over every completed "
                     "chunk, latency = chunk completion -> tokens in pinned host memory"
                     + ("; job streams placed least-loaded across GPUs" if world > 1 else "")}
    if fixed is not None:
        out["fixed_load"] = fixed
    return out


def serve_lines(args, dev, world):
    """Streams per GPU at p99 <= 160 ms.  One GPU: this package's engine for
    configs[2] (small) and configs[3] (large), each beside the reference's own
    engine on the same GPU (``reference_engine_search``).  N GPUs: configs[3],
    480 large streams placed across the N engines, then the search for the
    most the job serves."""
    import torch

    def guarded(fn, model, **kw):
        # one GPU: a search that fails (out of memory, say) is reported in its
        # entry instead of costing the bench line
        try:
            return fn(model, dev, **kw)
        except Exception as e:   # noqa: BLE001
            try:
                torch.cuda.synchronize(dev)
                torch.cuda.empty_cache()
            except Exception:   # noqa: BLE001  (a device error: the line reports it)
                pass
            return {"model": model, "error": f"{type(e).__name__}: {e}"[:400]}

    if args.serve_page_small:
        SERVE_PAGE["small"] = args.serve_page_small
    if args.serve_page_large:
        SERVE_PAGE["large"] = args.serve_page_large
    if world == 1:
        out = {}
        for model in ("small", "large"):
            ours = guarded(serving_search, model, measure_s=3.0 if model == "small" else 4.0,
                           max_trials=9 if model == "small" else 7,
                           fixed_total=480 if model == "large" else 160)
            ref = None
            if not args.no_reference_engine:
                ref = guarded(reference_engine_search, model,
                              max_trials=8 if model == "small" else 6,
                              measure_s=3.0 if model == "small" else 4.0)
            if ref and ref.get("streams_max") and ours.get("streams_max"):
                ours["vs_reference_engine"] = round(ours["streams_max"] / ref["streams_max"], 1)
            ours["reference_engine"] = ref
            out[model] = ours
        return out
    return {"large": serving_search("large", dev, measure_s=4.0, max_trials=6,
                                    fixed_total=480)}


def max_over_ranks(vals, device):
    """Element-wise max of per-rank timings over the process group (the step
    time of a weak-scaling run is its slowest rank's); identity on one rank."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return list(vals)
    t = torch.tensor(list(vals), dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def job_throughput(bytes_per_rank_step, world, ms):
    """Whole-job GB/s: every rank moved bytes_per_rank_step per step, in ms (max over ranks)."""
    return bytes_per_rank_step * world / (ms * 1e-3) / 1e9


# ---------------------------------------------------------------- B200 arm
def main():
    args = parse()
    if args.install_reference:
        print(install_reference(args.install_reference, args.wheelhouse))
        return
    if args.impl == "reference":
        run_reference_arm(args)
        return

    import torch
    import torch.distributed as dist

    from parakeet_b200.ops import PagedKVPool, pages_per_stream

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.profile_op == "features":   # the log-mel kernel alone, for ncu
        print(json.dumps(profile_features(args.model, args.steps, dev)))
        return
    if args.profile_op == "gemm":       # the projection GEMMs alone, for ncu
        print(json.dumps(profile_gemm(args.model, args.steps, dev)))
        return
    if args.profile_op and args.profile_op.startswith("scale_"):   # one op at 2048 streams, for ncu
        import torch
        dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        torch.cuda.set_device(dev)

        def run_only(fn):
            for _ in range(args.steps):
                fn()
            torch.cuda.synchronize()
            return 1.0
        r = ops_at_scale(args.model, dev, run_only, 1.0, only=args.profile_op[len("scale_"):])
        print(json.dumps({"profile_run": args.model, "op": args.profile_op, "steps": args.steps,
                          "device_error_word": r["device_error_word"]}))
        return
    if args.profile_op == "streaming":  # --steps audio -> tokens steps inside a profiler range
        print(json.dumps(streaming_step(args.model, args.steps, dev, profile=True,
                                        streams=args.pipeline_streams)))
        return
    c = SHAPES[args.model]
    L, D, H, att = c["layers"], c["dim"], c["heads"], c["att"]
    left, T = att[0], att[1] + 1
    W, P, dh = left + T, 2 * (left + T) - 1, D // H
    B = args.streams
    dt = torch.bfloat16
    sc = 1.0 / dh ** 0.5

    gen = torch.Generator().manual_seed(1)
    n_pages = B * pages_per_stream(left, T, PAGE)
    order = torch.randperm(n_pages, generator=gen)
    pool = PagedKVPool(L, D, H, att, B, num_pages=n_pages, dtype=dt, device=dev, page_order=order)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    rnd = lambda *s: (torch.randn(*s, generator=g, device=dev) * sc).to(dt)  # noqa: E731
    pos = rnd(L, P, D)
    bu, bv = rnd(L, H, dh), rnd(L, H, dh)
    NBUF = 4
    qkv = [rnd(L, B, T, 3 * D) for _ in range(NBUF)]
    out = torch.empty(L, B, T, D, dtype=dt, device=dev)
    slots = torch.arange(B, dtype=torch.int32, device=dev)
    lengths = torch.full((B,), T, dtype=torch.int32, device=dev)
    nb = alg_bytes(args.model)
    units = B * L
    step_bytes = (nb["append"] + nb["attention"]) * units

    # the rel-pos term of every (layer, stream, head, query) in one pre-pass
    # that reads each layer's pos rows once, instead of once per stream inside
    # the attention kernel (where they are L2 traffic 1.5x the K/V bytes' size)
    relpos_mode = args.relpos if pool.relpos_bd_cols > 0 else "in-kernel"
    prepass = relpos_mode != "in-kernel"
    bd_buf = (torch.empty(L, B, H, T, pool.relpos_bd_cols, dtype=torch.float32, device=dev)
              if prepass else None)

    def run_step(x, o, ev=None):
        # (on a side stream, concurrent with the step start, it measured slower:
        # the join costs the programmatic overlap of step start and attention)
        if ev is not None:
            ev[2].record()
        if relpos_mode == "prepass":
            pool.relpos_bd(0, x[..., :D], pos, bv, out=bd_buf)
        if ev is not None:
            ev[3].record()
        if relpos_mode == "fused":   # step start and pre-pass in one launch
            pool.begin_step(slots, lengths, relpos=(0, x[..., :D], pos, bv, bd_buf))
        else:
            pool.begin_step(slots, lengths)
        if ev is not None:
            ev[0].record()
        # append of the chunk's K/V rows fused into the attention call
        pool.attention(0, x[..., :D], pos, bu, bv, slots, lengths, o,
                       key=x[..., D:2 * D], value=x[..., 2 * D:], bd=bd_buf)
        if ev is not None:
            ev[1].record()
        pool.end_step(slots, lengths)

    def step(buf, ev=None):
        run_step(buf, out, ev)

    def make_ops():
        """The per-op breakdown: name -> (launch fn, algorithmic bytes, launches)."""
        kv_out = [torch.empty(B, W, D, dtype=dt, device=dev) for _ in range(2)]
        kv_all = [torch.empty(L, B, W, D, dtype=dt, device=dev) for _ in range(2)]
        x2 = rnd(B, T, 2 * D)
        wconv = rnd(D, 1, 9)
        lnw, lnb = rnd(D) + 1, rnd(D)
        yconv = torch.empty(B, T, D, dtype=dt, device=dev)
        ops = {
            "append": (lambda: pool.append(0, qkv[0][..., D:2 * D], qkv[0][..., 2 * D:], slots),
                       nb["append"] * units, 1),
            "attention": (lambda: pool.attention(0, qkv[0][..., :D], pos, bu, bv, slots, lengths, out),
                          nb["attention"] * units, 1),
            "attention+append": (lambda: pool.attention(0, qkv[0][..., :D], pos, bu, bv, slots,
                                                        lengths, out, key=qkv[0][..., D:2 * D],
                                                        value=qkv[0][..., 2 * D:]),
                                 (nb["attention"] + nb["append"]) * units, 1),
            "gather": (lambda: [pool.gather(l, slots, *kv_out) for l in range(L)],
                       nb["gather"] * units, L),
            "gather_all_layers": (lambda: pool.gather_layers(0, L, slots, *kv_all),
                                  nb["gather"] * units, 1),
            "conv": (lambda: [pool.conv_step(l, x2, wconv, slots, lengths, lnw, lnb, 1e-5, yconv)
                              for l in range(L)], nb["conv"] * units, L),
        }
        return ops

    # fill the 70-frame left context, then warm up
    for i in range(-(-left // T)):
        step(qkv[i % NBUF])
    for i in range(args.warmup):
        step(qkv[i % NBUF])
    torch.cuda.synchronize()
    if args.profile or args.profile_op:   # a short, fixed launch sequence for ncu; no report
        if args.profile_op:
            fn = make_ops()[args.profile_op][0]
            pool.begin_step(slots, lengths)
            for i in range(args.steps):
                fn()
        else:
            for i in range(args.steps):
                step(qkv[i % NBUF])
        torch.cuda.synchronize()
        print(json.dumps({"profile_run": args.model, "op": args.profile_op or "step",
                          "steps": args.steps, "device_error_word": pool.read_error()}))
        return

    clocks = ClockSampler(local)
    clocks.start()
    t_soak = time.perf_counter()
    while time.perf_counter() - t_soak < 1.0:   # bring clocks to load level, untimed
        for i in range(50):
            step(qkv[i % NBUF])
        torch.cuda.synchronize()

    K = args.steps
    # (a) eager steps with CUDA events around the attention kernel: roofline timing
    evs = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(4)) for _ in range(K)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record()
    for i in range(K):
        step(qkv[i % NBUF], evs[i])
    e1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    eager_ms = e0.elapsed_time(e1) / K
    # (a') eager steps queued behind a GPU-side spin: the host enqueues a step
    # more slowly than the GPU runs it, so in (a) the events around a launch
    # also time the host's gap before it; queued, the kernels run back to back
    # and the events time the launches alone (roofline.avg_launch_ms)
    KQ = min(K, 48)
    evq = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(4)) for _ in range(KQ)]
    torch.cuda.synchronize()
    # cycles at <= 2 GHz; at most 0.1 s (a profiler's serialised launches make eager_ms large)
    torch.cuda._sleep(int(min(0.1, 2e-3 + 2 * KQ * eager_ms * 1e-3) * 2.0e9))
    for i in range(KQ):
        step(qkv[i % NBUF], evq[i])
    torch.cuda.synchronize()
    attn_ms = sum(e[0].elapsed_time(e[1]) for e in evq) / KQ
    bd_ms = sum(e[2].elapsed_time(e[3]) for e in evq) / KQ
    start_ms = sum(e[3].elapsed_time(e[0]) for e in evq) / KQ

    # (b) the same steps replayed as CUDA graphs (one graph per input buffer): `value`
    ms = eager_ms
    graphs = []
    if not args.no_graph:
        for i in range(NBUF):
            gph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gph):
                step(qkv[i])
            graphs.append(gph)
        for i in range(max(3, args.warmup)):
            graphs[i % NBUF].replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        for i in range(K):
            graphs[i % NBUF].replay()
        g1.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms = g0.elapsed_time(g1) / K
    clk = clocks.stop()
    enc_line = dec_line = pre_line = fe_line = pipe_line = gemm_line = serve_line = None
    # the model-level lines are one GPU's measurements: run them on single-GPU
    # runs only, so that no rank waits in a collective while rank 0 measures
    if world == 1 and not args.no_breakdown:
        enc_line = encoder_step(args.model, 160 if args.model == "small" else 480, 20, dev)
        dec_line = rnnt_decode_step(args.model, 10, dev)
        pre_line = pre_encode_step(args.model, 10, dev)
        fe_line = feature_step(args.model, 50, dev)
        gemm_line = {m: gemm_step(m, 20, dev) for m in ("small", "large", "serving")}
        pipe_line = streaming_step(args.model, 10, dev)
    if not args.no_serve:
        serve_line = serve_lines(args, dev, world)
    err = pool.read_error()

    # ---- end to end through the public API, as a serving loop runs it: every step
    # copies its Q/K/V in from pinned host memory and its attention output back to
    # pinned host memory.  Three streams (copy in, compute, copy out) and three
    # buffer sets let step i's copies overlap steps i-1 and i+1; every step's
    # copies are inside the timed region.
    NB2 = 3
    hq = [b.cpu().pin_memory() for b in qkv]
    hout = [torch.empty(out.shape, dtype=dt).pin_memory() for _ in range(NB2)]
    dq = [torch.empty_like(qkv[0]) for _ in range(NB2)]
    dout = [torch.empty_like(out) for _ in range(NB2)]
    comp = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(NB2)]
    ev_comp = [torch.cuda.Event() for _ in range(NB2)]
    ev_out = [torch.cuda.Event() for _ in range(NB2)]

    def api_step(x, o):
        run_step(x, o)

    def e2e_issue(i):
        k = i % NB2
        with torch.cuda.stream(s_in):
            if i >= NB2:
                s_in.wait_event(ev_comp[k])            # dq[k] read by step i - NB2
            dq[k].copy_(hq[i % NBUF], non_blocking=True)
            ev_in[k].record(s_in)
        comp.wait_event(ev_in[k])
        if i >= NB2:
            comp.wait_event(ev_out[k])                 # dout[k] copied out by step i - NB2
        api_step(dq[k], dout[k])
        ev_comp[k].record(comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_comp[k])
            hout[k].copy_(dout[k], non_blocking=True)
            ev_out[k].record(s_out)

    def e2e_loop(n):
        start = torch.cuda.Event(enable_timing=True)
        start.record(comp)
        s_in.wait_event(start)
        s_out.wait_event(start)
        for i in range(n):
            e2e_issue(i)
        comp.wait_event(ev_out[(n - 1) % NB2])
        stop = torch.cuda.Event(enable_timing=True)
        stop.record(comp)
        return start, stop

    e2e_loop(max(3, args.warmup))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    f0, f1 = e2e_loop(K)
    torch.cuda.synchronize()
    e2e_ms = f0.elapsed_time(f1) / K
    # the copy-in alone, every rank at once (as in the loop): this rank's host
    # link rate, to read the e2e figure against (ranks share the host's links)
    if world > 1:
        dist.barrier()
    h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s_in):
        h0.record(s_in)
        for i in range(K):
            dq[i % NB2].copy_(hq[i % NBUF], non_blocking=True)
        h1.record(s_in)
    torch.cuda.synchronize()
    h2d_gbs_rank = hq[0].numel() * hq[0].element_size() * K / (h0.elapsed_time(h1) * 1e-3) / 1e9
    h2d_ranks = [h2d_gbs_rank]
    if world > 1:
        t = torch.zeros(world, dtype=torch.float64, device=dev)
        t[rank] = h2d_gbs_rank
        dist.all_reduce(t)
        h2d_ranks = t.tolist()
    if world > 1:
        dist.barrier()

    # ---- per-op breakdown (separate loops, same pool)
    breakdown = {}
    if not args.no_breakdown and rank == 0:
        flush_w = torch.empty(256 << 20, dtype=torch.uint8, device=dev)   # 2x L2
        flush_r = torch.ones(64 << 20, dtype=torch.int32, device=dev)     # 2x L2

        def timeit(fn, n=20):
            """Device time of fn's launches: captured once as a CUDA graph (no host
            launch cost), each replay timed with events after an L2 flush (a
            256 MB write, then a 256 MB read that writes its dirty lines back)."""
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            gph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gph):
                fn()
            gph.replay()
            total = 0.0
            for _ in range(n):
                flush_w.zero_()
                flush_r.sum()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                gph.replay()
                b.record()
                b.synchronize()
                total += a.elapsed_time(b)
            return total / n
        ops = make_ops()
        hbm, _ = peaks()
        pool.begin_step(slots, lengths)   # this step's pages and windows; every op re-runs it
        for name, (fn, nbytes, launches) in ops.items():
            t = timeit(fn)
            breakdown[name] = {"ms": round(t, 4), "GB/s": round(nbytes / t / 1e6, 1),
                               "frac": round(nbytes / t / 1e6 / hbm, 3), "launches": launches,
                               "bytes_per_stream_layer": nbytes // units}
        breakdown["at_2048_streams"] = ops_at_scale(args.model, dev, timeit, hbm)

    ms, e2e_ms, attn_ms, eager_ms = max_over_ranks([ms, e2e_ms, attn_ms, eager_ms], dev)

    if rank == 0:
        hbm, kind = peaks()
        kernel_name = ("paged_attn_stacked_kernel (append fused)" if H * T <= 16 and dh == 64
                       else "paged_attn_heads_kernel (+append_kernel)" if dh == 128 and 8 <= T <= 16
                       else "paged_attn_bf16_kernel (+append_kernel)")
        attn_bytes = step_bytes    # the fused kernel moves the append's bytes too
        achieved = attn_bytes / (attn_ms * 1e-3) / 1e9
        traffic = None
        tp = os.path.join(REPO, "profiles", "attention_traffic.json")
        if os.path.exists(tp):
            for tj in json.load(open(tp)):
                if tj.get("model") == args.model and tj.get("streams") == B:
                    traffic = tj.get("dram_bytes_per_launch")
        cpu = None
        if world == 1:
            gbs, done, el, threads, sample, ckind = cpu_reference(args, args.cpu_seconds)
            cpu = {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": ckind,
                   "sample": sample}
        value = job_throughput(step_bytes, world, ms)
        e2e = job_throughput(step_bytes, world, e2e_ms)
        line = {
            "metric": "paged-attn HBM GB/s (append + attention, algorithmic bytes)",
            "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "ms_per_step_eager": round(eager_ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": workload_config(args.model, B, world),
            "launch": "CUDA graph per step" if graphs else "eager",
            "roofline": {"bound": "hbm", "kernel": kernel_name,
                         "achieved": round(achieved, 1), "peak": hbm, "peak_kind": kind,
                         "unit": "GB/s", "frac": round(achieved / hbm, 3), "traffic": traffic,
                         "alg_bytes_per_launch": attn_bytes, "avg_launch_ms": round(attn_ms, 4)},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": qkv[0].numel() * 2, "d2h_bytes_per_step": out.numel() * 2,
                    "ms_per_step": round(e2e_ms, 4),
                    "pipeline": "copy-in, compute and copy-out streams, 3 buffer sets, eager API calls",
                    # the copy-in alone on every rank at once: the host-link rate per rank
                    "h2d_gbs_per_rank": [round(v, 1) for v in h2d_ranks]},
            # per step: [rel-pos pre-pass,] allocator+windows, attention+append, counters
            "gpu_launches": (4 if relpos_mode == "prepass" else 3) * K,
            "relpos": {"mode": relpos_mode,
                       "prepass_ms": round(bd_ms, 4) if relpos_mode == "prepass" else None,
                       "step_start_ms": round(start_ms, 4)},
            "clocks": clk,
            "device_error_word": err,
            "ops": breakdown,
            "encoder_step": enc_line,
            "rnnt_decode": dec_line,
            "pre_encode": pre_line,
            "features": fe_line,
            "gemm": gemm_line,
            "streaming_step": pipe_line,
            "streams_at_p99_160ms": serve_line,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
