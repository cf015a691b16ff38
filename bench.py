#!/usr/bin/env python
"""Decode-step GEMV benchmark of rumik_fast_b200 on B200 (the 36-layer decode-step projection set + the int8 audio head).

Headline (the BASELINE metric, decode-step GEMV HBM GB/s): one step = the 36-layer config-1 projection set (per
layer: QKV 5120x3072, o_proj 3072x3072, gate_up 16384x3072, down 3072x8192, int4 group-128) followed by the int8
audio head (16385x3072), replayed from one CUDA graph, the way rumik-fast's full-step benchmark runs it
(kernels/bench_gemv.py:83-113; engine/rumik_int4.py:225-245). Inputs follow the reference benchmark: fixed
activations (x_h for QKV/o/gate_up/head, x_i for down). The 144 projections run as one persistent
rb_gemv_int4_multi launch plus the head. The weights (1.98 GB) are larger than L2 (126 MB), so no L2 flush is
needed between steps.

The same JSON line carries sub-records, each timed by its own CUDA events:
  step      the real token-to-token decode step at position 511 (embedding row, 36 fused layers with attention,
            final norm, head, sampler; engine/rumik_fused.py:97-121): its tok/s is the line's "tok_s"
  prefill   config 3: the int4-weight matmul over the projection set at M = 34, 256, 1024 tokens
  gemv_c0   config 0: 36 distinct 8192x3072 GEMVs through gemv_int4_cuda in one CUDA graph, best of 3 rounds of
            20 replays (kernels/bench_cuda.py:18-32)
  chain     the headline step as an unmodified engine issues it: 145 stream-ordered gemv_int4_cuda/gemv_int8_cuda
            launches

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-extras]

Prints one JSON line (rank 0). value = algorithmic HBM bytes of a step / device time of a step, summed over
ranks (each rank runs an independent replica of the step: weak scaling).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
import types

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

LAYERS = 36
METRIC = "decode-step GEMV HBM GB/s"
UNIT = "GB/s"
PREFILL_TOKENS = (34, 256, 1024)
BATCHES = (4, 16)  # config 4: independent decode streams per GPU (batch 1 is the headline line)
# DRAM bytes (read + write) per launch of gemv_int4_tc_kernel on the 36-layer set: ncu capture of the 3-layer
# case of the current build scaled x12 by blocks streamed (profiles/gemv_int4_tc_3layer_traffic.md)
NCU_TRAFFIC_PER_LAUNCH = 1967102976
# The same for the one launch of the 144 projections and the int8 head's rows (the default step): 12 x the
# 3-layer projections + the head's share of a capture of the 3-layer list with the head (same profile)
NCU_TRAFFIC_STEP_LAUNCH = 2018034944


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-prefetch", action="store_true", help="do not stream weights before the PDL wait")
    ap.add_argument("--no-extras", action="store_true", help="headline only: no step/prefill/gemv_c0/chain records")
    ap.add_argument("--head", default="list_last", choices=["list", "list_last", "concurrent", "serial"],
                    help="set mode: the int8 head's rows as the first entry of the projection launch (list), its "
                         "own launch on a forked branch of the step graph (concurrent) or after the list (serial)")
    ap.add_argument("--mode", default="set", choices=["set", "chain"],
                    help="set: the 144 projections as one persistent launch (Int4GemvSet); chain: one launch each")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="length of the bounded CPU-baseline sample (0: skip it)")
    ap.add_argument("--layers", type=int, default=36,
                    help="decoder layers in the step (36 = config 1; fewer only for small profiling cases)")
    ap.add_argument("--pos", type=int, default=511, help="step workload: position of the token (cache slots read)")
    ap.add_argument("--attn", default="separate", choices=["fused", "separate", "persistent"],
                    help="step workload: per layer three launches with the attention in its own launch, or inside "
                         "the o_proj/down_proj launch (fused); or every layer in one launch of the whole-step "
                         "kernel (persistent)")
    ap.add_argument("--scales", default="fp16", choices=["fp16", "8bit"],
                    help="decode workload: the reference's fp16 scales, or 8-bit double-quantised ones")
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill", "step"],
                    help="decode: config 1 + 2 (the headline); prefill: config 3, the int4-weight matmul over the "
                         "36-layer projection set for --tokens prompt tokens; step: the full decode step alone")
    ap.add_argument("--tokens", type=int, default=256, help="prefill prompt length M (config 3: 34, 256, 1024)")
    ap.add_argument("--collective", default="nccl", choices=["peer", "nccl"],
                    help="tp only: per-layer reduction by the peer-memory kernel or by add + NCCL all-reduce")
    ap.add_argument("--parallel", default="replica", choices=["replica", "tp"],
                    help="replica: one independent decode stream per GPU (weak scaling); tp: one stream, every "
                         "projection sharded over the GPUs with one NCCL all-reduce per layer (strong scaling)")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def peaks():
    """(HBM GB/s, kind, bf16 TFLOP/s burst) from MEASURED_PEAKS.json, else the pool's fallback figures."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        j = json.load(open(p))
        return float(j["hbm_gbs"]), "measured", float(j.get("bf16_tflops", 1590.0))
    return 6650.0, "fallback", 1590.0


# ---------------------------------------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock, power and clock-event reasons of this GPU, polled through NVML about every millisecond while
    the timed regions run (read-only queries), so that even a timed region of a few milliseconds holds samples.
    Falls back to nvidia-smi at 200 ms when NVML is unavailable."""

    REASONS = (("hw_slowdown", 0x8), ("sw_thermal_slowdown", 0x20), ("hw_thermal_slowdown", 0x40),
               ("hw_power_brake_slowdown", 0x80), ("sw_power_cap", 0x4))
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = torch.device(device)
        self.rows, self.proc, self.thread, self.stop, self.nvml = [], None, None, False, None
        self.max_mhz = None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(self.device)
        try:
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID("GPU-" + str(props.uuid))
        except Exception:  # noqa: BLE001
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)

    def __enter__(self):
        try:
            nv, h = self._nvml_handle()
            self.nvml = (nv, h)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            return self
        except Exception:  # noqa: BLE001
            self.nvml = None
        try:
            idx = self.device.index or 0
            vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
            if vis.replace(",", "").isdigit():
                idx = int(vis.split(",")[idx])
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(idx), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read_smi, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _poll(self):
        nv, h = self.nvml
        while not self.stop:
            try:
                sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                reasons = int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
                self.rows.append((sm, reasons))
            except Exception:  # noqa: BLE001
                return
            time.sleep(0.001)

    def _read_smi(self):
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.proc.stdout:
            r = [c.strip() for c in line.split(",")]
            if len(r) < 9:
                continue
            bits = 0
            for nm, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    bits |= dict(self.REASONS)[nm]
            try:
                self.max_mhz = float(r[2])
                self.rows.append((float(r[1]), bits))
            except ValueError:
                pass

    def mark(self):
        return len(self.rows)

    def __exit__(self, *a):
        self.stop = True
        if self.proc:
            self.proc.terminate()
            self.proc.wait()
        if self.thread:
            self.thread.join(timeout=2)
        if self.nvml:
            try:
                self.nvml[0].nvmlShutdown()
            except Exception:  # noqa: BLE001
                pass

    def summary(self, start=0, end=None):
        rows = self.rows[start:end]
        if not rows:
            return None
        reasons = sorted({nm for _, bits in rows for nm, b in self.REASONS if bits & b})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": self.max_mhz,
                "samples": len(rows), "reasons": reasons, "source": "nvml" if self.nvml else "nvidia-smi"}


# ---------------------------------------------------------------------------------------------- workload
def build_workload(dev, seed, nlayers=LAYERS, scales="fp16"):
    """scales "8bit": every projection's fp16 scale / min repacked as 8-bit double-quantised scales
    (rumik_fast_b200.scales8), entries (q, Scales8, None)."""
    from rumik_fast_b200 import synthetic as syn
    gen = syn.generator(seed, dev)
    layers = [[syn.int4_weights(n, k, gen, dev) for _, n, k in syn.LAYER_SHAPES] for _ in range(nlayers)]
    if scales == "8bit":
        from rumik_fast_b200 import scales8
        layers = [[(q, scales8.pack(s, m), None) for q, s, m in L] for L in layers]
    head = syn.int8_weights(*syn.HEAD_SHAPE, gen, dev)
    xh = syn.activations((3072,), gen, dev)
    xi = syn.activations((8192,), gen, dev)
    outs = [torch.empty(n, device=dev, dtype=torch.float16) for _, n, _ in syn.LAYER_SHAPES]
    logits = torch.empty(syn.HEAD_SHAPE[0], device=dev, dtype=torch.float16)
    int4_bytes = nlayers * sum(syn.int4_bytes(n, k) for _, n, k in syn.LAYER_SHAPES)
    if scales == "8bit":  # 2 bytes per group instead of 4, plus a 4-byte factor per row
        int4_bytes -= nlayers * sum(2 * n * (k // 128) - 4 * n for _, n, k in syn.LAYER_SHAPES)
    head_bytes = syn.int8_bytes(*syn.HEAD_SHAPE)
    return dict(layers=layers, head=head, xh=xh, xi=xi, outs=outs, logits=logits, int4_bytes=int4_bytes,
                head_bytes=head_bytes)


def step_fn(w, mode="set", with_head=True, head="list"):
    """One decode step's projections: 36 x (QKV, o_proj, gate_up with x_h; down with x_i) + the int8 head.
    mode "set": the 144 int4 GEMVs as one persistent launch; the head (independent of them) by `head`:
      "list"       its int8 rows are the first entry of that launch (one more kind of work item);
      "list_last"  the same rows as the last entry (the default: the head's heavier blocks then fill the CTAs
                   that the projections' static deal leaves lightest);
      "concurrent" its own launch on a forked branch of the step's graph, launched first;
      "serial"     its own launch after the list.
    mode "chain": one launch per GEMV, in stream order, as an unmodified engine issues them."""
    import rumik_fast_b200 as rb
    layers, outs, xh, xi = w["layers"], w["outs"], w["xh"], w["xi"]
    side = None
    if mode == "set":
        entries = []
        for L in layers:
            entries += [(xh, *L[0], outs[0]), (xh, *L[1], outs[1]), (xh, *L[2], outs[2]), (xi, *L[3], outs[3])]
        if with_head and head in ("list", "list_last"):
            he = (xh, *w["head"], None, w["logits"])
            entries = [he] + entries if head == "list" else entries + [he]
            with_head = False
        projections = rb.Int4GemvSet(entries)
        side = torch.cuda.Stream() if head == "concurrent" else None
    else:
        def projections():
            for L in layers:
                rb.gemv_int4_cuda(xh, *L[0], out=outs[0])   # QKV
                rb.gemv_int4_cuda(xh, *L[1], out=outs[1])   # o_proj
                rb.gemv_int4_cuda(xh, *L[2], out=outs[2])   # gate_up
                rb.gemv_int4_cuda(xi, *L[3], out=outs[3])   # down

    def step():
        if with_head and side is not None:
            cur = torch.cuda.current_stream()
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                rb.gemv_int8_cuda(xh, *w["head"], out=w["logits"])
            projections()
            cur.wait_stream(side)
            return
        projections()
        if with_head:
            rb.gemv_int8_cuda(xh, *w["head"], out=w["logits"])
    return step


def capture(fn):
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


def timed(run, steps, warmup, world):
    """Device time of `steps` calls of run() (CUDA events on the current stream), max over ranks, in ms."""
    import torch.distributed as dist
    for _ in range(warmup):
        run()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        run()
    e.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = s.elapsed_time(e)
    if world > 1:
        t = torch.tensor([ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def free():
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


# ---------------------------------------------------------------------------------------------- CPU side
def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def host_layers(nlayers, seed):
    """Distinct config-1 layers, the int8 head and the two activation vectors as host torch tensors."""
    from rumik_fast_b200 import synthetic as syn
    g = torch.Generator().manual_seed(seed)
    layers = [[syn.int4_weights(n, k, g, "cpu") for _, n, k in syn.LAYER_SHAPES] for _ in range(nlayers)]
    head = syn.int8_weights(*syn.HEAD_SHAPE, g, "cpu")
    return layers, head, syn.activations((3072,), g, "cpu"), syn.activations((8192,), g, "cpu")


def cpu_layer(L, xh, xi):
    """One layer's four projections by the reference's CPU path (oracle/reference_cpu.py)."""
    from oracle import reference_cpu as R
    R.gemv_int4_torch(xh, *L[0])
    R.gemv_int4_torch(xh, *L[1])
    R.gemv_int4_torch(xh, *L[2])
    R.gemv_int4_torch(xi, *L[3])


def cpu_head(head, xh):
    from oracle import reference_cpu as R
    R.gemv_int8_torch(xh, *head, signed=True)


def cpu_baseline_sample(seconds):
    """The reference's CPU dequantise-then-matvec (torch on all host threads) over 8 distinct config-1 layers,
    cycled for about `seconds`, plus the head once: GB/s of algorithmic bytes."""
    from rumik_fast_b200 import synthetic as syn
    threads = cpu_threads()
    torch.set_num_threads(threads)
    layers, head, xh, xi = host_layers(8, 99)
    layer_bytes = sum(syn.int4_bytes(n, k) for _, n, k in syn.LAYER_SHAPES)
    cpu_layer(layers[0], xh, xi)  # warm the allocator and the thread pool
    t0 = time.perf_counter()
    cpu_head(head, xh)
    nbytes, n = syn.int8_bytes(*syn.HEAD_SHAPE), 0
    while time.perf_counter() - t0 < seconds:
        cpu_layer(layers[n % len(layers)], xh, xi)
        nbytes += layer_bytes
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(nbytes / dt / 1e9, 3), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"reference CPU path (torch dequantize(q, s, m) @ x.float(), kernels/int4_gemv.py:27-30, "
                      f"on {threads} threads): the int8 head + {n} config-1 layers cycled over 8 distinct layers, "
                      f"{dt:.1f} s"}


def run_reference(a):
    """The reference's own CPU path for the headline step, timed on the host cores: each step is the whole
    decode-step projection set (36 distinct layers) plus the int8 head, by torch dequantise-then-matvec on all
    host threads. Rank 0 only."""
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    from rumik_fast_b200 import synthetic as syn
    threads = cpu_threads()
    torch.set_num_threads(threads)  # torchrun sets OMP_NUM_THREADS=1 for N > 1: override it
    layers, head, xh, xi = host_layers(a.layers, 4242)
    step_bytes = a.layers * sum(syn.int4_bytes(n, k) for _, n, k in syn.LAYER_SHAPES) + syn.int8_bytes(*syn.HEAD_SHAPE)

    def step():
        for L in layers:
            cpu_layer(L, xh, xi)
        cpu_head(head, xh)
    # every step is a whole step; the counts are capped so that the run stays within a few minutes
    warm_budget, timed_budget = 30.0, 150.0
    t0 = time.perf_counter()
    step()
    est = time.perf_counter() - t0
    warmup = 1
    while warmup < a.warmup and (warmup + 1) * est <= warm_budget:
        step()
        warmup += 1
    steps = max(1, min(a.steps, int(timed_budget // max(est, 1e-3))))
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = time.perf_counter() - t0
    ms = dt / steps * 1e3
    gbs = step_bytes / (ms * 1e-3) / 1e9
    note = "" if (steps, warmup) == (a.steps, a.warmup) else (
        f"; {steps} timed / {warmup} warm-up steps of the {a.steps} / {a.warmup} asked, to stay within a few minutes")
    line = {"metric": METRIC, "value": round(gbs, 3), "unit": UNIT, "n_gpus": a.gpus, "steps": steps,
            "warmup": warmup, "ms_per_step": round(ms, 1), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic", "impl": "reference",
            "config": {"workload": f"config-1 {a.layers}-layer decode-step projection set (QKV 5120x3072, o "
                                   "3072x3072, gate_up 16384x3072, down 3072x8192; int4 g128) + config-2 int8 head "
                                   "16385x3072, batch 1: the reference's CPU path, torch dequantize(q, s, m) @ x.float() "
                                   "(kernels/int4_gemv.py:27-30, kernels/bench_cuda.py:38) per matrix" + note,
                       "batch": 1, "bytes_per_step": step_bytes, "threads": threads},
            "tok_s": round(1e3 / ms, 4),
            "cpu_baseline": {"value": round(gbs, 3), "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{steps} whole decode steps ({4 * a.layers} int4 GEMVs + the int8 head "
                                       "each), "
                                       f"{dt:.1f} s"},
            "e2e": {"value": round(gbs, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------------------------- sub-records
STEP_SHAPE = dict(H=3072, nq=24, nkv=8, hd=128, inter=8192, S=2048, eps=1e-5)


def build_step(dev, seed, nlayers, pos, attn_mode="separate"):
    """A whole decode step at the config-1 shapes (3072 hidden, 24 query / 8 key-value heads of 128, MLP 8192,
    36 layers, int8 head), laid out as rumik-fast's fused engine runs it (engine/rumik_fused.py:83-118), with the
    glue fused: per layer [add_ln + QKV + gate_up + rope/KV/silu*up] (one launch), attention (one launch),
    [o_proj + down_proj] (one launch); then the final add + LayerNorm and the int8 head. Random weights, a cache
    filled with random keys/values, and the token at position `pos` (slots 0..pos are read)."""
    import rumik_fast_b200 as rb
    from rumik_fast_b200 import fused
    from rumik_fast_b200 import synthetic as syn
    from rumik_fast_b200.attention import DecodeAttention
    c = STEP_SHAPE
    H, nq, nkv, hd, inter, S = c["H"], c["nq"], c["nkv"], c["hd"], c["inter"], c["S"]
    assert 0 <= pos < S
    gen = syn.generator(seed, dev)
    f16 = torch.float16
    vocab = 32768  # int8 token-embedding table (engine/fused.py:18-27); layer 0 gathers the token's row
    emb_q = torch.randint(-127, 128, (vocab, H), generator=gen, device=dev, dtype=torch.int16).to(torch.int8)
    emb_s = torch.rand(vocab, generator=gen, device=dev) * 0.02 + 0.001
    tok = torch.tensor([1234], device=dev, dtype=torch.int64)
    lnw = [(1 + 0.1 * syn.activations((H,), gen, dev).float()).to(f16) for _ in range(nlayers + 1)]
    inv = 1.0 / (10000.0 ** (torch.arange(0, hd, 2, device=dev).float() / hd))
    ang = torch.outer(torch.arange(S, device=dev).float(), inv).repeat_interleave(2, -1)
    cos, sin = ang.cos().to(f16), ang.sin().to(f16)
    kc = torch.randn(nlayers, nkv, S, hd, generator=gen, device=dev).to(f16)
    vc = torch.randn(nlayers, nkv, S, hd, generator=gen, device=dev).to(f16)
    xr = [torch.empty(H, device=dev, dtype=f16) for _ in range(2)]
    q_out, ob = (torch.empty(nq * hd, device=dev, dtype=f16) for _ in range(2))
    act = torch.empty(inter, device=dev, dtype=f16)
    buf_o, buf_d, hn = (torch.empty(H, device=dev, dtype=f16) for _ in range(3))
    logits = torch.empty(syn.HEAD_SHAPE[0], device=dev, dtype=f16)
    pos_t = torch.tensor([pos], device=dev, dtype=torch.int64)
    layer_in, attn, layer_out, pl_layers = [], [], [], []
    persistent = attn_mode == "persistent"
    xin = None
    for L in range(nlayers):
        xout = xr[L % 2]
        qkv = syn.int4_weights((nq + 2 * nkv) * hd, H, gen, dev)
        gu = fused.interleave_gate_up(*syn.int4_weights(2 * inter, H, gen, dev))
        if persistent:  # every layer in one launch of the whole-step kernel (DecodeLayers)
            wo = syn.int4_weights(H, nq * hd, gen, dev)
            wd = syn.int4_weights(H, inter, gen, dev)
            pl_layers.append(dict(qkv=qkv, gate_up=gu, o_proj=wo, down=wd, ln_w=lnw[L], k_cache=kc[L],
                                  v_cache=vc[L], rope=L % 4 != 3))
            continue
        ln = (fused.AddLn(xin, buf_o, buf_d, lnw[L], xout, eps=c["eps"]) if L else
              fused.AddLn.from_embedding(emb_q, emb_s, tok, lnw[0], xout, eps=c["eps"]))
        layer_in.append(fused.AddLnGemvPost(qkv, gu, add_ln=ln, pos=pos_t, cos=cos, sin=sin, k_cache=kc[L],
                                            v_cache=vc[L], q_out=q_out, act=act, n_q_heads=nq, n_kv_heads=nkv,
                                            rope=L % 4 != 3))
        wo = syn.int4_weights(H, nq * hd, gen, dev)
        wd = syn.int4_weights(H, inter, gen, dev)
        if attn_mode == "fused":  # attention inside the o_proj/down_proj launch
            layer_out.append(fused.AttnGemvSet([(act, *wd, buf_d), (ob, *wo, buf_o)], q=q_out, k_cache=kc[L],
                                               v_cache=vc[L], pos=pos_t, out=ob, n_q_heads=nq, n_kv_heads=nkv))
        else:
            attn.append(DecodeAttention(q_out, kc[L], vc[L], pos_t, ob, nq, nkv))
            layer_out.append(rb.Int4GemvSet([(ob, *wo, buf_o), (act, *wd, buf_d)]))
        xin = xout
    layers_launch = None
    if persistent:
        from rumik_fast_b200.decode_step import DecodeLayers
        layers_launch = DecodeLayers(pl_layers, pos=pos_t, cos=cos, sin=sin, emb_q=emb_q, emb_s=emb_s, tok=tok,
                                     n_q_heads=nq, n_kv_heads=nkv, eps=c["eps"])
        xin, buf_o, buf_d = layers_launch.last()
    final = fused.AddLn(xin, buf_o, buf_d, lnw[nlayers], None, eps=c["eps"], h_out=hn)
    head = syn.int8_weights(*syn.HEAD_SHAPE, gen, dev)
    # the sampling tail (engine/sample.py): stop predictor (LayerNorm, 512 x H bf16, GELU, 1 x 512), top-30,
    # Gumbel-max with in-graph uniforms; the sampled head row's id (< vocab) is the next step's token
    from rumik_fast_b200.sample import FusedSampler
    nz = 512
    eng = types.SimpleNamespace(
        hn=hn, H=H, dev=dev, audio_ids=torch.arange(syn.HEAD_SHAPE[0], device=dev, dtype=torch.int64),
        end_id=syn.HEAD_SHAPE[0] - 1, step_i=torch.zeros(1, dtype=torch.int64, device=dev), tok=tok,
        out=torch.zeros(4096, dtype=torch.int64, device=dev), temperature=0.8, top_k=30, min_new=8,
        stop={"0.weight": torch.ones(H, device=dev), "0.bias": torch.zeros(H, device=dev),
              "1.weight": (0.02 * torch.randn(nz, H, generator=gen, device=dev)).to(torch.bfloat16),
              "1.bias": torch.zeros(nz, device=dev), "3.weight": 0.05 * torch.randn(1, nz, generator=gen, device=dev),
              "3.bias": torch.full((1,), -100.0, device=dev)})  # never stops: every step draws a token
    sampler = FusedSampler(eng, lambda: logits)

    def step():
        if layers_launch is not None:
            layers_launch()
        for L in range(len(layer_in)):
            layer_in[L]()
            if attn:
                attn[L]()
            layer_out[L]()
        fused.add_layernorm(final)
        rb.gemv_int8_cuda(hn, *head, out=logits)
        sampler()

    shapes = [((nq + 2 * nkv) * hd, H), (2 * inter, H), (H, nq * hd), (H, inter)]
    wbytes = nlayers * sum(syn.int4_bytes(n, k) for n, k in shapes) + syn.int8_bytes(*syn.HEAD_SHAPE) + nz * H * 2
    kvbytes = nlayers * (2 * nkv * (pos + 1) * hd * 2 + 2 * nq * hd * 2)
    return dict(step=step, tok=tok, logits=logits, wbytes=wbytes + H, kvbytes=kvbytes,
                launches=(((nlayers + 35) // 36) if persistent else (2 if attn_mode == "fused" else 3) * nlayers) + 4,
                keep=(layer_in, attn, layer_out, final, head, kc, vc, emb_q, emb_s, sampler, eng, layers_launch))


def measure_step(dev, seed, nlayers, pos, attn_mode, steps, warmup, world, clk=None):
    """The whole decode step (fused glue + attention + head + sampler) from one CUDA graph, token id in and the
    drawn token out. Returns the record (tokens/s per GPU and the HBM roofline over the step's bytes)."""
    w = build_step(dev, seed, nlayers, pos, attn_mode)
    g = capture(w["step"])
    m0 = clk.mark() if clk else 0
    ms = timed(g.replay, steps, warmup, world)
    m1 = clk.mark() if clk else 0
    ms_step = ms / steps
    hx = w["tok"].cpu().pin_memory()
    hy = torch.empty(1, dtype=torch.int64).pin_memory()

    def e2e_step():  # token id in, next token id out
        w["tok"].copy_(hx, non_blocking=True)
        g.replay()
        hy.copy_(w["tok"], non_blocking=True)
    e2e_steps = max(1, steps // 2)
    ms_e2e = timed(e2e_step, e2e_steps, warmup, world) / e2e_steps
    peak, kind, _ = peaks()
    total = w["wbytes"] + w["kvbytes"]
    gbs = total / (ms_step * 1e-3) / 1e9
    rec = {"tok_s": round(world * 1e3 / ms_step, 1), "ms_per_step": round(ms_step, 5), "pos": pos, "layers": nlayers,
           "attention": attn_mode, "bytes_per_step": total, "weight_bytes": w["wbytes"], "kv_bytes": w["kvbytes"],
           "hbm_gbs": round(gbs, 1), "roofline_frac": round(gbs / peak, 4), "peak_gbs": peak, "peak_kind": kind,
           "e2e_tok_s": round(world * 1e3 / ms_e2e, 1), "e2e_h2d_bytes": 8, "e2e_d2h_bytes": 8,
           "launches_per_step": w["launches"],
           "clocks": clk.summary(m0, m1) if clk else None,
           "workload": f"{nlayers}-layer decode step at position {pos}: token id -> int8 embedding row (layer 0's "
                       "prologue); per layer add_ln + QKV 5120x3072 + gate_up 16384x3072 + rope/KV write/silu*up "
                       "(one launch), attention 24/8 heads x 128, o_proj 3072x3072 + down 3072x8192; final add_ln "
                       "+ int8 head 16385x3072; sampler (stop predictor, top-30, Gumbel-max; the drawn token feeds "
                       "the next step); one CUDA graph"}
    del g, w
    free()
    return rec


def measure_prefill(dev, seed, tokens, nlayers, steps, warmup, world, clk=None):
    """Config 3: Y = X W^T over the 36-layer projection set with X fp16 [M, K], one mm_int4 launch per matrix,
    replayed from one CUDA graph, for each M in `tokens`. Returns {M: record}."""
    from rumik_fast_b200 import synthetic as syn
    from rumik_fast_b200.mm_int4 import mm_int4, MmInt4Set
    gen = syn.generator(seed, dev)
    layers = [[syn.int4_weights(n, k, gen, dev) for _, n, k in syn.LAYER_SHAPES] for _ in range(nlayers)]
    wbytes = nlayers * sum(syn.int4_bytes(n, k) for _, n, k in syn.LAYER_SHAPES)
    hbm, hkind, tf_peak = peaks()
    tf_kind = hkind
    out = {}
    for M in tokens:
        xs = {k: syn.activations((M, k), gen, dev) for k in (3072, 8192)}
        ys = [torch.empty(M, n, device=dev, dtype=torch.float16) for _, n, _ in syn.LAYER_SHAPES]

        def step():
            for L in layers:
                for i, ((_, n, k), w) in enumerate(zip(syn.LAYER_SHAPES, L)):
                    mm_int4(xs[k], *w, out=ys[i])
        g = capture(step)
        m0 = clk.mark() if clk else 0
        ms = timed(g.replay, steps, warmup, world) / steps
        m1 = clk.mark() if clk else 0
        # the same products as persistent list launches (MmInt4Set, 52 products a launch)
        lst = MmInt4Set([(xs[k], *w, ys[i]) for L in layers for i, ((_, n, k), w) in enumerate(zip(syn.LAYER_SHAPES, L))])
        gl = capture(lst)
        ms_l = timed(gl.replay, steps, warmup, world) / steps
        flops = 2 * M * nlayers * sum(n * k for _, n, k in syn.LAYER_SHAPES)
        tf = flops / (ms * 1e-3) / 1e12
        gbs = wbytes / (ms * 1e-3) / 1e9
        bound = "hbm" if M < 64 else "tensor"
        frac = gbs / hbm if bound == "hbm" else tf / tf_peak
        tf_l, gbs_l = flops / (ms_l * 1e-3) / 1e12, wbytes / (ms_l * 1e-3) / 1e9
        frac_l = gbs_l / hbm if bound == "hbm" else tf_l / tf_peak
        out[str(M)] = {"tflops": round(world * tf, 1), "weight_gbs": round(gbs, 1), "ms_per_step": round(ms, 4),
                       "bound": bound, "roofline_frac": round(frac, 4),
                       "peak": hbm if bound == "hbm" else tf_peak,
                       "peak_unit": "GB/s" if bound == "hbm" else "TFLOP/s (bf16 dense, cuBLAS burst)",
                       "peak_kind": hkind if bound == "hbm" else tf_kind, "flops_per_step": flops,
                       "launches_per_step": 4 * nlayers, "clocks": clk.summary(m0, m1) if clk else None,
                       "list": {"tflops": round(world * tf_l, 1), "weight_gbs": round(gbs_l, 1),
                                "ms_per_step": round(ms_l, 4), "roofline_frac": round(frac_l, 4),
                                "launches_per_step": -(-4 * nlayers // 52),
                                "method": "rb_mm_int4_list: the same products in persistent launches of 52"}}
        del g, gl, lst, xs, ys
        free()
    del layers
    free()
    return out


def measure_batched(dev, seed, batches, nlayers, steps, warmup, world, clk=None):
    """Config 4's independent streams at batch B per GPU: one decode step's 144 projections for B tokens as
    mm_int4 calls (M = B: the weights are dequantised once per 128-row block for all B tokens) plus the int8 head
    at batch B (gemv_int8_cuda with x [B, K]), replayed from one CUDA graph. Returns {B: record}; batch 1 is the
    headline line itself."""
    from rumik_fast_b200 import synthetic as syn
    from rumik_fast_b200.mm_int4 import mm_int4, MmInt4Set
    import rumik_fast_b200 as rb
    gen = syn.generator(seed, dev)
    layers = [[syn.int4_weights(n, k, gen, dev) for _, n, k in syn.LAYER_SHAPES] for _ in range(nlayers)]
    head = syn.int8_weights(*syn.HEAD_SHAPE, gen, dev)
    wbytes = nlayers * sum(syn.int4_bytes(n, k) for _, n, k in syn.LAYER_SHAPES) + syn.int8_bytes(*syn.HEAD_SHAPE)
    hbm, hkind, _ = peaks()
    out = {}
    for B in batches:
        xs = {k: syn.activations((B, k), gen, dev) for k in (3072, 8192)}
        ys = [torch.empty(B, n, device=dev, dtype=torch.float16) for _, n, _ in syn.LAYER_SHAPES]
        logits = torch.empty(B, syn.HEAD_SHAPE[0], device=dev, dtype=torch.float16)

        def step():
            for L in layers:
                for i, ((_, n, k), w) in enumerate(zip(syn.LAYER_SHAPES, L)):
                    mm_int4(xs[k], *w, out=ys[i])
            rb.gemv_int8_cuda(xs[3072], *head, out=logits)
        g = capture(step)
        m0 = clk.mark() if clk else 0
        ms = timed(g.replay, steps, warmup, world) / steps
        m1 = clk.mark() if clk else 0
        # the projections as persistent list launches (rb_mm_int4_list), the head as before
        lst = MmInt4Set([(xs[k], *w, ys[i]) for L in layers for i, ((_, n, k), w) in enumerate(zip(syn.LAYER_SHAPES, L))])

        def step_list():
            lst()
            rb.gemv_int8_cuda(xs[3072], *head, out=logits)
        gl = capture(step_list)
        ms_l = timed(gl.replay, steps, warmup, world) / steps
        gbs = wbytes / (ms * 1e-3) / 1e9
        gbs_l = wbytes / (ms_l * 1e-3) / 1e9
        out[str(B)] = {"tok_s": round(world * B * 1e3 / ms, 1), "ms_per_step": round(ms, 4),
                       "weight_gbs": round(world * gbs, 1), "roofline_frac": round(gbs / hbm, 4), "peak_gbs": hbm,
                       "peak_kind": hkind, "launches_per_step": 4 * nlayers + 1,
                       "clocks": clk.summary(m0, m1) if clk else None,
                       "list": {"tok_s": round(world * B * 1e3 / ms_l, 1), "ms_per_step": round(ms_l, 4),
                                "weight_gbs": round(world * gbs_l, 1), "roofline_frac": round(gbs_l / hbm, 4),
                                "launches_per_step": -(-4 * nlayers // 52) + 1}}
        del g, gl, lst, xs, ys, logits
        free()
    del layers, head
    free()
    return out


def measure_c0(dev, seed, steps, warmup, world):
    """Config 0 the reference's way (kernels/bench_cuda.py:18-32): 36 distinct 8192x3072 int4 GEMVs through
    gemv_int4_cuda, captured in one CUDA graph; best of 3 rounds of max(steps, 20) replays (CUDA events)."""
    import rumik_fast_b200 as rb
    from rumik_fast_b200 import synthetic as syn
    gen = syn.generator(seed, dev)
    mats = [syn.int4_weights(8192, 3072, gen, dev) for _ in range(LAYERS)]
    x = syn.activations((3072,), gen, dev)
    y = torch.empty(8192, device=dev, dtype=torch.float16)
    g = capture(lambda: [rb.gemv_int4_cuda(x, *w, out=y) for w in mats])
    reps = max(steps, 20)
    best = min(timed(g.replay, reps, warmup if r == 0 else 3, world) / reps for r in range(3))
    per = best / LAYERS
    nb = syn.int4_bytes(8192, 3072)
    hbm, kind, _ = peaks()
    gbs = nb / (per * 1e-3) / 1e9
    rec = {"gbs": round(world * gbs, 1), "us_per_gemv": round(per * 1e3, 3), "bytes_per_gemv": nb,
           "roofline_frac": round(gbs / hbm, 4), "peak_gbs": hbm, "peak_kind": kind,
           "method": "36 distinct 8192x3072 matrices, one gemv_int4_cuda each, in one CUDA graph; best of 3 rounds "
                     f"x {reps} replays"}
    del g, mats
    free()
    return rec


def measure_chain(w, steps, warmup, world):
    """The headline step as an unmodified engine issues it: one gemv_int4_cuda per projection + the head."""
    g = capture(step_fn(w, "chain"))
    ms = timed(g.replay, steps, warmup, world) / steps
    hbm, kind, _ = peaks()
    nb = w["int4_bytes"] + w["head_bytes"]
    gbs = nb / (ms * 1e-3) / 1e9
    rec = {"gbs": round(world * gbs, 1), "ms_per_step": round(ms, 5), "launches_per_step": 4 * len(w["layers"]) + 1,
           "roofline_frac": round(gbs / hbm, 4)}
    del g
    free()
    return rec


# ---------------------------------------------------------------------------------------------- arms
def measure_tp(nlayers, collective, steps, warmup, rank, world, dev, clk):
    """Tensor-parallel decode step (config 4): every rank holds 1/world of each projection (column-parallel
    QKV/gate_up, row-parallel o/down, row-split int8 head); per layer one multi-GEMV launch of the rank's
    shards and one all-reduce of the 6 KB hidden vector, then the head and an all-gather of the logits.
    Every rank runs it (its collectives are the same on all ranks). Returns (ms per step, ms per step end to
    end, this rank's bytes per step, the whole model's bytes per step, clock summary, logits elements)."""
    from rumik_fast_b200 import synthetic as syn
    from rumik_fast_b200.tensor_parallel import TPDecodeStep
    gen = syn.generator(1234, dev)                    # the same full model on every rank; each keeps its shards
    layers = []
    for _ in range(nlayers):
        full = [syn.int4_weights(n, k, gen, dev) for _, n, k in syn.LAYER_SHAPES]
        layers.append((full[0], full[1], full[2], full[3]))
    head = syn.int8_weights(*syn.HEAD_SHAPE, gen, dev)
    x_h = syn.activations((3072,), gen, dev)
    x_attn = syn.activations((3072,), gen, dev)
    x_act = syn.activations((8192,), gen, dev)
    step = TPDecodeStep(layers, x_attn, x_act, head, rank, world, collective=collective)
    del layers, head
    torch.cuda.empty_cache()
    step.h[0].copy_(x_h)
    g = capture(step)
    full_bytes = nlayers * sum(syn.int4_bytes(n, k) for _, n, k in syn.LAYER_SHAPES) + syn.int8_bytes(*syn.HEAD_SHAPE)
    m0 = clk.mark() if clk else 0
    ms = timed(g.replay, steps, warmup, world)
    m1 = clk.mark() if clk else 0
    clocks = clk.summary(m0, m1) if clk else None
    ms_step = ms / steps
    hx = x_h.cpu().pin_memory()
    hl = torch.empty(step.logits_all.numel(), dtype=torch.float16).pin_memory()

    def e2e_step():
        step.h[0].copy_(hx, non_blocking=True)
        g.replay()
        hl.copy_(step.logits_all, non_blocking=True)
    e2e_steps = max(1, steps // 2)
    ms_e2e = timed(e2e_step, e2e_steps, warmup, world) / e2e_steps
    rank_bytes = step.bytes
    del g, e2e_step
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    step.close()
    del step
    free()
    return ms_step, ms_e2e, rank_bytes, full_bytes, clocks, hl.numel()


def tp_record(ms_tp, rank_bytes, full_bytes, world, collective, ms_one_gpu):
    """The bench line's `tp` sub-record at N > 1: the tensor-parallel step beside this run's one-GPU step."""
    peak, kind, _ = peaks()
    rank_gbs = rank_bytes / (ms_tp * 1e-3) / 1e9
    return {"ms_per_step": round(ms_tp, 5), "tok_s": round(1e3 / ms_tp, 1), "world": world, "collective": collective,
            "model_gbs": round(full_bytes / (ms_tp * 1e-3) / 1e9, 1), "rank_gbs": round(rank_gbs, 1),
            "rank_roofline_frac": round(rank_gbs / peak, 4), "peak_kind": kind,
            "one_gpu_ms_per_step": round(ms_one_gpu, 5), "speedup_vs_one_gpu": round(ms_one_gpu / ms_tp, 3),
            "limit": "per layer: one multi-GEMV launch of the rank's shards plus a 6 KB all-reduce of the hidden "
                     "vector, each latency-bound (a few microseconds of launch, ramp and tail per launch)",
            "workload": "config-4 tensor-parallel step: the config-1 36-layer projection set + int8 head sharded "
                        "(column-parallel QKV/gate_up, row-parallel o/down, row-split head), one all-reduce per "
                        "layer, batch 1; one_gpu = the same bytes on one GPU as this run's single projection-set "
                        "launch"}


def run_tp(a, rank, world, dev):
    """Tensor-parallel decode step alone (--parallel tp): the step as the line's value."""
    with ClockSampler(dev) as clk:
        ms_step, ms_e2e, rank_bytes, full_bytes, clocks, nlog = measure_tp(
            a.layers, a.collective, a.steps, a.warmup, rank, world, dev, clk)
    peak, peak_kind, _ = peaks()
    rank_gbs = rank_bytes / (ms_step * 1e-3) / 1e9
    if rank == 0:
        gbs = full_bytes / (ms_step * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": round(gbs, 1), "unit": UNIT, "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
            "config": {"workload": "config-4 tensor-parallel decode step: config-1 36-layer projection set + "
                                   "int8 head sharded over the GPUs (column-parallel QKV/gate_up, row-parallel "
                                   "o/down), one NCCL all-reduce of the hidden vector per layer, batch 1",
                       "batch": 1, "bytes_per_step": full_bytes, "parallelism": f"tp{world}",
                       "launches": "per layer: one multi-GEMV launch + " + (
                           "one peer-memory reduction kernel" if a.collective == "peer" else "add + NCCL all-reduce")
                       + "; head + all-gather", "collective": a.collective,
                       "l2": "no flush: 1.98 GB of weights per step over all ranks > 126 MB L2 per GPU"},
            "tok_s": round(1e3 / ms_step, 1),
            "e2e": {"value": round(full_bytes / (ms_e2e * 1e-3) / 1e9, 1), "unit": UNIT,
                    "h2d_bytes_per_step": 3072 * 2, "d2h_bytes_per_step": nlog * 2,
                    "ms_per_step": round(ms_e2e, 5)},
            "roofline": {"bound": "hbm", "achieved": round(rank_gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(rank_gbs / peak, 4), "peak_kind": peak_kind,
                         "kernel": "whole tensor-parallel step per rank (GEMVs + all-reduces)", "traffic": None,
                         "algorithmic_bytes_per_launch": None},
            "cpu_baseline": None, "clocks": clocks,
            "gpu_launches": a.steps * (a.layers + 1), "mode": "tp",
        }
        print(json.dumps(line), flush=True)
    return 0


def init_dist(dev, world):
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)


def end_dist(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def run_ours(a):
    import rumik_fast_b200 as rb
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    init_dist(dev, world)
    rb.set_weight_prefetch(not a.no_prefetch)
    if a.parallel == "tp":
        rc = run_tp(a, rank, world, dev)
        end_dist(world)
        return rc
    if a.scales == "8bit" and a.mode != "set":
        raise SystemExit("--scales 8bit runs on the projection-set kernel (--mode set)")
    w = build_workload(dev, seed=1234 + rank, nlayers=a.layers, scales=a.scales)
    g_step = capture(step_fn(w, a.mode, head=a.head))
    g_int4 = capture(step_fn(w, a.mode, with_head=False))
    int4_bytes = w["int4_bytes"]
    w_head_bytes = w["head_bytes"]
    step_bytes = int4_bytes + w_head_bytes
    logits_bytes = w["logits"].numel() * 2

    with ClockSampler(dev) as clk:
        m0 = clk.mark()
        ms = timed(g_step.replay, a.steps, a.warmup, world)
        m1 = clk.mark()
        ms_step = ms / a.steps

        # the int4 projections alone over the same steps: the dominant kernel when the head has its own launch,
        # and what the head costs inside the step (step - projections)
        ms4 = timed(g_int4.replay, max(1, a.steps // 2), a.warmup, world) / max(1, a.steps // 2)
        launches4 = 1 if a.mode == "set" else a.layers * 4
        one_launch = a.mode == "set" and a.head in ("list", "list_last")  # the step IS one list launch
        if one_launch:
            roof_bytes, roof_ms, roof_launches = step_bytes, ms_step, 1
        else:
            roof_bytes, roof_ms, roof_launches = int4_bytes, ms4, launches4
        achieved = (roof_bytes / roof_launches) / (roof_ms / roof_launches * 1e-3) / 1e9
        peak, peak_kind, _ = peaks()

        # end to end through the public API: pinned host inputs -> device, step, logits -> pinned host
        hx, hi = w["xh"].cpu().pin_memory(), w["xi"].cpu().pin_memory()
        hl = torch.empty_like(w["logits"], device="cpu").pin_memory()

        def e2e_step():
            w["xh"].copy_(hx, non_blocking=True)
            w["xi"].copy_(hi, non_blocking=True)
            g_step.replay()
            hl.copy_(w["logits"], non_blocking=True)
        e2e_steps = max(1, a.steps // 2)
        ms_e2e = timed(e2e_step, e2e_steps, a.warmup, world) / e2e_steps
        del g_step, g_int4, e2e_step
        free()

        extras = {}
        if not a.no_extras and a.layers == LAYERS and a.scales == "fp16" and a.mode == "set":
            extras["chain"] = measure_chain(w, a.steps, a.warmup, world)
            del w
            free()
            extras["gemv_c0"] = measure_c0(dev, 5 + rank, a.steps, a.warmup, world)
            extras["step"] = measure_step(dev, 777 + rank, LAYERS, 511, "separate", a.steps, a.warmup, world, clk)
            extras["batched"] = measure_batched(dev, 99 + rank, BATCHES, LAYERS, a.steps, a.warmup, world, clk)
            extras["prefill"] = measure_prefill(dev, 4321 + rank, PREFILL_TOKENS, LAYERS, a.steps, a.warmup, world,
                                                clk)
            if world > 1:  # the same projection set + head tensor-parallel over the ranks
                ms_tp, _, rb_, fb_, _, _ = measure_tp(LAYERS, a.collective, a.steps, a.warmup, rank, world, dev, None)
                extras["tp"] = tp_record(ms_tp, rb_, fb_, world, a.collective, ms_step)
    clocks = clk.summary(m0, m1)

    if rank == 0:
        gbs = world * step_bytes / (ms_step * 1e-3) / 1e9
        cpu = cpu_baseline_sample(a.cpu_seconds) if world == 1 and a.cpu_seconds > 0 else None
        line = {
            "metric": METRIC, "value": round(gbs, 1), "unit": UNIT, "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
            "config": {"workload": "config-1 36-layer decode-step projection set (QKV 5120x3072, o 3072x3072, "
                                   "gate_up 16384x3072, down 3072x8192; int4 g128) + config-2 int8 head "
                                   "16385x3072, batch 1, in one CUDA graph",
                       "launches": ("144 projections and the int8 head's rows in one persistent launch"
                                    if a.head in ("list", "list_last") else f"144 projections in one persistent launch + the "
                                    f"head ({a.head})") if a.mode == "set" else "145 stream-ordered launches",
                       "batch": 1, "bytes_per_step": step_bytes, "parallelism": f"replica x{world}",
                       "weight_prefetch": not a.no_prefetch,
                       "l2": "no flush: 1.98 GB of weights per step > 126 MB L2",
                       "scales": "fp16 scale + min per group (the reference format)" if a.scales == "fp16" else
                       "8-bit double-quantised scales (rumik_fast_b200.scales8): 2 bytes per group + 4 per row"},
            "tok_s": extras["step"]["tok_s"] if "step" in extras else None,
            "tok_s_independent_set": round(world * 1e3 / ms_step, 1),
            "pct_of_peak": round(100 * gbs / world / peak, 1),
            "e2e": {"value": round(world * step_bytes / (ms_e2e * 1e-3) / 1e9, 1), "unit": UNIT,
                    "h2d_bytes_per_step": (3072 + 8192) * 2, "d2h_bytes_per_step": logits_bytes,
                    "ms_per_step": round(ms_e2e, 5)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "kernel": ("gemv_int4_tc_kernel (144 projections + the int8 head's rows)" if one_launch
                                    else "gemv_int4_tc_kernel") if a.mode == "set" else "gemv_int4_kernel",
                         "traffic": (NCU_TRAFFIC_STEP_LAUNCH if one_launch else NCU_TRAFFIC_PER_LAUNCH)
                         if a.mode == "set" and a.layers == LAYERS else None,
                         "algorithmic_bytes_per_launch": roof_bytes // roof_launches},
            "head": {"placement": a.head if a.mode == "set" else "chain", "bytes": w_head_bytes,
                     "step_minus_projections_us": round((ms_step - ms4) * 1e3, 2),
                     "marginal_gbs": round(w_head_bytes / max(ms_step - ms4, 1e-6) / 1e6, 1),
                     "marginal_frac": round(w_head_bytes / max(ms_step - ms4, 1e-6) / 1e6 / peak, 4)},
            "cpu_baseline": cpu,
            "clocks": clocks,
            "gpu_launches": a.steps * (1 if one_launch else launches4 + 1),
            "mode": a.mode,
        }
        line.update(extras)
        print(json.dumps(line), flush=True)
    end_dist(world)
    return 0


def run_prefill(a):
    """Config 3 alone (--workload prefill --tokens M): the prefill record as the line's value."""
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    init_dist(dev, world)
    M = a.tokens
    with ClockSampler(dev) as clk:
        rec = measure_prefill(dev, 4321 + rank, (M,), a.layers, a.steps, a.warmup, world, clk)[str(M)]
    if rank == 0:
        line = {"metric": "prefill int4-weight matmul TFLOP/s", "value": rec["tflops"], "unit": "TFLOP/s",
                "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": rec["ms_per_step"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
                "data": "synthetic",
                "config": {"workload": f"config-3 prefill: X fp16 [{M}, K] against the {a.layers}-layer projection "
                                       "set, one mm_int4 launch per matrix, in one CUDA graph", "tokens": M,
                           "parallelism": f"replica x{world}", "l2": "no flush: weights per step > 126 MB L2"},
                "prefill": rec, "clocks": rec["clocks"], "gpu_launches": a.steps * rec["launches_per_step"],
                "mode": "prefill"}
        print(json.dumps(line), flush=True)
    end_dist(world)
    return 0


def run_step(a):
    """The full decode step alone (--workload step): the step record as the line's value."""
    import rumik_fast_b200 as rb
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    init_dist(dev, world)
    rb.set_weight_prefetch(not a.no_prefetch)
    with ClockSampler(dev) as clk:
        rec = measure_step(dev, 777 + rank, a.layers, a.pos, a.attn, a.steps, a.warmup, world, clk)
    if rank == 0:
        line = {"metric": "full decode step tok/s", "value": rec["tok_s"], "unit": "tok/s", "n_gpus": world,
                "steps": a.steps, "warmup": a.warmup, "ms_per_step": rec["ms_per_step"], "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
                "config": {"workload": rec["workload"], "pos": a.pos, "parallelism": f"replica x{world}",
                           "l2": "no flush: 2.0 GB of weights per step > 126 MB L2"},
                "step": rec, "clocks": rec["clocks"], "gpu_launches": a.steps * rec["launches_per_step"],
                "mode": "step"}
        print(json.dumps(line), flush=True)
    end_dist(world)
    return 0


def main():
    a = parse()
    if a.scales != "fp16" and (a.workload != "decode" or a.parallel != "replica"):
        raise SystemExit("--scales 8bit applies to the decode workload's projection set (replicas)")
    if a.impl == "reference":
        return run_reference(a)
    if a.workload == "prefill":
        return run_prefill(a)
    if a.workload == "step":
        return run_step(a)
    return run_ours(a)


if __name__ == "__main__":
    sys.exit(main())
