"""Benchmark: compressed-KV decode attention (SMAQ hot path) on B200.

Default workload: Llama-3-70B KV shape -- 80 layers, 64 query / 8 KV
heads, head_dim 128, bf16 -- 4 sequences x 131072 compressed history tokens (block-VQ keys:
8-dim blocks, 256-entry fp16-valued codebook k-means-fit on 16K calibration keys; 2-bit values
in groups of 32) plus a 128-token exact bf16 window, one decode token per sequence.  A step is
the attention of all 80 layers for one decode token of every sequence.  With N ranks the KV
heads are split over the ranks (N <= 8, no collective: each rank's query heads only read its
own KV heads), so the total work is fixed: ``scaling: strong``.  At N = 1 the line also carries
``cfg1``: configs[1] (Llama-3-8B, 32 layers, 32/8 heads, 16 x 32768 tokens) measured the same
way, the 32K-context point of the metric.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference] [--workload W]

``--workload decode`` is configs[1] alone (N > 1: every rank serves its own 16 sequences,
``scaling: weak``); ``--workload paged`` is configs[3] (Qwen2.5-7B KV shape, 64 sequences of
1K-64K tokens in a 16-token paged store, 4-bit scalar keys, 64-token window); ``--workload
append`` is configs[2] (8 x 8192 new tokens x 8 KV heads quantized into store rows: tcgen05
rotation + 3-bit scalar key codes, 2-bit values; GB/s counts input plus output bytes).

Timing: every decode step (one ``smaq_decode`` call per layer through ``smaq_b200.ops.decode``,
each one kernel launch) is captured once in a CUDA graph and replayed; CUDA events on the
replay stream bracket the K timed steps.  ``e2e`` replays a second graph whose every layer
also copies that layer's query rows host -> device (pinned) before its decode and its output
rows device -> host after it.  The KV cache of one step is far larger than L2 (126 MB), so no
L2 flush is needed between steps.

``--impl reference`` times the reference implementation itself (gauravsaini/smaq, installed
unmodified under baseline/_ref) on the host CPU: ``compute_hybrid_attention`` over a
``CompressedKVStore`` holding one sequence of the workload, all host threads, scaled to the
step.  Inputs: seeded synthetic data with the spectral key distribution (no dataset).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from dataclasses import dataclass, field

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "compressed-KV decode attn tokens/s & HBM GB/s (% of roofline) at 32K/128K ctx"
REF_DIR = os.path.join(REPO, "baseline", "_ref")

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the decode kernel,
# read from one ncu capture of the same kernel on the same per-launch shape; keyed by
# (batch, history tokens, window, query heads, kv heads) of one launch.
NCU_TRAFFIC: dict = {
    (4, 131072, 128, 64, 8): 270_843_648 + 5_184_000,     # configs[4], decode_v3_kernel<8>
    (16, 32768, 128, 32, 8): 277_166_336 + 8_543_232,     # configs[1], decode_v3_kernel<4>
}
# the same for the paged configs[3] launch (decode_s_kernel) and the configs[2] key kernel
NCU_TRAFFIC_PAGED = 1_145_590_000 + 8_393_984


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="smaq_b200", choices=["smaq_b200", "reference"])
    ap.add_argument("--workload", default="longctx", choices=["longctx", "decode", "append", "append_bvq", "paged", "scores"])
    ap.add_argument("--layers", type=int, default=0, help="build fewer layers (profiling runs only; 0: the config's)")
    ap.add_argument("--no-cfg1", action="store_true", help="longctx at N=1: skip the configs[1], [2] and [3] sub-measurements")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", dest="graph", action="store_false", help="launch every layer from Python")
    ap.add_argument("--no-overlap", dest="overlap", action="store_false",
                    help="plain stream ordering between layer launches (default: each layer's launch overlaps "
                         "the previous one's end; no layer writes another layer's history rows or the lengths)")
    return ap.parse_args(argv)


def peak_hbm():
    try:
        return float(json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ----------------------------------------------------------------------------- decode workloads
@dataclass
class DecodeSpec:
    name: str
    layers: int
    batch: int            # sequences this rank decodes
    ctx: int
    window: int
    hq: int               # query heads on this rank
    hkv: int              # kv heads on this rank
    hq_total: int
    hkv_total: int
    scaling: str
    parallelism: str
    world: int = 1
    extra: dict = field(default_factory=dict)

    def config(self):
        return {"workload": self.name, "layers": self.layers, "batch": self.batch if self.scaling == "strong"
                else self.batch * self.world, "n_q_heads": self.hq_total, "n_kv_heads": self.hkv_total,
                "head_dim": 128, "history_tokens": self.ctx, "window_tokens": self.window,
                "keys": "block-VQ 8x256 (fp16 codebook)", "values": "2-bit g32", "parallelism": self.parallelism,
                "per_gpu": {"batch": self.batch, "n_q_heads": self.hq, "n_kv_heads": self.hkv},
                "l2": "inputs larger than L2 (no flush)"}

    def bytes_per_layer(self) -> int:
        """Algorithmic HBM bytes of one layer's decode on this rank: packed history rows
        (16 B block indices + 32 B value codes + 8 B value scales + 8 B value zeros per
        token-head), the exact bf16 window K and V, the bf16 query in and output out."""
        D = 128
        hist = self.ctx * (D // 8 + D // 4 + 2 * 2 * (D // 32))
        recent = self.window * 2 * D * 2
        qo = self.hq * D * 2 * 2
        return self.batch * (self.hkv * (hist + recent) + qo)


def decode_spec(workload: str, world: int, layers_override: int = 0) -> DecodeSpec:
    if workload == "longctx":
        from smaq_b200.distributed import make_plan
        plan = make_plan(world, 8)
        if plan.seq_splits > 1:
            raise SystemExit("longctx: more ranks than KV heads is not benchmarked")
        g = plan.head_groups
        s = DecodeSpec("cfg4_llama3_70b_bvq_longctx", 80, 4, 131072, 128, 64 // g, 8 // g, 64, 8, "strong",
                       f"kv-head x{g}", world)
    else:
        s = DecodeSpec("cfg1_llama3_8b_bvq_decode", 32, 16, 32768, 128, 32, 8, 32, 8, "weak",
                       f"replicas x{world} (independent sequences)", world)
    if layers_override:
        s.layers = layers_override
    return s


class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power)}


def make_codebook(dev):
    """256-entry block-VQ codebook fit by seeded k-means on 16K calibration keys, fp16 values."""
    import torch
    from smaq_b200 import ops, synthetic as syn
    from smaq_b200.block_vq import SMAQBlockVQ
    vq = SMAQBlockVQ(128, device=dev)
    ck = torch.from_numpy(syn.keys((16384,), 128, seed=21)).to(dev)
    cq = torch.from_numpy(syn.calibration_queries(16384, 128, seed=syn.SEED_CAL_Q)).to(dev)
    vq.fit(ck, cq, seed=syn.SEED_KMEANS)
    for name in ("E_blocks", "E_inv_blocks", "centroids", "decoded_centroids"):
        getattr(vq, name).copy_(getattr(vq, name).half().float())
    vq.cb16 = ops.fp16_codebook(vq.decoded_centroids)
    assert vq.cb16 is not None
    return vq


def spectral_keys_gpu(n, gen, U, lam_sqrt, outl, dtype):
    import torch
    z = torch.randn((n, 128), generator=gen, device=U.device, dtype=torch.float32) * lam_sqrt
    x = z @ U.T
    x[:, outl] *= 8.0
    return x.to(dtype)


def build_layers(spec: DecodeSpec, dev, vq, seed0: int, head0: int = 0):
    """Per layer: store rows [B, Hkv, ctx, ...] (decode layout), exact window, queries, outputs.
    ``head0``: first global KV head of this rank (keys and values of a KV head do not depend on
    how the heads are sharded)."""
    import torch
    from smaq_b200 import ops, synthetic as syn
    from smaq_b200._lib import SMAQ_KEYS_BVQ, SMAQ_LAYOUT_DECODE
    U_np, outl = syn.basis(128)
    U = torch.from_numpy(U_np.astype(np.float32)).to(dev)
    lam = torch.from_numpy(np.sqrt(syn.spectrum(128)).astype(np.float32)).to(dev)
    outl = torch.from_numpy(outl).to(dev)
    B, H, T, D, W = spec.batch, spec.hkv, spec.ctx, 128, spec.window
    bf = torch.bfloat16
    layers = []
    for li in range(spec.layers):
        L = {
            "codes": torch.empty((B, H, T, 16), dtype=torch.uint8, device=dev),
            "vdata": torch.empty((B, H, T, 32), dtype=torch.uint8, device=dev),
            "vs": torch.empty((B, H, T, 4), dtype=bf, device=dev),
            "vz": torch.empty((B, H, T, 4), dtype=bf, device=dev),
            "rk": torch.empty((B, W, H, D), dtype=bf, device=dev),
            "rv": torch.empty((B, W, H, D), dtype=bf, device=dev),
            "q": torch.empty((B, spec.hq, D), dtype=bf, device=dev),
            "out": torch.empty((B, spec.hq, D), dtype=bf, device=dev),
        }
        G = spec.hq // spec.hkv
        for hl in range(H):
            gen = torch.Generator(device=dev).manual_seed(seed0 * 100003 + li * 131 + head0 + hl)
            for b in range(B):
                k = spectral_keys_gpu(T, gen, U, lam, outl, bf).reshape(T, 1, D)
                v = torch.randn((T, 1, D), generator=gen, device=dev, dtype=torch.float32).to(bf)
                ops.append(k, v, n_heads=1, slot_offset=(b * H + hl) * T, page_size=T, key_format=SMAQ_KEYS_BVQ,
                           E_blocks=vq.E_blocks, centroids=vq.centroids, key_codes=L["codes"], v_data=L["vdata"],
                           v_scales=L["vs"], v_zeros=L["vz"], layout=SMAQ_LAYOUT_DECODE)
            L["rk"][:, :, hl] = spectral_keys_gpu(B * W, gen, U, lam, outl, bf).reshape(B, W, D)
            L["rv"][:, :, hl] = torch.randn((B, W, D), generator=gen, device=dev, dtype=torch.float32).to(bf)
            L["q"][:, hl * G:(hl + 1) * G] = torch.randn((B, G, D), generator=gen, device=dev,
                                                        dtype=torch.float32).to(bf)
        layers.append(L)
    torch.cuda.synchronize()
    return layers


def decode_layer(spec: DecodeSpec, L, vq, hl, rl, ws, overlap: bool):
    from smaq_b200 import ops
    from smaq_b200._lib import SMAQ_KEYS_BVQ, SMAQ_LAYOUT_DECODE
    return ops.decode(L["q"], n_kv_heads=spec.hkv, key_format=SMAQ_KEYS_BVQ, centroids=vq.decoded_centroids,
                      key_codes=L["codes"], v_data=L["vdata"], v_scales=L["vs"], v_zeros=L["vz"], hist_len=hl,
                      page_size=spec.ctx, recent_k=L["rk"], recent_v=L["rv"], recent_len=rl, out=L["out"],
                      workspace=ws, layout=SMAQ_LAYOUT_DECODE, centroids_f16=vq.cb16, overlap_prior=overlap)


def time_decode(spec: DecodeSpec, dev, vq, steps: int, warmup: int, overlap: bool, use_graph: bool, barrier):
    """Device time of one step (all layers), of one layer launch alone, and of one end-to-end
    step (per-layer host<->device copies of queries and outputs)."""
    import torch
    from smaq_b200 import ops
    layers = build_layers(spec, dev, vq, seed0=1 + spec.extra.get("rank", 0), head0=spec.extra.get("head0", 0))
    hl = torch.full((spec.batch,), spec.ctx, dtype=torch.int32, device=dev)
    rl = torch.full((spec.batch,), spec.window, dtype=torch.int32, device=dev)
    ws = torch.empty(ops.decode_workspace_bytes(spec.batch, spec.hq, spec.hkv, 128), dtype=torch.uint8, device=dev)
    hQ = torch.empty((spec.layers,) + tuple(layers[0]["q"].shape), dtype=torch.bfloat16).pin_memory()
    hO = torch.empty_like(hQ).pin_memory()
    for i, L in enumerate(layers):
        hQ[i].copy_(L["q"].cpu())

    def step():
        for L in layers:
            decode_layer(spec, L, vq, hl, rl, ws, overlap)

    def e2e_step():
        for i, L in enumerate(layers):
            L["q"].copy_(hQ[i], non_blocking=True)
            decode_layer(spec, L, vq, hl, rl, ws, overlap)
            hO[i].copy_(L["out"], non_blocking=True)

    for _ in range(max(3, warmup)):
        step()
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    run, run_e2e = step, e2e_step
    if use_graph:
        g, ge = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                step()
            with torch.cuda.graph(ge, stream=stream):
                e2e_step()
        torch.cuda.synchronize()
        run, run_e2e = g.replay, ge.replay
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn, n):
        with torch.cuda.stream(stream):
            for _ in range(max(3, warmup)):
                fn()
            torch.cuda.synchronize()
            barrier()
            torch.cuda.synchronize()
            e0.record(stream)
            for _ in range(n):
                fn()
            e1.record(stream)
            torch.cuda.synchronize()
            barrier()
        return e0.elapsed_time(e1) / n

    clocks = Clocks(dev.index or 0)
    clocks.start()
    time.sleep(0.3)
    ms = timed(run, steps)
    ck = clocks.stop()
    e2e_ms = timed(run_e2e, steps)
    # one layer launch alone between two events (cold start of that launch: no overlap)
    iso = []
    with torch.cuda.stream(stream):
        for L in layers[: min(8, len(layers))]:
            torch.cuda.synchronize()
            e0.record(stream)
            decode_layer(spec, L, vq, hl, rl, ws, False)
            e1.record(stream)
            torch.cuda.synchronize()
            iso.append(e0.elapsed_time(e1))
    ops.decode_status(spec.batch, spec.hkv, ws)
    del layers
    torch.cuda.empty_cache()
    return {"ms": ms, "e2e_ms": e2e_ms, "iso_ms": statistics.median(iso), "clocks": ck,
            "h2d": hQ.numel() * hQ.element_size(), "d2h": hO.numel() * hO.element_size()}


def decode_line(spec: DecodeSpec, t: dict, steps: int, warmup: int) -> dict:
    peak, src = peak_hbm()
    bpl = spec.bytes_per_layer()
    launch_ms = t["ms"] / spec.layers
    achieved = bpl / (launch_ms * 1e-3) / 1e9
    tokens = spec.batch if spec.scaling == "strong" else spec.batch * spec.world
    traffic = NCU_TRAFFIC.get((spec.batch, spec.ctx, spec.window, spec.hq, spec.hkv))
    return {
        "metric": METRIC, "value": tokens / (t["ms"] * 1e-3), "unit": "tokens/s", "n_gpus": spec.world,
        "steps": steps, "warmup": max(3, warmup), "ms_per_step": t["ms"], "higher_is_better": True,
        "scaling": spec.scaling, "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": spec.config(),
        "hbm_gbs": spec.world * bpl * spec.layers / (t["ms"] * 1e-3) / 1e9,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "traffic_source": "ncu dram bytes per launch, same per-launch shape"
                     if traffic else None, "peak_source": src,
                     "kernel": "one fused decode launch per layer (history + window + merge)",
                     "algorithmic_bytes_per_launch": bpl, "launch_us": launch_ms * 1e3,
                     "launch_us_isolated": t["iso_ms"] * 1e3,
                     "launch_time": "timed region / launches (CUDA-graph replay, consecutive launches overlap); "
                                    "isolated = one launch alone between two events"},
        "e2e": {"value": tokens / (t["e2e_ms"] * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": t["h2d"],
                "d2h_bytes_per_step": t["d2h"],
                "note": "per layer: pinned host -> device copy of its query rows, decode, device -> host copy of "
                        "its output rows; one CUDA-graph replay per step"},
        "gpu_launches": spec.layers * steps,
        "clocks": t["clocks"],
    }


def run_decode(a, rank: int, world: int):
    import torch
    import torch.distributed as dist
    from smaq_b200 import build
    build.build()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    spec = decode_spec(a.workload, world, a.layers)
    if spec.scaling == "weak":
        spec.extra["rank"] = rank     # replicas: every rank its own sequences
    else:
        from smaq_b200.distributed import make_plan
        spec.extra["head0"] = make_plan(world, 8).kv_heads(rank).start
    vq = make_codebook(dev)
    t = time_decode(spec, dev, vq, a.steps, a.warmup, a.overlap, a.graph, barrier)
    if world > 1:
        v = torch.tensor([t["ms"], t["e2e_ms"], t["iso_ms"]], device=dev)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        t["ms"], t["e2e_ms"], t["iso_ms"] = v.tolist()
    line = decode_line(spec, t, a.steps, a.warmup)
    if world == 1 and a.workload == "longctx" and not a.no_cfg1:
        s1 = decode_spec("decode", 1)
        t1 = time_decode(s1, dev, vq, a.steps, a.warmup, a.overlap, a.graph, barrier)
        l1 = decode_line(s1, t1, a.steps, a.warmup)
        line["cfg1"] = {k: l1[k] for k in ("value", "unit", "ms_per_step", "config", "hbm_gbs", "roofline", "e2e",
                                           "clocks")}
        # configs[2] (append) and configs[3] (paged scalar-key decode), same steps, no CPU sample
        sub = argparse.Namespace(**{**vars(a), "layers": 0, "no_cpu_baseline": True})
        keep = ("metric", "value", "unit", "ms_per_step", "config", "roofline", "e2e", "gpu_launches", "clocks")
        l2 = run_append(sub, 0, 1, emit=False)
        line["cfg2"] = {k: l2[k] for k in keep if k in l2}
        l3 = run_paged(sub, 0, 1, emit=False)
        line["cfg3"] = {k: l3[k] for k in keep if k in l3}
    if rank == 0:
        if world == 1 and not a.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(spec)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# ----------------------------------------------------------------------------- reference (CPU)
def import_reference():
    """The reference package installed unmodified under baseline/_ref (None if absent)."""
    if not os.path.isdir(os.path.join(REF_DIR, "smaq")):
        return None
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import smaq
    if not os.path.abspath(smaq.__file__).startswith(REF_DIR):
        return None
    return smaq


def _timed_runs(fn, seconds_cap: float, max_runs: int = 5):
    runs = []
    t_end = time.perf_counter() + seconds_cap
    while True:
        t0 = time.perf_counter()
        fn()
        runs.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end or len(runs) >= max_runs:
            return statistics.median(runs), len(runs)


def reference_decode_sample(spec: DecodeSpec, key_format: str = "bvq", bits: int = 4, seconds_cap: float = 20.0,
                            max_runs: int = 5, warmup: int = 1):
    """The reference's compute_hybrid_attention on CPU (all host threads) for one layer and one
    sequence of the workload, scaled to a full step.  The store is the reference's own
    CompressedKVStore, filled through append_chunk."""
    import torch
    from smaq_b200 import synthetic as syn
    smaq = import_reference()
    if smaq is None:
        return None
    from smaq.score import compute_hybrid_attention
    from smaq.store import CompressedKVStore
    from smaq.strategies import SMAQBlockVQStrategy, SMAQFullMetricScalarStrategy
    torch.set_num_threads(os.cpu_count() or 1)
    cpu = torch.device("cpu")
    D = 128
    ctx, hq, hkv, window, layers = spec.ctx, spec.hq_total, spec.hkv_total, spec.window, spec.layers
    batch = spec.batch if spec.scaling == "strong" else spec.batch * spec.world
    if key_format == "bvq":
        strat = SMAQBlockVQStrategy(D, device=cpu)
        strat.fit(torch.from_numpy(syn.calibration_queries(4096, D)), torch.from_numpy(syn.keys((4096,), D, seed=21)))
    else:
        strat = SMAQFullMetricScalarStrategy(D, bits=bits, device=cpu)
        strat.fit(torch.from_numpy(syn.calibration_queries(512, D)))
    store = CompressedKVStore(D, hkv, device=cpu, key_strategy=strat, key_bits=bits)
    chunk = 8192
    for t0 in range(0, ctx, chunk):
        n = min(chunk, ctx - t0)
        k = torch.from_numpy(syn.keys((n, hkv), D, seed=1000 + t0 // chunk)).to(torch.bfloat16)
        v = torch.from_numpy(syn.values((n, hkv), D, seed=2000 + t0 // chunk)).to(torch.bfloat16)
        store.append_chunk(k, v)
    rk = torch.from_numpy(syn.keys((window, hkv), D, seed=3)).to(torch.bfloat16)
    rv = torch.from_numpy(syn.values((window, hkv), D, seed=4)).to(torch.bfloat16)
    q = torch.from_numpy(syn.queries((1, hq), D, seed=5)).to(torch.bfloat16)
    for _ in range(max(1, warmup)):   # the first call also builds the reference's flat cache
        compute_hybrid_attention(q, store, rk, rv, hq)
    t, n_runs = _timed_runs(lambda: compute_hybrid_attention(q, store, rk, rv, hq), seconds_cap, max_runs)
    step_s = t * layers * batch
    return {"value": batch / step_s, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "reference",
            "sample": f"reference compute_hybrid_attention (baseline/_ref, torch {torch.__version__} CPU), 1 layer x "
                      f"1 sequence ({ctx} history + {window} window tokens, {hq}/{hkv} heads), median of {n_runs} "
                      f"runs = {t * 1e3:.1f} ms, scaled x{layers * batch}"}


def port_decode_sample(spec: DecodeSpec, seconds_cap: float = 20.0):
    """Fallback when the reference is not installed: the numpy restatement (fp32) on one layer x
    one sequence, scaled."""
    from oracle import smaq_oracle as O
    from smaq_b200 import synthetic as syn
    rng = np.random.default_rng(5)
    H, T, D, W = spec.hkv_total, spec.ctx, 128, spec.window
    idx = rng.integers(0, 256, size=(H, T, 16))
    dec = rng.standard_normal((16, 256, 8)).astype(np.float32)
    vdata = rng.integers(0, 256, size=(H, T, 32), dtype=np.uint8)
    vs = np.abs(rng.standard_normal((H, T, 4))).astype(np.float32)
    vz = rng.standard_normal((H, T, 4)).astype(np.float32)
    q = syn.queries((1, spec.hq_total), D, seed=9)
    rk = syn.keys((W, H), D, seed=10)
    rv = syn.values((W, H), D, seed=11)

    def one():
        K = O.bvq_dequantize(idx, dec, work=np.float32)
        V = O.dequantize_values(vdata, vs, vz, 2, 32)
        O.hybrid_attention(q, "bf16", K, V, rk, rv, spec.hq_total, H, work=np.float32)

    t, n_runs = _timed_runs(one, seconds_cap)
    batch = spec.batch if spec.scaling == "strong" else spec.batch * spec.world
    return {"value": batch / (t * spec.layers * batch), "unit": "tokens/s", "cores": 1, "kind": "port",
            "sample": f"numpy restatement, 1 layer x 1 sequence ({T} + {W} tokens), median of {n_runs} runs = "
                      f"{t * 1e3:.1f} ms, scaled x{spec.layers * batch}"}


def cpu_baseline(spec: DecodeSpec, seconds_cap: float = 20.0, max_runs: int = 5, warmup: int = 1):
    return (reference_decode_sample(spec, seconds_cap=seconds_cap, max_runs=max_runs, warmup=warmup)
            or port_decode_sample(spec, seconds_cap))


def run_reference(a, rank: int, world: int):
    if rank != 0:
        return
    spec = decode_spec(a.workload, world, a.layers)
    # one store is built, then K timed calls (each one layer x one sequence), median taken
    info = cpu_baseline(spec, seconds_cap=120.0, max_runs=max(1, a.steps), warmup=max(1, a.warmup))
    v = info["value"]
    tokens = spec.batch if spec.scaling == "strong" else spec.batch * world
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1e3 * tokens / v,
            "higher_is_better": True, "scaling": spec.scaling, "vs_baseline": None, "dtype": "bf16-io/f32",
            "data": "synthetic", "config": spec.config(),
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": info["cores"], "kind": info["kind"],
                             "sample": info["sample"]},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- append
APPEND_METRIC = "compressed-KV append GB/s (in+out)"
AP_B, AP_T, AP_H, AP_D, AP_BITS = 8, 8192, 8, 128, 3


def append_config():
    return {"workload": "cfg2_append_bf16", "batch": AP_B, "new_tokens": AP_T, "n_kv_heads": AP_H, "head_dim": AP_D,
            "keys": "scalar 3-bit (metric rotation on tcgen05, 3-split bf16)", "values": "2-bit g32",
            "l2": "inputs larger than L2 (no flush)"}


def append_bytes():
    rows = AP_B * AP_T * AP_H
    k_in = v_in = rows * AP_D * 2
    k_out = rows * (AP_D // 2 + 2)            # 3-bit codes two per byte + bf16 norm
    v_out = rows * (AP_D // 4 + 2 * 2 * (AP_D // 32))
    return k_in, v_in, k_out, v_out


def append_cpu_sample(seconds_cap: float = 20.0, max_runs: int = 5):
    """The reference's CompressedKVStore.append_chunk (smaq/store.py:83-95: SMAQ 3-bit scalar
    keys + 2-bit values, bf16) on the host CPU with all threads, on a bounded sample of
    token-heads, scaled to the full batch.  Falls back to the torch CPU restatement of the same
    ops when the reference is not installed."""
    import torch
    from smaq_b200 import synthetic as syn
    torch.set_num_threads(os.cpu_count() or 1)
    tokens = 8192
    rows = tokens * AP_H
    k = torch.from_numpy(syn.keys((tokens, AP_H), AP_D, seed=31)).to(torch.bfloat16)
    v = torch.from_numpy(syn.values((tokens, AP_H), AP_D, seed=32)).to(torch.bfloat16)
    calq = torch.from_numpy(syn.calibration_queries(512, AP_D))
    smaq = import_reference()
    if smaq is not None:
        from smaq.store import CompressedKVStore
        from smaq.strategies import SMAQFullMetricScalarStrategy
        strat = SMAQFullMetricScalarStrategy(AP_D, bits=AP_BITS, device=torch.device("cpu"))
        strat.fit(calq)
        store = CompressedKVStore(AP_D, AP_H, key_bits=AP_BITS, device=torch.device("cpu"), key_strategy=strat)

        def one():
            store.append_chunk(k, v)
        kind, what = "reference", "reference CompressedKVStore.append_chunk (baseline/_ref)"
    else:
        from oracle import smaq_oracle as O
        from smaq_b200.quantizer import SMAQQuantizer
        quant = SMAQQuantizer(AP_D, bits=AP_BITS, device=torch.device("cpu"))
        quant.fit(calq)
        E, bnd = quant.E.float(), quant.decision_boundaries.float().contiguous()
        kr, vr = k.reshape(rows, AP_D), v.reshape(rows, AP_D)

        def one():
            O.torch_append(kr, vr, E, bnd, AP_BITS)
        kind, what = "port", "torch CPU restatement of the append ops"
    t, n_runs = _timed_runs(one, seconds_cap, max_runs)
    total = sum(append_bytes())
    scale = AP_B * AP_T * AP_H / rows
    return {"value": total / (t * scale) / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(), "kind": kind,
            "sample": f"{what}, {tokens} tokens x {AP_H} heads, median of {n_runs} runs = {t * 1e3:.1f} ms, "
                      f"scaled x{scale:.0f}"}


def append_inputs(dev, rank: int = 0):
    """configs[2] inputs and destination rows on ``dev``: keys/values [B*T, H, D] bf16 with the
    spectral key distribution, the fitted 3-bit scalar quantizer, and decode-layout rows."""
    import torch
    from smaq_b200 import synthetic as syn
    from smaq_b200.quantizer import SMAQQuantizer
    quant = SMAQQuantizer(AP_D, bits=AP_BITS, device=dev)
    quant.fit(torch.from_numpy(syn.calibration_queries(512, AP_D)).to(dev))
    U_np, outl = syn.basis(AP_D)
    U = torch.from_numpy(U_np.astype(np.float32)).to(dev)
    lam = torch.from_numpy(np.sqrt(syn.spectrum(AP_D)).astype(np.float32)).to(dev)
    outl = torch.from_numpy(outl).to(dev)
    gen = torch.Generator(device=dev).manual_seed(100 + rank)
    N = AP_B * AP_T
    k = spectral_keys_gpu(N * AP_H, gen, U, lam, outl, torch.bfloat16).reshape(N, AP_H, AP_D)
    v = torch.randn((N, AP_H, AP_D), generator=gen, device=dev, dtype=torch.float32).to(torch.bfloat16)
    rows = N * AP_H
    out = {"codes": torch.empty((rows, AP_D // 2), dtype=torch.uint8, device=dev),
           "norms": torch.empty((rows,), dtype=torch.bfloat16, device=dev),
           "vd": torch.empty((rows, AP_D // 4), dtype=torch.uint8, device=dev),
           "vs": torch.empty((rows, AP_D // 32), dtype=torch.bfloat16, device=dev)}
    out["vz"] = torch.empty_like(out["vs"])
    return k, v, quant, out


def append_step(k, v, quant, o, keys=True, values=True):
    """One configs[2] append: every sequence's 8192 new tokens land in its own store page
    (page_size 8192), decode layout."""
    from smaq_b200 import ops
    from smaq_b200._lib import SMAQ_KEYS_SCALAR, SMAQ_LAYOUT_DECODE
    ops.append(k if keys else None, v if values else None, n_heads=AP_H, page_size=AP_T,
               key_format=SMAQ_KEYS_SCALAR, key_bits=AP_BITS, E=quant.E, boundaries=quant.decision_boundaries,
               key_codes=o["codes"], key_norms=o["norms"], v_data=o["vd"], v_scales=o["vs"], v_zeros=o["vz"],
               layout=SMAQ_LAYOUT_DECODE)


def run_append(a, rank: int, world: int, emit: bool = True):
    import torch
    import torch.distributed as dist
    from smaq_b200 import build
    build.build()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    k, v, quant, o = append_inputs(dev, rank)
    codes, norms, vd, vs, vz = o["codes"], o["norms"], o["vd"], o["vs"], o["vz"]

    def step(kk=k, vv=v, keys=True, values=True):
        append_step(kk, vv, quant, o, keys, values)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(max(3, a.warmup)):
        step()
    torch.cuda.synchronize()
    # one step captured as a CUDA graph (two kernel launches), replayed K times
    g = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream()
    with torch.cuda.stream(cs):
        with torch.cuda.graph(g, stream=cs):
            step()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    ms = e0.elapsed_time(e1) / a.steps
    ck = clocks.stop()
    # the keys kernel alone (dominant launch) for the roofline
    for _ in range(2):
        step(values=False)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(a.steps):
        step(values=False)
    e1.record()
    torch.cuda.synchronize()
    key_ms = e0.elapsed_time(e1) / a.steps
    # end to end: pinned host K/V -> device, append, compressed rows back to the host
    hk = torch.empty(k.shape, dtype=k.dtype).pin_memory()
    hv = torch.empty(v.shape, dtype=v.dtype).pin_memory()
    hk.copy_(k.cpu())
    hv.copy_(v.cpu())
    outs = [codes, norms, vd, vs, vz]
    houts = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in outs]
    dk, dv = torch.empty_like(k), torch.empty_like(v)

    def e2e_step():
        dk.copy_(hk, non_blocking=True)
        dv.copy_(hv, non_blocking=True)
        step(dk, dv)
        for h, t in zip(houts, outs):
            h.copy_(t, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    barrier()
    e0.record()
    for _ in range(a.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1) / a.steps
    if world > 1:
        t = torch.tensor([ms, e2e_ms, key_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms, key_ms = t.tolist()
    k_in, v_in, k_out, v_out = append_bytes()
    total = k_in + v_in + k_out + v_out
    try:
        peaks = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))
        peak_gbs, peak_tf, src = float(peaks["hbm_gbs"]), float(peaks["bf16_tflops"]), "measured"
    except Exception:
        peak_gbs, peak_tf, src = 6650.0, 1590.0, "fallback"
    key_bytes = k_in + k_out
    achieved = key_bytes / (key_ms * 1e-3) / 1e9
    flops = 3 * 2 * (AP_B * AP_T * AP_H) * AP_D * AP_D    # three bf16 splits of the d x d rotation
    if rank == 0:
        line = {
            "metric": APPEND_METRIC, "value": world * total / (ms * 1e-3) / 1e9, "unit": "GB/s", "n_gpus": world,
            "steps": a.steps, "warmup": max(3, a.warmup), "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16-io/f32-accum", "data": "synthetic",
            "config": append_config(),
            "tokens_per_s": world * AP_B * AP_T / (ms * 1e-3),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak_gbs, "unit": "GB/s",
                         "frac": achieved / peak_gbs, "traffic": None, "peak_source": src,
                         "kernel": "tc_scalar_key_kernel (keys: bf16 in, codes + norms out)",
                         "algorithmic_bytes_per_launch": key_bytes,
                         "tensor_tflops": flops / (key_ms * 1e-3) / 1e12,
                         "tensor_frac": flops / (key_ms * 1e-3) / 1e12 / peak_tf},
            "e2e": {"value": world * total / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": k_in + v_in,
                    "d2h_bytes_per_step": sum(t.numel() * t.element_size() for t in outs)},
            "gpu_launches": 2 * a.steps,
            "clocks": ck,
        }
        if not emit:
            return line
        if world == 1 and not a.no_cpu_baseline:
            line["cpu_baseline"] = append_cpu_sample()
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_append_reference(a, rank: int):
    if rank != 0:
        return
    info = append_cpu_sample(seconds_cap=120.0, max_runs=max(1, a.steps))
    v = info["value"]
    total = sum(append_bytes())
    line = {"impl": "reference", "metric": APPEND_METRIC, "value": v, "unit": "GB/s",
            "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": 1e3 * total / (v * 1e9), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16-io/f32-matmul", "data": "synthetic", "config": append_config(),
            "cpu_baseline": {"value": v, "unit": "GB/s", "cores": info["cores"], "kind": info["kind"],
                             "sample": info["sample"]},
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- paged
PG_B, PG_HQ, PG_HKV, PG_LAYERS, PG_PAGE, PG_W, PG_BITS = 64, 28, 4, 28, 16, 64, 4


def paged_lengths():
    from smaq_b200 import synthetic as syn
    return syn.seq_lengths(PG_B, 1024, 65536)


def paged_bytes_per_layer(lens) -> int:
    D = 128
    per_tok = (D // 2 + 2) + (D // 4 + 2 * 2 * (D // 32))     # 4-bit codes + norm, values
    return int(sum(lens)) * PG_HKV * per_tok + PG_B * (PG_HKV * PG_W * 2 * D * 2 + PG_HQ * D * 2 * 2)


def paged_config():
    return {"workload": "cfg3_qwen2.5_7b_paged_scalar4", "layers": PG_LAYERS, "batch": PG_B, "n_q_heads": PG_HQ,
            "n_kv_heads": PG_HKV, "head_dim": 128, "page_size": PG_PAGE, "lengths": "U[1024, 65536] seed 4",
            "window_tokens": PG_W, "keys": "scalar 4-bit", "values": "2-bit g32",
            "l2": "inputs larger than L2 (no flush)"}


def paged_cpu_sample(seconds_cap: float = 20.0, max_runs: int = 5):
    """The reference's compute_hybrid_attention (4-bit SMAQ scalar keys) on the host CPU for one
    layer x one sequence of the mean length, scaled to the step; the numpy restatement when the
    reference is not installed."""
    lens = paged_lengths()
    n = int(np.mean(lens))
    spec = DecodeSpec("cfg3_qwen2.5_7b_paged_scalar4", PG_LAYERS, PG_B, n, PG_W, PG_HQ, PG_HKV, PG_HQ, PG_HKV,
                      "weak", "single GPU")
    info = reference_decode_sample(spec, key_format="scalar", bits=PG_BITS, seconds_cap=seconds_cap,
                                   max_runs=max_runs)
    if info is not None:
        return info
    from oracle import smaq_oracle as O
    from smaq_b200 import synthetic as syn
    rng = np.random.default_rng(6)
    D = 128
    codes = rng.integers(0, 256, size=(PG_HKV, n, 64), dtype=np.uint8)
    norms = np.abs(rng.standard_normal((PG_HKV, n))).astype(np.float32)
    Einv = np.linalg.qr(rng.standard_normal((D, D)))[0].astype(np.float32)
    cent = np.linspace(-2, 2, 16).astype(np.float32)
    vdata = rng.integers(0, 256, size=(PG_HKV, n, 32), dtype=np.uint8)
    vs = np.abs(rng.standard_normal((PG_HKV, n, 4))).astype(np.float32)
    vz = rng.standard_normal((PG_HKV, n, 4)).astype(np.float32)
    q = syn.queries((1, PG_HQ), D, seed=9)
    rk = syn.keys((PG_W, PG_HKV), D, seed=10)
    rv = syn.values((PG_W, PG_HKV), D, seed=11)

    def one():
        K = O.scalar_score_keys(codes, norms, PG_BITS, Einv, cent, D)
        V = O.dequantize_values(vdata, vs, vz, 2, 32)
        O.hybrid_attention(q, "bf16", K, V, rk, rv, PG_HQ, PG_HKV, work=np.float32)

    t, n_runs = _timed_runs(one, seconds_cap, max_runs)
    return {"value": PG_B / (t * PG_LAYERS * PG_B), "unit": "tokens/s", "cores": 1, "kind": "port",
            "sample": f"numpy restatement, 1 layer x 1 sequence of {n} tokens, median of {n_runs} runs = "
                      f"{t * 1e3:.1f} ms, scaled x{PG_LAYERS * PG_B}"}


def build_paged_layers(n_layers: int, dev, rank: int = 0):
    """configs[3] on ``dev``: per layer a shuffled 16-token paged store (decode layout) filled
    through slot mappings, block table, exact window, queries, outputs.  Returns
    ``(layers, quantizer, lengths)``."""
    import torch
    from smaq_b200 import ops, synthetic as syn
    from smaq_b200._lib import SMAQ_KEYS_SCALAR, SMAQ_LAYOUT_DECODE
    from smaq_b200.quantizer import SMAQQuantizer
    D = 128
    lens = paged_lengths()
    quant = SMAQQuantizer(D, bits=PG_BITS, device=dev)
    quant.fit(torch.from_numpy(syn.calibration_queries(512, D)).to(dev))
    U_np, outl = syn.basis(D)
    U = torch.from_numpy(U_np.astype(np.float32)).to(dev)
    lam = torch.from_numpy(np.sqrt(syn.spectrum(D)).astype(np.float32)).to(dev)
    outl = torch.from_numpy(outl).to(dev)
    pages = [(int(n) + PG_PAGE - 1) // PG_PAGE for n in lens]
    n_pages, maxp = sum(pages), max(pages)
    rng = np.random.default_rng(40 + rank)
    bf = torch.bfloat16
    layers = []
    for li in range(n_layers):
        gen = torch.Generator(device=dev).manual_seed(1000 * (rank + 1) + li)
        perm = rng.permutation(n_pages)
        bt = np.zeros((PG_B, maxp), np.int32)
        o = 0
        for b in range(PG_B):
            bt[b, :pages[b]] = perm[o:o + pages[b]]
            o += pages[b]
        L = {"codes": torch.empty((n_pages, PG_HKV, PG_PAGE, D // 2), dtype=torch.uint8, device=dev),
             "norms": torch.empty((n_pages, PG_HKV, PG_PAGE), dtype=bf, device=dev),
             "vdata": torch.empty((n_pages, PG_HKV, PG_PAGE, D // 4), dtype=torch.uint8, device=dev),
             "vs": torch.empty((n_pages, PG_HKV, PG_PAGE, D // 32), dtype=bf, device=dev),
             "vz": torch.empty((n_pages, PG_HKV, PG_PAGE, D // 32), dtype=bf, device=dev),
             "bt": torch.from_numpy(bt).to(dev)}
        for b in range(PG_B):
            n = int(lens[b])
            k = spectral_keys_gpu(n * PG_HKV, gen, U, lam, outl, bf).reshape(n, PG_HKV, D)
            v = torch.randn((n, PG_HKV, D), generator=gen, device=dev, dtype=torch.float32).to(bf)
            t = torch.arange(n, device=dev)
            slots = L["bt"][b, t // PG_PAGE].to(torch.int64) * PG_PAGE + t % PG_PAGE
            ops.append(k, v, n_heads=PG_HKV, slots=slots, page_size=PG_PAGE, key_format=SMAQ_KEYS_SCALAR,
                       key_bits=PG_BITS, E=quant.E, boundaries=quant.decision_boundaries, key_codes=L["codes"],
                       key_norms=L["norms"], v_data=L["vdata"], v_scales=L["vs"], v_zeros=L["vz"],
                       layout=SMAQ_LAYOUT_DECODE)
        L["rk"] = spectral_keys_gpu(PG_B * PG_W * PG_HKV, gen, U, lam, outl, bf).reshape(PG_B, PG_W, PG_HKV, D)
        L["rv"] = torch.randn((PG_B, PG_W, PG_HKV, D), generator=gen, device=dev, dtype=torch.float32).to(bf)
        L["q"] = torch.randn((PG_B, PG_HQ, D), generator=gen, device=dev, dtype=torch.float32).to(bf)
        L["out"] = torch.empty((PG_B, PG_HQ, D), dtype=bf, device=dev)
        layers.append(L)
    torch.cuda.synchronize()
    return layers, quant, lens


def paged_decode(L, quant, hl, rl, ws, overlap: bool):
    from smaq_b200 import ops
    from smaq_b200._lib import SMAQ_KEYS_SCALAR, SMAQ_LAYOUT_DECODE
    return ops.decode(L["q"], n_kv_heads=PG_HKV, key_format=SMAQ_KEYS_SCALAR, key_bits=PG_BITS, E_inv=quant.E_inv,
                      centroids=quant.centroids, key_norms=L["norms"], key_codes=L["codes"], v_data=L["vdata"],
                      v_scales=L["vs"], v_zeros=L["vz"], hist_len=hl, page_size=PG_PAGE, block_table=L["bt"],
                      recent_k=L["rk"], recent_v=L["rv"], recent_len=rl, out=L["out"], workspace=ws,
                      layout=SMAQ_LAYOUT_DECODE, overlap_prior=overlap)


def run_paged(a, rank: int, world: int, emit: bool = True):
    import torch
    from smaq_b200 import build, ops
    build.build()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    D = 128
    n_layers = a.layers or PG_LAYERS
    layers, quant, lens = build_paged_layers(n_layers, dev, rank)
    hl = torch.from_numpy(lens.astype(np.int32)).to(dev)
    rl = torch.full((PG_B,), PG_W, dtype=torch.int32, device=dev)
    ws = torch.empty(ops.decode_workspace_bytes(PG_B, PG_HQ, PG_HKV, D), dtype=torch.uint8, device=dev)
    hQ = torch.empty((n_layers, PG_B, PG_HQ, D), dtype=torch.bfloat16).pin_memory()
    hO = torch.empty_like(hQ).pin_memory()
    for i, L in enumerate(layers):
        hQ[i].copy_(L["q"].cpu())

    def step():
        for L in layers:
            paged_decode(L, quant, hl, rl, ws, a.overlap)

    def e2e_step():
        for i, L in enumerate(layers):
            L["q"].copy_(hQ[i], non_blocking=True)
            paged_decode(L, quant, hl, rl, ws, a.overlap)
            hO[i].copy_(L["out"], non_blocking=True)

    for _ in range(max(3, a.warmup)):
        step()
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    run, run_e2e = step, e2e_step
    if a.graph:
        g, ge = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                step()
            with torch.cuda.graph(ge, stream=stream):
                e2e_step()
        torch.cuda.synchronize()
        run, run_e2e = g.replay, ge.replay
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn):
        with torch.cuda.stream(stream):
            for _ in range(max(3, a.warmup)):
                fn()
            torch.cuda.synchronize()
            e0.record(stream)
            for _ in range(a.steps):
                fn()
            e1.record(stream)
            torch.cuda.synchronize()
        return e0.elapsed_time(e1) / a.steps

    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.3)
    ms = timed(run)
    ck = clocks.stop()
    e2e_ms = timed(run_e2e)
    ops.decode_status(PG_B, PG_HKV, ws)
    bpl = paged_bytes_per_layer(lens)
    peak, src = peak_hbm()
    achieved = bpl * n_layers / (ms * 1e-3) / 1e9
    # tokens/s of a full 28-layer step (ms scaled when fewer layers were built for profiling)
    ms_full = ms * PG_LAYERS / n_layers
    line = {"metric": METRIC, "value": PG_B / (ms_full * 1e-3), "unit": "tokens/s", "n_gpus": 1, "steps": a.steps,
            "warmup": max(3, a.warmup), "ms_per_step": ms_full, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": paged_config(),
            "hbm_gbs": achieved,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": NCU_TRAFFIC_PAGED,
                         "traffic_source": "ncu dram bytes per launch, same per-launch shape",
                         "peak_source": src,
                         "kernel": "one fused scalar-key decode launch per layer (paged)",
                         "algorithmic_bytes_per_launch": bpl},
            "e2e": {"value": PG_B / (e2e_ms * PG_LAYERS / n_layers * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": hQ.numel() * hQ.element_size(),
                    "d2h_bytes_per_step": hO.numel() * hO.element_size(),
                    "note": "per layer: query rows host -> device, decode, output rows device -> host"},
            "gpu_launches": n_layers * a.steps, "clocks": ck}
    del layers
    torch.cuda.empty_cache()
    if not emit:
        return line
    if not a.no_cpu_baseline:
        line["cpu_baseline"] = paged_cpu_sample()
    if rank == 0:
        print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- main

# ----------------------------------------------------------------------------- block-VQ append
def run_append_bvq(a, rank: int):
    """configs[2]'s append batch with block-VQ keys (the configs[1]/[4] key format: 8-dim blocks,
    256-entry codebook) and 2-bit values: SMAQBlockVQ.quantize (smaq/block_vq.py:216-244) plus
    quantize_values through one smaq_append per step."""
    import torch
    from smaq_b200 import build, ops
    from smaq_b200._lib import SMAQ_KEYS_BVQ, SMAQ_LAYOUT_DECODE
    build.build()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    vq = make_codebook(dev)
    k, v, _, o = append_inputs(dev, rank)
    rows = k.shape[0] * k.shape[1]
    codes = torch.empty((rows, AP_D // 8), dtype=torch.uint8, device=dev)

    def step(keys=True, values=True):
        ops.append(k if keys else None, v if values else None, n_heads=AP_H, page_size=AP_T, key_format=SMAQ_KEYS_BVQ,
                   E_blocks=vq.E_blocks, centroids=vq.centroids, key_codes=codes, v_data=o["vd"], v_scales=o["vs"],
                   v_zeros=o["vz"], layout=SMAQ_LAYOUT_DECODE)

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn):
        for _ in range(max(3, a.warmup)):
            fn()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(a.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / a.steps

    clocks = Clocks(dev.index or 0)
    clocks.start()
    time.sleep(0.3)
    ms = timed(step)
    ck = clocks.stop()
    key_ms = timed(lambda: step(values=False))
    k_in = v_in = rows * AP_D * 2
    k_out = rows * (AP_D // 8)
    v_out = rows * (AP_D // 4 + 2 * 2 * (AP_D // 32))
    total = k_in + v_in + k_out + v_out
    peak, src = peak_hbm()
    flops = rows * (AP_D // 8) * 256 * 8 * 2          # shaped-key . centroid for every code of every block
    line = {"metric": "compressed-KV append GB/s (in+out), block-VQ keys", "value": total / (ms * 1e-3) / 1e9,
            "unit": "GB/s", "n_gpus": 1, "steps": a.steps, "warmup": max(3, a.warmup), "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16-io/f32-distances",
            "data": "synthetic",
            "config": {"workload": "append_bvq", "batch": AP_B, "new_tokens": AP_T, "n_kv_heads": AP_H,
                       "head_dim": AP_D, "keys": "block-VQ 8x256", "values": "2-bit g32",
                       "l2": "inputs larger than L2 (no flush)"},
            "roofline": {"bound": "issue (mma.sync scores + argmin epilogue)",
                         "achieved": (k_in + k_out) / (key_ms * 1e-3) / 1e9,
                         "peak": peak, "unit": "GB/s", "frac": (k_in + k_out) / (key_ms * 1e-3) / 1e9 / peak,
                         "traffic": None, "peak_source": src,
                         "kernel": "bvq_mma_kernel (m16n8k8 bf16, codebook in three bf16 terms)",
                         "key_kernel_us": key_ms * 1e3, "distance_tflops": flops / (key_ms * 1e-3) / 1e12,
                         "tensor_tflops_bf16": 3 * flops / (key_ms * 1e-3) / 1e12},
            "gpu_launches": 2 * a.steps, "clocks": ck}
    if not a.no_cpu_baseline:
        line["cpu_baseline"] = append_bvq_cpu_sample(vq)
    if rank == 0:
        print(json.dumps(line), flush=True)


def append_bvq_cpu_sample(vq, seconds_cap: float = 20.0, max_runs: int = 3):
    """The reference's CompressedKVStore.append_chunk with SMAQBlockVQStrategy on the host CPU,
    all threads, 1024 tokens x 8 heads, scaled to the batch."""
    import torch
    from smaq_b200 import synthetic as syn
    torch.set_num_threads(os.cpu_count() or 1)
    tokens = 1024
    k = torch.from_numpy(syn.keys((tokens, AP_H), AP_D, seed=31)).to(torch.bfloat16)
    v = torch.from_numpy(syn.values((tokens, AP_H), AP_D, seed=32)).to(torch.bfloat16)
    smaq = import_reference()
    if smaq is None:
        return {"value": None, "unit": "GB/s", "cores": 0, "kind": "reference", "sample": "reference not installed"}
    from smaq.store import CompressedKVStore
    from smaq.strategies import SMAQBlockVQStrategy
    cpu = torch.device("cpu")
    strat = SMAQBlockVQStrategy(AP_D, device=cpu)
    q = strat.quantizer
    for name in ("E_blocks", "E_inv_blocks", "centroids", "decoded_centroids"):
        setattr(q, name, getattr(vq, name).detach().to(cpu))
    store = CompressedKVStore(AP_D, AP_H, device=cpu, key_strategy=strat)
    t, n = _timed_runs(lambda: store.append_chunk(k, v), seconds_cap, max_runs)
    rows = tokens * AP_H
    per_row = AP_D * 2 * 2 + AP_D // 8 + AP_D // 4 + 2 * 2 * (AP_D // 32)
    scale = AP_B * AP_T * AP_H / rows
    return {"value": rows * per_row / t / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "reference",
            "sample": f"reference CompressedKVStore.append_chunk with SMAQBlockVQStrategy (baseline/_ref), {tokens} "
                      f"tokens x {AP_H} heads, median of {n} runs = {t * 1e3:.1f} ms (rate; x{scale:.0f} for the batch)"}


# ----------------------------------------------------------------------------- standalone scores / attend
SC_H, SC_G, SC_N, SC_BITS = 8, 8, 131072, 4


def scores_config():
    return {"workload": "hf_cache_scores_attend", "n_kv_heads": SC_H, "queries_per_kv_head": SC_G,
            "history_tokens": SC_N, "head_dim": 128, "keys": f"scalar {SC_BITS}-bit", "values": "2-bit g32",
            "query": "fp32 (scores out fp32, the reference's Triton output type)", "weights": "fp32",
            "l2": "inputs larger than L2 (no flush)"}


def scores_inputs(dev):
    """HF-style cache history of SC_H kv heads x SC_N tokens, with SC_G query rows per head."""
    import torch
    from smaq_b200 import synthetic as syn
    from smaq_b200.kv_cache import quantize_values
    from smaq_b200.quantizer import SMAQQuantizer
    D = 128
    quant = SMAQQuantizer(D, bits=SC_BITS, device=dev)
    quant.fit(torch.from_numpy(syn.calibration_queries(512, D)).to(dev))
    U_np, outl = syn.basis(D)
    U = torch.from_numpy(U_np.astype(np.float32)).to(dev)
    lam = torch.from_numpy(np.sqrt(syn.spectrum(D)).astype(np.float32)).to(dev)
    gen = torch.Generator(device=dev).manual_seed(7)
    k = spectral_keys_gpu(SC_H * SC_N, gen, U, lam, torch.from_numpy(outl).to(dev), torch.bfloat16)
    kq = quant.quantize(k.reshape(SC_H, SC_N, D))
    v = torch.randn((SC_H, SC_N, D), generator=gen, device=dev, dtype=torch.float32).to(torch.bfloat16)
    vq = quantize_values(v)
    q = torch.randn((SC_H, SC_G, D), generator=gen, device=dev, dtype=torch.float32)
    return quant, kq, vq, q


def run_scores(a, rank: int):
    """One step: scores of every kv head's query rows against its compressed keys
    (smaq_key_scores), a torch softmax, and the weighted value sum (smaq_attend_values).  The
    reference's own GPU scoring kernel (its Triton fast path, smaq/triton_kernels.py:139-187,
    one call per kv head) is timed beside it on the same inputs."""
    import torch
    from smaq_b200 import build, ops
    build.build()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    quant, kq, vq, q = scores_inputs(dev)
    scale = 128 ** -0.5
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]

    def step():
        s = quant.attention_score(q, kq, scale=scale)
        w = torch.softmax(s, dim=-1)
        return ops.attend_values(w, vq.data, vq.scales, vq.zeros)

    for _ in range(max(3, a.warmup)):
        step()
    torch.cuda.synchronize()
    ts, ta = [], []
    for _ in range(a.steps):
        ev[0].record()
        s = quant.attention_score(q, kq, scale=scale)
        ev[1].record()
        w = torch.softmax(s, dim=-1)
        ev[2].record()
        ops.attend_values(w, vq.data, vq.scales, vq.zeros)
        ev[3].record()
        torch.cuda.synchronize()
        ts.append(ev[0].elapsed_time(ev[1]))
        ta.append(ev[2].elapsed_time(ev[3]))
    t_step = statistics.median([x + y for x, y in zip(ts, ta)]) * 1e-3
    t_s, t_a = statistics.median(ts) * 1e-3, statistics.median(ta) * 1e-3
    rows = SC_H * SC_N
    b_scores = rows * (64 + 2 + SC_G * 4)           # codes + norm in, fp32 scores out
    b_attend = rows * (SC_G * 4 + 32 + 8 + 8)       # weights + value codes + scales + zeros in
    peak, src = peak_hbm()
    ref_gpu = None
    smaq = import_reference()
    if smaq is not None:
        try:
            from smaq.triton_kernels import _triton_attention_scores
            from smaq.quantizer import SMAQQuantized, SMAQQuantizer as RefQ
            rq = RefQ(128, bits=SC_BITS, device=dev)
            rq.E.copy_(quant.E)
            rq.E_inv.copy_(quant.E_inv)
            per = [(q[h], SMAQQuantized(indices=kq.indices[h], norms=kq.norms[h], bits=SC_BITS)) for h in range(SC_H)]
            for _ in range(3):
                for qh, kh in per:
                    _triton_attention_scores(rq, qh, kh)
            torch.cuda.synchronize()
            tr = []
            for _ in range(a.steps):
                ev[4].record()
                for qh, kh in per:
                    _triton_attention_scores(rq, qh, kh)
                ev[5].record()
                torch.cuda.synchronize()
                tr.append(ev[4].elapsed_time(ev[5]) * 1e-3)
            t_r = statistics.median(tr)
            ref_gpu = {"kernel": "reference _smaq_scores_kernel (Triton, baseline/_ref), one call per kv head",
                       "ms": t_r * 1e3, "gbs": b_scores / t_r / 1e9, "speedup_of_smaq_key_scores": t_r / t_s}
        except Exception as exc:  # the reference's GPU kernel is informational here
            ref_gpu = {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}
    line = {"metric": "standalone compressed-history scores + attend GB/s", "value": (b_scores + b_attend) / t_step / 1e9,
            "unit": "GB/s", "n_gpus": 1, "steps": a.steps, "warmup": max(3, a.warmup), "ms_per_step": t_step * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32-query/bf16-rows",
            "data": "synthetic", "config": scores_config(),
            "kernels": {"smaq_key_scores": {"us": t_s * 1e6, "gbs": b_scores / t_s / 1e9,
                                            "frac": b_scores / t_s / 1e9 / peak},
                        "smaq_attend_values": {"us": t_a * 1e6, "gbs": b_attend / t_a / 1e9,
                                               "frac": b_attend / t_a / 1e9 / peak}},
            "roofline": {"bound": "hbm", "achieved": (b_scores + b_attend) / t_step / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": (b_scores + b_attend) / t_step / 1e9 / peak, "traffic": None, "peak_source": src,
                         "algorithmic_bytes_per_step": b_scores + b_attend},
            "reference_gpu": ref_gpu, "gpu_launches": 3 * a.steps}
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    a = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if a.workload == "append":
        (run_append_reference(a, rank) if a.impl == "reference" else run_append(a, rank, world))
        return
    if a.workload == "paged":
        if a.impl == "reference":
            if rank == 0:
                info = paged_cpu_sample(seconds_cap=120.0, max_runs=max(1, a.steps))
                print(json.dumps({"impl": "reference", "metric": METRIC, "value": info["value"], "unit": "tokens/s",
                                  "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
                                  "ms_per_step": 1e3 * PG_B / info["value"], "higher_is_better": True,
                                  "scaling": "weak", "vs_baseline": None, "dtype": "bf16-io/f32", "data": "synthetic",
                                  "config": paged_config(), "cpu_baseline": info,
                                  "e2e": {"value": info["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                                          "d2h_bytes_per_step": 0}}), flush=True)
        else:
            run_paged(a, rank, world)
        return
    if a.workload == "append_bvq":
        if a.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the block-VQ append line carries the reference's "
                                  "CPU rate as cpu_baseline"}), flush=True)
        else:
            run_append_bvq(a, rank)
        return
    if a.workload == "scores":
        if a.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the scores workload times the reference's GPU "
                              "scoring kernel inside the smaq_b200 line (reference_gpu)"}), flush=True)
        else:
            run_scores(a, rank)
        return
    if a.impl == "reference":
        run_reference(a, rank, world)
        return
    run_decode(a, rank, world)


if __name__ == "__main__":
    main()
