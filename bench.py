"""Benchmark: compressed-KV decode attention (SMAQ hot path) on B200.

Default workload: Llama-3-8B KV shape -- 32 layers, 32 query / 8 KV
heads, head_dim 128, bf16 -- batch 16 sequences x 32768 compressed history tokens (block-VQ
keys: 8-dim blocks, 256-entry fp16-valued codebook k-means-fit on 16K calibration keys; 2-bit
values in groups of 32) plus a 128-token exact bf16 window, one decode token per sequence.
A step = the attention of all 32 layers for one decode token of every sequence.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference] [--workload append]

``--workload paged`` measures configs[3] (Qwen2.5-7B KV shape, 64 sequences of 1K-64K tokens in
a 16-token paged store, 4-bit scalar keys, 64-token window); ``--workload longctx`` configs[4]
(Llama-3-70B KV shape, 4 x 128K, KV heads sharded over the ranks, strong scaling).
``--workload append`` measures BASELINE.json configs[2] instead: a batch of 8 x 8192 new tokens x
8 KV heads x head_dim 128 in bf16 quantized into store rows (tcgen05 rotation + 3-bit scalar key
codes, 2-bit values in groups of 32); GB/s counts input plus output bytes.

N > 1 (torchrun, one rank per GPU): every rank serves its own 16 sequences (sequences are
independent units; no collective on the data path) -> ``scaling: weak``.

Inputs: seeded synthetic data with the spectral key distribution (no dataset).  The KV cache
of one step (8.9 GB) is far larger than L2 (126 MB), so no explicit L2 flush is needed.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "compressed-KV decode attn tokens/s & HBM GB/s (% of roofline) at 32K/128K ctx"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="smaq_b200", choices=["smaq_b200", "reference"])
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--ctx", type=int, default=32768)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--window", type=int, default=128)
    ap.add_argument("--hq", type=int, default=32)
    ap.add_argument("--hkv", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ctas", type=int, default=0, help="decode grid size (0: one CTA per SM)")
    ap.add_argument("--no-overlap", dest="overlap", action="store_false",
                    help="plain stream ordering between layer launches (default: each layer's launch overlaps "
                         "the previous one's end; no layer writes another layer's history rows or the lengths)")
    ap.add_argument("--workload", default="decode", choices=["decode", "append", "longctx", "paged"])
    ap.add_argument("--paged-layers", type=int, default=28, help="layers of the paged workload (profiling only)")
    return ap.parse_args()


def config_of(a):
    if a.workload == "longctx":
        return {"workload": "cfg4_llama3_70b_bvq_longctx", "layers": a.layers, "batch": a.batch,
                "n_q_heads": a.hq_total, "n_kv_heads": a.hkv_total, "head_dim": 128, "history_tokens": a.ctx,
                "window_tokens": a.window, "keys": "block-VQ 8x256 (fp16 codebook)", "values": "2-bit g32",
                "parallelism": f"kv-head x{a.head_groups}" + (f", sequence x{a.seq_splits}" if a.seq_splits > 1 else ""),
                "per_gpu": {"n_q_heads": a.hq, "n_kv_heads": a.hkv}, "l2": "inputs larger than L2 (no flush)"}
    return {"workload": "cfg1_llama3_8b_bvq_decode", "layers": a.layers, "batch_per_gpu": a.batch,
            "n_q_heads": a.hq, "n_kv_heads": a.hkv, "head_dim": 128, "history_tokens": a.ctx,
            "window_tokens": a.window, "keys": "block-VQ 8x256 (fp16 codebook)", "values": "2-bit g32",
            "l2": "inputs larger than L2 (no flush)"}


def bytes_per_layer(a) -> int:
    """Algorithmic HBM bytes of one layer's decode (roofline)."""
    D = 128
    hist = a.ctx * (D // 8 + D // 4 + 2 * 2 * (D // 32))      # 16 B idx + 32 B codes + 8 B scales + 8 B zeros
    recent = a.window * 2 * D * 2                              # exact bf16 K and V
    qo = a.hq * D * 2 * 2                                      # query in, output out (bf16)
    return a.batch * (a.hkv * (hist + recent) + qo)


# ----------------------------------------------------------------------------- clocks
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


# ----------------------------------------------------------------------------- workload
def make_codebook(dev):
    """256-entry block-VQ codebook fit by seeded k-means on 16K calibration keys, fp16 values."""
    import torch
    from smaq_b200 import synthetic as syn
    from smaq_b200.block_vq import SMAQBlockVQ
    vq = SMAQBlockVQ(128, device=dev)
    ck = torch.from_numpy(syn.keys((16384,), 128, seed=21)).to(dev)
    cq = torch.from_numpy(syn.calibration_queries(16384, 128, seed=syn.SEED_CAL_Q)).to(dev)
    vq.fit(ck, cq, seed=syn.SEED_KMEANS)
    for name in ("E_blocks", "E_inv_blocks", "centroids", "decoded_centroids"):
        getattr(vq, name).copy_(getattr(vq, name).half().float())
    from smaq_b200 import ops
    vq.cb16 = ops.fp16_codebook(vq.decoded_centroids)
    assert vq.cb16 is not None
    return vq


def spectral_keys_gpu(n, gen, U, lam_sqrt, outl, dtype):
    import torch
    z = torch.randn((n, 128), generator=gen, device=U.device, dtype=torch.float32) * lam_sqrt
    x = z @ U.T
    x[:, outl] *= 8.0
    return x.to(dtype)


def build_layers(a, dev, vq, seed0: int):
    """Per layer: batched store rows [B, Hkv, ctx, ...], recent window, queries."""
    import torch
    from smaq_b200 import ops, synthetic as syn
    from smaq_b200._lib import SMAQ_KEYS_BVQ, SMAQ_LAYOUT_DECODE
    U_np, outl = syn.basis(128)
    U = torch.from_numpy(U_np.astype(np.float32)).to(dev)
    lam = torch.from_numpy(np.sqrt(syn.spectrum(128)).astype(np.float32)).to(dev)
    outl = torch.from_numpy(outl).to(dev)
    B, H, T, D, W = a.batch, a.hkv, a.ctx, 128, a.window
    bf = torch.bfloat16
    layers = []
    for li in range(a.layers):
        gen = torch.Generator(device=dev).manual_seed(seed0 * 1000 + li)
        L = {
            "codes": torch.empty((B, H, T, 16), dtype=torch.uint8, device=dev),
            "vdata": torch.empty((B, H, T, 32), dtype=torch.uint8, device=dev),
            "vs": torch.empty((B, H, T, 4), dtype=bf, device=dev),
            "vz": torch.empty((B, H, T, 4), dtype=bf, device=dev),
        }
        for b in range(B):
            k = spectral_keys_gpu(T * H, gen, U, lam, outl, bf).reshape(T, H, D)
            v = torch.randn((T, H, D), generator=gen, device=dev, dtype=torch.float32).to(bf)
            ops.append(k, v, n_heads=H, slot_offset=b * T, page_size=T, key_format=SMAQ_KEYS_BVQ,
                       E_blocks=vq.E_blocks, centroids=vq.centroids, key_codes=L["codes"], v_data=L["vdata"],
                       v_scales=L["vs"], v_zeros=L["vz"], layout=SMAQ_LAYOUT_DECODE)
        L["rk"] = spectral_keys_gpu(B * W * H, gen, U, lam, outl, bf).reshape(B, W, H, D)
        L["rv"] = torch.randn((B, W, H, D), generator=gen, device=dev, dtype=torch.float32).to(bf)
        L["q"] = (torch.randn((B, a.hq, D), generator=gen, device=dev, dtype=torch.float32)).to(bf)
        L["out"] = torch.empty((B, a.hq, D), dtype=bf, device=dev)
        layers.append(L)
    torch.cuda.synchronize()
    return layers


def decode_layer(a, L, vq, hl, rl, ws, q=None, out=None):
    from smaq_b200 import ops
    from smaq_b200._lib import SMAQ_KEYS_BVQ, SMAQ_LAYOUT_DECODE
    return ops.decode(L["q"] if q is None else q, n_kv_heads=a.hkv, key_format=SMAQ_KEYS_BVQ,
                      centroids=vq.decoded_centroids, key_codes=L["codes"], v_data=L["vdata"], v_scales=L["vs"],
                      v_zeros=L["vz"], hist_len=hl, page_size=a.ctx, recent_k=L["rk"], recent_v=L["rv"],
                      recent_len=rl, out=L["out"] if out is None else out, workspace=ws, layout=SMAQ_LAYOUT_DECODE,
                      centroids_f16=vq.cb16, num_ctas=getattr(a, "ctas", 0), overlap_prior=getattr(a, "overlap", False))


def stack_io(layers):
    """Put every layer's query rows in one device buffer and its outputs in another (each layer
    keeps views), with pinned host mirrors, so an end-to-end step moves all queries host->device
    in one copy and all outputs device->host in one copy."""
    import torch
    Q = torch.stack([L["q"] for L in layers])
    O = torch.stack([L["out"] for L in layers])
    for i, L in enumerate(layers):
        L["q"], L["out"] = Q[i], O[i]
    hQ = torch.empty_like(Q, device="cpu").pin_memory()
    hQ.copy_(Q.cpu())
    hO = torch.empty_like(O, device="cpu").pin_memory()
    return Q, O, hQ, hO


# ----------------------------------------------------------------------------- CPU baseline
def cpu_sample(a, seconds_cap: float = 20.0):
    """Time the CPU port of the reference path (oracle, fp32 like the reference's torch ops) on
    one layer x one sequence, and scale to the metric's unit."""
    from oracle import smaq_oracle as O
    from smaq_b200 import synthetic as syn
    try:
        from threadpoolctl import threadpool_info
        cores = max([i.get("num_threads", 1) for i in threadpool_info()] + [1])
    except Exception:
        cores = os.cpu_count() or 1
    rng = np.random.default_rng(5)
    H, T, D, W = a.hkv, a.ctx, 128, a.window
    idx = rng.integers(0, 256, size=(H, T, 16))
    dec = rng.standard_normal((16, 256, 8)).astype(np.float32)
    vdata = rng.integers(0, 256, size=(H, T, 32), dtype=np.uint8)
    vs = np.abs(rng.standard_normal((H, T, 4))).astype(np.float32)
    vz = rng.standard_normal((H, T, 4)).astype(np.float32)
    q = syn.queries((1, a.hq), D, seed=9)
    rk = syn.keys((W, H), D, seed=10)
    rv = syn.values((W, H), D, seed=11)
    runs = []
    t_end = time.perf_counter() + seconds_cap
    while True:
        t0 = time.perf_counter()
        K = O.bvq_dequantize(idx, dec, work=np.float32)           # the reference materialises k_hat
        V = O.dequantize_values(vdata, vs, vz, 2, 32)
        O.hybrid_attention(q, "bf16", K, V, rk, rv, a.hq, H, work=np.float32)
        runs.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end or len(runs) >= 5:
            break
    t = statistics.median(runs)
    step_s = t * a.layers * a.batch                                 # one layer x one sequence -> full step
    return {"value": a.batch / step_s, "unit": "tokens/s", "cores": int(cores), "kind": "port",
            "sample": f"1 layer x 1 sequence ({T} history + {W} window tokens, {H} kv heads), "
                      f"median of {len(runs)} runs = {t*1e3:.1f} ms, scaled x{a.layers * a.batch}"}


def run_reference(a, rank: int, world: int):
    if rank != 0:
        return
    for _ in range(max(0, a.warmup)):
        pass
    vals = []
    info = None
    for _ in range(max(1, a.steps)):
        info = cpu_sample(a, seconds_cap=max(2.0, 60.0 / max(1, a.steps)))
        vals.append(info["value"])
    v = statistics.median(vals)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1e3 * a.batch / v, "higher_is_better": True,
            "scaling": "strong" if a.workload == "longctx" else "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_of(a),
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": info["cores"], "kind": "port",
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


def append_cpu_sample(seconds_cap: float = 20.0):
    """The reference's append path restated in torch CPU ops (oracle.torch_append: norm, divide,
    fp32 matmul, searchsorted, pack; value codec) on all host threads, on a bounded sample of
    token-heads, scaled to the full batch."""
    import torch
    from oracle import smaq_oracle as O
    from smaq_b200 import synthetic as syn
    from smaq_b200.quantizer import SMAQQuantizer
    torch.set_num_threads(os.cpu_count() or 1)
    rows = 65536
    k = torch.from_numpy(syn.keys((rows,), AP_D, seed=31)).to(torch.bfloat16)
    v = torch.from_numpy(syn.values((rows,), AP_D, seed=32)).to(torch.bfloat16)
    quant = SMAQQuantizer(AP_D, bits=AP_BITS, device=torch.device("cpu"))
    quant.fit(torch.from_numpy(syn.calibration_queries(512, AP_D)))
    E, bnd = quant.E.float(), quant.decision_boundaries.float().contiguous()
    runs = []
    t_end = time.perf_counter() + seconds_cap
    while True:
        t0 = time.perf_counter()
        O.torch_append(k, v, E, bnd, AP_BITS)
        runs.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end or len(runs) >= 5:
            break
    t = statistics.median(runs)
    total = sum(append_bytes())
    scale = AP_B * AP_T * AP_H / rows
    return {"value": total / (t * scale) / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{rows} token-heads, median of {len(runs)} runs = {t*1e3:.1f} ms, scaled x{scale:.0f}"}


def run_append(a, rank: int, world: int):
    import torch
    import torch.distributed as dist
    from smaq_b200 import build, ops, synthetic as syn
    from smaq_b200._lib import SMAQ_KEYS_SCALAR, SMAQ_LAYOUT_DECODE
    from smaq_b200.quantizer import SMAQQuantizer
    build.build()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
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
    codes = torch.empty((rows, AP_D // 2), dtype=torch.uint8, device=dev)
    norms = torch.empty((rows,), dtype=torch.bfloat16, device=dev)
    vd = torch.empty((rows, AP_D // 4), dtype=torch.uint8, device=dev)
    vs = torch.empty((rows, AP_D // 32), dtype=torch.bfloat16, device=dev)
    vz = torch.empty_like(vs)
    E, bnd = quant.E.contiguous(), quant.decision_boundaries.contiguous()

    def step(kk=k, vv=v, keys=True, values=True):
        # every sequence's 8192 new tokens land in its own store page (page_size 8192)
        ops.append(kk if keys else None, vv if values else None, n_heads=AP_H, page_size=AP_T,
                   key_format=SMAQ_KEYS_SCALAR, key_bits=AP_BITS, E=E, boundaries=bnd, key_codes=codes,
                   key_norms=norms, v_data=vd, v_scales=vs, v_zeros=vz, layout=SMAQ_LAYOUT_DECODE)

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
        if world == 1 and not a.no_cpu_baseline:
            line["cpu_baseline"] = append_cpu_sample()
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_append_reference(a, rank: int):
    if rank != 0:
        return
    vals, info = [], None
    for _ in range(max(1, a.steps)):
        info = append_cpu_sample(seconds_cap=max(2.0, 60.0 / max(1, a.steps)))
        vals.append(info["value"])
    v = statistics.median(vals)
    total = sum(append_bytes())
    line = {"impl": "reference", "metric": APPEND_METRIC, "value": v, "unit": "GB/s",
            "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": 1e3 * total / (v * 1e9), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16-io/f32-matmul", "data": "synthetic", "config": append_config(),
            "cpu_baseline": {"value": v, "unit": "GB/s", "cores": info["cores"], "kind": "port",
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


def paged_cpu_sample(seconds_cap: float = 20.0):
    """The reference's hybrid attention (oracle port, fp32) for one layer x one sequence of the
    mean length, scaled to the step."""
    from oracle import smaq_oracle as O
    from smaq_b200 import synthetic as syn
    lens = paged_lengths()
    n = int(np.mean(lens))
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
    runs = []
    t_end = time.perf_counter() + seconds_cap
    while True:
        t0 = time.perf_counter()
        K = O.scalar_score_keys(codes, norms, PG_BITS, Einv, cent, D)
        V = O.dequantize_values(vdata, vs, vz, 2, 32)
        O.hybrid_attention(q, "bf16", K, V, rk, rv, PG_HQ, PG_HKV, work=np.float32)
        runs.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end or len(runs) >= 5:
            break
    t = statistics.median(runs)
    step_s = t * PG_LAYERS * PG_B
    return {"value": PG_B / step_s, "unit": "tokens/s", "cores": 1, "kind": "port",
            "sample": f"1 layer x 1 sequence of {n} tokens, median of {len(runs)} runs = {t*1e3:.1f} ms, "
                      f"scaled x{PG_LAYERS * PG_B}"}


def run_paged(a, rank: int, world: int):
    import torch
    from smaq_b200 import build, ops, synthetic as syn
    from smaq_b200._lib import SMAQ_KEYS_SCALAR, SMAQ_LAYOUT_DECODE
    from smaq_b200.quantizer import SMAQQuantizer
    build.build()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    D = 128
    lens = paged_lengths()
    n_layers = a.paged_layers
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
    hl = torch.from_numpy(lens.astype(np.int32)).to(dev)
    rl = torch.full((PG_B,), PG_W, dtype=torch.int32, device=dev)
    ws = torch.empty(ops.decode_workspace_bytes(PG_B, PG_HQ, PG_HKV, D), dtype=torch.uint8, device=dev)

    def dec(L, q=None):
        ops.decode(L["q"] if q is None else q, n_kv_heads=PG_HKV, key_format=SMAQ_KEYS_SCALAR, key_bits=PG_BITS,
                   E_inv=quant.E_inv, centroids=quant.centroids, key_norms=L["norms"], key_codes=L["codes"],
                   v_data=L["vdata"], v_scales=L["vs"], v_zeros=L["vz"], hist_len=hl, page_size=PG_PAGE,
                   block_table=L["bt"], recent_k=L["rk"], recent_v=L["rv"], recent_len=rl, out=L["out"], workspace=ws,
                   layout=SMAQ_LAYOUT_DECODE, overlap_prior=a.overlap)

    def step():
        for L in layers:
            dec(L)

    for _ in range(max(3, a.warmup)):
        step()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.steps
    ck = clocks.stop()
    Q, O, hQ, hO = stack_io(layers)

    def e2e_step():
        Q.copy_(hQ, non_blocking=True)
        step()
        hO.copy_(O, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(a.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / a.steps
    bpl = paged_bytes_per_layer(lens)
    try:
        peak = float(json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))["hbm_gbs"])
    except Exception:
        peak = 6650.0
    achieved = bpl * n_layers / (ms * 1e-3) / 1e9
    # tokens/s of a full 28-layer step (ms scaled when fewer layers were built for profiling)
    ms_full = ms * PG_LAYERS / n_layers
    line = {"metric": METRIC, "value": PG_B / (ms_full * 1e-3), "unit": "tokens/s", "n_gpus": 1, "steps": a.steps,
            "warmup": max(3, a.warmup), "ms_per_step": ms_full, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32-accum/bf16-io", "data": "synthetic", "config": paged_config(),
            "hbm_gbs": achieved,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": None, "kernel": "smaq_decode (scalar keys, paged) per step",
                         "algorithmic_bytes_per_launch": bpl},
            "e2e": {"value": PG_B / (e2e_ms * PG_LAYERS / n_layers * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": hQ.numel() * hQ.element_size(),
                    "d2h_bytes_per_step": hO.numel() * hO.element_size()},
            "gpu_launches": n_layers * a.steps, "clocks": ck}
    if not a.no_cpu_baseline:
        line["cpu_baseline"] = paged_cpu_sample()
    if rank == 0:
        print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- main
def main():
    a = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if a.workload == "append":
        if a.impl == "reference":
            run_append_reference(a, rank)
        else:
            run_append(a, rank, world)
        return
    if a.workload == "paged":
        if a.impl == "reference":
            if rank == 0:
                info = paged_cpu_sample(seconds_cap=max(2.0, 60.0 / max(1, a.steps)))
                print(json.dumps({"impl": "reference", "metric": METRIC, "value": info["value"], "unit": "tokens/s",
                                  "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
                                  "ms_per_step": 1e3 * PG_B / info["value"], "higher_is_better": True,
                                  "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                                  "config": paged_config(), "cpu_baseline": info,
                                  "e2e": {"value": info["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                                          "d2h_bytes_per_step": 0}}), flush=True)
        else:
            run_paged(a, rank, world)
        return
    if a.workload == "longctx":
        # Llama-3-70B KV shape, 4 x 128K, 80 layers; strong scaling,
        # KV heads sharded over the ranks (smaq_b200.distributed.make_plan)
        from smaq_b200.distributed import make_plan
        plan = make_plan(world, 8)
        if plan.seq_splits > 1:
            raise SystemExit("longctx: more ranks than KV heads is not benchmarked")
        a.batch, a.ctx, a.layers, a.window = 4, 131072, 80, 128
        a.hq_total, a.hkv_total = 64, 8
        a.head_groups, a.seq_splits = plan.head_groups, plan.seq_splits
        if a.impl != "reference":  # the CPU reference arm times the whole (unsharded) layer
            a.hq, a.hkv = 64 // plan.head_groups, 8 // plan.head_groups
        else:
            a.hq, a.hkv = 64, 8
    if a.impl == "reference":
        run_reference(a, rank, world)
        return
    import torch
    import torch.distributed as dist
    from smaq_b200 import build
    build.build()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    vq = make_codebook(dev)
    layers = build_layers(a, dev, vq, seed0=rank + 1)
    hl = torch.full((a.batch,), a.ctx, dtype=torch.int32, device=dev)
    rl = torch.full((a.batch,), a.window, dtype=torch.int32, device=dev)
    from smaq_b200 import ops
    ws = torch.empty(ops.decode_workspace_bytes(a.batch, a.hq, a.hkv, 128, a.ctas), dtype=torch.uint8, device=dev)

    def step():
        for L in layers:
            decode_layer(a, L, vq, hl, rl, ws)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(max(3, a.warmup)):
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
        step()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    ms = e0.elapsed_time(e1) / a.steps
    ck = clocks.stop()
    # per-layer decode call time (plan + decode + merge kernels) for the roofline
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in layers]
    for _ in range(2):
        for L, (s0, s1) in zip(layers, evs):
            s0.record()
            decode_layer(a, L, vq, hl, rl, ws)
            s1.record()
        torch.cuda.synchronize()
    layer_ms = statistics.mean(s0.elapsed_time(s1) for s0, s1 in evs)
    # end to end through the public API with host buffers: H2D queries, decode, D2H outputs
    Q, O, hQ, hO = stack_io(layers)

    def e2e_step():
        Q.copy_(hQ, non_blocking=True)
        step()
        hO.copy_(O, non_blocking=True)

    for _ in range(2):
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
        t = torch.tensor([ms, e2e_ms, layer_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms, layer_ms = t.tolist()
    bpl = bytes_per_layer(a)
    peak_gbs = None
    peak_src = "fallback 6650 GB/s"
    try:
        peak_gbs = float(json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))["hbm_gbs"])
        peak_src = "measured"
    except Exception:
        peak_gbs = 6650.0
    # average launch duration over the timed region: one decode launch per layer and nothing
    # else in a step (consecutive launches overlap when --no-overlap is not given)
    launch_ms = ms / a.layers
    achieved = bpl / (launch_ms * 1e-3) / 1e9
    # DRAM bytes per launch from one ncu capture of this workload (profiles/decode_bvq_cfg1_kernel.md)
    default_shape = (a.batch, a.ctx, a.window, a.hq, a.hkv) == (16, 32768, 128, 32, 8)
    traffic = 284.2e6 if default_shape else None
    h2d = hQ.numel() * hQ.element_size()
    d2h = hO.numel() * hO.element_size()
    if rank == 0:
        strong = a.workload == "longctx"
        tokens = a.batch if strong else a.batch * world
        line = {
            "metric": METRIC, "value": tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
            "steps": a.steps, "warmup": max(3, a.warmup), "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "f32-accum/bf16-io",
            "data": "synthetic", "config": config_of(a),
            "hbm_gbs": world * bpl * a.layers / (ms * 1e-3) / 1e9,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak_gbs, "unit": "GB/s",
                         "frac": achieved / peak_gbs, "traffic": traffic, "peak_source": peak_src,
                         "kernel": "smaq_decode per layer (one decode_v3_kernel launch)",
                         "algorithmic_bytes_per_launch": bpl, "launch_us": launch_ms * 1e3,
                         "launch_us_isolated": layer_ms * 1e3,
                         "launch_time": "timed region / launches; isolated = one launch between two events"},
            "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": a.layers * a.steps,
            "clocks": ck,
        }
        if world == 1 and not a.no_cpu_baseline:
            line["cpu_baseline"] = cpu_sample(a)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
