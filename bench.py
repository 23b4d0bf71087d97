#!/usr/bin/env python
"""Benchmark: compressed-KV decode attention on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (config 1): batch 32 per GPU, 32 query heads / 8 kv heads,
head_dim 128, 8192 cached tokens per sequence, 32 layers, 4-bit K and V
packed. One step = for every layer: quantize-append the new token's K and V
of all 32 sequences, then decode attention for the 32 query heads over the
whole context (lc_decode_step: the append launch also rotates the queries). Synthetic seeded data: K, V ~ N(0, 1) with 4 outlier channels
per kv head scaled x8; queries ~ N(0, 1/sqrt(128)) read as a standard
deviation, softmax scale 1. The 9 GB cache is far larger than L2 (126 MB),
so every step streams it from HBM (no flush needed).

`value` is whole-job decode tokens/s with inputs resident in HBM. `e2e`
drives the same step through the public API from pinned host memory: every
step copies its inputs (all layers' queries and new K/V) to the device,
runs the layers, and reads every output back. The copies go in four chunks
of layers on an upload and a download stream, so they overlap the other
chunks' compute; two device buffer sets let steps be issued back to back,
and the timed region ends when the last step's outputs are in host memory.
Under
torchrun each rank runs its own 32 sequences (weak scaling, no collective on
the data path).

`--impl reference` times the reference's CPU path (the oracle's C++
restatement of turboquant-cache SimpleCache: attend_keys, softmax,
attend_values) on a bounded sample on all host cores.
"""
from __future__ import annotations

import argparse
import faulthandler
import importlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "compressed-KV decode attn GB/s & tokens/s vs HBM roofline; quantize-append GB/s"
CFG = dict(batch=32, hq=32, hkv=8, dim=128, ctx=8192, layers=32, k_bits=4, v_bits=4)
BYTES_PER_TOKEN_HEAD = 8 * 8 + 8 * 8 + 4 + 4  # 4-bit d=128: 8 K words + 8 V words + 2 sigma = 136 B


def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


def profile_traffic():
    """dram bytes per decode launch from the committed ncu summary, if present."""
    p = os.path.join(ROOT, "profiles", "k_decode_pair_config1.md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []

    def __enter__(self):
        self.nvml = False
        try:  # NVML in a thread: a sample every few ms, so short timed regions get many
            import pynvml

            pynvml.nvmlInit()
            self.h = None
            try:  # the CUDA device by PCI address (NVML and CUDA orders can differ)
                import torch

                pr = torch.cuda.get_device_properties(self.device)
                bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
                self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(self.device)
            self.nvml = True
            self.stop = threading.Event()
            self.t = threading.Thread(target=self._poll, args=(pynvml,), daemon=True)
            self.t.start()
            return self
        except Exception:
            self.nvml = False
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.device)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def _poll(self, nv):
        bits = [("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
                ("sw_power_cap", 0x4)]
        while not self.stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                mx = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
                get = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    nv.nvmlDeviceGetCurrentClocksThrottleReasons
                r = get(self.h)
                flags = ["Active" if r & b else "Not Active" for _, b in bits]
                self.lines.append(",".join([str(self.device), str(sm), str(mx), "0", hex(r)] + flags))
            except Exception:
                pass
            self.stop.wait(0.004)

    def __exit__(self, *a):
        if self.nvml:
            self.stop.set()
            self.t.join(timeout=2)
            return
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------
# CPU baseline: the oracle (C++ restatement of SimpleCache decode)
# ----------------------------------------------------------------------------
def cpu_attend_sample(seq_data, hq: int, hkv: int, dim: int, threads: int, budget_s: float, seed: int = 7):
    """Time decode for one (sequence, layer) of config 1 on the CPU oracle.

    seq_data: per kv head (k_words [n,W], k_sigma [n], v_words, v_sigma).
    Runs query heads until `budget_s` of wall time or all hq heads are done;
    returns seconds for all hq heads (extrapolated) and the heads run.
    """
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import pyoracle as orc
    from concurrent.futures import ThreadPoolExecutor

    orc.build()
    t = orc.Tables.generate(dim, CFG["k_bits"], 64, 42)
    comp = orc.Compressor(t)
    sc = orc.SimpleCache(comp, comp, 1, hkv, dim)
    for h, (kw, ks, vw, vs) in enumerate(seq_data):
        sc.load(0, h, 0, kw, ks)
        sc.load(0, h, 1, vw, vs)
    q = (orc.gauss_f32(seed, hq * dim).reshape(hq, dim) * np.float32(dim ** -0.5)).astype(np.float32)
    G = hq // hkv
    done = 0
    t0 = time.perf_counter()
    with ThreadPoolExecutor(max_workers=threads) as ex:
        while done < hq:
            batch = list(range(done, min(hq, done + threads)))
            list(ex.map(lambda h: sc.attend(0, h // G, q[h], 1.0), batch))
            done += len(batch)
            if time.perf_counter() - t0 > budget_s:
                break
    el = time.perf_counter() - t0
    return el * hq / done, done


def synth_seq_on_cpu(n: int, hkv: int, dim: int, seed: int):
    """One sequence of config-1 K/V compressed by the oracle (reference arm)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import pyoracle as orc
    from concurrent.futures import ThreadPoolExecutor

    orc.build()
    t = orc.Tables.generate(dim, CFG["k_bits"], 64, 42)
    comp = orc.Compressor(t)

    def one(h):
        out = []
        for side in (0, 1):
            x = orc.gauss_f32(seed * 1000 + 2 * h + side, n * dim).reshape(n, dim)
            rng = np.random.default_rng(seed + h)
            x[:, rng.choice(dim, 4, replace=False)] *= np.float32(8.0)
            s1, _, _, sc = comp.compress(x)
            out += [s1, sc]
        return out

    with ThreadPoolExecutor(max_workers=os.cpu_count() or 1) as ex:
        return list(ex.map(one, range(hkv)))


def run_reference(args):
    rank, _, world = env_rank()
    if rank != 0:
        return  # rank 0 alone times the CPU reference
    hq, hkv, dim, ctx, L, B = CFG["hq"], CFG["hkv"], CFG["dim"], CFG["ctx"], CFG["layers"], CFG["batch"]
    threads = os.cpu_count() or 1
    data = synth_seq_on_cpu(ctx, hkv, dim, 11)
    per = []
    for k in range(args.warmup + args.steps):
        s, heads = cpu_attend_sample(data, hq, hkv, dim, threads, budget_s=2.0, seed=100 + k)
        if k >= args.warmup:
            per.append(s)
    sample_s = statistics.median(per)
    step_s = sample_s * L * B  # one (seq, layer) sample scaled to the whole step
    tok_s = B / step_s
    line = {
        "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": {"workload": "config1 decode: batch 32, 32q/8kv, d128, ctx 8192, 32 layers, 4-bit K/V",
                   "sample": "one (sequence, layer) per step, scaled by layers x batch"},
        "cpu_baseline": {"value": tok_s, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": f"1 of {L * B} (sequence, layer) pairs per step: {hq} query heads over "
                                   f"{ctx} tokens, oracle C++ restatement of SimpleCache, {threads} threads"},
        "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------
# Scale-out workloads of config 4 (and config 1 split by kv heads), measured
# at every N beside the default line: strong scaling, fixed total work.
# ----------------------------------------------------------------------------
def _bf16_kv(torch, gen, dev, B, hkv, n, D, scale_vec):
    x = torch.randn((B, hkv, n, D), generator=gen, device=dev, dtype=torch.float32) * scale_vec
    return x.to(torch.bfloat16).contiguous()


def _outlier_scale(torch, hkv, D, dev):
    sel = torch.Generator(device="cpu")
    sel.manual_seed(99)
    v = torch.ones(hkv, D)
    for h in range(hkv):
        v[h, torch.randperm(D, generator=sel)[:4]] = 8.0
    return v.to(dev).view(1, hkv, 1, D)


def _time_steps(torch, dist, step, steps, warm, world):
    """Device time of `steps` calls of step() on torch's current stream, max over ranks (ms)."""
    for _ in range(warm):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def _request_shard(args, lc, torch, dist, dev, local, rank, world, codec, peak):
    """Config 4, first half: 256 concurrent requests at context 32768 (4-bit,
    GQA 32/8, d 128) split by request over the ranks, no collective."""
    total, ctx, L, hq, hkv, D = 256, 32768, args.c4_layers, CFG["hq"], CFG["hkv"], CFG["dim"]
    B = total // world
    steps, warm = max(3, args.steps // 2), 3
    pps = (ctx + steps + warm + 8 + 255) // 256 + 1
    cache = lc.CudaKvCache(L, hkv, D, codec, codec, max_seqs=B, max_pages=L * B * pps + 64, max_pages_per_seq=pps,
                           device=local)
    gen = torch.Generator(device=dev)
    gen.manual_seed(5000 + rank)
    sv = _outlier_scale(torch, hkv, D, dev)
    ids = list(range(B))
    t0 = time.time()
    for layer in range(L):
        for c0 in range(0, ctx, 2048):
            cache.append(layer, ids, _bf16_kv(torch, gen, dev, B, hkv, 2048, D, sv),
                         _bf16_kv(torch, gen, dev, B, hkv, 2048, D, sv))
    torch.cuda.synchronize()
    fill_s = time.time() - t0
    qs = (torch.randn((L, B, hq, D), generator=gen, device=dev) * D ** -0.5).to(torch.bfloat16)
    k1 = [_bf16_kv(torch, gen, dev, B, hkv, 1, D, sv) for _ in range(L)]
    v1 = [_bf16_kv(torch, gen, dev, B, hkv, 1, D, sv) for _ in range(L)]
    out = torch.empty((L, B, hq, D), device=dev, dtype=torch.bfloat16)

    def step():
        for layer in range(L):
            cache.decode_step(layer, ids, k1[layer], v1[layer], qs[layer], hq, 1.0, out=out[layer],
                              out_dtype=lc.LC_BF16)

    ms = _time_steps(torch, dist, step, steps, warm, world)
    n0 = cache.ring_state(0, 0)["view_len"]
    cache.timing(1)
    for _ in range(2):
        step()
    dec_ms, dec_n, _, _, other_ms = cache.timing(0)
    launch_ms = dec_ms / max(dec_n, 1)
    bytes_launch = B * hkv * BYTES_PER_TOKEN_HEAD * (n0 + 1.5)
    achieved = bytes_launch / (launch_ms / 1e3) / 1e9
    cache.close()
    del qs, k1, v1, out
    torch.cuda.empty_cache()
    return {"value": total * steps / (ms / 1e3), "unit": "tok/s", "scaling": "strong", "ms_per_step": ms / steps,
            "workload": f"config4: {total} requests x {ctx} tokens over {world} GPU(s) ({B} per GPU), {L} layers, "
                        f"32q/8kv, d128, 4-bit K/V; append + decode per layer",
            "per_gpu": {"requests": B, "decode_avg_launch_us": launch_ms * 1e3, "decode_gbs": achieved,
                        "roofline_frac": achieved / peak, "merge_and_rotation_ms_per_step": other_ms / 2},
            "fill_s": fill_s}


def _head_shard(args, lc, torch, dist, dev, local, rank, world, codec, peak):
    """Config 1 split by kv-head groups: rank r holds kv heads [r * 8/N,
    (r + 1) * 8/N) of all 32 sequences and their query groups; no collective
    (each q head reads only its kv head)."""
    B, hq, hkv, D, ctx, L = CFG["batch"], CFG["hq"], CFG["hkv"], CFG["dim"], CFG["ctx"], args.heads_layers
    split = importlib.import_module("lumen-rs_b200.split")
    h0, h1 = split.head_shard(hkv, rank, world)
    hk = h1 - h0
    G = hq // hkv
    steps, warm = max(3, args.steps // 2), 3
    pps = (ctx + steps + warm + 8 + 255) // 256 + 1
    cache = lc.CudaKvCache(L, hk, D, codec, codec, max_seqs=B, max_pages=L * B * pps + 64, max_pages_per_seq=pps,
                           device=local)
    gen = torch.Generator(device=dev)
    gen.manual_seed(6000 + rank)
    sv = _outlier_scale(torch, hkv, D, dev)[:, h0:h1]
    ids = list(range(B))
    for layer in range(L):
        for c0 in range(0, ctx, 2048):
            cache.append(layer, ids, _bf16_kv(torch, gen, dev, B, hk, 2048, D, sv),
                         _bf16_kv(torch, gen, dev, B, hk, 2048, D, sv))
    qs = (torch.randn((L, B, hk * G, D), generator=gen, device=dev) * D ** -0.5).to(torch.bfloat16)
    k1 = [_bf16_kv(torch, gen, dev, B, hk, 1, D, sv) for _ in range(L)]
    v1 = [_bf16_kv(torch, gen, dev, B, hk, 1, D, sv) for _ in range(L)]
    out = torch.empty((L, B, hk * G, D), device=dev, dtype=torch.bfloat16)

    def step():
        for layer in range(L):
            cache.decode_step(layer, ids, k1[layer], v1[layer], qs[layer], hk * G, 1.0, out=out[layer],
                              out_dtype=lc.LC_BF16)

    ms = _time_steps(torch, dist, step, steps, warm, world)
    n0 = cache.ring_state(0, 0)["view_len"]
    cache.timing(1)
    for _ in range(2):
        step()
    dec_ms, dec_n, _, _, _ = cache.timing(0)
    launch_ms = dec_ms / max(dec_n, 1)
    achieved = B * hk * BYTES_PER_TOKEN_HEAD * (n0 + 1.5) / (launch_ms / 1e3) / 1e9
    cache.close()
    del qs, k1, v1, out
    torch.cuda.empty_cache()
    return {"value": B * steps / (ms / 1e3), "unit": "tok/s", "scaling": "strong", "ms_per_step": ms / steps,
            "workload": f"config1 by kv-head groups: {B} sequences x {ctx} tokens, {hkv} kv heads split {world} "
                        f"way(s) ({hk} kv / {hk * G} q heads per GPU), {L} layers, 4-bit K/V",
            "per_gpu": {"kv_heads": hk, "decode_avg_launch_us": launch_ms * 1e3, "decode_gbs": achieved,
                        "roofline_frac": achieved / peak}}


def _longctx_split(args, lc, torch, dist, dev, local, rank, world, codec, peak, n_ctx, L, steps, warm):
    """Config 4, second half: one n_ctx-token sequence split by tokens over
    the ranks. Per layer each rank decodes its shard's partials, the library
    exchanges them (peer stores over NVLink) and merges (lc_decode_attn_split)."""
    split = importlib.import_module("lumen-rs_b200.split")
    hq, hkv, D = CFG["hq"], CFG["hkv"], CFG["dim"]
    lo, hi = split.shard_range(n_ctx, rank, world)
    owner = rank == split.owner_of_next(world)
    extra = steps + warm + 8 if owner else 0
    pages = (hi - lo + extra + 255) // 256 + 1
    cache = lc.CudaKvCache(L, hkv, D, codec, codec, max_seqs=1, max_pages=L * pages + 16, max_pages_per_seq=pages,
                           device=local)
    gen = torch.Generator(device=dev)
    gen.manual_seed(4242 + rank)
    sv = _outlier_scale(torch, hkv, D, dev)
    t0 = time.time()
    for layer in range(L):
        for c0 in range(lo, hi, 16384):
            n = min(16384, hi - c0)
            cache.append(layer, [0], _bf16_kv(torch, gen, dev, 1, hkv, n, D, sv),
                         _bf16_kv(torch, gen, dev, 1, hkv, n, D, sv))
    torch.cuda.synchronize()
    fill_s = time.time() - t0
    group = split.make_group(hq, D, local) if world > 1 else lc.SplitGroup(1, 0, lc.SplitGroup.new_id(), hq, D,
                                                                            device=local)
    dec = split.SplitSequenceDecoder(cache, 0, lc_group=group)
    qs = (torch.randn((L, 1, hq, D), generator=gen, device=dev) * D ** -0.5).to(torch.bfloat16)
    k1 = [_bf16_kv(torch, gen, dev, 1, hkv, 1, D, sv) for _ in range(L)]
    v1 = [_bf16_kv(torch, gen, dev, 1, hkv, 1, D, sv) for _ in range(L)]
    out = torch.empty((L, hq, D), device=dev, dtype=torch.float32)

    def step():
        for layer in range(L):
            if owner:
                cache.append(layer, [0], k1[layer], v1[layer])
            dec.decode(layer, qs[layer], hq, 1.0, out=out[layer])

    ms = _time_steps(torch, dist, step, steps, warm, world)
    status = group.status()
    # the same layers' local partials alone (no exchange, no merge of ranks)
    m = torch.empty((hq,), device=dev)
    l_ = torch.empty((hq,), device=dev)
    o = torch.empty((hq, D), device=dev)

    def local_step():
        for layer in range(L):
            cache.decode_partials(layer, [0], qs[layer], hq, 1.0, m=m, l=l_, o=o)

    local_ms = _time_steps(torch, dist, local_step, steps, warm, world)
    peer = group.info()["peer_stores"]
    if world > 1:
        dist.barrier()  # every rank past its last exchange before buffers are freed
    group.close()
    cache.close()
    del qs, k1, v1, out
    torch.cuda.empty_cache()
    kv_bytes = n_ctx * hkv * BYTES_PER_TOKEN_HEAD * L
    return {"value": steps / (ms / 1e3), "unit": "tok/s", "scaling": "strong", "ms_per_step": ms / steps,
            "ms_per_layer": ms / steps / L, "local_partials_ms_per_layer": local_ms / steps / L,
            "exchange_and_merge_ms_per_layer": (ms - local_ms) / steps / L,
            "exchange": ("peer stores over NVLink + release flags (lc_decode_attn_split)" if peer else
                         "in-place ncclAllGather (lc_decode_attn_split)") if world > 1 else "none (one rank)",
            "group_status": status, "decode_gbs": kv_bytes / (ms / steps / 1e3) / 1e9,
            "workload": f"config4 long context: 1 sequence of {n_ctx} tokens split over {world} GPU(s), {L} layers, "
                        f"32q/8kv, d128, 4-bit K/V", "fill_s": fill_s}


def scale_out(args, lc, torch, dist, dev, local, rank, world, codec, peak):
    res = {}
    res["config4_request_shard"] = _request_shard(args, lc, torch, dist, dev, local, rank, world, codec, peak)
    res["config1_head_shard"] = _head_shard(args, lc, torch, dist, dev, local, rank, world, codec, peak)
    res["config4_longctx_split"] = _longctx_split(args, lc, torch, dist, dev, local, rank, world, codec, peak,
                                                  1 << 20, args.longctx_layers, max(3, args.steps // 2), 3)
    return res


# ----------------------------------------------------------------------------
# Our arm
# ----------------------------------------------------------------------------
def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    rank, local, world = env_rank()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    lc = importlib.import_module("lumen-rs_b200")
    B, hq, hkv, D, ctx, L = CFG["batch"], CFG["hq"], CFG["hkv"], CFG["dim"], CFG["ctx"], args.layers
    steps, warm = args.steps, args.warmup
    total_new = steps + warm + args.e2e_steps + 8
    pages_per_seq = (ctx + total_new + 255) // 256 + 1
    codec = lc.TurboQuantCompressor(lc.TurboQuantConfig(CFG["k_bits"], 64, 42, 1000, D))
    cache = lc.CudaKvCache(L, hkv, D, codec, codec, max_seqs=B, max_pages=L * B * pages_per_seq + 64,
                           max_pages_per_seq=pages_per_seq, device=local)
    ids = list(range(B))
    stream_ptr = cache.stream()
    s = torch.cuda.ExternalStream(stream_ptr, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + 7919 * rank)
    sel = torch.Generator(device="cpu")
    sel.manual_seed(99)
    outl = torch.stack([torch.randperm(D, generator=sel)[:4] for _ in range(hkv)])  # [hkv, 4]
    scale_vec = torch.ones(hkv, D)
    for h in range(hkv):
        scale_vec[h, outl[h]] = 8.0
    scale_vec = scale_vec.to(dev).view(1, hkv, 1, D)

    def kv_block(n):
        x = torch.randn((B, hkv, n, D), generator=gen, device=dev, dtype=torch.float32) * scale_vec
        return x.to(torch.bfloat16).contiguous()

    # ---- fill the cache: 8192 tokens per sequence per layer (untimed) ----
    t_fill = time.time()
    with torch.cuda.stream(s):
        for layer in range(L):
            for c0 in range(0, ctx, 2048):
                k, v = kv_block(2048), kv_block(2048)
                torch.cuda.current_stream().synchronize()
                cache.append(layer, ids, k, v, stream=stream_ptr)
    torch.cuda.synchronize()
    fill_s = time.time() - t_fill

    # per-step inputs, device resident
    qs = (torch.randn((L, B, hq, D), generator=gen, device=dev) * D ** -0.5).to(torch.bfloat16)
    k1 = torch.stack([kv_block(1) for _ in range(L)])
    v1 = torch.stack([kv_block(1) for _ in range(L)])
    out = torch.empty((L, B, hq, D), device=dev, dtype=torch.bfloat16)
    torch.cuda.synchronize()

    def step():
        # per layer: append the new token and attend (lc_decode_step; the
        # append launch also rotates the queries)
        for layer in range(L):
            cache.decode_step(layer, ids, k1[layer], v1[layer], qs[layer], hq, 1.0, out=out[layer],
                              out_dtype=lc.LC_BF16, stream=stream_ptr)

    for _ in range(warm):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ctx0 = cache.ring_state(0, 0)["view_len"]
    launches0 = cache.kernel_launches()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        ev0.record(s)
        h0 = time.perf_counter()
        for _ in range(steps):
            step()
        host_ms = (time.perf_counter() - h0) * 1e3 / steps
        ev1.record(s)
        ev1.synchronize()
    elapsed_ms = ev0.elapsed_time(ev1)
    launches = cache.kernel_launches() - launches0  # timed region only
    # the host time to issue the same step from one native call
    # (lc_decode_step_layers: the same launches, the layer loop in C++),
    # against the per-layer calls timed above
    import numpy as np

    ids_np = np.asarray(ids, np.int32)
    torch.cuda.synchronize()
    hl_steps = max(2, min(steps, 5))
    h0 = time.perf_counter()
    for _ in range(hl_steps):
        cache.decode_step_layers(0, ids_np, k1, v1, qs, hq, 1.0, out=out, out_dtype=lc.LC_BF16, stream=stream_ptr)
    host_layers_ms = (time.perf_counter() - h0) * 1e3 / hl_steps
    torch.cuda.synchronize()
    ctx1 = cache.ring_state(0, 0)["view_len"]
    # per-kernel device times: CUDA events around each launch, a separate pass
    t_steps = max(2, min(steps, 5))
    cache.timing(1)
    for _ in range(t_steps):
        step()
    dec_ms, dec_n, app_ms, app_n, other_ms = cache.timing(0)
    ctx2 = cache.ring_state(0, 0)["view_len"]
    # the same step with R folded into the query and output projections, as
    # the reference's Gemma path does (gemma4_moe.rs:4705-4765): the decode
    # takes rotated queries and returns rotated outputs (per-launch events)
    rot_flags = lc.LC_Q_ROTATED | lc.LC_OUT_ROTATED
    cache.timing(1)
    for _ in range(t_steps):
        for layer in range(L):
            cache.decode_step(layer, ids, k1[layer], v1[layer], qs[layer], hq, 1.0, flags=rot_flags, out=out[layer],
                              out_dtype=lc.LC_BF16, stream=stream_ptr)
    rdec_ms, rdec_n, _, _, _ = cache.timing(0)
    ctx3 = cache.ring_state(0, 0)["view_len"]
    # the dominant kernel back to back, as the step issues it: every layer's
    # decode with the queries handed over rotated (f32, as lc_decode_step's
    # append launch writes them), one event pair around the whole sequence.
    # Events around every launch (above) break the programmatic overlap of a
    # launch with the previous kernel's tail and add their own gaps.
    qf = qs.float()
    reps = 3

    def decode_pass():
        for layer in range(L):
            cache.decode_attn(layer, ids, qf[layer], hq, 1.0, flags=lc.LC_Q_ROTATED, out=out[layer],
                              out_dtype=lc.LC_BF16, stream=stream_ptr)

    decode_pass()
    torch.cuda.synchronize()
    b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    b0.record(s)
    for _ in range(reps):
        decode_pass()
    b1.record(s)
    b1.synchronize()
    b2b_ms = b0.elapsed_time(b1) / (reps * L)
    del qf
    if world > 1:
        t = torch.tensor([elapsed_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    ms_step = elapsed_ms / steps
    tok_s = world * B * steps / (elapsed_ms / 1e3)
    # algorithmic bytes: every attended token's packed K/V words and sigmas, once per kv head
    kv_bytes_per_launch = B * hkv * BYTES_PER_TOKEN_HEAD * (ctx0 + 1 + ctx1) / 2.0
    kv_bytes_timed = B * hkv * BYTES_PER_TOKEN_HEAD * (ctx1 + 1 + ctx2) / 2.0
    dec_avg_ms = dec_ms / max(dec_n, 1)
    b2b_bytes = B * hkv * BYTES_PER_TOKEN_HEAD * ctx3
    achieved = b2b_bytes / (b2b_ms / 1e3) / 1e9
    achieved_isolated = kv_bytes_timed / (dec_avg_ms / 1e3) / 1e9
    rdec_avg_ms = rdec_ms / max(rdec_n, 1)
    rot_achieved = B * hkv * BYTES_PER_TOKEN_HEAD * (ctx2 + 1 + ctx3) / 2.0 / (rdec_avg_ms / 1e3) / 1e9
    peak, peak_kind = measured_peaks()
    decode_gbs = world * kv_bytes_per_launch * L * steps / (elapsed_ms / 1e3) / 1e9
    # append: bf16 in (2 x 256 B per vector pair of K,V), packed words + sigma out
    app_vecs = B * hkv * 2
    app_bytes = app_vecs * (D * 2 + 8 * 8 + 4)
    app_avg_ms = app_ms / max(app_n, 1)

    # ---- config 3's prefill quantize-append on a separate cache: 16
    # sequences x 2048-token chunks (8 kv heads, d128, 4-bit, bf16 K/V with
    # outlier channels), 4 timed chunks after one warm-up chunk ----
    pB, pchunk, pn = 16, 2048, 4
    ppages = ((pn + 1) * pchunk + 255) // 256 + 1
    pcache = lc.CudaKvCache(1, hkv, D, codec, codec, max_seqs=pB, max_pages=pB * ppages + 8,
                            max_pages_per_seq=ppages, device=local)
    pks = [kv_block(pchunk)[:pB].contiguous() for _ in range(2)]
    pvs = [kv_block(pchunk)[:pB].contiguous() for _ in range(2)]
    pids = list(range(pB))
    pcache.append(0, pids, pks[0], pvs[0])
    torch.cuda.synchronize()
    pe0, pe1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pe0.record()
    for c in range(pn):
        pcache.append(0, pids, pks[c & 1], pvs[c & 1])
    pe1.record()
    pe1.synchronize()
    p_ms = pe0.elapsed_time(pe1) / pn
    p_vecs = pB * pchunk * hkv * 2
    p_bytes = p_vecs * (D * 2 + 8 * 8 + 4)  # bf16 in; packed words + sigma out
    pcache.close()
    del pks, pvs

    # ---- e2e through the public API, every rank: each step copies its inputs
    # (all layers' q and new K/V) from pinned host memory to the device, runs
    # the layers, and reads all outputs back to pinned host memory ----
    # One record per layer in pinned host memory: [q | new K | new V] (bf16).
    nq, nk = B * hq * D, B * hkv * D
    inh = torch.empty((L, nq + 2 * nk), dtype=torch.bfloat16).pin_memory()
    inh[:, :nq].copy_(qs.view(L, -1).cpu())
    inh[:, nq:nq + nk].copy_(k1.view(L, -1).cpu())
    inh[:, nq + nk:].copy_(v1.view(L, -1).cpu())
    oh = torch.empty((L, B, hq, D), dtype=torch.bfloat16).pin_memory()
    # two sets of device buffers, so step k + 1's uploads overlap step k's
    # layers; events keep a set from being refilled (or its outputs
    # overwritten) before the step that used it is done with it
    ind = [torch.empty_like(inh, device=dev) for _ in range(2)]
    od = [torch.empty_like(out) for _ in range(2)]
    qd = [[ind[b][l, :nq].view(B, hq, D) for l in range(L)] for b in range(2)]
    kd = [[ind[b][l, nq:nq + nk].view(B, hkv, 1, D) for l in range(L)] for b in range(2)]
    vd = [[ind[b][l, nq + nk:].view(B, hkv, 1, D) for l in range(L)] for b in range(2)]

    # Copies run in chunks of layers on two copy streams: a chunk's inputs go
    # up while earlier layers compute, and its outputs come back while later
    # layers compute. The host does not wait between steps; the timed region
    # ends when the last step's last output is in host memory.
    up, down = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    chunk = max(1, L // 4)
    bounds = [(c, min(c + chunk, L)) for c in range(0, L, chunk)]
    ev_in = [[torch.cuda.Event() for _ in bounds] for _ in range(2)]
    ev_out = [[torch.cuda.Event() for _ in bounds] for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]   # the set's last layer has run
    ev_read = [torch.cuda.Event() for _ in range(2)]   # the set's outputs are in host memory
    for e in ev_used + ev_read:
        e.record(torch.cuda.current_stream())

    def e2e_step(k):
        st = k & 1
        comp = torch.cuda.current_stream()
        up.wait_event(ev_used[st])
        with torch.cuda.stream(up):
            for i, (c0, c1) in enumerate(bounds):
                ind[st][c0:c1].copy_(inh[c0:c1], non_blocking=True)
                ev_in[st][i].record(up)
        comp.wait_event(ev_read[st])  # od[st] is read back by then
        for i, (c0, c1) in enumerate(bounds):
            comp.wait_event(ev_in[st][i])
            for layer in range(c0, c1):
                cache.decode_step(layer, ids, kd[st][layer], vd[st][layer], qd[st][layer], hq, 1.0,
                                  out=od[st][layer], out_dtype=lc.LC_BF16)
            ev_out[st][i].record(comp)
            down.wait_event(ev_out[st][i])
            with torch.cuda.stream(down):
                oh[c0:c1].copy_(od[st][c0:c1], non_blocking=True)
        ev_used[st].record(comp)
        ev_read[st].record(down)

    e2e_step(0)
    e2e_step(1)
    down.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for k in range(args.e2e_steps):
        e2e_step(k)
    down.synchronize()
    torch.cuda.synchronize()
    e2e_s = (time.perf_counter() - t0) / max(args.e2e_steps, 1)
    if world > 1:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    h2d = L * (B * hq * D * 2 + 2 * B * hkv * D * 2)
    d2h = L * B * hq * D * 2

    result = None
    if rank == 0:
        # ---- CPU baseline: oracle decode of one (seq, layer) sample ----
        cpu = None
        if not args.no_cpu:
            f = cache.fetch(0, 0)
            data = [(f["k_words"][h], f["k_sigma"][h], f["v_words"][h], f["v_sigma"][h]) for h in range(hkv)]
            budget = args.cpu_budget if world == 1 else args.cpu_budget / 4
            sample_s, heads = cpu_attend_sample(data, hq, hkv, D, threads=1, budget_s=budget)
            cpu_tok_s = B / (sample_s * L * B)
            cpu = {"value": cpu_tok_s, "unit": "tok/s", "cores": 1, "kind": "port",
                   "sample": f"{heads} of {hq} query heads of one (sequence, layer) over {ctx1} tokens "
                             f"(attend_keys + softmax + attend_values, oracle C++), scaled to {L} layers x {B} seqs"}
        result = {
            "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": world, "steps": steps, "warmup": warm,
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16 tensor-core products (K/V centroid tables f16; queries and P as f16 hi+lo pairs, f32-accurate), f32 accumulation and softmax", "data": "synthetic",
            "config": {"workload": f"config1 decode: batch 32/GPU, 32q/8kv, d128, ctx 8192 (+1 per step), "
                                   f"{L} layers, 4-bit K/V packed; append + decode per layer",
                       "global_batch": world * B, "seq_len": ctx, "parallelism": f"request-shard x{world}",
                       "l2": "inputs larger than L2 (9.1 GB cache per GPU)",
                       "queries": "bf16 N(0, std 1/sqrt(128)), scale 1.0"},
            "decode_gbs": decode_gbs,
            "append": {"gbs": app_bytes / (app_avg_ms / 1e3) / 1e9, "vectors_per_s": app_vecs / (app_avg_ms / 1e3),
                       "avg_launch_us": app_avg_ms * 1e3, "mode": "strict bit-exact",
                       "what": "the decode step's append: one token of 32 sequences x 8 kv heads, K and V"},
            "prefill_append": {"gbs": p_bytes / (p_ms / 1e3) / 1e9, "vectors_per_s": p_vecs / (p_ms / 1e3),
                               "ms_per_chunk": p_ms, "mode": "strict bit-exact",
                               "what": "config 3's chunk append: 16 sequences x 2048 tokens x 8 kv heads, K and V, "
                                       "bf16 in, packed words + sigma out"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": profile_traffic(),
                         "kernel": "k_decode_pair<4, fused>", "avg_launch_us": b2b_ms * 1e3,
                         "launches": reps * L, "bytes_per_launch": b2b_bytes, "peak_source": f"{peak_kind} hbm_gbs",
                         "timing": "CUDA events around 3 x 32 back-to-back decode launches (all layers, queries "
                                   "rotated as lc_decode_step hands them over), on the cache stream",
                         "isolated": {"avg_launch_us": dec_avg_ms * 1e3, "launches": dec_n,
                                      "frac": achieved_isolated / peak,
                                      "timing": "an event pair around every launch inside the step"}},
            "weights_rotated": {"flags": "LC_Q_ROTATED | LC_OUT_ROTATED (R folded into Wq / Wo as in the "
                                         "reference's Gemma path)",
                                "avg_launch_us": rdec_avg_ms * 1e3, "achieved_gbs": rot_achieved,
                                "frac": rot_achieved / peak, "launches": rdec_n},
            "cpu_baseline": cpu,
            "e2e": {"value": world * B / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_s * 1e3, "per": "GPU (bytes), whole job (value)",
                    "copies": "4 chunks of layers each way, pinned host memory, on an upload and a download "
                              "stream overlapped with the other chunks' compute; two device buffer sets, steps "
                              "issued back to back; wall clock over all steps to the last output in host memory"},
            "gpu_launches": launches,
            "breakdown_ms_per_step": {"decode_attn": dec_ms / t_steps, "append": app_ms / t_steps,
                                      "other_kernels": other_ms / t_steps, "host_issue": host_ms,
                                      "host_issue_one_call": host_layers_ms},
            "clocks": clk.summary(),
            "fill_s": fill_s,
        }
    cache.close()
    del qs, k1, v1, out, ind, od, inh, oh, qd, kd, vd
    torch.cuda.empty_cache()
    if not args.no_scale_out:
        # strong-scaling workloads of config 4 (and config 1 by kv heads),
        # every rank in the same order; rank 0 reports them on this line
        so = scale_out(args, lc, torch, dist, dev, local, rank, world, codec, measured_peaks()[0])
        if rank == 0:
            result.update(so)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ----------------------------------------------------------------------------
# Config 4, second half: one 1,048,576-token sequence split by sequence
# ----------------------------------------------------------------------------
def run_longctx(args):
    import torch
    import torch.distributed as dist

    rank, local, world = env_rank()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    lc = importlib.import_module("lumen-rs_b200")
    codec = lc.TurboQuantCompressor(lc.TurboQuantConfig(CFG["k_bits"], 64, 42, 1000, CFG["dim"]))
    peak, _ = measured_peaks()
    with ClockSampler(local) as clk:
        r = _longctx_split(args, lc, torch, dist, dev, local, rank, world, codec, peak, args.ctx_tokens, args.layers,
                           args.steps, args.warmup)
    if rank == 0:
        line = {"metric": METRIC, "value": r["value"], "unit": "tok/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "f16 tensor-core products (K/V centroid tables f16; queries and P as f16 hi+lo pairs, f32-accurate), f32 accumulation and softmax",
                "data": "synthetic",
                "config": {"workload": r["workload"], "global_batch": 1, "seq_len": args.ctx_tokens,
                           "parallelism": f"sequence-split x{world}"},
                "clocks": clk.summary(), "mode": "longctx"}
        line.update({k: v for k, v in r.items() if k not in line and k != "workload"})
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ----------------------------------------------------------------------------
# Config 2: mixed precision with rotating windows
# ----------------------------------------------------------------------------
def run_window(args):
    import torch

    rank, local, world = env_rank()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    lc = importlib.import_module("lumen-rs_b200")
    B, hq, hkv, D = 16, 16, 8, 256
    win, glob_ctx = 1024, 32768
    layers = [win] * 5 + [0]  # 5 sliding layers per global layer
    L = len(layers)
    kc = lc.TurboQuantCompressor(lc.TurboQuantConfig(3, 64, 42, 1000, D))
    vc = lc.TurboQuantCompressor(lc.TurboQuantConfig(2, 64, 42, 1000, D))
    steps, warm = args.steps, args.warmup
    pages_g = (glob_ctx + steps + warm + 8 + 255) // 256 + 1
    pages_w = win // 256 + 2
    cache = lc.CudaKvCache(L, hkv, D, kc, vc, max_seqs=B, max_pages=B * (5 * 2 * pages_w + pages_g) + 64,
                           max_pages_per_seq=pages_g, device=local, layer_max_size=layers, layer_keep=[0] * L,
                           store_flags=lc.LC_STORE_DIGEST)
    gen = torch.Generator(device=dev)
    gen.manual_seed(5 + rank)
    ids = list(range(B))

    def kv(n):
        return (torch.randn((B, hkv, n, D), generator=gen, device=dev)).to(torch.bfloat16)

    t_fill = time.time()
    for layer, ms in enumerate(layers):
        if ms:  # sliding: one window-sized chunk, then single-token steps wrapping the ring 3 more times
            cache.append(layer, ids, kv(win), kv(win))
            k1f, v1f = kv(1), kv(1)
            for _ in range(3 * win):
                cache.append(layer, ids, k1f, v1f)
        else:
            for c0 in range(0, glob_ctx, 2048):
                cache.append(layer, ids, kv(2048), kv(2048))
    torch.cuda.synchronize()
    fill_s = time.time() - t_fill
    qs = (torch.randn((L, B, hq, D), generator=gen, device=dev) * D ** -0.5).to(torch.bfloat16)
    k1 = torch.stack([kv(1) for _ in range(L)])
    v1 = torch.stack([kv(1) for _ in range(L)])
    out = torch.empty((L, B, hq, D), device=dev, dtype=torch.bfloat16)

    def step():
        # lc_decode_step per layer: the append launch also rotates the step's
        # queries, which the decode kernel reads as given
        for layer in range(L):
            cache.decode_step(layer, ids, k1[layer], v1[layer], qs[layer], hq, 1.0 / D ** 0.5, out=out[layer],
                              out_dtype=lc.LC_BF16)

    for _ in range(warm):
        step()
    torch.cuda.synchronize()
    views = [cache.ring_state(0, l)["view_len"] for l in range(L)]
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record()
        for _ in range(steps):
            step()
        ev1.record()
        ev1.synchronize()
    ms_step = ev0.elapsed_time(ev1) / steps
    # per-launch device times (CUDA events around each launch), a separate pass
    t_steps = max(2, min(steps, 5))
    cache.timing(1)
    for _ in range(t_steps):
        step()
    dec_ms, dec_n, app_ms, app_n, other_ms = cache.timing(0)
    bpt = 8 * lc.packed_words(D, 3) + 8 * lc.packed_words(D, 2) + 8  # 176 B per (token, kv head)
    kv_bytes = B * hkv * bpt * sum(views)
    # the global layer's decode kernel alone: per-launch CUDA events (the
    # partials kernel; the query rotation and the slot merge are timed apart),
    # 738 MB of packed KV per launch, above L2
    g_layer = layers.index(0)
    n_g = 10
    torch.cuda.synchronize()
    cache.timing(1)
    for _ in range(n_g):
        cache.decode_attn(g_layer, ids, qs[g_layer], hq, 1.0 / D ** 0.5, out=out[g_layer], out_dtype=lc.LC_BF16)
    g_ms, g_n, _, _, g_other = cache.timing(0)
    g_us = g_ms / max(1, g_n) * 1e3
    g_bytes = B * hkv * bpt * views[g_layer]
    peak, peak_kind = measured_peaks()
    g_gbs = g_bytes / (g_us * 1e-6) / 1e9
    # the same global-layer call page-sparse (LC_SPARSE_PAGES: max(pages / 8,
    # 64) of the 64-token pages by their digest bound, with the sink, the 4
    # recent pages and the tail); the first call digests every full page
    cache.decode_attn(g_layer, ids, qs[g_layer], hq, 1.0 / D ** 0.5, flags=lc.LC_SPARSE_PAGES,
                      out=out[g_layer], out_dtype=lc.LC_BF16)
    torch.cuda.synchronize()
    ev0.record()
    for _ in range(n_g):
        cache.decode_attn(g_layer, ids, qs[g_layer], hq, 1.0 / D ** 0.5, flags=lc.LC_SPARSE_PAGES,
                          out=out[g_layer], out_dtype=lc.LC_BF16)
    ev1.record()
    ev1.synchronize()
    sparse_us = ev0.elapsed_time(ev1) / n_g * 1e3
    for _ in range(3):
        cache.decode_attn(g_layer, ids, qs[g_layer], hq, 1.0 / D ** 0.5, out=out[g_layer], out_dtype=lc.LC_BF16)
    torch.cuda.synchronize()
    ev0.record()
    for _ in range(n_g):
        cache.decode_attn(g_layer, ids, qs[g_layer], hq, 1.0 / D ** 0.5, out=out[g_layer], out_dtype=lc.LC_BF16)
    ev1.record()
    ev1.synchronize()
    dense_call_us = ev0.elapsed_time(ev1) / n_g * 1e3
    print(json.dumps({
        "metric": METRIC, "value": B / (ms_step / 1e3), "unit": "tok/s", "n_gpus": 1, "steps": steps,
        "warmup": warm, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16 tensor-core products (K/V centroid tables f16; queries and P as f16 hi+lo pairs, f32-accurate), f32 accumulation and softmax", "data": "synthetic",
        "mode": "window",
        "config": {"workload": f"config2: batch {B}, {hq}q/{hkv}kv, d{D}, 3-bit K / 2-bit V, 5 sliding layers "
                               f"(ring {win}, wrapped 4x) + 1 global layer ({glob_ctx} tokens); lc_decode_step "
                               f"(append + decode) per layer", "views": views},
        "decode_gbs": kv_bytes / (ms_step / 1e3) / 1e9, "bytes_per_token_head": bpt,
        "breakdown_ms_per_step": {"decode_attn": dec_ms / t_steps, "append": app_ms / t_steps,
                                  "other_kernels (query rotation, merge)": other_ms / t_steps},
        "global_layer_sparse": {"call_us": sparse_us, "dense_call_us": dense_call_us,
                                "speedup": dense_call_us / sparse_us,
                                "what": "lc_decode_attn of the 32,771-token global layer with LC_SPARSE_PAGES "
                                        "(digest selection, then the tensor-core kernel over the chosen pages) "
                                        "against the same call dense; whole calls, CUDA events"},
        "roofline": {"bound": "hbm", "kernel": "k_decode_mma32 (global layer)", "achieved": g_gbs, "peak": peak,
                     "unit": "GB/s", "frac": g_gbs / peak, "us_per_launch": g_us, "bytes_per_launch": g_bytes,
                     "other_kernels_us": g_other / n_g * 1e3, "peak_source": f"{peak_kind} hbm_gbs"},
        "clocks": clk.summary(), "fill_s": fill_s,
    }), flush=True)
    cache.close()


# ----------------------------------------------------------------------------
# Config 3: prefill quantize-append in 2048-token chunks + prefix reuse
# ----------------------------------------------------------------------------
def run_sparse(args):
    """Page-sparse decode (LC_SPARSE_PAGES) against dense decode on one cache:
    config 4's per-GPU share, 32 requests x 32768 tokens, GQA 32/8, d128,
    4-bit; the same decode steps timed both ways (no appends in the timed
    steps, so the digests are up to date after the warm-up)."""
    import torch

    rank, local, world = env_rank()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    lc = importlib.import_module("lumen-rs_b200")
    B, hq, hkv, D, ctx = 32, CFG["hq"], CFG["hkv"], CFG["dim"], 32768
    L = min(args.layers, 4)
    codec = lc.TurboQuantCompressor(lc.TurboQuantConfig(CFG["k_bits"], 64, 42, 1000, D))
    pages = (ctx + 255) // 256 + 1
    cache = lc.CudaKvCache(L, hkv, D, codec, codec, max_seqs=B, max_pages=L * B * pages + 64,
                           max_pages_per_seq=pages, store_flags=lc.LC_STORE_DIGEST, device=local)
    gen = torch.Generator(device=dev)
    gen.manual_seed(4242 + rank)
    ids = list(range(B))
    for layer in range(L):
        for c0 in range(0, ctx, 2048):
            k = torch.randn((B, hkv, 2048, D), generator=gen, device=dev).to(torch.bfloat16)
            v = torch.randn((B, hkv, 2048, D), generator=gen, device=dev).to(torch.bfloat16)
            cache.append(layer, ids, k, v)
    q = (torch.randn((L, B, hq, D), generator=gen, device=dev) * D ** -0.5).to(torch.bfloat16)
    out_d = torch.empty((L, B, hq, D), device=dev, dtype=torch.float32)
    out_s = torch.empty((L, B, hq, D), device=dev, dtype=torch.float32)

    def step(flags, out):
        for layer in range(L):
            cache.decode_attn(layer, ids, q[layer], hq, 1.0, flags=flags, out=out[layer], out_dtype=lc.LC_F32)

    res = {}
    with ClockSampler(local) as clk:
        for name, flags, out in (("dense", 0, out_d), ("sparse", lc.LC_SPARSE_PAGES, out_s)):
            for _ in range(args.warmup):
                step(flags, out)
            torch.cuda.synchronize()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
            for _ in range(args.steps):
                step(flags, out)
            ev1.record()
            ev1.synchronize()
            res[name] = ev0.elapsed_time(ev1) / args.steps
    P = ctx // 64
    keep = max(P // 8, 64)
    bytes_dense = L * B * hkv * ctx * BYTES_PER_TOKEN_HEAD
    print(json.dumps({
        "metric": METRIC, "value": B / (res["sparse"] / 1e3), "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": res["sparse"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16 tensor-core products (K/V centroid tables f16; queries and P as f16 hi+lo pairs, f32-accurate), f32 accumulation and softmax",
        "data": "synthetic", "mode": "sparse",
        "config": {"workload": f"config4 per-GPU share: {B} requests x {ctx} tokens, {hq}q/{hkv}kv, d{D}, 4-bit, "
                               f"{L} layers; page-sparse decode (64-token pages, keep max(pages/8, 64) + sink + "
                               f"recent + tail) vs dense", "kept_fraction": keep * 64 / ctx},
        "dense": {"tok_s": B / (res["dense"] / 1e3), "ms_per_step": res["dense"],
                  "decode_gbs": bytes_dense / (res["dense"] / 1e3) / 1e9},
        "speedup_vs_dense": res["dense"] / res["sparse"],
        "max_abs_sparse_vs_dense": float((out_s - out_d).abs().max()),
        "clocks": clk.summary(),
    }), flush=True)
    cache.close()


def run_prefill(args):
    import torch

    rank, local, world = env_rank()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    lc = importlib.import_module("lumen-rs_b200")
    hkv, D, L = CFG["hkv"], CFG["dim"], 1
    B, n_new, chunk, prefix, n_req = 16, 16384, 2048, 4096, 64
    codec = lc.TurboQuantCompressor(lc.TurboQuantConfig(CFG["k_bits"], 64, 42, 1000, D))
    pages = (n_new + chunk + 255) // 256 + 1
    cache = lc.CudaKvCache(L, hkv, D, codec, codec, max_seqs=B + 1 + n_req,
                           max_pages=(B + 1) * pages + n_req * 2 + 64, max_pages_per_seq=pages, device=local)
    gen = torch.Generator(device=dev)
    gen.manual_seed(77 + rank)
    sel = torch.Generator(device="cpu")
    sel.manual_seed(99)
    scale_vec = torch.ones(hkv, D)
    for h in range(hkv):
        scale_vec[h, torch.randperm(D, generator=sel)[:4]] = 8.0
    scale_vec = scale_vec.to(dev).view(1, hkv, 1, D)
    ks = [(torch.randn((B, hkv, chunk, D), generator=gen, device=dev) * scale_vec).to(torch.bfloat16)
          for _ in range(n_new // chunk)]
    vs = [(torch.randn((B, hkv, chunk, D), generator=gen, device=dev) * scale_vec).to(torch.bfloat16)
          for _ in range(n_new // chunk)]
    ids = list(range(B))
    # warm-up on a throwaway fill, then release
    for r in range(args.warmup):
        cache.append(0, ids, ks[r % len(ks)], vs[r % len(vs)])
    for b in ids:
        cache.release(b)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record()
        for c in range(n_new // chunk):
            cache.append(0, ids, ks[c], vs[c])
        ev1.record()
        ev1.synchronize()
    ms = ev0.elapsed_time(ev1)
    vectors = B * n_new * hkv * 2
    bytes_alg = vectors * (D * 2 + 8 * 8 + 4)  # bf16 in; packed words + sigma out
    # prefill attention: one more 2048-token chunk on sequence 0 (view 16384 +
    # 2048), its queries attending causally over the view (lc_prefill_attn)
    cache.append(0, [0], ks[0][:1].contiguous(), vs[0][:1].contiguous())
    hq = CFG["hq"]
    qp = (torch.randn((chunk, hq, D), generator=gen, device=dev) * D ** -0.5).to(torch.bfloat16)
    outq = torch.empty((chunk, hq, D), device=dev, dtype=torch.bfloat16)
    for _ in range(2):
        cache.prefill_attn(0, 0, qp, hq, D ** -0.5, out=outq, out_dtype=lc.LC_BF16)
    torch.cuda.synchronize()
    reps = 5
    cache.timing(1)
    ev0.record()
    for _ in range(reps):
        cache.prefill_attn(0, 0, qp, hq, D ** -0.5, out=outq, out_dtype=lc.LC_BF16)
    ev1.record()
    ev1.synchronize()
    pf_ms = ev0.elapsed_time(ev1) / reps
    pk_ms, pk_n, _, _, po_ms = cache.timing(0)
    view = n_new + chunk
    pf_bytes = view * hkv * (8 * lc.packed_words(D, 4) * 2 + 8)  # the view's packed K/V read once: 136 B per (token, kv head)
    visible = chunk * (view - chunk) + chunk * (chunk + 1) // 2  # (query token, key) pairs under the causal mask
    pf_flops = 4.0 * D * hq * visible  # QK and PV multiply-adds
    peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
    bf16_peak = peaks.get("bf16_tflops", 1590.0)
    prefill_attn = {
        "chunk_tokens": chunk, "view_tokens": view, "ms_per_chunk": pf_ms,
        "kernel_ms": pk_ms / max(1, pk_n), "other_kernels_ms": po_ms / max(1, pk_n),
        "query_tokens_per_s": chunk / (pf_ms / 1e3),
        "kv_gbs": pf_bytes / (pf_ms / 1e3) / 1e9, "kv_bytes_per_chunk": pf_bytes,
        "useful_tflops": pf_flops / (pk_ms / max(1, pk_n) / 1e3) / 1e12,
        "tensor_frac_of_bf16_peak": pf_flops / (pk_ms / max(1, pk_n) / 1e3) / 1e12 / bf16_peak,
        "note": "k_prefill_tiled, one launch: queries rotated on the tensor cores, each 64-key tile dequantized "
                "once per (kv head, 32 query tokens x 4 heads), QK as two m16n8k16 MMAs (hi / lo query) and PV as "
                "one, output normalised and un-rotated in the same kernel",
    }
    # prefix reuse: one 4096-token prefix shared by 64 requests through the block table
    src = B
    cache.append(0, [src], ks[0][:1, :, :prefix // 2].contiguous(), vs[0][:1, :, :prefix // 2].contiguous())
    cache.append(0, [src], ks[1][:1, :, :prefix // 2].contiguous(), vs[1][:1, :, :prefix // 2].contiguous())
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for r in range(n_req):
        cache.fork(src, B + 1 + r, prefix)
    torch.cuda.synchronize()
    fork_us = (time.perf_counter() - t0) * 1e6 / n_req
    q = (torch.randn((n_req, CFG["hq"], D), generator=gen, device=dev) * D ** -0.5).to(torch.bfloat16)
    outp = torch.empty((n_req, CFG["hq"], D), device=dev, dtype=torch.bfloat16)
    rq = [B + 1 + r for r in range(n_req)]
    cache.decode_attn(0, rq, q, CFG["hq"], 1.0, out=outp, out_dtype=lc.LC_BF16)
    ref0 = torch.empty((1, CFG["hq"], D), device=dev, dtype=torch.bfloat16)
    cache.decode_attn(0, [src], q[:1], CFG["hq"], 1.0, out=ref0, out_dtype=lc.LC_BF16)
    torch.cuda.synchronize()
    fork_vs_src = float((outp[:1].float() - ref0.float()).abs().max())
    print(json.dumps({
        "metric": METRIC, "value": bytes_alg / (ms / 1e3) / 1e9, "unit": "GB/s", "n_gpus": 1, "steps": 1,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 (strict reference order)", "data": "synthetic", "mode": "prefill",
        "config": {"workload": f"config3 prefill: {B} sequences x {n_new} new tokens appended in {chunk}-token "
                               f"chunks, 8 kv heads, d128, 4-bit, bf16 K/V with outlier channels; "
                               f"{n_req} requests forked from one {prefix}-token prefix (256-token pages)"},
        "append": {"vectors_per_s": vectors / (ms / 1e3), "bytes_per_vector": D * 2 + 8 * 8 + 4,
                   "ms_per_chunk": ms / (n_new // chunk)},
        "prefix": {"fork_us_per_request": fork_us, "pages_shared_per_request": prefix // 256,
                   "max_abs_fork_vs_source_decode": fork_vs_src},
        "prefill_attn": prefill_attn,
        "clocks": clk.summary(),
    }), flush=True)
    cache.close()


def main():
    faulthandler.enable()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--layers", type=int, default=CFG["layers"], help="layers (32 = config 1; fewer for profiling)")
    ap.add_argument("--cpu-budget", type=float, default=20.0, help="seconds of CPU-baseline sampling")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--mode", default="decode", choices=["decode", "longctx", "prefill", "window", "sparse"],
                    help="decode: config 1 request-sharded; longctx: config 4's 1M-token sequence split by "
                         "sequence; prefill: config 3 chunked quantize-append and prefix reuse; window: config 2 "
                         "mixed precision with rotating windows")
    ap.add_argument("--ctx-tokens", type=int, default=1 << 20, help="longctx: tokens of the split sequence")
    ap.add_argument("--no-scale-out", action="store_true",
                    help="skip the strong-scaling workloads reported beside the default line")
    ap.add_argument("--c4-layers", type=int, default=4, help="layers of config 4's 256 x 32K request-shard run")
    ap.add_argument("--heads-layers", type=int, default=8, help="layers of the kv-head-shard run of config 1")
    ap.add_argument("--longctx-layers", type=int, default=8, help="layers of the 1M-token split run")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args)
    elif args.mode == "longctx":
        run_longctx(args)
    elif args.mode == "prefill":
        run_prefill(args)
    elif args.mode == "sparse":
        run_sparse(args)
    elif args.mode == "window":
        run_window(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
