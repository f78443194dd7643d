#!/usr/bin/env python3
"""Benchmark of the B200 decode-attention hot path (one JSON line on rank 0).

Metric: decode-attention achieved HBM GB/s (% of peak) and
seq-steps/s at 1/2/4/8 B200.  Default workload = BASELINE config 4, the one
the metric's "at 1/2/4/8 B200" is quoted on: long-context split-KV
flash-decoding, batch 4, context 131072, 14 Q / 2 KV heads, head_dim 64,
bf16 KV ~ N(0,1); the KV sequence is sharded evenly over the N GPUs and the
per-shard softmax records are exchanged over NVLink peer memory inside the
merge kernel (--exchange nccl: all-gathered over NCCL instead) and merged on
every GPU.  A step is one decode step of all 24 Qwen2-0.5B layers: per layer
RoPE on q/k, the owner's cache-write of the new row, split-KV attention, the
exchange and the merge.

  value       whole-job algorithmic bytes / step time, inputs resident in HBM
  e2e         the same through the C ABI with pinned HOST buffers, every
              step's host->device inputs and device->host outputs included
  roofline    dominant kernel (decode attention), bytes per launch over its
              CUDA-event launch time, vs the measured HBM copy bandwidth
  cpu_baseline  the reference's own CPU code (oracle/_ref, compiled from
              tmac_gguf.cpp:990-1016 / :1090-1128) on a bounded sample

Usage: python bench.py [--gpus N] [--steps K] [--warmup W]
                       [--impl tg|reference]
                       [--workload longctx|batched|cfg2|cfg1|prefill|qkv|qkv_batched]
For N > 1 launch with torch.distributed.run (one rank per GPU).
"""
from __future__ import annotations

import argparse
import ctypes as C
import csv
import datetime
import importlib.util
import io
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "tmac_gguf.cpp_b200")

N_HEAD, N_KV, HD = 14, 2, 64
QD, KD = N_HEAD * HD, N_KV * HD

WORKLOADS = {
    # BASELINE config 4
    "longctx": dict(B=4, ctx=131072, layers=24, dtype="bf16", split=True,
                    desc="config4: long-context split-KV decode, B=4, ctx=131072, bf16 KV, "
                         "KV sharded over the GPUs, softmax records exchanged and merged"),
    # BASELINE config 3
    "batched": dict(B=256, ctx=4096, layers=24, dtype="bf16", split=False,
                    desc="config3: batched decode, B=256 per GPU, ctx=4096, bf16 KV, "
                         "24 layers with independent seeds, sequences partitioned per GPU"),
    # BASELINE config 2
    "cfg2": dict(B=64, ctx=256, layers=24, dtype="f32", split=False, ragged=True,
                 desc="config2: batched decode, B=64, ctx~U[1,256], fp32 KV, 24 layers"),
    # BASELINE config 1
    "cfg1": dict(B=1, ctx=256, layers=24, dtype="f32", split=False,
                 desc="config1: single sequence, pos=255, fp32 KV, 24 layers"),
    # config 1 and config 3 run as the whole attention block of a layer
    # (tmac_gguf.cpp:1045-1140): the Q/K/V projection (Q5_0 q/k, Q8_0 v)
    # with biases, RoPE and cache-write fused in one kernel, attention, and
    # the Q5_0 attn_output matvec with its residual add into the hidden state
    "qkv": dict(B=1, ctx=256, layers=24, dtype="f32", split=False, qkv=True,
                desc="config1 as attention blocks: x -> Q5_0/Q8_0 q/k/v projection + bias + "
                     "RoPE + cache-write -> attention -> Q5_0 attn_output + residual, B=1, "
                     "pos=255, fp32 KV, 24 layers"),
    "qkv_batched": dict(B=256, ctx=4096, layers=24, dtype="bf16", split=False, qkv=True,
                        desc="config3 as attention blocks: x -> Q5_0/Q8_0 q/k/v projection + "
                             "bias + RoPE + cache-write -> attention -> Q5_0 attn_output + "
                             "residual, B=256, ctx=4096, bf16 KV, 24 layers"),
    # BASELINE config 5
    "prefill": dict(B=16, ctx=2048, layers=1, dtype="bf16", split=False, prefill=True,
                    desc="config5: causal prefill, B=16 per GPU, S=2048, 14Q/2KV heads, d=64, "
                         "RoPE in fp32 then bf16 q/k/v, fp32 accumulate, tcgen05"),
}


# DRAM bytes (read, write) per launch of the dominant kernel, from one ncu
# capture of that kernel on a B200 at N = 1 (dram__bytes_read.sum and
# dram__bytes_write.sum).  For a KV shard of 1/N of the context the launch
# streams 1/N of the rows, so the figure is scaled by the shard's share.
NCU_TRAFFIC = {
    "longctx": (268508928, 3666176),
    "batched": (538675200, 5082112),
    "prefill": (75751936, 67844352),
}


def ncu_traffic(workload, share=1.0):
    t = NCU_TRAFFIC.get(workload)
    return None if t is None else (t[0] + t[1]) * share


def load_package():
    name = "tmac_gguf_cpp_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(
        name, os.path.join(PKG_DIR, "__init__.py"), submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load_oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # noqa: E402
    return oracle


def stamp_summary(st, n_sms):
    """In-step timing of the bf16 decode steps from their %globaltimer
    stamps, uint64 [step][row][4] in ns (decode CTA c in row c: start,
    dependency released, tiles done, end; merge CTA m in row n_sms + m:
    start, decode data available, -, end):
      launch_us  decode dependency released (earliest CTA) -> the step's last
                 CTA ended (decode and merge kernel: one layer in the step)
      tiles_us   released -> the last decode CTA finished its tiles
      tail_us    last tile finished -> step end (merge of split sequences
                 and, across GPUs, the record exchange)
      period_us  between consecutive steps' ends (one layer)
      early_us   how long before the release the first decode CTA started
                 (its pre-wait prologue and tile loads)"""
    st = st.astype(np.int64)
    dec, mrg = st[:, :n_sms, :], st[:, n_sms:, :]
    big = np.iinfo(np.int64).max
    rel = np.where(dec[:, :, 1] > 0, dec[:, :, 1], big).min(axis=1)
    start = np.where(dec[:, :, 0] > 0, dec[:, :, 0], big).min(axis=1)
    tiles = dec[:, :, 2].max(axis=1)
    end = np.maximum(dec[:, :, 3].max(axis=1), mrg[:, :, 3].max(axis=1))
    out = {"steps": int(st.shape[0]),
           "launch_us": float(np.mean(end - rel)) / 1e3,
           "tiles_us": float(np.mean(tiles - rel)) / 1e3,
           "tail_us": float(np.mean(end - tiles)) / 1e3,
           "early_us": float(np.mean(rel - start)) / 1e3}
    if st.shape[0] > 1:
        out["period_us"] = float(np.mean(np.diff(end))) / 1e3
    return out


def torch_reference_check(kv, layer, q_rot, out, pos, world, tol, dist=None):
    """Independent check of one layer's output: attention of the rotated q
    (the kernels write it back) over this rank's cache rows in float64 torch
    on the GPU, every rank's softmax record combined, compared with the
    library's output (tmac_gguf.cpp:1093-1128 semantics: scale 1/sqrt(64),
    causal window 0..pos, query head h on KV head h / 7)."""
    import torch
    B = len(pos)
    g = N_HEAD // N_KV
    kvh = torch.arange(N_HEAD, device="cuda") // g
    ms, ls, os_ = [], [], []
    for s in range(B):
        n_loc = int(min(max(int(pos[s]) + 1 - kv.shard_start, 0), kv.max_ctx))
        if n_loc == 0:
            ms.append(torch.full((N_HEAD,), -1e300, dtype=torch.float64, device="cuda"))
            ls.append(torch.zeros(N_HEAD, dtype=torch.float64, device="cuda"))
            os_.append(torch.zeros(N_HEAD, HD, dtype=torch.float64, device="cuda"))
            continue
        kr, vr = kv.read_rows(layer, s, 0, n_loc)
        to32 = lambda a: torch.from_numpy(
            (np.ascontiguousarray(a).view(np.uint16).astype(np.uint32) << 16).view(np.float32))
        K = to32(kr).cuda().double().reshape(n_loc, N_KV, HD)[:, kvh, :]
        V = to32(vr).cuda().double().reshape(n_loc, N_KV, HD)[:, kvh, :]
        q = q_rot[s].double().reshape(N_HEAD, HD)
        sc = torch.einsum("hd,nhd->hn", q, K) / 8.0
        m = sc.max(dim=1).values
        w = torch.exp(sc - m[:, None])
        ms.append(m)
        ls.append(w.sum(dim=1))
        os_.append(torch.einsum("hn,nhd->hd", w, V))
    m, l, o = torch.stack(ms), torch.stack(ls), torch.stack(os_)
    if world > 1:
        gm = [torch.zeros_like(m) for _ in range(world)]
        gl = [torch.zeros_like(l) for _ in range(world)]
        go = [torch.zeros_like(o) for _ in range(world)]
        dist.all_gather(gm, m)
        dist.all_gather(gl, l)
        dist.all_gather(go, o)
        M = torch.stack(gm).max(dim=0).values
        wt = [torch.exp(mi - M) for mi in gm]
        l = sum(li * wi for li, wi in zip(gl, wt))
        o = sum(oi * wi[..., None] for oi, wi in zip(go, wt))
    ref = (o / l[..., None]).reshape(B, QD)
    err = float((out.double() - ref).abs().max())
    return {"max_abs": err, "tol": tol, "ok": bool(err <= tol), "layer": layer,
            "sequences": B,
            "against": "float64 torch attention over the same bf16 cache rows and rotated q, "
                       "every rank's softmax record combined"}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def tensor_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["bf16_tflops"]), "measured (burst)"
    return 1590.0, "fallback"


def positions(wl, seed=1234):
    """Global position of each sequence's current token (past_len)."""
    if wl.get("ragged"):
        rng = np.random.default_rng(seed)
        return rng.integers(0, wl["ctx"], size=wl["B"]).astype(np.int32)
    return np.full(wl["B"], wl["ctx"] - 1, dtype=np.int32)


def algo_bytes_step(wl, pos):
    """Algorithmic HBM bytes of one decode step over all layers and
    sequences (whole job): K and V rows read once, the new row written,
    q read and the output written (fp32)."""
    s_kv = 2 if wl["dtype"] == "bf16" else 4
    n = pos.astype(np.int64) + 1
    per_layer = int(np.sum(n * 2 * KD * s_kv + 2 * KD * s_kv + 2 * QD * 4))
    return per_layer * wl["layers"]


L2_BYTES = 126 * 1024 * 1024  # B200 L2


def qkv_weight_bytes():
    """Bytes of one layer's projection weights: W_q and W_k in Q5_0 (22-byte
    blocks of 32), W_v in Q8_0 (34-byte blocks)."""
    nb = QD // 32
    return (QD + KD) * nb * 22 + KD * nb * 34


def wo_weight_bytes():
    """Bytes of one layer's attn_output weight (Q5_0, QD x QD)."""
    return QD * (QD // 32) * 22


def qkv_kernel_bytes(wl, B):
    """Algorithmic bytes of one projection launch: the weights once, x read,
    rotated q written, the new k / v rows written."""
    s_kv = 2 if wl["dtype"] == "bf16" else 4
    return qkv_weight_bytes() + B * (QD * 4 + QD * 4 + 2 * KD * s_kv)


def attn_output_bytes(B):
    """Algorithmic bytes of one attn_output launch: W_o once, the context
    read, the hidden state read and written."""
    return wo_weight_bytes() + B * 3 * QD * 4


def synth_qblocks(rng, wtype, rows, cols, d_scale):
    """Random GGML blocks (Q5_0 = 6, Q8_0 = 8) with finite fp16 scales."""
    bs = 22 if wtype == 6 else 34
    nb = rows * (cols // 32)
    blk = rng.integers(0, 256, size=(nb, bs), dtype=np.uint8)
    d = (d_scale * rng.uniform(0.5, 1.5, nb) * rng.choice([-1.0, 1.0], nb)).astype(np.float16)
    blk[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    return blk.reshape(rows, -1)


def kernel_bytes_launch(wl, pos, shard_start, shard_len, split):
    """Algorithmic bytes of one decode launch on one rank: this shard's K and
    V rows read once, the new row written by its owner, q read and the
    output written (the fused kernel does RoPE, cache-write and attention)."""
    s_kv = 2 if wl["dtype"] == "bf16" else 4
    p1 = pos.astype(np.int64) + 1
    n_loc = np.clip(p1 - shard_start, 0, shard_len)
    owner = (pos >= shard_start) & (pos < shard_start + shard_len)
    return int(np.sum(n_loc * 2 * KD * s_kv) + int(owner.sum()) * 2 * KD * s_kv
               + len(pos) * 2 * QD * 4)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,"
              "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None

    def stop(self, t0, t1):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = []
        for r in csv.reader(io.StringIO(out)):
            if len(r) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(r[0].strip(), "%Y/%m/%d %H:%M:%S.%f").timestamp()
                idx = int(r[1])
                sm = float(r[2])
                smax = float(r[3])
            except ValueError:
                continue
            if idx not in self.gpus:
                continue
            rows.append((ts, sm, smax, [x.strip() for x in r[6:10]]))
        if not rows:
            return None
        inside = [x for x in rows if t0 - 0.05 <= x[0] <= t1 + 0.05] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for x in inside for i, v in enumerate(x[3])
                          if v.lower() == "active"})
        return {"sm_mhz": statistics.median(x[1] for x in inside),
                "sm_max_mhz": max(x[2] for x in inside),
                "reasons": reasons, "samples": len(inside)}


# ---------------------------------------------------------------- CPU legs

def cpu_units(O, wl, n_units, seed=7):
    """n_units independent (sequence, layer) units for the reference CPU
    code: fp32 caches holding bf16-rounded N(0,1) values (the reference
    only has fp32 caches), at the workload's positions.  At most 32 distinct
    cache arrays are allocated; further units reuse them."""
    pos = positions(wl)
    n_distinct = min(n_units, 32)
    caches = []
    for u in range(n_distinct):
        p = int(pos[u % len(pos)])
        gen = O.normal_bf16 if wl["dtype"] == "bf16" else O.normal
        k = gen(O.derive_seed(seed, u, 0, 4), (p + 1) * KD).reshape(p + 1, KD)
        v = gen(O.derive_seed(seed, u, 0, 5), (p + 1) * KD).reshape(p + 1, KD)
        caches.append((k, v, p))
    ks = [caches[u % n_distinct][0] for u in range(n_units)]
    vs = [caches[u % n_distinct][1] for u in range(n_units)]
    ps = np.array([caches[u % n_distinct][2] for u in range(n_units)], np.int32)
    q = np.stack([O.normal(O.derive_seed(seed, u, 0, 1), QD) for u in range(n_units)])
    return q, ks, vs, ps


def unit_bytes(wl, ps):
    s_kv = 2 if wl["dtype"] == "bf16" else 4
    return int(np.sum((ps.astype(np.int64) + 1) * 2 * KD * s_kv + 2 * QD * 4))


def time_reference_cpu(O, wl, n_units, n_threads, reps=1):
    q, ks, vs, ps = cpu_units(O, wl, n_units)
    best = None
    for _ in range(reps):
        t = time.perf_counter()
        O.ref_attention_units_mt(q, ks, vs, ps, n_threads)
        dt = time.perf_counter() - t
        best = dt if best is None else min(best, dt)
    return unit_bytes(wl, ps) / best / 1e9, best, int(np.sum(ps + 1))


def qkv_cpu_weights(O):
    """One layer's attention-block weights for the CPU legs (Q5_0 q/k, Q8_0
    v, biases, Q5_0 attn_output)."""
    return (O.qblocks(O.TYPE_Q5_0, 101, QD, QD, 0.004), O.qblocks(O.TYPE_Q5_0, 102, KD, QD, 0.004),
            O.qblocks(O.TYPE_Q8_0, 103, KD, QD, 0.0005), O.normal(104, QD) * np.float32(0.1),
            O.normal(105, KD) * np.float32(0.1), O.normal(106, KD) * np.float32(0.1),
            O.qblocks(O.TYPE_Q5_0, 107, QD, QD, 0.004))


def run_reference_qkv_units(O, W, x, ks, vs, ps, n_threads):
    """The reference's attention block (tmac_gguf.cpp:1045-1140: quantized
    projections, biases, RoPE, cache-write, attention, attn_output matmul,
    residual add) on every unit, fanned out over n_threads (ctypes drops the
    GIL during each call)."""
    from concurrent.futures import ThreadPoolExecutor
    h0 = O.normal(108, QD)

    def one(u):
        O.ref_attention_block(*W, x[u], h0, ks[u], vs[u], int(ps[u]), v_type=O.TYPE_Q8_0)

    if n_threads <= 1:
        for u in range(len(ps)):
            one(u)
        return
    with ThreadPoolExecutor(n_threads) as ex:
        list(ex.map(one, range(len(ps))))


def time_reference_qkv_cpu(O, wl, n_units, n_threads):
    x, ks, vs, ps = cpu_units(O, wl, n_units)
    W = qkv_cpu_weights(O)
    t = time.perf_counter()
    run_reference_qkv_units(O, W, x, ks, vs, ps, n_threads)
    dt = time.perf_counter() - t
    return ((unit_bytes(wl, ps) + n_units * (qkv_weight_bytes() + wo_weight_bytes() + 2 * QD * 4))
            / dt / 1e9, dt, int(np.sum(ps + 1)))


def run_reference_arm(args, wl, rank, world):
    """--impl reference: the reference's CPU implementation of the path,
    all host threads, bounded sample per step (rank 0 only)."""
    if rank != 0:
        return
    O = load_oracle()
    kind = "reference" if O.ref_available() else "port"
    if kind == "port":
        run = lambda q, ks, vs, ps, nt: O.attention_units_mt(q, ks, vs, ps, nt)
    else:
        run = lambda q, ks, vs, ps, nt: O.ref_attention_units_mt(q, ks, vs, ps, nt)
    threads = os.cpu_count() or 1
    total_units = wl["B"] * wl["layers"]
    # whole layers of the batch, enough units to keep every thread busy
    n_units = min(total_units, max(wl["B"], (threads // wl["B"]) * wl["B"]))
    q, ks, vs, ps = cpu_units(O, wl, n_units)
    extra = 0
    if wl.get("qkv"):
        if kind == "reference":
            W = qkv_cpu_weights(O)
            run = lambda q, ks, vs, ps, nt: run_reference_qkv_units(O, W, q, ks, vs, ps, nt)
            extra = n_units * (qkv_weight_bytes() + wo_weight_bytes() + 2 * QD * 4)
        else:
            print(json.dumps({"impl": "reference", "unavailable":
                              "the projection workloads need the reference build "
                              "oracle/_ref/libref.so"}), flush=True)
            return
    for _ in range(args.warmup):
        run(q, ks, vs, ps, threads)
    t = time.perf_counter()
    for _ in range(args.steps):
        run(q, ks, vs, ps, threads)
    dt = time.perf_counter() - t
    gbs = (unit_bytes(wl, ps) + extra) * args.steps / dt / 1e9
    sample = (f"{n_units} of the {total_units} (sequence, layer) units of one step per "
              f"timed step ({n_units // wl['B']} layer(s) x {wl['B']} sequences), fp32 "
              f"caches of the workload's values, {threads} threads")
    line = {
        "metric": "decode-attn achieved HBM GB/s (algorithmic bytes / time)",
        "value": gbs, "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong" if wl["split"] else "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (splitmix64 + Box-Muller N(0,1))",
        "config": {"workload": wl["desc"], "cpu_sample": sample},
        "seq_steps_per_s": n_units / wl["layers"] * args.steps / dt,
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": sample},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def prefill_flops(B, S, n_head=N_HEAD, hd=HD):
    """Algorithmic causal FLOPs: query t attends t+1 keys; QK and PV are 2
    FLOPs per multiply-add each."""
    return 4.0 * hd * n_head * B * S * (S + 1) / 2.0


def run_prefill_bench(args, wl, rank, world, local, be, tg, barrier, max_over_ranks, sampler):
    import torch
    B, S = wl["B"], wl["ctx"]
    kv = tg.KVCache(be, 1, B, S, dtype=tg.DTYPE_BF16)
    g = torch.Generator(device="cuda")
    g.manual_seed(2000 + rank)
    q = torch.randn(B, S, QD, device="cuda", generator=g)
    k = torch.randn(B, S, KD, device="cuda", generator=g)
    v = torch.randn(B, S, KD, device="cuda", generator=g)
    out = torch.zeros(B, S, QD, device="cuda")
    stream = torch.cuda.ExternalStream(be.stream())
    kv.prefill(0, B, S, q, k, v, out)
    be.synchronize()
    be.graph_begin()
    kv.prefill(0, B, S, q, k, v, out)
    graph = be.graph_end()
    for _ in range(args.warmup):
        graph.launch()
    be.synchronize()
    barrier()
    launches0 = be.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.time()
    e0.record(stream)
    for _ in range(args.steps):
        graph.launch()
    e1.record(stream)
    be.synchronize()
    t1 = time.time()
    launches = be.launch_count() - launches0
    barrier()
    ms_step = max_over_ranks(e0.elapsed_time(e1)) / args.steps
    clocks = sampler.stop(t0, t1) if sampler else None
    flops = prefill_flops(B, S)
    value = flops * world / (ms_step * 1e-3) / 1e12
    be.profile_enable(True)
    be.graph_begin()
    kv.prefill(0, B, S, q, k, v, out)
    gprof = be.graph_end()
    be.profile_enable(False)
    kms, kn = 0.0, 0
    for _ in range(max(3, min(args.steps, 20))):
        gprof.launch()
        a, n = be.profile_read()
        kms += a
        kn += n
    gprof.destroy()
    k_ms = kms / max(kn, 1)
    peak, peak_kind = tensor_peak()
    achieved = flops / (k_ms * 1e-3) / 1e12
    achieved = -max_over_ranks(-achieved) if world > 1 else achieved
    # end to end: fp32 inputs from pinned host memory, output back to host
    qh = torch.randn(B, S, QD).pin_memory()
    kh = torch.randn(B, S, KD).pin_memory()
    vh = torch.randn(B, S, KD).pin_memory()
    oh = torch.zeros(B, S, QD).pin_memory()
    for _ in range(2):
        kv.prefill(0, B, S, qh, kh, vh, oh)
    barrier()
    n_e2e = max(3, args.steps // 4)
    t = time.perf_counter()
    for _ in range(n_e2e):
        kv.prefill(0, B, S, qh, kh, vh, oh)
    e2e_s = max_over_ranks(time.perf_counter() - t)
    e2e = flops * world * n_e2e / e2e_s / 1e12
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        O = load_oracle()
        if O.ref_available():
            Ss = 1024
            qs = O.round_bf16(O.normal(11, Ss * QD)).reshape(Ss, QD)
            ks = O.round_bf16(O.normal(12, Ss * KD)).reshape(Ss, KD)
            vs = O.round_bf16(O.normal(13, Ss * KD)).reshape(Ss, KD)
            kc = np.zeros_like(ks)
            vc = np.zeros_like(vs)
            ctx_o = np.empty(QD, np.float32)
            R = O.ref()
            tt = time.perf_counter()
            for t_ in range(Ss):
                qq = np.ascontiguousarray(qs[t_])
                R.tgref_cache_write_attention(qq, np.ascontiguousarray(ks[t_]),
                                              np.ascontiguousarray(vs[t_]), ctx_o,
                                              kc.reshape(-1), vc.reshape(-1), t_)
            dt = time.perf_counter() - tt
            cpu = {"value": prefill_flops(1, Ss) / dt / 1e12, "unit": "TFLOP/s", "cores": 1,
                   "kind": "reference",
                   "sample": f"1 sequence x {Ss} tokens processed token by token by the "
                             f"reference code (tmac_gguf.cpp:1090-1128), single-threaded, "
                             f"{dt:.2f} s"}
    if rank == 0:
        line = {
            "metric": "causal prefill attention TFLOP/s (algorithmic causal FLOPs / time)",
            "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1))",
            "config": {"workload": wl["desc"], "batch": B, "seq_len": S, "n_head": N_HEAD,
                       "n_kv_head": N_KV, "head_dim": HD,
                       "parallelism": f"sequence-partitioned x{world}",
                       "l2": "inputs 151 MB fp32 per step > L2"},
            "gpu_launches": launches,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak, "peak_kind": peak_kind,
                         "kernel": "prefill_attn_kernel", "flops_per_launch": flops,
                         "launch_ms": k_ms, "traffic": ncu_traffic(args.workload),
                         "traffic_unit": "bytes per launch (ncu dram__bytes_read + write)"},
            "e2e": {"value": e2e, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": B * S * (QD + 2 * KD) * 4,
                    "d2h_bytes_per_step": B * S * QD * 4},
            "clocks": clocks, "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    graph.destroy()
    kv.destroy()


# ---------------------------------------------------------------- GPU arm

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="tg", choices=["tg", "reference"])
    ap.add_argument("--workload", default="longctx", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", default="auto", choices=["auto", "peer", "nccl"],
                    help="split-KV record exchange for N > 1 (tg_comm_set_exchange)")
    ap.add_argument("--ctx", type=int, default=0,
                    help="override the workload's context length (small cases for "
                         "profiler captures; the reported config says so)")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the independent check of layer 0's output")
    ap.add_argument("--ring", type=int, default=0, choices=[0, 128, 192],
                    help="decode K/V ring per CTA in KB (tg_set_decode_tuning; 0 automatic)")
    ap.add_argument("--preload", type=int, default=0, choices=[0, 1],
                    help="tile loads before the grid-dependency wait when safe (1) or never")
    ap.add_argument("--layers", type=int, default=0,
                    help="override the layers per step (small profiling cases)")
    args = ap.parse_args()
    wl = dict(WORKLOADS[args.workload])
    if args.layers > 0:
        wl["layers"] = args.layers
    if args.ctx > 0:
        wl["ctx"] = args.ctx
        wl["desc"] = wl["desc"] + f" [context overridden to {args.ctx}]"
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference_arm(args, wl, rank, world)
    if args.warmup < 3:
        args.warmup = 3

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    tg = load_package()
    tg.set_decode_tuning(args.ring, args.preload)
    be = tg.CudaBackend(local)
    if wl.get("prefill"):
        def barrier_p():
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()

        def max_p(x):
            if world == 1:
                return x
            t = torch.tensor([x], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())
        sampler = ClockSampler(set(range(world))) if local == 0 else None
        time.sleep(0.3 if sampler else 0)
        run_prefill_bench(args, wl, rank, world, local, be, tg, barrier_p, max_p, sampler)
        be.shutdown()
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    split = wl["split"] and world > 1
    if split:
        uid = [tg.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        be.comm_init(uid[0], rank, world, timeout_ms=120000)
        be.set_exchange({"auto": tg.EXCHANGE_AUTO, "peer": tg.EXCHANGE_PEER,
                         "nccl": tg.EXCHANGE_NCCL}[args.exchange])

    B, L = wl["B"], wl["layers"]
    pos = positions(wl)
    if wl["split"]:
        shard_start, shard_len = tg.shard_range(wl["ctx"], world, rank)
        gctx = wl["ctx"]
    else:
        shard_start, shard_len, gctx = 0, wl["ctx"], wl["ctx"]
    dtype = tg.DTYPE_BF16 if wl["dtype"] == "bf16" else tg.DTYPE_F32
    kv = tg.KVCache(be, L, B, max(shard_len, 1), dtype=dtype, shard_start=shard_start,
                    global_ctx=gctx)
    kv.fill_normal(0x5EED0000 + 7919 * rank)

    g = torch.Generator(device="cuda")
    g.manual_seed(1000 + (0 if wl["split"] else rank))
    q = torch.randn(L, B, QD, device="cuda", generator=g)
    kn = torch.randn(L, B, KD, device="cuda", generator=g)
    vn = torch.randn(L, B, KD, device="cuda", generator=g)
    out = torch.zeros(L, B, QD, device="cuda")
    pos_d = torch.from_numpy(pos).cuda()
    stream = torch.cuda.ExternalStream(be.stream())

    qkv = bool(wl.get("qkv"))
    if qkv:
        # One weight set per layer (device-resident model constants); the
        # step's input is the normed hidden state x, in q's place.
        rng = np.random.default_rng(77 + rank)
        weights, w_out = [], []
        for _ in range(L):
            wq = torch.from_numpy(synth_qblocks(rng, 6, QD, QD, 0.004)).cuda()
            wk = torch.from_numpy(synth_qblocks(rng, 6, KD, QD, 0.004)).cuda()
            wv = torch.from_numpy(synth_qblocks(rng, 8, KD, QD, 0.0005)).cuda()
            bq = torch.randn(QD, device="cuda", generator=g) * 0.1
            bk = torch.randn(KD, device="cuda", generator=g) * 0.1
            bv = torch.randn(KD, device="cuda", generator=g) * 0.1
            weights.append(tg.QKVWeights(wq, wk, wv, QD, v_type=tg.WTYPE_Q8_0, b_q=bq,
                                         b_k=bk, b_v=bv))
            w_out.append(torch.from_numpy(synth_qblocks(rng, 6, QD, QD, 0.004)).cuda())

    def step(qs, ks, vs, ps, os_):
        for l in range(L):
            if qkv:   # x = qs[l]; the residual stream os_[l] is read and written
                kv.attention_block(l, weights[l], w_out[l], qs[l], ps, os_[l],
                                   o_type=tg.WTYPE_Q5_0)
            elif split:
                kv.decode_layer_splitkv(l, qs[l], ks[l], vs[l], ps, os_[l])
            else:
                kv.decode_layer(l, qs[l], ks[l], vs[l], ps, os_[l])

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident timed region -----------------------------------
    # One decode step (all layers) is captured into a CUDA graph after a
    # first direct run has sized the scratch buffers; the graph is replayed.
    step(q, kn, vn, pos_d, out)
    be.synchronize()
    be.graph_begin()
    step(q, kn, vn, pos_d, out)
    graph = be.graph_end()
    for _ in range(args.warmup):
        graph.launch()
    be.synchronize()
    sampler = ClockSampler(set(range(world))) if local == 0 else None
    time.sleep(0.3 if sampler else 0)
    # A step whose inputs fit twice in L2 is timed alone between L2 flushes
    # (a 512 MB write on the same stream, outside the events); larger steps
    # stream their inputs from HBM on their own and run back to back.
    wbytes = L * (qkv_weight_bytes() + wo_weight_bytes()) if qkv else 0
    gpu_step_bytes = algo_bytes_step(wl, pos) / (world if wl["split"] else 1) + wbytes
    flush = gpu_step_bytes < 2 * L2_BYTES
    flush_buf = torch.empty(512 << 20, dtype=torch.uint8, device="cuda") if flush else None

    def l2_flush():
        if flush:
            with torch.cuda.stream(stream):
                flush_buf.add_(1)

    barrier()
    launches0 = be.launch_count()
    t_wall0 = time.time()
    if flush:
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        for a, b in evs:
            l2_flush()
            a.record(stream)
            graph.launch()
            b.record(stream)
    else:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            graph.launch()
        e1.record(stream)
    be.synchronize()
    t_wall1 = time.time()
    launches = be.launch_count() - launches0
    barrier()
    ms_local = sum(a.elapsed_time(b) for a, b in evs) if flush else e0.elapsed_time(e1)
    ms_total = max_over_ranks(ms_local)
    clocks = sampler.stop(t_wall0, t_wall1) if sampler else None
    ms_step = ms_total / args.steps
    # The attention block also reads and writes the hidden state (x stands in
    # for q in the attention bytes; the context stays on the device).
    hbytes = L * B * 2 * QD * 4 if qkv else 0
    bytes_step = (algo_bytes_step(wl, pos) + wbytes + hbytes) * (1 if wl["split"] else world)
    seqs_step = B * (1 if wl["split"] else world)
    value = bytes_step / (ms_step * 1e-3) / 1e9

    # ---- roofline: decode-kernel launches timed with CUDA events -----------
    # A second graph of the same step carries event records around every
    # decode-attention launch; each replay re-records them on the stream.
    be.profile_enable(tg.PROFILE_PROJECTION if qkv else tg.PROFILE_ATTENTION)
    be.graph_begin()
    step(q, kn, vn, pos_d, out)
    gprof = be.graph_end()
    be.profile_enable(False)
    kms, kn_launch = 0.0, 0
    for _ in range(max(3, min(args.steps, 50))):
        l2_flush()
        gprof.launch()
        ms_i, n_i = be.profile_read()
        kms += ms_i
        kn_launch += n_i
    gprof.destroy()
    # Projection workloads time both projection-class launches of a layer
    # (the Q/K/V kernel and attn_output): bytes per launch is their mean.
    k_bytes = ((qkv_kernel_bytes(wl, B) + attn_output_bytes(B)) / 2 if qkv
               else kernel_bytes_launch(wl, pos, shard_start, shard_len, split))
    k_avg_ms = kms / max(kn_launch, 1)
    hbm_peak, peak_kind = peaks()
    achieved = k_bytes / (k_avg_ms * 1e-3) / 1e9
    achieved_min = max_over_ranks(-achieved)  # slowest rank's kernel
    achieved = -achieved_min if world > 1 else achieved

    # ---- in-step timing of the bf16 decode steps (globaltimer stamps) ------
    instep = None
    fused = kv.uses_tensor_cores() and not qkv
    if fused:
        be.profile_enable(tg.PROFILE_STAMPS)
        be.graph_begin()
        step(q, kn, vn, pos_d, out)
        gst = be.graph_end()
        be.profile_enable(False)
        sums = []
        for _ in range(max(3, min(args.steps, 20))):
            l2_flush()
            gst.launch()
            sums.append(stamp_summary(be.profile_read_stamps(), be.num_sms()))
        gst.destroy()
        instep = {k: float(np.mean([x[k] for x in sums])) for k in sums[0]}
        for k in ("launch_us", "tiles_us", "tail_us", "period_us"):  # slowest rank
            if k in instep:
                instep[k] = max_over_ranks(instep[k])
        k_in_ms = instep["launch_us"] / 1e3
        achieved_in = k_bytes / (k_in_ms * 1e-3) / 1e9

    # ---- parity of one layer against an independent reference -----------
    parity = None
    if fused and not args.no_parity:
        be.synchronize()
        parity = torch_reference_check(kv, 0, q[0], out[0], pos, world, 2e-3,
                                       dist if world > 1 else None)

    # ---- end to end through the C ABI with pinned host buffers ---------------
    qh = torch.randn(L, B, QD).pin_memory()
    kh = torch.randn(L, B, KD).pin_memory()
    vh = torch.randn(L, B, KD).pin_memory()
    oh = torch.zeros(L, B, QD).pin_memory()
    ph = torch.from_numpy(pos.copy()).pin_memory()

    def e2e_step():
        be.metal_batch_begin()
        step(qh, kh, vh, ph, oh)
        be.metal_batch_end()

    # Through the C ABI (include/tg_cuda_backend.h, the boundary the
    # reference's C++ forward loop calls), arguments converted once per
    # buffer: every step's host->device inputs and device->host outputs
    # inside tg_batch_begin / tg_batch_end.  The same loop through the
    # Python wrapper is reported beside it.
    hb, kvb = be.handle, kv.handle
    if qkv:
        fn = tg.lib().tg_attention_block_splitkv if split else tg.lib().tg_attention_block
        args_l = [(hb, kvb, l, B, C.byref(weights[l].desc), tg.WTYPE_Q5_0, w_out[l].data_ptr(),
                   qh[l].data_ptr(), ph.data_ptr(), oh[l].data_ptr()) for l in range(L)]
    else:
        fn = tg.lib().tg_decode_layer_splitkv if split else tg.lib().tg_decode_layer
        args_l = [(hb, kvb, l, B, qh[l].data_ptr(), kh[l].data_ptr(), vh[l].data_ptr(),
                   ph.data_ptr(), oh[l].data_ptr()) for l in range(L)]

    def c_step(timed=False):
        t_call = 0
        be.metal_batch_begin()
        for a in args_l:
            t0c = time.perf_counter_ns()
            rc = fn(*a)
            t_call += time.perf_counter_ns() - t0c
            if rc != 0:
                raise tg.TGError(rc, tg.lib().tg_last_error().decode())
        be.metal_batch_end()
        return t_call

    for _ in range(args.warmup):
        c_step()
    barrier()
    e2e_steps = max(3, args.steps // 2)
    c_ns = 0
    t = time.perf_counter()
    for _ in range(e2e_steps):
        c_ns += c_step()
    e2e_s = max_over_ranks(time.perf_counter() - t)
    e2e_value = bytes_step * e2e_steps / e2e_s / 1e9
    cabi_us_call = c_ns / (e2e_steps * L) / 1e3
    for _ in range(2):
        e2e_step()
    barrier()
    host_s = 0.0
    t = time.perf_counter()
    for _ in range(e2e_steps):
        be.metal_batch_begin()
        th = time.perf_counter()
        step(qh, kh, vh, ph, oh)
        host_s += time.perf_counter() - th
        be.metal_batch_end()
    py_s = max_over_ranks(time.perf_counter() - t)
    py_value = bytes_step * e2e_steps / py_s / 1e9
    host_us_call = host_s / (e2e_steps * L) * 1e6
    if qkv:   # x and the hidden state in, hidden out; weights and caches stay
        h2d = L * B * QD * 4 * 2 + L * B * 4
        d2h = L * B * QD * 4
    else:
        h2d = L * B * (QD + 2 * KD) * 4 + L * B * 4
        d2h = L * B * (2 * QD + KD) * 4

    # ---- CPU baseline (rank 0, one GPU only) -------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        O = load_oracle()
        if O.ref_available():
            n_units = 2 if wl["ctx"] > 8192 else 24
            if qkv:
                gbs, dt, npos = time_reference_qkv_cpu(O, wl, n_units, 1)
            else:
                gbs, dt, npos = time_reference_cpu(O, wl, n_units, 1)
            cpu = {"value": gbs, "unit": "GB/s", "cores": 1, "kind": "reference",
                   "sample": f"{n_units} (sequence, layer) units at the workload's positions "
                             f"({npos} cache rows, {dt:.2f} s), reference code single-threaded "
                             "as it runs" + ("; its attention block from x (tmac_gguf.cpp:"
                                             "1045-1140: Q5_0/Q8_0 projections, attention, "
                                             "attn_output, residual)" if qkv else "")
                             + "; fp32 caches of bf16-rounded values, bytes counted as "
                             "the workload's"}

    if rank == 0:
        line = {
            "metric": "decode-attn achieved HBM GB/s (algorithmic bytes / time)",
            "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong" if wl["split"] else "weak", "vs_baseline": None,
            "dtype": wl["dtype"], "data": "synthetic (seeded N(0,1))",
            "config": {"workload": wl["desc"], "batch": B, "context": wl["ctx"],
                       "layers_per_step": L, "n_head": N_HEAD, "n_kv_head": N_KV,
                       "head_dim": HD, "parallelism": f"split-kv x{world}" if wl["split"]
                       else f"sequence-partitioned x{world}",
                       "l2": ("L2 flushed between timed steps (512 MB write outside the "
                              "events): %.1f MB of inputs per GPU per step" % (gpu_step_bytes / 1e6))
                             if flush else "inputs larger than L2: %.0f MB per GPU per step"
                             % (gpu_step_bytes / 1e6),
                       "exchange": ({tg.EXCHANGE_PEER: "nvlink peer stores in the merge kernel",
                                     tg.EXCHANGE_NCCL: "ncclAllGather + merge kernel"}
                                    .get(be.exchange, "none") if split else "none")},
            "seq_steps_per_s": seqs_step / (ms_step * 1e-3),
            "hbm_frac_of_measured": value / (hbm_peak * world),
            "gpu_launches": launches,
            "roofline": {"bound": "hbm",
                         "achieved": achieved_in if fused else achieved, "peak": hbm_peak,
                         "unit": "GB/s", "frac": (achieved_in if fused else achieved) / hbm_peak,
                         "peak_kind": peak_kind,
                         "timing": ("in-step: %globaltimer stamps of every CTA, decode "
                                    "dependency released -> last decode / merge CTA ended, "
                                    "mean over the step's layers (the decode + merge pair)"
                                    if fused else "CUDA events around each launch"),
                         "kernel": ("projection kernels (q/k/v + attn_output), "
                                    + ("qkv_tc_kernel" if B >= 9 else "qkv_kernel"))
                         if qkv else
                         ("decode_fused_kernel" if kv.uses_tensor_cores()
                          else ("decode_small_kernel" if kv.max_ctx <= 1024 and
                                shard_start == 0 and not split else "decode_generic_kernel")),
                         "bytes_per_launch": k_bytes,
                         "launch_ms": k_in_ms if fused else k_avg_ms,
                         "launch_ms_alone": k_avg_ms, "achieved_alone": achieved,
                         "traffic": ncu_traffic(args.workload,
                                                shard_len / wl["ctx"] if wl["split"] else 1.0),
                         "traffic_unit": "bytes per launch (ncu dram__bytes_read + write)"},
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "api": "C ABI (tg_decode_layer[_splitkv] / tg_attention_block[_splitkv]) "
                           "called from ctypes with page-locked host buffers, one call per "
                           "layer inside tg_batch_begin / tg_batch_end",
                    "c_abi_us_per_layer_call": cabi_us_call,
                    "python_api": {"value": py_value,
                                   "host_us_per_layer_call": host_us_call}},
            "instep_us": instep,
            "merge_exchange_us_per_layer": instep["tail_us"] if instep else None,
            "parity": parity,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    graph.destroy()
    kv.destroy()
    if split:
        be.comm_destroy()
    be.shutdown()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
