"""Benchmark of the B200 KV-cache hot path (one JSON line on rank 0).

Default workload — batched decode attention, LLaMA-3-8B attention shape:
32 q heads, 8 kv heads, head_dim 128, fp16 cache, 32 layers, 64 sequences
with cached lengths drawn once (seed 20261201) uniform in [512, 32768], K/V
~ N(0,1).  One step = for every layer: fused RoPE+append of each sequence's
new token and split-K decode attention over the grown cache, in one launch
per layer (hx_append_decode_attention; ``--separate``: K1 then K2 as two
launches), i.e. one decode token for each of the 64 sequences.  Metric:
aggregate decode tok/s; the decode kernel's achieved HBM GB/s is in
``roofline``.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--collective p2p|nccl] [--separate] [--no-overlap] [--no-cpu-baseline]
                  [--no-c1-32k]

At N=1 the same JSON line also carries ``c1_32k``: batch-1 decode on the
Qwen2.5-7B attention shape (28 q heads, 4 kv heads, head_dim 128) over
32,769 positions, 28 layers captured in one CUDA graph and timed as
replays, with its microseconds per layer and its fraction of the measured
HBM peak and of 8 TB/s.

Multi-GPU (torchrun, one process per GPU, NCCL): at 8 GPUs each rank holds
one kv head (4 q heads) of every sequence; at 2 or 4 GPUs each rank holds a
length-balanced subset of the sequences with all 8 kv heads.  After every
layer the per-rank attention outputs are gathered: by default the decode
kernels store every output row straight into every rank's output buffer over
NVLink peer memory, then the ranks exchange an epoch flag
(``--collective p2p``); with ``--collective nccl`` an NCCL all-gather follows
each decode call.

``--impl reference`` times the reference's CPU attention algorithm (the
oracle restatement of hxinfer-engine/src/layer/attention.cpp:49-85 with the
GQA mapping of attention_score_cuda.cu:20-21; the reference's own CPU layer
is MHA-only) on a bounded sample of the same workload, scaled to the full
step, on rank 0; other ranks exit.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SEED = 20261201
HQ, HKV, HD, LAYERS, NSEQ = 32, 8, 128, 32, 64
# Layers whose decode call is bracketed by CUDA events in the timed steps.
EVENT_STRIDE = 4
# One metric string for both arms, so the two lines can be compared directly.
METRIC = "decode tok/s (batched decode attention)"
# DRAM bytes (read + write) of one decode launch / its algorithmic bytes,
# from an ncu capture of the same kernel on 16 sequences x 8192 positions
# (541.6 MB of DRAM traffic for 537.1 MB of K+V+q+out); the traffic of the
# bench's 4.4 GB launches scales with the tiles read, so `roofline.traffic`
# is this ratio times the launch's algorithmic bytes.
DECODE_TRAFFIC_RATIO = 1.008


def lengths_c4():
    return np.random.default_rng(SEED).integers(512, 32769, NSEQ).astype(np.int64)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ------------------------------------------------------------------ partitioning

def partition(world: int, rank: int, lengths):
    """(mode, seq indices, kv-head indices, padded rows) for this rank; every
    rank's output block is padded to the largest shard's row count so the
    all-gather is uniform."""
    from hxinfer_b200.dist import plan
    mode, shards = plan(world, HKV, lengths)
    seqs, heads = shards[rank]
    return mode, seqs, heads, max(len(s) for s, _ in shards)


# ------------------------------------------------------------------ clocks

class ClockSampler:
    def __init__(self, uuids):
        self.uuids = set(uuids)
        self.proc = None
        self.path = None
        self.out = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        self.out = open(self.path, "w")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=uuid,clocks.sm,clocks.max.sm,power.draw,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.out, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait()
        if self.out:
            self.out.close()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            for line in open(self.path):
                f = [x.strip() for x in line.split(",")]
                if len(f) < 8 or (self.uuids and f[0] not in self.uuids):
                    continue
                try:
                    sm.append(float(f[1]))
                    mx.append(float(f[2]))
                except ValueError:
                    continue
                for n, v in zip(names, f[4:8]):
                    if v.lower() == "active":
                        reasons.add(n)
            os.unlink(self.path)
        except OSError:
            pass
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ CPU baseline

def cpu_decode_rate(lengths, n_sample_seqs: int, nthreads: int, min_seconds: float = 3.0):
    """Oracle decode attention (reference CPU loop + GQA mapping) on a sample of
    sequences of one layer; returns (tokens/s scaled to the full 32-layer,
    64-sequence step, description)."""
    from oracle import oracle as O
    rng = np.random.default_rng(SEED + 7)
    idx = list(range(n_sample_seqs))
    ks = [O.f16(rng.standard_normal((int(lengths[i]) + 1, HKV * HD))) for i in idx]
    vs = [O.f16(rng.standard_normal((int(lengths[i]) + 1, HKV * HD))) for i in idx]
    q = O.f16(rng.standard_normal((len(idx), HQ * HD)))
    reps, t0 = 0, time.perf_counter()
    while True:
        O.decode_attention_batch(q, ks, vs, HQ, HKV, HD, nthreads=nthreads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    t_sample = el / reps
    sample_pos = sum(int(lengths[i]) + 1 for i in idx)
    full_pos = int(sum(int(x) + 1 for x in lengths))
    t_step = t_sample * (full_pos / sample_pos) * LAYERS
    desc = (f"{len(idx)} of {len(lengths)} sequences ({sample_pos} positions), 1 of {LAYERS} "
            f"layers, {reps} reps; scaled by positions x layers to the full step")
    return len(lengths) / t_step, desc, t_sample


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    lengths = lengths_c4()
    nthreads = os.cpu_count() or 1
    rates = []
    for _ in range(args.warmup):
        cpu_decode_rate(lengths, 2, nthreads, min_seconds=0.0)
    descs = ""
    sample_s = []
    for _ in range(args.steps):
        r, descs, t_sample = cpu_decode_rate(lengths, 2, nthreads, min_seconds=1.0)
        rates.append(r)
        sample_s.append(t_sample)
    val = statistics.median(rates)
    med_sample = statistics.median(sample_s)
    line = {"impl": "reference", "metric": METRIC,
            "value": val, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup,
            # extrapolated: one sample covers 2 of the 64 sequences of 1 of the
            # 32 layers; the time actually measured per sample is sample_ms
            "ms_per_step": 1000.0 * NSEQ / val, "ms_per_step_kind": "extrapolated from sample_ms",
            "sample_ms": 1000.0 * med_sample,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic N(0,1) K/V rounded to fp16",
            "config": {"workload": "batched_decode_llama3_8b_attention", "layers": LAYERS,
                       "q_heads": HQ, "kv_heads": HKV, "head_dim": HD, "sequences": NSEQ,
                       "lengths": "U[512,32768] seed 20261201"},
            "cpu_baseline": {"value": val, "unit": "tok/s", "cores": nthreads, "kind": "port",
                             "sample": descs, "sample_ms": 1000.0 * med_sample},
            "e2e": {"value": val, "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm

def run_batched_decode(args):
    import torch
    import torch.distributed as dist

    from hxinfer_b200 import kv

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    lengths = lengths_c4()
    mode, seqs, heads, n_pad = partition(world, rank, lengths)
    hkv = len(heads)
    hq = hkv * (HQ // HKV)
    n = len(seqs)
    W, K = args.warmup, args.steps
    extra = W + 2 * K + 2
    my_len = np.array([int(lengths[s]) for s in seqs], np.int64)
    cap = int(my_len.max()) + extra
    nblocks = int(sum(math.ceil((int(L) + extra) / 64) for L in my_len))
    cache = kv.KVCache(LAYERS, hkv, HD, n, cap, num_blocks=nblocks, overlap=args.overlap)
    for i, L in enumerate(my_len):
        cache.reserve(i, int(L) + extra)
    cache.fill_normal(SEED + 1000 * rank)
    table = kv.RopeTable(HD, cap, 5e5)

    g = torch.Generator(device=dev)
    g.manual_seed(SEED + rank)
    q_in = torch.randn((LAYERS, n, hq * HD), generator=g, device=dev).half()
    k_in = torch.randn((LAYERS, n, hkv * HD), generator=g, device=dev).half()
    v_in = torch.randn((LAYERS, n, hkv * HD), generator=g, device=dev).half()
    q_rot = torch.empty_like(q_in)
    out = torch.zeros((LAYERS, n_pad, hq * HD), dtype=torch.float16, device=dev)
    p2p = world > 1 and args.collective == "p2p"
    gathered = torch.empty((LAYERS, world, n_pad, hq * HD), dtype=torch.float16, device=dev) \
        if world > 1 and not p2p else None
    peer = None
    if p2p:
        # every rank's decode stores its rows straight into every rank's
        # [2][LAYERS][NSEQ][HQ*HD] buffer (reference output layout, no
        # assembly); steps alternate between the two halves, so a rank writes
        # a half again only after every rank has read it back (the step in
        # between ends with an epoch exchange that follows that read)
        def exchange(blob):
            allb = [None] * world
            dist.all_gather_object(allb, blob)
            return allb
        layer_bytes = NSEQ * HQ * HD * 2
        peer = kv.PeerGather(rank, world, 2 * LAYERS * layer_bytes, exchange)
        assembled = peer.view(torch.float16, shape=(2, LAYERS, NSEQ, HQ * HD))
        out_rows = torch.tensor(seqs, dtype=torch.int32, device=dev)
        head0 = heads[0] * (HQ // HKV)
        epoch = [0]
        # Each layer's epoch exchange waits on a side stream, so the next
        # layer's append and decode stream HBM while this layer's rows drain
        # to the peers; a step ends when its last exchange has completed.
        side = torch.cuda.Stream()

    def attend(l, si, q, k, v, timed_events=False, out_buf=None):
        """One layer of a decode step: the new tokens' RoPE + append and the
        decode attention, in one launch (hx_append_decode_attention), or with
        --separate as K1 then K2 (hx_rope_append, hx_decode_attention).
        Without the gather the rows go to out_buf (default `out`)."""
        pos, lens = pos_tab[si], len_tab[si]
        o = out if out_buf is None else out_buf
        if args.separate:
            cache.rope_append(l, k, v, seq_ids, pos, q=q, num_q_heads=hq, table=table,
                              q_out=q_rot[l])
        if timed_events:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        if p2p:
            epoch[0] += 1
            place = dict(out_offset=((si % 2) * LAYERS + l) * layer_bytes, out_rows=out_rows,
                         out_row_heads=HQ, out_head0=head0, workspace=ws)
            if args.separate:
                cache.decode_gather(l, q_rot[l], seq_ids, lens, hq, peer, **place)
            else:
                cache.append_decode_gather(l, q, k, v, seq_ids, lens, hq, peer, table=table, **place)
        elif args.separate:
            cache.decode(l, q_rot[l], seq_ids, lens, hq, out=o[l], workspace=ws)
        else:
            cache.append_decode(l, q, k, v, seq_ids, lens, hq, table=table, out=o[l],
                                workspace=ws)
        if timed_events:
            e1.record(stream)
            ev_pairs.append((e0, e1))
        if p2p:
            done = torch.cuda.Event()
            done.record(stream)
            side.wait_event(done)
            peer.wait(epoch[0], stream=side)
        elif world > 1:
            dist.all_gather_into_tensor(gathered[l], o[l])
    seq_ids = torch.arange(n, dtype=torch.int32, device=dev)
    total_steps = W + 2 * K
    base = torch.from_numpy(my_len.astype(np.int32)).to(dev)
    pos_tab = torch.stack([base + s for s in range(total_steps)])  # append position per step
    len_tab = pos_tab + 1
    ws = torch.zeros(cache.workspace_bytes(n, hq), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    ev_pairs = []

    def step(si, timed_events=False):
        # The roofline's launch time comes from CUDA events around the decode
        # call of every EVENT_STRIDE-th layer of the timed steps (all layers
        # do the same work): an event record between two launches also ends
        # their programmatic overlap, so fewer of them disturb the step less.
        for l in range(LAYERS):
            attend(l, si, q_in[l], k_in[l], v_in[l], timed_events and l % EVENT_STRIDE == 0)
        if p2p:
            stream.wait_stream(side)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for s in range(W):
        step(s)
    barrier()
    kv.device_status()

    uuids = []
    try:
        uuids = ["GPU-" + str(torch.cuda.get_device_properties(local).uuid)]
    except Exception:
        pass
    if world > 1:
        allu = [None] * world
        dist.all_gather_object(allu, uuids)
        uuids = [u for x in allu for u in x]
    sampler = ClockSampler(uuids) if rank == 0 else None
    if sampler:
        sampler.__enter__()
    barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for s in range(W, W + K):
        step(s, timed_events=True)
    t1.record(stream)
    barrier()
    if sampler:
        sampler.__exit__()
    ms = max_over_ranks(t0.elapsed_time(t1))
    kv.device_status()
    dec_ms = [a.elapsed_time(b) for a, b in ev_pairs]
    dec_avg_ms = max_over_ranks(sum(dec_ms) / len(dec_ms))

    # algorithmic bytes of one decode call (this rank): K+V read over the
    # grown cache + q read + out write, averaged over the timed steps; the
    # one-launch form also reads the new k and v rows and writes them to the
    # cache
    mean_len = float(np.mean([np.sum(my_len + s + 1) for s in range(W, W + K)]))
    dec_bytes = 2 * mean_len * hkv * HD * 2 + 2 * n * hq * HD * 2
    if not args.separate:
        dec_bytes += 2 * (2 * n * hkv * HD * 2)
    achieved = dec_bytes / (dec_avg_ms * 1e-3) / 1e9
    peak, peak_kind = peaks()

    # ---- end to end: host (pinned) q/k/v in, attention outputs out, every step.
    # Served as a pipeline: device inputs and (without the gather) outputs are
    # double-buffered, and a copy stream uploads step i+1's inputs and reads
    # back step i's outputs while the neighbouring step computes.  With the
    # gather the read-back stays on the compute stream after the step's
    # exchange, since peers write the same gather region again two steps on.
    q_h = q_in.cpu().pin_memory()
    k_h = k_in.cpu().pin_memory()
    v_h = v_in.cpu().pin_memory()
    if p2p:
        # this rank reads back its share of the assembled output rows
        r0, r1 = rank * NSEQ // world, (rank + 1) * NSEQ // world
        out_h = torch.empty((LAYERS, r1 - r0, HQ * HD), dtype=torch.float16).pin_memory()
    else:
        out_h = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    q_d = [torch.empty_like(q_in) for _ in range(2)]
    k_d = [torch.empty_like(k_in) for _ in range(2)]
    v_d = [torch.empty_like(v_in) for _ in range(2)]
    outs = [out, torch.zeros_like(out)]  # padding rows read back as zeros in both
    copy = torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]

    def upload(i):
        """Inputs of the i-th end-to-end step into buffer i % 2 (copy stream),
        once step i - 2 has finished reading that buffer."""
        b = i % 2
        if i >= 2:
            copy.wait_event(ev_done[b])
        with torch.cuda.stream(copy):
            q_d[b].copy_(q_h, non_blocking=True)
            k_d[b].copy_(k_h, non_blocking=True)
            v_d[b].copy_(v_h, non_blocking=True)
        ev_in[b].record(copy)

    def e2e_step(i, si):
        b = i % 2
        stream.wait_event(ev_in[b])
        for l in range(LAYERS):
            attend(l, si, q_d[b][l], k_d[b][l], v_d[b][l], out_buf=outs[b])
        if p2p:
            stream.wait_stream(side)
            out_h.copy_(assembled[si % 2, :, r0:r1], non_blocking=True)
            ev_done[b].record(stream)
        else:
            ev_done[b].record(stream)
            copy.wait_event(ev_done[b])
            with torch.cuda.stream(copy):
                out_h.copy_(outs[b], non_blocking=True)

    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    copy.wait_event(e0)
    upload(0)
    for i, s in enumerate(range(W + K, W + 2 * K)):
        if i + 1 < K:
            upload(i + 1)
        e2e_step(i, s)
    stream.wait_stream(copy)
    e1.record(stream)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    kv.device_status()
    h2d = (q_h.numel() + k_h.numel() + v_h.numel()) * 2
    d2h = out_h.numel() * 2
    if world > 1:
        t = torch.tensor([h2d, d2h], dtype=torch.float64, device=dev)
        dist.all_reduce(t)
        h2d, d2h = int(t[0].item()), int(t[1].item())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        nthreads = os.cpu_count() or 1
        rate, desc, _ = cpu_decode_rate(lengths, 2, nthreads, min_seconds=10.0)
        cpu = {"value": rate, "unit": "tok/s", "cores": nthreads, "kind": "port", "sample": desc}

    clocks = sampler.summary() if sampler else None
    tok_s = NSEQ * K / (ms * 1e-3)
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": tok_s, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16 storage / f32 accumulate", "data": "synthetic",
            "config": {"workload": "batched_decode_llama3_8b_attention", "layers": LAYERS,
                       "q_heads": HQ, "kv_heads": HKV, "head_dim": HD, "sequences": NSEQ,
                       "lengths": "U[512,32768] seed 20261201",
                       "mean_len": float(np.mean(lengths)),
                       "kv_bytes_per_step": float(2 * (lengths.sum() + NSEQ) * HKV * HD * 2 * LAYERS),
                       "parallelism": f"{mode}x{world}",
                       "collective": ("p2p gather fused into the decode kernels" if p2p else
                                      "nccl all_gather_into_tensor" if world > 1 else "none"),
                       "l2": "inputs larger than L2 (KV cache >> 126 MB)",
                       "step": ("K1 then K2, two launches per layer" if args.separate else
                                "RoPE + append + decode in one launch per layer"),
                       "launch": ("programmatic dependent (HX_KV_OVERLAP_LAUNCH)" if args.overlap
                                  else "stream-ordered")},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "kernel": ("decode_attention_kernel (+ decode_combine_kernel when not "
                                    "folded), one hx_decode_attention call" if args.separate else
                                    "decode_attention_kernel with the new tokens' RoPE + append "
                                    "(+ decode_combine_kernel when not folded), one "
                                    "hx_append_decode_attention call"),
                         "bytes_per_launch": dec_bytes, "avg_launch_ms": dec_avg_ms,
                         "traffic": DECODE_TRAFFIC_RATIO * dec_bytes,
                         "traffic_source": "ncu dram__bytes_read+write, 16x8192 capture, "
                                           "scaled by tiles read"},
            "hbm_gbs_step": float(2 * (lengths.sum() + NSEQ) * HKV * HD * 2 * LAYERS) / (ms / K * 1e-3) / 1e9,
            "cpu_baseline": cpu,
            "e2e": {"value": NSEQ * K / (e2e_ms * 1e-3), "unit": "tok/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "copies": ("pinned host buffers; uploads " + ("and read-backs " if not p2p else "")
                               + "on a second stream, double-buffered, overlapping the "
                               "neighbouring step's compute")},
            "gpu_launches": K * LAYERS * ((1 if args.separate else 0)
                                          + kv.decode_kernel_count(n * hkv, HD, HQ // HKV)
                                          + (1 if p2p else 0)),
            "clocks": clocks,
        }
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()  # no rank unmaps its buffer while a peer may still write it
    if peer is not None:
        peer.close()
    cache.close()
    table.close()
    if rank == 0:
        if world == 1 and not args.no_c1_32k:
            del q_in, k_in, v_in, q_rot, out, q_d, k_d, v_d
            torch.cuda.empty_cache()
            line["c1_32k"] = run_c1_32k(args)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_c1_32k(args, layers: int = 28, ctx: int = 32768, replays: int = 50):
    """Batch-1 decode on the Qwen2.5-7B attention shape (28 q heads, 4 kv
    heads, head_dim 128, RoPE theta 1e6): one new token appended at position
    32768 and attended over 32,769 positions, for each of 28 layers.  The 28
    layers are captured in one CUDA graph and timed as replays with CUDA
    events; `decode_us_per_layer` is the decode call alone (q already
    rotated), `step_us_per_layer` adds the RoPE + append launch in front of
    it, and `one_launch_step_us_per_layer` is the whole step as one
    hx_append_decode_attention launch per layer.  The 28
    layers hold 1.88 GB of K/V, so no layer's 67 MB is still in L2 when it
    is read again."""
    import torch

    from hxinfer_b200 import kv

    hq, hkv = 28, 4
    dev = torch.device("cuda", torch.cuda.current_device())
    cap = ctx + 1
    cache = kv.KVCache(layers, hkv, HD, 1, cap, overlap=True)
    cache.reserve(0, cap)
    cache.fill_normal(SEED + 32)
    table = kv.RopeTable(HD, cap, 1e6)
    g = torch.Generator(device=dev)
    g.manual_seed(SEED + 33)
    q = torch.randn((layers, 1, hq * HD), generator=g, device=dev).half()
    k = torch.randn((layers, 1, hkv * HD), generator=g, device=dev).half()
    v = torch.randn((layers, 1, hkv * HD), generator=g, device=dev).half()
    q_rot = torch.empty_like(q)
    out = torch.empty_like(q)
    sid = torch.zeros(1, dtype=torch.int32, device=dev)
    pos = torch.full((1,), ctx, dtype=torch.int32, device=dev)
    lens = pos + 1
    ws = torch.zeros(cache.workspace_bytes(1, hq), dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream()

    def step(mode):
        for l in range(layers):
            if mode == "one_launch":
                cache.append_decode(l, q[l], k[l], v[l], sid, lens, hq, table=table, out=out[l],
                                    workspace=ws, stream=stream)
                continue
            if mode == "step":
                cache.rope_append(l, k[l], v[l], sid, pos, q=q[l], num_q_heads=hq, table=table,
                                  q_out=q_rot[l], stream=stream)
            cache.decode(l, q_rot[l], sid, lens, hq, out=out[l], workspace=ws, stream=stream)

    res = {}
    with torch.cuda.stream(stream):
        step("step")  # kernel attributes are set outside the capture
        step("one_launch")
        torch.cuda.synchronize()
        for name, app in (("decode", "decode"), ("step", "step"), ("one_launch", "one_launch")):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                step(app)
            for _ in range(3):
                graph.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(replays):
                graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            res[name] = 1e3 * e0.elapsed_time(e1) / (replays * layers)
            del graph
    kv.device_status()
    cache.close()
    table.close()
    kv_bytes = 2 * (ctx + 1) * hkv * HD * 2
    dec_bytes = kv_bytes + 2 * hq * HD * 2                  # + q read, out write
    step_bytes = dec_bytes + 2 * hkv * HD * 2 * 2 + hq * HD * 2 * 2  # + k/v in, row out, q in/out
    peak, peak_kind = peaks()
    dec_gbs = dec_bytes / (res["decode"] * 1e-6) / 1e9
    return {"workload": "qwen2.5-7b attention, batch 1, 32769 positions, 28 layers, CUDA graph",
            "decode_us_per_layer": res["decode"], "step_us_per_layer": res["step"],
            "one_launch_step_us_per_layer": res["one_launch"],
            "decode_bytes_per_layer": dec_bytes, "step_bytes_per_layer": step_bytes,
            "decode_gbs": dec_gbs, "frac_measured_peak": dec_gbs / peak, "peak_kind": peak_kind,
            "frac_8tbs": dec_gbs / 8000.0,
            "target_us_per_layer": dec_bytes / (0.75 * 8000e9) * 1e6,
            "step_gbs": step_bytes / (res["step"] * 1e-6) / 1e9,
            "one_launch_step_gbs": step_bytes / (res["one_launch"] * 1e-6) / 1e9,
            "replays": replays, "launch": "programmatic dependent (HX_KV_OVERLAP_LAUNCH)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-c1-32k", action="store_true",
                    help="skip the batch-1 Qwen 32k decode sub-record (N=1 only)")
    ap.add_argument("--separate", action="store_true",
                    help="K1 and K2 as two launches per layer (hx_rope_append then "
                         "hx_decode_attention) instead of hx_append_decode_attention")
    ap.add_argument("--overlap", dest="overlap", action="store_true", default=True,
                    help="launch the decode kernels as programmatic dependents "
                         "(HX_KV_OVERLAP_LAUNCH; the default)")
    ap.add_argument("--no-overlap", dest="overlap", action="store_false",
                    help="plain stream-ordered launches")
    ap.add_argument("--collective", default="p2p", choices=["p2p", "nccl"],
                    help="N>1: gather fused into the decode kernels over NVLink peer memory "
                         "(p2p) or an NCCL all-gather after each decode call (nccl)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
        return
    run_batched_decode(args)


if __name__ == "__main__":
    main()
