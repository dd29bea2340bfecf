"""Small, self-contained cases of the hot-path kernels, sized for profiling.

    python -m hxinfer_b200.profile_case decode  --shape llama3 --seqs 16 --len 8192 --layers 1 --iters 5
    python -m hxinfer_b200.profile_case decode  --shape qwen   --seqs 1  --len 32769 --layers 28 --iters 20
    python -m hxinfer_b200.profile_case decode  --shape llama3_kvhead --seqs 64 --len 16874 --layers 8 --iters 20
    python -m hxinfer_b200.profile_case decode  --shape llama3_kvhead --seqs 64 --ragged --layers 8 --iters 20 --overlap --gather
    python -m hxinfer_b200.profile_case snapshot --shape qwen  --len 2048 --layers 28 --iters 20
    python -m hxinfer_b200.profile_case prefill --shape llama2 --len 1024 --layers 4 --iters 5
    python -m hxinfer_b200.profile_case c2 --len 1024 --steps 1024 --layers 1
    python -m hxinfer_b200.profile_case c5 --len 2048 --new 256 --steps 128 --layers 28 --conts 32
    python -m hxinfer_b200.profile_case qkv --shape qwen --seqs 1 --layers 28 --iters 20
    python -m hxinfer_b200.profile_case convert --mib 1024 --iters 10
    torchrun --nproc-per-node 8 -m hxinfer_b200.profile_case oproj --seqs 64 --iters 50

Each case fills a cache with N(0,1) fp16, runs the kernels `iters` times and
prints one JSON line with the CUDA-event time per iteration and the
algorithmic bytes, so the same command serves a timing check and an ncu
capture (keep the device footprint to a few GB: inputs larger than the
126 MB L2, small enough for ncu's memory save/restore between passes).
"""
from __future__ import annotations

import argparse
import json
import math

import torch

from . import kv

# (q heads, kv heads, rope theta); llama3_kvhead is one rank's shard of the
# LLaMA-3 attention when 8 ranks split the kv heads (one kv head, 4 q heads)
SHAPES = {"llama3": (32, 8, 5e5), "qwen": (28, 4, 1e6), "llama2": (32, 32, 1e4),
          "llama3_kvhead": (4, 1, 5e5)}


def decode_case(a):
    """Decode steps over `layers` layers, timed as CUDA-graph replays (so the
    host's launch rate does not limit small cases): per layer the fused
    RoPE+append (K1) then the split-K decode (K2); also K2 alone."""
    hq, hkv, theta = SHAPES[a.shape]
    hd, n, L, layers = 128, a.seqs, a.len, a.layers
    if a.ragged:  # the batched decode workload's lengths: U[512, 32768], seed 20261201
        import numpy as np
        lens_h = np.random.default_rng(20261201).integers(512, 32769, n).astype(np.int64)
        L = int(lens_h.max())
    cap = L + 2
    cache = kv.KVCache(layers, hkv, hd, n, cap, overlap=a.overlap)
    for s in range(n):
        cache.reserve(s, cap)
    cache.fill_normal(7)
    table = kv.RopeTable(hd, cap, theta)
    g = torch.Generator(device="cuda")
    g.manual_seed(1)
    q = torch.randn((layers, n, hq * hd), generator=g, device="cuda").half()
    k = torch.randn((layers, n, hkv * hd), generator=g, device="cuda").half()
    v = torch.randn((layers, n, hkv * hd), generator=g, device="cuda").half()
    q_rot = torch.empty_like(q)
    out = torch.empty_like(q)
    sid = torch.arange(n, dtype=torch.int32, device="cuda")
    ws = torch.zeros(cache.workspace_bytes(n, hq), dtype=torch.uint8, device="cuda")
    if a.ragged:
        lens = torch.tensor(lens_h, dtype=torch.int32, device="cuda")
        pos = lens - 1
    else:
        pos = torch.full((n,), L - 1, dtype=torch.int32, device="cuda")
        lens = pos + 1
    stream = torch.cuda.Stream()

    gather = None
    if a.gather:
        # a one-rank gather endpoint: the gathering kernels store the rows into
        # this rank's own buffer, which isolates their cost from the exchange
        row_bytes = hq * hd * 2
        gather = kv.PeerGather(0, 1, 2 * n * row_bytes, lambda b: [b])
        g_rows = torch.arange(n, dtype=torch.int32, device="cuda")

    def step(with_append):
        for l in range(layers):
            if with_append == "one_launch_gather":
                cache.append_decode_gather(l, q[l], k[l], v[l], sid, lens, hq, gather,
                                           out_offset=(l & 1) * n * row_bytes, out_rows=g_rows,
                                           out_row_heads=hq, out_head0=0, table=table,
                                           workspace=ws, stream=stream)
                continue
            if with_append == "one_launch":
                cache.append_decode(l, q[l], k[l], v[l], sid, lens, hq, table=table, out=out[l],
                                    workspace=ws, stream=stream)
                continue
            if with_append:
                cache.rope_append(l, k[l], v[l], sid, pos, q=q[l], num_q_heads=hq, table=table,
                                  q_out=q_rot[l], stream=stream)
            cache.decode(l, q_rot[l], sid, lens, hq, out=out[l], workspace=ws, stream=stream)

    res = {}
    with torch.cuda.stream(stream):
        step(True)  # warm-up (sets kernel attributes outside capture)
        step("one_launch")
        if gather is not None:
            step("one_launch_gather")
        torch.cuda.synchronize()
        kinds = [("step", True), ("decode_only", False), ("one_launch", "one_launch")]
        if gather is not None:
            kinds.append(("one_launch_gather", "one_launch_gather"))
        for name, app in kinds:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                step(app)
            graph.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(a.iters):
                graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            res[name] = e0.elapsed_time(e1) / (a.iters * layers)
    kv.device_status()
    if gather is not None:
        gather.close()
    nbytes = 2 * int(lens.sum().item()) * hkv * hd * 2
    print(json.dumps({"case": "decode", "shape": a.shape, "seqs": n,
                      "len": "U[512,32768]" if a.ragged else L, "layers": layers,
                      "overlap": a.overlap,
                      "graph_us_per_layer_step": 1e3 * res["step"],
                      "graph_us_per_layer_decode": 1e3 * res["decode_only"],
                      "graph_us_per_layer_one_launch_step": 1e3 * res["one_launch"],
                      "graph_us_per_layer_one_launch_gather_world1":
                          1e3 * res["one_launch_gather"] if gather is not None else None,
                      "bytes_per_launch": nbytes,
                      "decode_gbs": nbytes / (res["decode_only"] * 1e-3) / 1e9,
                      "step_gbs": nbytes / (res["step"] * 1e-3) / 1e9}))


def snapshot_case(a):
    hq, hkv, _ = SHAPES[a.shape]
    hd, L, layers = 128, a.len, a.layers
    cache = kv.KVCache(layers, hkv, hd, 2, L)
    cache.reserve(0, L)
    cache.reserve(1, L)
    cache.fill_normal(3)
    snap = torch.empty(cache.snapshot_bytes(L), dtype=torch.uint8, device="cuda")
    ts, tr = [], []
    for _ in range(a.iters):
        e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        e[0].record()
        cache.snapshot(0, L, snap)
        e[1].record()
        cache.restore(1, L, snap)
        e[2].record()
        ts.append(e)
    torch.cuda.synchronize()
    kv.device_status()
    snap_ms = sum(x[0].elapsed_time(x[1]) for x in ts[1:]) / max(1, len(ts) - 1)
    rest_ms = sum(x[1].elapsed_time(x[2]) for x in ts[1:]) / max(1, len(ts) - 1)
    payload = cache.snapshot_bytes(L)
    print(json.dumps({"case": "snapshot", "shape": a.shape, "len": L, "layers": layers,
                      "payload_bytes": payload, "snapshot_ms": snap_ms, "restore_ms": rest_ms,
                      "snapshot_payload_gbs": payload / (snap_ms * 1e-3) / 1e9,
                      "restore_payload_gbs": payload / (rest_ms * 1e-3) / 1e9}))


def prefill_case(a):
    """Causal prefill of `len` fresh tokens (start 0), all q heads of the shape.
    The `layers` x `iters` launches are captured in one CUDA graph and timed
    as replays (CUDA events around the replays), so the host's launch time
    between launches is not counted."""
    hq, hkv, theta = SHAPES[a.shape]
    hd, n = 128, a.len
    cache = kv.KVCache(a.layers, hkv, hd, 1, n + a.start)
    cache.reserve(0, n + a.start)
    cache.fill_normal(11)
    g = torch.Generator(device="cuda")
    g.manual_seed(2)
    q = torch.randn((n, hq * hd), generator=g, device="cuda").half()
    out = torch.empty_like(q)
    for l in range(a.layers):  # warm-up, outside the graph
        cache.prefill(l, q, 0, a.start, hq, out=out)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for it in range(a.iters):
            for l in range(a.layers):
                cache.prefill(l, q, 0, a.start, hq, out=out)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    kv.device_status()
    avg = e0.elapsed_time(e1) / (reps * a.iters * a.layers)
    # unmasked (query, key) pairs x 4 flops per pair per dim
    pairs = sum(a.start + i + 1 for i in range(n))
    flops = 4.0 * hq * hd * pairs
    print(json.dumps({"case": "prefill", "shape": a.shape, "len": n, "start": a.start,
                      "layers": a.layers, "timing": "cuda graph", "prefill_ms_avg": avg,
                      "flops_per_launch": flops, "tflops": flops / (avg * 1e-3) / 1e12}))


def c2_case(a):
    """LLaMA-2-7B MHA shape (32 q = 32 kv heads, theta 1e4), batch 1: K1 appends
    a 1024-token prompt, K3 prefills it, then 1024 decode steps each append one
    token (K1) and attend over the grown cache (K2).  The decode steps are
    captured once in a CUDA graph (every step's positions baked in) and timed
    as replays, so host launch time is not counted."""
    hq = hkv = 32
    hd, n0, steps, layers = 128, a.len, a.steps, a.layers
    cap = n0 + steps
    cache = kv.KVCache(layers, hkv, hd, 1, cap)
    cache.reserve(0, cap)
    table = kv.RopeTable(hd, cap, 1e4)
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    dev = torch.device("cuda")
    qp = torch.randn((n0, hq * hd), generator=g, device=dev).half()
    kp = torch.randn((n0, hkv * hd), generator=g, device=dev).half()
    vp = torch.randn((n0, hkv * hd), generator=g, device=dev).half()
    qd = torch.randn((steps, 1, hq * hd), generator=g, device=dev).half()
    kd = torch.randn((steps, 1, hkv * hd), generator=g, device=dev).half()
    vd = torch.randn((steps, 1, hkv * hd), generator=g, device=dev).half()
    q_rot = torch.empty_like(qp)
    qd_rot = torch.empty_like(qd)
    out_p = torch.empty_like(qp)
    out_d = torch.empty_like(qd)
    sid0 = torch.zeros(n0, dtype=torch.int32, device=dev)
    pos0 = torch.arange(n0, dtype=torch.int32, device=dev)
    sid = torch.zeros(1, dtype=torch.int32, device=dev)
    pos_tab = torch.arange(n0, n0 + steps, dtype=torch.int32, device=dev).view(steps, 1)
    len_tab = pos_tab + 1
    ws = torch.zeros(cache.workspace_bytes(1, hq), dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream()

    def prefill():
        for l in range(layers):
            cache.rope_append(l, kp, vp, sid0, pos0, q=qp, num_q_heads=hq, table=table,
                              q_out=q_rot, stream=stream)
            cache.prefill(l, q_rot, 0, 0, hq, out=out_p, stream=stream)

    def decode_all():
        for t in range(steps):
            for l in range(layers):
                cache.rope_append(l, kd[t], vd[t], sid, pos_tab[t], q=qd[t], num_q_heads=hq,
                                  table=table, q_out=qd_rot[t], stream=stream)
                cache.decode(l, qd_rot[t], sid, len_tab[t], hq, out=out_d[t], workspace=ws,
                             stream=stream)

    def decode_all_one_launch():  # the same steps, one hx_append_decode_attention each
        for t in range(steps):
            for l in range(layers):
                cache.append_decode(l, qd[t], kd[t], vd[t], sid, len_tab[t], hq, table=table,
                                    out=out_d[t], workspace=ws, stream=stream)

    with torch.cuda.stream(stream):
        prefill()
        decode_all()  # warm-up, sets kernel attributes outside capture
        decode_all_one_launch()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            decode_all()
        graph1 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph1, stream=stream):
            decode_all_one_launch()
        e = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
        e[0].record(stream)
        prefill()
        e[1].record(stream)
        graph.replay()
        e[2].record(stream)
        graph.replay()
        e[3].record(stream)
        graph1.replay()
        e[4].record(stream)
        graph1.replay()
        e[5].record(stream)
        torch.cuda.synchronize()
    kv.device_status()
    pre_ms = e[0].elapsed_time(e[1])
    dec_ms = e[2].elapsed_time(e[3])
    dec1_ms = e[4].elapsed_time(e[5])
    pairs = n0 * (n0 + 1) // 2
    pre_flops = 4.0 * hq * hd * pairs * layers
    dec_bytes = 2.0 * hkv * hd * 2 * sum(range(n0 + 1, n0 + steps + 1)) * layers
    print(json.dumps({"case": "c2", "shape": "llama2", "prompt": n0, "decode_steps": steps,
                      "layers": layers, "prefill_ms": pre_ms,
                      "prefill_tflops_incl_append": pre_flops / (pre_ms * 1e-3) / 1e12,
                      "decode_ms": dec_ms, "decode_us_per_step_layer": 1e3 * dec_ms / (steps * layers),
                      "one_launch_decode_us_per_step_layer": 1e3 * dec1_ms / (steps * layers),
                      "decode_kv_bytes": dec_bytes,
                      "decode_gbs": dec_bytes / (dec_ms * 1e-3) / 1e9}))


def c5_case(a):
    """Prefix-cache reuse on the Qwen2.5-7B attention shape (28 layers, 28 q /
    4 kv heads, theta 1e6), attention-layer level (q/k/v are synthetic; the
    projections and the rest of the model are not run).  A `prefix`-token
    prompt is appended (K1) and prefilled (K3) once on sequence 0 and
    snapshotted (K4).  Each of `conts` continuations then restores the
    snapshot into sequence 1, appends and prefills `new` tokens at positions
    prefix .. prefix+new-1, and decodes `steps` tokens (K1 + K2 per layer, one
    CUDA graph).  The alternative recomputes: sequence 2 appends and prefills
    all prefix+new tokens from position 0, then decodes the same steps."""
    hq, hkv, theta = 28, 4, 1e6
    hd, layers, P, NP, ND, NC = 128, a.layers, a.len, a.new, a.steps, a.conts
    cap = P + NP + ND
    dev = torch.device("cuda")
    cache = kv.KVCache(layers, hkv, hd, 3, cap)
    for s in range(3):
        cache.reserve(s, cap)
    table = kv.RopeTable(hd, cap, theta)
    g = torch.Generator(device="cuda")
    g.manual_seed(9)

    def rnd(*shape):
        return torch.randn(shape, generator=g, device=dev).half()

    qp, kp, vp = rnd(P + NP, hq * hd), rnd(P + NP, hkv * hd), rnd(P + NP, hkv * hd)
    qd, kd, vd = rnd(ND, 1, hq * hd), rnd(ND, 1, hkv * hd), rnd(ND, 1, hkv * hd)
    q_rot = torch.empty_like(qp)
    out_p = torch.empty_like(qp)
    qd_rot = torch.empty_like(qd)
    out_d = torch.empty_like(qd)
    ws = torch.zeros(cache.workspace_bytes(1, hq), dtype=torch.uint8, device=dev)
    snap = torch.empty(cache.snapshot_bytes(P), dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream()
    sid = {s: torch.full((P + NP,), s, dtype=torch.int32, device=dev) for s in range(3)}
    pos_all = torch.arange(P + NP, dtype=torch.int32, device=dev)

    def prefill(seq, start, n):
        sl = slice(start, start + n)
        for l in range(layers):
            cache.rope_append(l, kp[sl], vp[sl], sid[seq][:n], pos_all[sl], q=qp[sl], num_q_heads=hq,
                              table=table, q_out=q_rot[sl], stream=stream)
            cache.prefill(l, q_rot[sl], seq, start, hq, out=out_p[sl], stream=stream)

    dpos = torch.arange(P + NP, cap, dtype=torch.int32, device=dev).view(ND, 1)
    dlen = dpos + 1

    def decode(seq):
        s1 = sid[seq][:1]
        for t in range(ND):
            for l in range(layers):
                cache.rope_append(l, kd[t], vd[t], s1, dpos[t], q=qd[t], num_q_heads=hq,
                                  table=table, q_out=qd_rot[t], stream=stream)
                cache.decode(l, qd_rot[t], s1, dlen[t], hq, out=out_d[t], workspace=ws,
                             stream=stream)

    def ev():
        e = torch.cuda.Event(enable_timing=True)
        e.record(stream)
        return e

    with torch.cuda.stream(stream):
        prefill(0, 0, P)
        cache.snapshot(0, P, snap, stream=stream)
        cache.restore(1, P, snap, stream=stream)
        prefill(1, P, NP)
        prefill(2, 0, P + NP)
        decode(1)  # warm-up outside capture
        torch.cuda.synchronize()
        graphs = {}
        for seq in (1, 2):
            graphs[seq] = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graphs[seq], stream=stream):
                decode(seq)
        # prefix once, then snapshot
        e = [ev()]
        prefill(0, 0, P)
        e.append(ev())
        cache.snapshot(0, P, snap, stream=stream)
        e.append(ev())
        t_restore, t_new, t_dec, t_recompute, t_dec2 = [], [], [], [], []
        for _ in range(NC):
            c = [ev()]
            cache.restore(1, P, snap, stream=stream)
            c.append(ev())
            prefill(1, P, NP)
            c.append(ev())
            graphs[1].replay()
            c.append(ev())
            prefill(2, 0, P + NP)
            c.append(ev())
            graphs[2].replay()
            c.append(ev())
            torch.cuda.synchronize()
            t_restore.append(c[0].elapsed_time(c[1]))
            t_new.append(c[1].elapsed_time(c[2]))
            t_dec.append(c[2].elapsed_time(c[3]))
            t_recompute.append(c[3].elapsed_time(c[4]))
            t_dec2.append(c[4].elapsed_time(c[5]))
        torch.cuda.synchronize()
    kv.device_status()
    med = lambda x: sorted(x)[len(x) // 2]  # noqa: E731
    payload = cache.snapshot_bytes(P)
    reuse_ms = med(t_restore) + med(t_new) + med(t_dec)
    recompute_ms = med(t_recompute) + med(t_dec2)
    toks = NP + ND
    print(json.dumps({
        "case": "c5", "shape": "qwen", "layers": layers, "prefix": P, "new": NP, "decode_steps": ND,
        "continuations": NC, "payload_bytes": payload,
        "prefix_prefill_ms": e[0].elapsed_time(e[1]), "snapshot_ms": e[1].elapsed_time(e[2]),
        "snapshot_payload_gbs": payload / (e[1].elapsed_time(e[2]) * 1e-3) / 1e9,
        "restore_ms": med(t_restore), "restore_payload_gbs": payload / (med(t_restore) * 1e-3) / 1e9,
        "new_prefill_ms": med(t_new), "decode_ms": med(t_dec),
        "reuse_ms_per_continuation": reuse_ms,
        "recompute_prefill_ms": med(t_recompute), "recompute_ms_per_continuation": recompute_ms,
        "reuse_tok_s": toks / (reuse_ms * 1e-3), "recompute_tok_s": toks / (recompute_ms * 1e-3),
        "speedup": recompute_ms / reuse_ms}))
    cache.close()
    table.close()


def qkv_case(a):
    """Decode-step QKV projection of one layer for `seqs` tokens: the fused
    hx_qkv_rope_append against the unfused chain (three cuBLAS GEMMs through
    torch, then K1), both captured in CUDA graphs over `layers` layers so the
    weights (layers x (Hq + 2 Hkv) x 128 x hidden x 2 B) stream from HBM."""
    hq, hkv, theta = SHAPES[a.shape]
    hidden = {"qwen": 3584, "llama3": 4096, "llama2": 4096}[a.shape]
    hd, n, layers = 128, a.seqs, a.layers
    dev = torch.device("cuda")
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    ws = [[(torch.randn((m * hd, hidden), generator=g, device=dev) * 0.02).half()
           for m in (hq, hkv, hkv)] for _ in range(layers)]
    bs = [(torch.randn((m * hd,), generator=g, device=dev) * 0.02).half() for m in (hq, hkv, hkv)]
    x = torch.randn((n, hidden), generator=g, device=dev).half()
    cache = kv.KVCache(layers, hkv, hd, n, 64, overlap=a.overlap)
    for s in range(n):
        cache.reserve(s, 64)
    table = kv.RopeTable(hd, 64, theta)
    sid = torch.arange(n, dtype=torch.int32, device=dev)
    pos = torch.full((n,), 10, dtype=torch.int32, device=dev)
    q_out = torch.empty((n, hq * hd), dtype=torch.float16, device=dev)
    stream = torch.cuda.Stream()

    def fused():
        for l in range(layers):
            cache.qkv_rope_append(l, x, ws[l][0], ws[l][1], ws[l][2], sid, pos, hq, table=table,
                                  bq=bs[0], bk=bs[1], bv=bs[2], q_out=q_out, stream=stream)

    def chain():
        for l in range(layers):
            q = x @ ws[l][0].T
            k = x @ ws[l][1].T
            v = x @ ws[l][2].T
            cache.rope_append(l, k, v, sid, pos, q=q, num_q_heads=hq, table=table, bq=bs[0],
                              bk=bs[1], bv=bs[2], q_out=q_out, stream=stream)

    res = {}
    with torch.cuda.stream(stream):
        for name, fn in (("fused", fused), ("cublas_chain", chain)):
            fn()
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                fn()
            graph.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(a.iters):
                graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            res[name] = 1e3 * e0.elapsed_time(e1) / (a.iters * layers)
    kv.device_status()
    wbytes = (hq + 2 * hkv) * hd * hidden * 2
    print(json.dumps({"case": "qkv", "shape": a.shape, "tokens": n, "layers": layers, "overlap": a.overlap,
                      "weight_bytes_per_layer": wbytes,
                      "fused_us_per_layer": res["fused"], "chain_us_per_layer": res["cublas_chain"],
                      "fused_gbs": wbytes / (res["fused"] * 1e-6) / 1e9,
                      "chain_gbs": wbytes / (res["cublas_chain"] * 1e-6) / 1e9}))


def convert_case(a):
    """Checkpoint dtype conversion on the device (hx_convert): BF16 -> FP16
    in place (the loader's common case; 2 + 2 bytes per element) and
    FP32 -> FP16 out of place (4 + 2 bytes per element), --mib MiB of source."""
    n16 = a.mib * (1 << 20) // 2
    n32 = a.mib * (1 << 20) // 4
    g = torch.Generator(device="cuda").manual_seed(1)
    bf = torch.randn(n16, device="cuda", generator=g).to(torch.bfloat16)
    f32 = torch.randn(n32, device="cuda", generator=g)
    h16 = torch.empty(n32, dtype=torch.float16, device="cuda")
    res = {}
    for name, run, nbytes in (
            ("bf16_to_fp16_inplace", lambda: kv.convert(bf.view(torch.float16), bf), 4 * n16),
            ("fp32_to_fp16", lambda: kv.convert(h16, f32), 6 * n32)):
        run()  # warm-up
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(a.iters + 1)]
        ev[0].record()
        for i in range(a.iters):
            run()
            ev[i + 1].record()
        torch.cuda.synchronize()
        ms = [ev[i].elapsed_time(ev[i + 1]) for i in range(a.iters)]
        best = min(ms)
        res[name] = {"ms_best": best, "ms_mean": sum(ms) / len(ms), "bytes": nbytes,
                     "gbs_best": nbytes / (best * 1e-3) / 1e9}
    kv.device_status()
    print(json.dumps({"case": "convert", "mib": a.mib, **res}))


def oproj_case(a):
    """The output projection after a sharded decode or prefill, two ways, on
    WORLD_SIZE ranks (torchrun, one GPU each), LLaMA-3-8B shape (dim 4096,
    32 q heads).  Each rank holds the attention rows of its q-head slice,
    [rows, 4096 / world].
      replicated:    all-gather the slices (NCCL), then every rank runs the
                     full [rows, 4096] x [4096, 4096]^T projection (the
                     reference's o_proj, attention.cpp:87, after the gather);
                     `replicated_gemm` is its GEMM alone, i.e. the cost when
                     the gather is fused into the decode kernels;
      row-parallel:  each rank multiplies its slice by its [4096, 4096 / world]
                     column block of the weight, then an all-reduce (NCCL)
                     sums the [rows, 4096] partials.
    Each arm runs `layers` layers (weights streamed from HBM) captured in one
    CUDA graph; device time per layer with CUDA events over `iters` replays,
    the max over ranks.  `seqs` rows for a decode step, `len` rows for a
    prefill."""
    import os

    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", torch.cuda.current_device()))
    dev = torch.device("cuda")
    dim, layers = 4096, a.layers
    if dim % world:
        raise ValueError("world must divide 4096")
    sl = dim // world
    g = torch.Generator(device="cuda")
    g.manual_seed(17 + rank)
    res = {}
    for rows in sorted({a.seqs, a.len}):
        w_full = [(torch.randn((dim, dim), generator=g, device=dev) * 0.02).half() for _ in range(layers)]
        w_cols = [w[:, rank * sl:(rank + 1) * sl].contiguous() for w in w_full]
        x_sl = torch.randn((rows, sl), generator=g, device=dev).half()
        x_full = torch.empty((rows, dim), dtype=torch.float16, device=dev)
        gathered = torch.empty((world, rows, sl), dtype=torch.float16, device=dev)
        y = torch.empty((rows, dim), dtype=torch.float16, device=dev)

        def replicated():
            for l in range(layers):
                if world > 1:
                    dist.all_gather_into_tensor(gathered, x_sl)
                    x_full.copy_(gathered.permute(1, 0, 2).reshape(rows, dim))
                else:
                    x_full.copy_(x_sl)
                torch.matmul(x_full, w_full[l].t(), out=y)

        def replicated_gemm():
            for l in range(layers):
                torch.matmul(x_full, w_full[l].t(), out=y)

        def row_parallel():
            for l in range(layers):
                torch.matmul(x_sl, w_cols[l].t(), out=y)
                if world > 1:
                    dist.all_reduce(y)

        for name, fn in (("replicated", replicated), ("replicated_gemm", replicated_gemm),
                         ("row_parallel", row_parallel)):
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                for _ in range(3):
                    fn()
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                fn()
            graph.replay()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(a.iters):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            del graph  # released before the process group (it holds NCCL calls)
            us = torch.tensor([1e3 * e0.elapsed_time(e1) / (a.iters * layers)], device=dev)
            if world > 1:
                dist.all_reduce(us, op=dist.ReduceOp.MAX)
            res[f"{name}_us_rows{rows}"] = us.item()
        del w_full, w_cols
    if rank == 0:
        print(json.dumps({"case": "oproj", "world": world, "dim": dim, "layers": layers,
                          "slice": sl, "timing": "CUDA graph, max over ranks", **res}))
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["decode", "snapshot", "prefill", "c2", "c5", "qkv", "convert", "oproj"])
    ap.add_argument("--mib", type=int, default=1024, help="convert: MiB of source data")
    ap.add_argument("--shape", default="llama3", choices=sorted(SHAPES))
    ap.add_argument("--seqs", type=int, default=16)
    ap.add_argument("--len", type=int, default=8192)
    ap.add_argument("--layers", type=int, default=1)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--start", type=int, default=0)
    ap.add_argument("--steps", type=int, default=1024, help="c2, c5: decode steps after the prompt")
    ap.add_argument("--new", type=int, default=256, help="c5: tokens prefilled after the restored prefix")
    ap.add_argument("--conts", type=int, default=32, help="c5: continuations of the prefix")
    ap.add_argument("--gather", action="store_true",
                    help="decode: also time the gathering one-launch step with a one-rank endpoint")
    ap.add_argument("--ragged", action="store_true",
                    help="decode: lengths U[512, 32768] (seed 20261201), as the batched bench")
    ap.add_argument("--overlap", action="store_true",
                    help="programmatic dependent launch of append -> decode (HX_KV_OVERLAP_LAUNCH)")
    a = ap.parse_args()
    if a.case != "oproj":  # oproj picks LOCAL_RANK's device itself
        torch.cuda.set_device(0)
    {"decode": decode_case, "snapshot": snapshot_case, "prefill": prefill_case,
     "c2": c2_case, "c5": c5_case, "qkv": qkv_case, "convert": convert_case,
     "oproj": oproj_case}[a.case](a)


if __name__ == "__main__":
    main()
