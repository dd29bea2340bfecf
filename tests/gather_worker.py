"""One rank of the multi-GPU gather test (launched by test_gpu_gather.py
through torch.distributed.run, one process per GPU; host exchange over gloo).

For each case every rank builds the same synthetic K/V and q on the host,
loads its shard (hxinfer_b200.dist.plan) into its own cache and runs, over
several steps and layers,
  * hx_decode_attention on its shard (the per-rank result), and
  * hx_decode_attention_gather into every rank's gather buffer + hx_dist_wait.
Checks on every rank:
  * the gathered buffer equals, bit for bit, the per-rank results placed by
    hxinfer_b200.dist.assemble (all ranks' results exchanged on the host);
  * it matches the unsharded decode of the whole cache within the decode
    attention tolerance (max abs 2e-3, max rel 1e-2 of the output scale).
The cases cover sequence and kv-head sharding, a rank without sequences, fp32
output and a call with enough segments for the two-CTAs-per-SM decode shape.
Then, for the same cases, the one-launch step (hx_append_decode_attention_
gather: bias-free RoPE + append of each sequence's newest token, then the
gathering decode) is checked bit for bit against hx_rope_append followed by
hx_decode_attention_gather on a second copy of the shard.
Then rank 0 waits for an epoch that no rank posts: the bounded device wait
must end with HX_ERR_TIMEOUT in the status word and leave the context usable.
Prints "RANK <r> OK" at the end.
"""
from __future__ import annotations

import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from hxinfer_b200 import kv  # noqa: E402
from hxinfer_b200 import dist as hxdist  # noqa: E402
from hxinfer_b200._lib import HX_ERR_TIMEOUT, HXError  # noqa: E402

HD = 128
LAYERS = 2
STEPS = 3

# (name, q heads, kv heads, lengths, output dtype)
CASES = [
    ("sequences", 8, 4, [700, 1, 129, 4096, 64, 2000, 333], torch.float16),
    ("kv_heads", 4, 2, [1500, 65, 3000, 17], torch.float16),
    ("one_sequence", 8, 4, [2500], torch.float32),  # the other ranks hold no sequence
    # >= 64 (sequence, kv head) segments per rank: the two-CTAs-per-SM decode shape
    ("many_segments", 16, 4, [int(x) for x in np.random.default_rng(9).integers(1, 1500, 40)],
     torch.float16),
]


def exchange_fn(world):
    def exchange(blob):
        out = [None] * world
        dist.all_gather_object(out, blob)
        return out
    return exchange


def run_case(rank, world, dev, name, hq, hkv, lengths, out_dtype):
    n_all = len(lengths)
    group = hq // hkv
    mode, shards = hxdist.plan(world, hkv, lengths)
    seqs, heads = shards[rank]
    n = len(seqs)
    cap = max(lengths) + 1
    g = torch.Generator().manual_seed(1234 + n_all)
    K = [[torch.randn((L, hkv * HD), generator=g).half() for L in lengths] for _ in range(LAYERS)]
    V = [[torch.randn((L, hkv * HD), generator=g).half() for L in lengths] for _ in range(LAYERS)]
    Q = torch.randn((LAYERS, n_all, hq * HD), generator=g).half()

    def cols(t, hs, width):  # columns of kv/q heads hs, each `width` wide
        return torch.cat([t[..., h * width:(h + 1) * width] for h in hs], dim=-1)

    # this rank's shard
    cache = kv.KVCache(LAYERS, len(heads), HD, max(n, 1), cap)
    for i, s in enumerate(seqs):
        cache.reserve(i, lengths[s])
        for l in range(LAYERS):
            cache.write(l, i, 0, cols(K[l][s], heads, HD).contiguous().to(dev),
                        cols(V[l][s], heads, HD).contiguous().to(dev))
    qh = [h * group + j for h in heads for j in range(group)]
    q_loc = cols(Q[:, seqs], qh, HD).contiguous().to(dev) if n else \
        torch.empty((LAYERS, 0, len(qh) * HD), dtype=torch.float16, device=dev)
    sid = torch.arange(n, dtype=torch.int32, device=dev)
    lens = torch.tensor([lengths[s] for s in seqs], dtype=torch.int32, device=dev)
    rows = torch.tensor(seqs, dtype=torch.int32, device=dev)
    esize = 4 if out_dtype == torch.float32 else 2
    layer_bytes = n_all * hq * HD * esize
    peer = kv.PeerGather(rank, world, LAYERS * layer_bytes, exchange_fn(world))
    ws = torch.zeros(max(cache.workspace_bytes(max(n, 1), len(qh)), 16), dtype=torch.uint8,
                     device=dev)

    plain = []
    epoch = 100 * (CASES.index(next(c for c in CASES if c[0] == name)) + 1)
    for step in range(STEPS):
        for l in range(LAYERS):
            epoch += 1
            cache.decode_gather(l, q_loc[l], sid, lens, len(qh), peer, out_offset=l * layer_bytes,
                                out_rows=rows, out_row_heads=hq, out_head0=heads[0] * group,
                                out_dtype=out_dtype, workspace=ws)
            peer.wait(epoch)
            if step == 0:
                plain.append(cache.decode(l, q_loc[l], sid, lens, len(qh), out_dtype=out_dtype)
                             if n else torch.empty((0, len(qh) * HD), dtype=out_dtype, device=dev))
    kv.device_status()
    got = peer.view(out_dtype, shape=(LAYERS, n_all, hq * HD)).cpu()

    parts = [None] * world
    dist.all_gather_object(parts, [p.cpu().numpy() for p in plain])
    for l in range(LAYERS):
        exp = hxdist.assemble(mode, [parts[r][l] for r in range(world)], shards, n_all, hq, HD)
        if not np.array_equal(got[l].numpy(), exp):
            bad = np.argwhere(got[l].numpy() != exp)
            raise AssertionError(f"{name}: layer {l} gathered rows differ from the per-rank "
                                 f"results at {bad[:5].tolist()} ({len(bad)} elements)")

    # unsharded decode of the whole cache on this GPU
    full = kv.KVCache(LAYERS, hkv, HD, n_all, cap)
    for s, L in enumerate(lengths):
        full.reserve(s, L)
        for l in range(LAYERS):
            full.write(l, s, 0, K[l][s].to(dev), V[l][s].to(dev))
    sid_a = torch.arange(n_all, dtype=torch.int32, device=dev)
    len_a = torch.tensor(lengths, dtype=torch.int32, device=dev)
    for l in range(LAYERS):
        ref = full.decode(l, Q[l].to(dev), sid_a, len_a, hq, out_dtype=torch.float32).cpu()
        err = (got[l].float() - ref).abs().max().item()
        scale = ref.abs().max().item()
        assert err <= max(2e-3, 1e-2 * scale), f"{name}: layer {l} max abs error {err}"
    kv.device_status()
    torch.cuda.synchronize()
    dist.barrier()  # nobody unmaps while a peer may still write
    peer.close()
    full.close()
    cache.close()
    return epoch


def run_fused_case(rank, world, dev, name, hq, hkv, lengths, out_dtype, epoch):
    """The newest position of every sequence arrives as raw q / k / v rows:
    append_decode_gather on one copy of the shard against rope_append +
    decode_gather on another; both gathered buffers must be equal."""
    n_all = len(lengths)
    group = hq // hkv
    mode, shards = hxdist.plan(world, hkv, lengths)
    seqs, heads = shards[rank]
    n = len(seqs)
    cap = max(lengths) + 1
    g = torch.Generator().manual_seed(4321 + n_all)
    K = [torch.randn((L, hkv * HD), generator=g).half() for L in lengths]
    V = [torch.randn((L, hkv * HD), generator=g).half() for L in lengths]
    Q = torch.randn((n_all, hq * HD), generator=g).half()

    def cols(t, hs, width):
        return torch.cat([t[..., h * width:(h + 1) * width] for h in hs], dim=-1)

    caches = [kv.KVCache(1, len(heads), HD, max(n, 1), cap) for _ in range(2)]
    for c in caches:
        for i, s in enumerate(seqs):
            c.reserve(i, lengths[s])
            if lengths[s] > 1:  # history; the newest position comes with the step
                c.write(0, i, 0, cols(K[s][:-1], heads, HD).contiguous().to(dev),
                        cols(V[s][:-1], heads, HD).contiguous().to(dev))
    qh = [h * group + j for h in heads for j in range(group)]
    q_loc = cols(Q[seqs], qh, HD).contiguous().to(dev) if n else \
        torch.empty((0, len(qh) * HD), dtype=torch.float16, device=dev)
    k_new = cols(torch.stack([K[s][-1] for s in seqs]), heads, HD).contiguous().to(dev) if n else \
        torch.empty((0, len(heads) * HD), dtype=torch.float16, device=dev)
    v_new = cols(torch.stack([V[s][-1] for s in seqs]), heads, HD).contiguous().to(dev) if n else \
        torch.empty((0, len(heads) * HD), dtype=torch.float16, device=dev)
    table = kv.RopeTable(HD, cap, 1e6)
    sid = torch.arange(n, dtype=torch.int32, device=dev)
    lens = torch.tensor([lengths[s] for s in seqs], dtype=torch.int32, device=dev)
    rows = torch.tensor(seqs, dtype=torch.int32, device=dev)
    esize = 4 if out_dtype == torch.float32 else 2
    layer_bytes = n_all * hq * HD * esize
    peer = kv.PeerGather(rank, world, 2 * layer_bytes, exchange_fn(world))
    place = dict(out_rows=rows, out_row_heads=hq, out_head0=heads[0] * group, out_dtype=out_dtype)
    q_rot = torch.empty_like(q_loc)
    if n:
        caches[0].rope_append(0, k_new, v_new, sid, lens - 1, q=q_loc, num_q_heads=len(qh),
                              table=table, q_out=q_rot)
    epoch += 1
    caches[0].decode_gather(0, q_rot, sid, lens, len(qh), peer, out_offset=0, **place)
    peer.wait(epoch)
    epoch += 1
    caches[1].append_decode_gather(0, q_loc, k_new, v_new, sid, lens, len(qh), peer,
                                   out_offset=layer_bytes, table=table, **place)
    peer.wait(epoch)
    kv.device_status()
    got = peer.view(out_dtype, shape=(2, n_all, hq * HD)).cpu()
    if not torch.equal(got[0], got[1]):
        bad = (got[0] != got[1]).nonzero()
        raise AssertionError(f"{name}: one-launch step differs from append + decode at "
                             f"{bad[:5].tolist()} ({len(bad)} elements)")
    torch.cuda.synchronize()
    dist.barrier()
    peer.close()
    table.close()
    for c in caches:
        c.close()
    return epoch


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("gloo", timeout=timedelta(seconds=90))
    epoch = 0
    for case in CASES:
        epoch = run_case(rank, world, dev, *case)
        dist.barrier()
    epoch = 10000
    for case in CASES:
        epoch = run_fused_case(rank, world, dev, *case, epoch)
        dist.barrier()

    # bounded wait that runs out: nobody posts this epoch
    peer = kv.PeerGather(rank, world, 4096, exchange_fn(world))
    if rank == 0:
        peer.wait(12345)
        try:
            kv.device_status()
            raise AssertionError("the wait for an epoch nobody posted did not time out")
        except HXError as e:
            assert e.status == HX_ERR_TIMEOUT, e
        kv.device_status()  # cleared; the context still works
        torch.ones(4, device=dev).sum().item()
    torch.cuda.synchronize()
    dist.barrier()
    peer.close()
    print(f"RANK {rank} OK", flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
