"""Multi-rank partitioning of batched decode attention, on CPU ranks (gloo).

Each of 2 ranks computes its shard (its sequences or its kv heads) with the
CPU oracle; the shards are all-gathered (padded to a common row count, as
the GPU path does) and assembled into the reference output layout
[sequence][q_head*head_dim].  The result must equal the single-process oracle
bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hxinfer_b200 import dist as D

HQ, HD = 8, 128


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _case(hkv, seed=5):
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    lengths = [int(x) for x in rng.integers(1, 300, 7)]
    q = O.f16(rng.standard_normal((len(lengths), HQ * HD)))
    ks = [O.f16(rng.standard_normal((L, hkv * HD))) for L in lengths]
    vs = [O.f16(rng.standard_normal((L, hkv * HD))) for L in lengths]
    return lengths, q, ks, vs


def _worker(rank, world, port, hkv, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as O
        lengths, q, ks, vs = _case(hkv)
        mode, shards = D.plan(world, hkv, lengths)
        seqs, heads = shards[rank]
        group = HQ // hkv
        qcols = np.concatenate([np.arange(h * group * HD, (h + 1) * group * HD) for h in heads])
        kcols = np.concatenate([np.arange(h * HD, (h + 1) * HD) for h in heads])
        part = O.decode_attention_batch(q[seqs][:, qcols], [ks[s][:, kcols] for s in seqs],
                                        [vs[s][:, kcols] for s in seqs], len(heads) * group,
                                        len(heads), HD)
        n_pad = max(len(sh[0]) for sh in shards)
        buf = torch.zeros((n_pad, part.shape[1]), dtype=torch.float32)
        buf[:len(seqs)] = torch.from_numpy(part)
        gathered = [torch.zeros_like(buf) for _ in range(world)]
        dist.all_gather(gathered, buf)
        parts = [g[:len(sh[0])].numpy() for g, sh in zip(gathered, shards)]
        full = D.assemble(mode, parts, shards, len(lengths), HQ, HD)
        if rank == 0:
            result_q.put((mode, full))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("hkv,mode", [(2, "kv_heads"), (4, "sequences")])
def test_two_rank_gather_matches_single_process(oracle, hkv, mode):
    world = 2
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, hkv, q_out)) for r in range(world)]
    for p in procs:
        p.start()
    got_mode, full = q_out.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    lengths, q, ks, vs = _case(hkv)
    want = oracle.decode_attention_batch(q, ks, vs, HQ, hkv, HD)
    assert got_mode == mode
    assert np.array_equal(full.view(np.uint32), want.view(np.uint32))


def test_plan_shapes():
    lengths = [int(x) for x in np.random.default_rng(4).integers(512, 32769, 64)]
    for world in (2, 4):
        mode, shards = D.plan(world, 8, lengths)
        assert mode == "sequences"
        sizes = [len(s) for s, _ in shards]
        assert max(sizes) - min(sizes) <= 1
        assert sorted(i for s, _ in shards for i in s) == list(range(64))
        loads = [sum(lengths[i] for i in s) for s, _ in shards]
        assert max(loads) / min(loads) < 1.1
    mode, shards = D.plan(8, 8, lengths)
    assert mode == "kv_heads" and [h for _, h in shards] == [[r] for r in range(8)]
    assert all(len(s) == 64 for s, _ in shards)


def test_assemble_with_a_rank_without_sequences():
    """Fewer sequences than ranks: the empty shard contributes no rows."""
    mode, shards = D.plan(2, 4, [300])
    assert mode == "sequences" and shards[1][0] == []
    part0 = np.arange(8 * 4, dtype=np.float32).reshape(1, 32)
    part1 = np.zeros((0, 32), np.float32)
    out = D.assemble(mode, [part0, part1], shards, 1, 8, 4)
    assert np.array_equal(out, part0)


def test_peer_gather_views_must_fit_the_buffer():
    """View arguments are checked on the host before any device pointer is
    used (an out-of-bounds view of peer-mapped memory would fault on use)."""
    import torch
    from hxinfer_b200 import kv
    pg = kv.PeerGather.__new__(kv.PeerGather)  # no endpoint: only the checks run
    pg.bytes, pg.ptr, pg.handle = 1024, 0, None
    for offset, shape in ((0, (513,)), (1000, (16,)), (-2, None), (1, None), (2048, None)):
        with pytest.raises(ValueError):
            pg.view(torch.float16, offset, shape)
