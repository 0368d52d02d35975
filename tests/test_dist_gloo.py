"""Multi-rank host logic on CPU (gloo, world_size 2): sequence sharding and batch sharding.

Each rank builds ITS OWN paged cache holding only its page-aligned token range
(bpt.dist.token_shards), computes its merged partial state with the numpy oracle, packs it in
the layout bpt.dist.state_buffer / split_state define, and the ranks exchange states with
all_gather_into_tensor exactly as decode_sequence_sharded does; merging the gathered states
must reproduce single-rank attention over the whole sequence. A rank that never joins the
collective must surface as an error on the other rank within the process-group timeout.
"""
import datetime
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

LOG2E = float(np.log2(np.e))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s=30):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _rank_cache(k, v, lens, ranges, block_size, seed):
    """Paged cache holding tokens [lo, hi) of each sequence, re-paged from token 0."""
    from oracle import cache as oc
    g = oc.rng(seed)
    sub_lens = [hi - lo for (lo, hi) in ranges]
    S = max(max(sub_lens), 1)
    ks = np.zeros((k.shape[0], S) + k.shape[2:], k.dtype)
    vs = np.zeros_like(ks)
    for b, (lo, hi) in enumerate(ranges):
        ks[b, :hi - lo] = k[b, lo:hi]
        vs[b, :hi - lo] = v[b, lo:hi]
    kc, vc, bt, _ = oc.build_paged_cache(ks, vs, sub_lens, block_size, g, "spare", 2)
    return kc, vc, bt, np.asarray(sub_lens, np.int32)


def _seq_shard_worker(rank, world, port, result_path):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "kvq-decode_b200")]
    from bpt.dist import split_state, state_buffer, token_shards
    from oracle import attention as oa
    from oracle import cache as oc
    _init(rank, world, port)
    lens, Hq, Hkv, D, bs = [1000, 37, 16], 32, 8, 128, 16
    g = oc.rng(123)                                # same inputs on every rank
    q, k, v = oc.make_qkv(g, lens, Hq, Hkv, D)
    ranges = [token_shards(n, bs, world)[rank] for n in lens]
    kc, vc, bt, sl = _rank_cache(k, v, lens, ranges, bs, seed=500 + rank)
    o, lse = oa.paged_decode_attention_partial(q, kc, vc, bt, sl, np.zeros_like(sl), sl)
    send = state_buffer(len(lens), Hq, D, "cpu")
    so, sl2 = split_state(send, len(lens), Hq, D)
    so.copy_(torch.from_numpy(o))
    sl2.copy_(torch.from_numpy(lse * LOG2E))      # states travel in log2 units
    recv = torch.empty(world * send.numel(), dtype=torch.float32)
    dist.all_gather_into_tensor(recv, send)
    blocks = recv.view(world, -1)
    os_, ls_ = zip(*[split_state(blocks[r], len(lens), Hq, D) for r in range(world)])
    merged = oa.merge_states(np.stack([x.numpy() for x in os_]),
                             np.stack([x.numpy() for x in ls_]) / LOG2E)
    if rank == 0:
        kf, vf, btf, nb = oc.build_paged_cache(k, v, lens, bs, oc.rng(9), "spare", 4)
        full = oa.paged_decode_attention_ref(q, kf, vf, btf, np.asarray(lens),
                                             out_dtype=np.float32)
        np.save(result_path, np.abs(merged - full).max())
    dist.barrier()
    dist.destroy_process_group()


def _batch_shard_worker(rank, world, port, result_path):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "kvq-decode_b200")]
    from bpt.dist import shard_range
    from oracle import attention as oa
    from oracle import cache as oc
    _init(rank, world, port)
    B, Hq, Hkv, D, bs = 6, 32, 8, 128, 16
    g = oc.rng(77)
    lens = [int(x) for x in g.integers(1, 300, size=B)]
    q, k, v = oc.make_qkv(g, lens, Hq, Hkv, D)
    lo, hi = shard_range(B, world, rank)
    kc, vc, bt, _ = oc.build_paged_cache(k[lo:hi], v[lo:hi], lens[lo:hi], bs, oc.rng(rank),
                                         "spare", 2)
    out = oa.paged_decode_attention_ref(q[lo:hi], kc, vc, bt, np.asarray(lens[lo:hi]),
                                        out_dtype=np.float32)
    res = torch.empty(B, Hq, D)
    dist.all_gather_into_tensor(res, torch.from_numpy(out))
    if rank == 0:
        kf, vf, btf, _ = oc.build_paged_cache(k, v, lens, bs, oc.rng(5), "spare", 2)
        full = oa.paged_decode_attention_ref(q, kf, vf, btf, np.asarray(lens),
                                             out_dtype=np.float32)
        np.save(result_path, np.abs(res.numpy() - full).max())
    dist.barrier()
    dist.destroy_process_group()


def _missing_rank_worker(rank, world, port, result_path):
    _init(rank, world, port, timeout_s=3)
    if rank == 1:
        return  # never joins the collective and leaves without tearing down
    t = torch.zeros(4)
    try:
        dist.all_gather_into_tensor(torch.zeros(8), t)
        np.save(result_path, np.array(0))
    except Exception:
        np.save(result_path, np.array(1))


def _run(worker, tmp_path, world=2):
    port = _free_port()
    path = str(tmp_path / "result.npy")
    mp.start_processes(worker, args=(world, port, path), nprocs=world, join=True,
                       start_method="spawn")
    return np.load(path)


def test_sequence_sharding_protocol_matches_single_rank(tmp_path):
    assert float(_run(_seq_shard_worker, tmp_path)) < 1e-5


def test_batch_sharding_matches_single_rank(tmp_path):
    assert float(_run(_batch_shard_worker, tmp_path)) < 1e-6


def test_token_shards_are_page_aligned_and_cover_the_sequence():
    from bpt.dist import shard_range, token_shards
    for n, bs, w in [(1000, 16, 2), (131072, 16, 8), (5, 16, 4), (0, 16, 2), (4097, 64, 3)]:
        sh = token_shards(n, bs, w)
        assert sh[0][0] == 0 and sh[-1][1] == n
        for (a, b), (c, _) in zip(sh, sh[1:]):
            assert b == c and a <= b and (a % bs == 0 or a == n)
    assert [shard_range(10, 4, r) for r in range(4)] == [(0, 2), (2, 5), (5, 7), (7, 10)]


def test_a_rank_that_never_joins_is_detected(tmp_path):
    """The surviving rank's collective must fail with an error (process-group timeout),
    not hang: the failure is made on the host, no GPU is involved."""
    port = _free_port()
    path = str(tmp_path / "result.npy")
    ctx = mp.start_processes(_missing_rank_worker, args=(2, port, path), nprocs=2, join=False,
                             start_method="spawn")
    while not ctx.join(timeout=60):
        pass
    assert int(np.load(path)) == 1
