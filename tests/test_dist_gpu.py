"""Multi-GPU decode over NCCL (needs >= 2 GPUs; one process per GPU).

* sequence sharding: every rank holds only its page-aligned token range of each sequence
  (FP16 and INT4 KIVI caches); decode_sequence_sharded (local split-KV + state merge + one
  all_gather_into_tensor + rank-state merge) must equal the single-GPU result, and so must the
  fused NVLink exchange (SequenceShardExchange: split kernel + one peer-store kernel), over
  repeated calls and CUDA-graph replays;
* batch sharding: each rank decodes its own sequences; gather_outputs equals single-GPU.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, result_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "kvq-decode_b200")]
    from bpt import paged_decode_attention
    from bpt.dist import SequenceShardExchange, decode_batch_sharded, \
        decode_sequence_sharded, gather_outputs, shard_range, token_shards
    from bpt.quant import empty_kivi_cache, paged_decode_attention_kivi, quantize_append
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    Hq, Hkv, D = 32, 8, 128
    errs = {}

    def paged(k, v, lens, bs, seed):
        """Contiguous [B, S, H, D] -> (kc, vc, bt) with a random page permutation."""
        g = torch.Generator().manual_seed(seed)
        pages = [(n + bs - 1) // bs for n in lens]
        nb = sum(pages) + 1
        perm = torch.randperm(nb, generator=g)
        bt = torch.zeros(len(lens), max(max(pages), 1), dtype=torch.int32)
        kc = torch.zeros(nb, bs, Hkv, D, dtype=k.dtype, device=dev)
        vc = torch.zeros_like(kc)
        off = 0
        for b, p in enumerate(pages):
            ids = perm[off:off + p]
            off += p
            bt[b, :p] = ids.to(torch.int32)
            for i, pid in enumerate(ids.tolist()):
                lo, hi = i * bs, min((i + 1) * bs, lens[b])
                kc[pid, :hi - lo] = k[b, lo:hi]
                vc[pid, :hi - lo] = v[b, lo:hi]
        return kc, vc, bt.to(dev)

    # ---------------- FP16 sequence sharding
    g = torch.Generator(device=dev).manual_seed(1)
    lens = [70000, 4097, 16]
    B, bs = len(lens), 16
    q = torch.randn(B, Hq, D, generator=g, device=dev, dtype=torch.float16)
    k = torch.randn(B, max(lens), Hkv, D, generator=g, device=dev, dtype=torch.float16)
    v = torch.randn(B, max(lens), Hkv, D, generator=g, device=dev, dtype=torch.float16)
    ranges = [token_shards(n, bs, world)[rank] for n in lens]
    sub = [hi - lo for lo, hi in ranges]
    ks = torch.zeros(B, max(max(sub), 1), Hkv, D, dtype=torch.float16, device=dev)
    vs = torch.zeros_like(ks)
    for b, (lo, hi) in enumerate(ranges):
        ks[b, :hi - lo] = k[b, lo:hi]
        vs[b, :hi - lo] = v[b, lo:hi]
    kc, vc, bt = paged(ks, vs, sub, bs, seed=10 + rank)
    sl = torch.tensor(sub, dtype=torch.int32, device=dev)
    out = decode_sequence_sharded(q, kc, vc, bt, sl)
    kf, vf, btf = paged(k, v, lens, bs, seed=99)
    ref = paged_decode_attention(q, kf, vf, btf, torch.tensor(lens, dtype=torch.int32,
                                                               device=dev))
    errs["fp16_seq"] = (out.float() - ref.float()).abs().max().item()

    # ---------------- the same through the fused NVLink exchange (eager, then graph replays)
    ex = SequenceShardExchange(B, Hq, D)
    fused = None
    for _ in range(3):
        fused = decode_sequence_sharded(q, kc, vc, bt, sl, exchange=ex)
    torch.cuda.synchronize()
    errs["fp16_seq_fused"] = (fused.float() - ref.float()).abs().max().item()
    errs["fused_vs_nccl"] = (fused.float() - out.float()).abs().max().item()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    gout = torch.empty_like(fused)
    with torch.cuda.stream(side):
        decode_sequence_sharded(q, kc, vc, bt, sl, exchange=ex, out=gout)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            decode_sequence_sharded(q, kc, vc, bt, sl, exchange=ex, out=gout)
    torch.cuda.synchronize()
    for _ in range(4):
        gout.zero_()
        graph.replay()
    torch.cuda.synchronize()
    errs["fp16_seq_fused_graph"] = (gout.float() - ref.float()).abs().max().item()
    errs["fused_status"] = float(ex.status.item())
    del graph
    ex.close()

    # ---------------- INT4 KIVI sequence sharding (page-aligned shards -> identical codes)
    bs = 64
    lens = [40000, 130]
    B = len(lens)
    k = torch.randn(B, max(lens), Hkv, D, generator=g, device=dev, dtype=torch.float16)
    v = torch.randn(B, max(lens), Hkv, D, generator=g, device=dev, dtype=torch.float16)
    q = torch.randn(B, Hq, D, generator=g, device=dev, dtype=torch.float16)

    def kivi_cache(kk, vv, ll, seed):
        pages = [(n + bs - 1) // bs for n in ll]
        nb = sum(pages) + 1
        gg = torch.Generator().manual_seed(seed)
        perm = torch.randperm(nb, generator=gg)
        btk = torch.zeros(len(ll), max(max(pages), 1), dtype=torch.int32)
        off = 0
        for b, p in enumerate(pages):
            btk[b, :p] = perm[off:off + p].to(torch.int32)
            off += p
        btk = btk.to(dev)
        c = empty_kivi_cache(nb, bs, Hkv, D, "int4", dev)
        n_t = torch.tensor(ll, dtype=torch.int32, device=dev)
        quantize_append(c, kk, vv, n_t, torch.zeros_like(n_t), btk)
        return c, btk, n_t

    ranges = [token_shards(n, bs, world)[rank] for n in lens]
    sub = [hi - lo for lo, hi in ranges]
    ks = torch.zeros(B, max(max(sub), 1), Hkv, D, dtype=torch.float16, device=dev)
    vs = torch.zeros_like(ks)
    for b, (lo, hi) in enumerate(ranges):
        ks[b, :hi - lo] = k[b, lo:hi]
        vs[b, :hi - lo] = v[b, lo:hi]
    c_loc, bt_loc, sl_loc = kivi_cache(ks, vs, sub, 20 + rank)
    out = decode_sequence_sharded(q, None, None, bt_loc, sl_loc, kivi_cache=c_loc)
    c_full, bt_full, sl_full = kivi_cache(k, v, lens, 7)
    ref = paged_decode_attention_kivi(q, c_full, bt_full, sl_full)
    errs["int4_seq"] = (out.float() - ref.float()).abs().max().item()
    ex = SequenceShardExchange(B, Hq, D)
    fused = decode_sequence_sharded(q, None, None, bt_loc, sl_loc, kivi_cache=c_loc, exchange=ex)
    torch.cuda.synchronize()
    errs["int4_seq_fused"] = (fused.float() - ref.float()).abs().max().item()
    ex.close()

    # ---------------- FP16 batch sharding
    Bt, bs = 4 * world, 16
    lens = [int(x) for x in torch.randint(1, 20000, (Bt,), generator=torch.Generator()
                                          .manual_seed(3)).tolist()]
    k = torch.randn(Bt, max(lens), Hkv, D, generator=g, device=dev, dtype=torch.float16)
    v = torch.randn(Bt, max(lens), Hkv, D, generator=g, device=dev, dtype=torch.float16)
    q = torch.randn(Bt, Hq, D, generator=g, device=dev, dtype=torch.float16)
    lo, hi = shard_range(Bt, world, rank)
    kc, vc, bt = paged(k[lo:hi], v[lo:hi], lens[lo:hi], bs, seed=30 + rank)
    out_loc = decode_batch_sharded(q[lo:hi].contiguous(), kc, vc, bt,
                                   torch.tensor(lens[lo:hi], dtype=torch.int32, device=dev))
    allout = gather_outputs(out_loc)
    kf, vf, btf = paged(k, v, lens, bs, seed=31)
    ref = paged_decode_attention(q, kf, vf, btf, torch.tensor(lens, dtype=torch.int32,
                                                               device=dev))
    errs["fp16_batch"] = (allout.float() - ref.float()).abs().max().item()

    if rank == 0:
        np.save(os.path.join(result_dir, "errs.npy"), errs, allow_pickle=True)
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()


def test_sharded_decode_matches_single_gpu(tmp_path):
    world = min(torch.cuda.device_count(), 8)
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    errs = np.load(tmp_path / "errs.npy", allow_pickle=True).item()
    # split boundaries differ (per-rank splits + rank merge) -> fp32 rounding only
    assert errs["fp16_seq"] < 2e-3, errs
    assert errs["fp16_seq_fused"] < 2e-3 and errs["fp16_seq_fused_graph"] < 2e-3, errs
    assert errs["fused_vs_nccl"] < 1e-3 and errs["fused_status"] == 0, errs
    assert errs["int4_seq"] < 2e-3 and errs["int4_seq_fused"] < 2e-3, errs
    assert errs["fp16_batch"] < 2e-3, errs
