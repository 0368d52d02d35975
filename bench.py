#!/usr/bin/env python
"""bpt benchmark: achieved HBM bandwidth of paged-KV GQA decode on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl bpt|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU, NCCL)

A step is one single-layer decode call over one batch (Llama-3-8B layer: Hq=32, Hkv=8, D=128)
of synthetic paged KV with seeded ragged lengths and a random-permutation block table, inputs
resident in HBM. Multi-GPU runs shard by batch (each rank owns its own batch and KV pool, no
collective on the data path): weak scaling; the time is the max over ranks.

Prints ONE JSON line (rank 0). `value` is the whole-job achieved bandwidth in TB/s:
algorithmic bytes of all ranks' calls / max-over-ranks device time. `roofline` reports the
dominant kernel (the split-KV decode kernel) against the measured HBM copy peak. `e2e` is the
same metric through the public API with per-step host->device copies of the step's inputs
(q, block table, sequence lengths) from pinned memory and a device->host read of the output;
the KV cache is resident state, like weights. `--impl reference` times the reference's CPU
algorithm (the numpy port in oracle/) on the host cores on a bounded sample of the workload.
"""
import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "kvq-decode_b200"))
sys.path.insert(0, ROOT)

HQ, HKV, D = 32, 8, 128
FALLBACK_HBM_GBS = 6650.0
B200_SPEC_GBS = 8000.0

# BASELINE configs[1] (FP16 batch) and configs[2] (FP16 batch 1); default = the largest
# single-GPU configuration of the FP16 batch family.
WORKLOADS = {
    "fp16_b64_ctx64k": dict(fmt="fp16", batch=64, ctx=65536, block_size=16, ragged=True),
    "fp16_b32_ctx64k": dict(fmt="fp16", batch=32, ctx=65536, block_size=16, ragged=True),
    "fp16_b16_ctx64k": dict(fmt="fp16", batch=16, ctx=65536, block_size=16, ragged=True),
    "fp16_b8_ctx64k": dict(fmt="fp16", batch=8, ctx=65536, block_size=16, ragged=True),
    "fp16_b64_ctx16k": dict(fmt="fp16", batch=64, ctx=16384, block_size=16, ragged=True),
    "fp16_b32_ctx16k": dict(fmt="fp16", batch=32, ctx=16384, block_size=16, ragged=True),
    "fp16_b16_ctx16k": dict(fmt="fp16", batch=16, ctx=16384, block_size=16, ragged=True),
    "fp16_b8_ctx16k": dict(fmt="fp16", batch=8, ctx=16384, block_size=16, ragged=True),
    "fp16_b1_ctx4k": dict(fmt="fp16", batch=1, ctx=4096, block_size=16, ragged=False),
    "fp16_b1_ctx16k": dict(fmt="fp16", batch=1, ctx=16384, block_size=16, ragged=False),
    "fp16_b1_ctx64k": dict(fmt="fp16", batch=1, ctx=65536, block_size=16, ragged=False),
    "fp16_b1_ctx128k": dict(fmt="fp16", batch=1, ctx=131072, block_size=16, ragged=False),
}
# BASELINE configs[3] (INT8 / FP8-E4M3 KIVI, bs=64) and configs[4] (INT4 KIVI, bs=64)
for _fmt in ("int8", "fp8", "int4"):
    for _b in (1, 8, 32, 64):
        for _ctx, _tag in ((8192, "8k"), (32768, "32k"), (131072, "128k")):
            WORKLOADS[f"{_fmt}_b{_b}_ctx{_tag}"] = dict(fmt=_fmt, batch=_b, ctx=_ctx,
                                                        block_size=64, ragged=False)
DEFAULT_WORKLOAD = "fp16_b64_ctx64k"
# published reference number for the same metric (A100-80GB, best split, B=32 ctx=16k,
# docs/NOTES.md:99 of the reference): 1638 GB/s
REFERENCE_PUBLISHED_TBPS = 1.638


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["bpt", "reference", "reference-triton", "flashinfer"],
                    default="bpt",
                    help="reference: the reference's CPU algorithm (numpy port) on the host "
                         "cores; reference-triton: the reference's own Triton FP16 kernel "
                         "(installed under baseline/_ref) on this GPU, same inputs; flashinfer: "
                         "FlashInfer's paged decode (the library in this image) on this GPU, "
                         "same inputs")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=DEFAULT_WORKLOAD)
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--seqshard", action="store_true",
                    help="shard every sequence's tokens over the ranks (strong scaling; the "
                         "ranks exchange their partial softmax states)")
    ap.add_argument("--exchange", choices=["nvlink", "nccl"], default="nvlink",
                    help="sequence sharding: fused NVLink peer-store kernel (default) or one "
                         "NCCL all-gather")
    ap.add_argument("--eager", action="store_true",
                    help="time eager calls instead of CUDA-graph replays of the call")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=1,
                    help="decode L independent layers (own KV cache, q, table each) per step, "
                         "captured in one CUDA graph: L=32 is a whole Llama-3-8B decode step's "
                         "attention")
    ap.add_argument("--splits", type=int, default=0,
                    help="force the split count per sequence (0: the planner's choice)")
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="budget of the CPU-baseline sample")
    return ap.parse_args()


def workload_lens(wl, rank, seed):
    from bpt.cache import ragged_lengths
    if wl["ragged"]:
        return ragged_lengths(wl["batch"], wl["ctx"], seed + 7919 * rank)
    return [wl["ctx"]] * wl["batch"]


def config_index(wl):
    if wl["fmt"] == "fp16":
        return 1 if wl["batch"] > 1 else 2
    return 4 if wl["fmt"] == "int4" else 3


def config_dict(name, wl, n_gpus, seqshard=False, exchange="nvlink"):
    return {
        "workload": f"{name}: BASELINE configs[{config_index(wl)}] "
                    f"{wl['fmt']} paged KV, Llama-3-8B layer (Hq={HQ}, Hkv={HKV}, D={D}), "
                    f"B={wl['batch']} per GPU, ctx={wl['ctx']}"
                    + (" seq_len~U[0.75ctx,ctx]" if wl["ragged"] else "")
                    + f", block_size={wl['block_size']}, random-permutation block table"
                    + ("" if wl["fmt"] == "fp16" else
                       ", KIVI (keys per page/head/channel, values per token/head; K ~ N(0,1)"
                       " with 4 seeded x10 outlier channels per kv head), quantized on the GPU"),
        "kv_dtype": wl["fmt"], "batch_per_gpu": wl["batch"], "ctx": wl["ctx"],
        "block_size": wl["block_size"], "q_heads": HQ, "kv_heads": HKV, "head_dim": D,
        "parallelism": (f"sequence-sharded x{n_gpus} (page-aligned token ranges per rank, "
                        + ("partial softmax states exchanged by one fused kernel storing into "
                           "the peers' memory over NVLink)" if exchange == "nvlink" else
                           "partial softmax states merged after one NCCL all-gather)")
                        if seqshard else
                        f"batch-sharded x{n_gpus} (independent sequences per rank)"),
        "l2": "no flush: per-step working set (GBs of KV) far exceeds the 126 MB L2",
    }


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, STREAM copy)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback (no MEASURED_PEAKS.json)"


def split_kernel_name(fmt, block_size):
    """The stage-1 kernel a decode call of this format launches (Llama-3-8B head shape)."""
    if fmt == "fp16":
        return "split_kv_fp16_mma_kernel"
    if fmt in ("int8", "int4") and block_size >= 32:   # group 4, 8 kv heads
        return f"kivi_tc_decode_kernel<{fmt}>"
    if fmt in ("int8", "int4"):
        return f"kivi_int_decode_kernel<{fmt}>"
    return f"kivi_decode_kernel<{fmt}>"


def ncu_traffic(kernel, algorithmic_bytes):
    """DRAM bytes per launch of the stage-1 kernel: the committed ncu ratio (read + write over
    algorithmic bytes, profiles/dram_traffic.json) scaled to this workload, or (None, None)."""
    path = os.path.join(ROOT, "profiles", "dram_traffic.json")
    try:
        with open(path) as f:
            e = json.load(f)["kernels"].get(kernel)
        if not e:
            return None, None
        note = (f"ncu dram__bytes_read.sum + dram__bytes_write.sum of {kernel} on "
                f"{e['capture_workload']} = {e['ratio']:.5f} x algorithmic bytes, scaled to this "
                "workload's algorithmic bytes")
        return float(e["ratio"]) * algorithmic_bytes, note
    except Exception:
        return None, None


class quiet_stdout:
    """Silence file descriptor 1 (C/C++ writes included, e.g. NCCL's version banner at
    communicator creation) so rank 0 prints exactly one JSON line on stdout."""

    def __enter__(self):
        sys.stdout.flush()
        self.saved = os.dup(1)
        self.null = os.open(os.devnull, os.O_WRONLY)
        os.dup2(self.null, 1)
        return self

    def __exit__(self, *a):
        sys.stdout.flush()
        os.dup2(self.saved, 1)
        os.close(self.saved)
        os.close(self.null)


class ClockSampler:
    """NVML SM-clock and clock-event-reason sampling while the timed region runs."""
    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, device_index):
        self.samples, self.reasons, self.ok = [], 0, False
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = self._handle(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # pragma: no cover - NVML missing
            self.err = str(e)

    def _handle(self, idx):
        import torch
        try:
            p = torch.cuda.get_device_properties(idx)
            bus = f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
            return self.nv.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return self.nv.nvmlDeviceGetHandleByIndex(idx)

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": self.err}
        names = [v for k, v in self.REASONS.items() if self.reasons & k and k != 0x1]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples)}


# ----------------------------------------------------------------------------- CPU oracle

def oracle_sample_inputs(n, block_size, fmt, seed):
    """One sequence of n tokens for the CPU oracle: (q, k_cache, v_cache, bt, sl, nbytes_fn).
    Quantized formats return the *codes* cache; the timed oracle step dequantizes it (the
    reference's algorithm applied to the KIVI cache: dequantize, then fp32 attention)."""
    import numpy as np
    from oracle import kivi
    g = np.random.Generator(np.random.PCG64(seed))
    pages = (n + block_size - 1) // block_size
    q = g.standard_normal((1, HQ, D), dtype=np.float32).astype(np.float16)
    bt = g.permutation(pages).astype(np.int32)[None]
    sl = np.asarray([n], np.int32)
    if fmt == "fp16":
        kc = g.standard_normal((pages, block_size, HKV, D), dtype=np.float32).astype(np.float16)
        vc = g.standard_normal((pages, block_size, HKV, D), dtype=np.float32).astype(np.float16)
        return q, (kc, vc), bt, sl
    cache = kivi.empty_cache(pages, block_size, HKV, D, fmt)
    k = g.standard_normal((1, pages * block_size, HKV, D), dtype=np.float32)
    k[..., :4] *= 10.0
    v = g.standard_normal((1, pages * block_size, HKV, D), dtype=np.float32)
    kivi.quantize_append(cache, k.astype(np.float16), v.astype(np.float16), [n], [0],
                         bt, block_size, fmt)
    return q, cache, bt, sl


def oracle_step(q, kv, bt, sl, fmt):
    from oracle import attention as oa
    from oracle import kivi
    import numpy as np
    if fmt == "fp16":
        return oa.paged_decode_attention_ref(q, kv[0], kv[1], bt, sl)
    kd, vd = kivi.dequantize_cache(kv, fmt)
    return oa.paged_decode_attention_ref(q, kd, vd, bt, sl, out_dtype=np.float16)


def cpu_oracle_sample(lens, block_size, fmt, seed, budget_s):
    """Time the CPU oracle (reference algorithm, src/bpt/reference.py:20-49; for KIVI caches
    preceded by the numpy dequantization) on whole sequences of the workload's length (capped
    at 32k tokens) until ~budget_s seconds. Returns (GB/s, seconds, bytes, description)."""
    from bpt.roofline import decode_call_bytes
    n = min(int(lens[0]), 32768)
    q, kv, bt, sl = oracle_sample_inputs(n, block_size, fmt, seed)
    oracle_step(q, kv, bt, sl, fmt)  # warm-up
    done, t0 = 0, time.perf_counter()
    while True:
        oracle_step(q, kv, bt, sl, fmt)
        done += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    nbytes = decode_call_bytes([n] * done, block_size, HQ, HKV, D, fmt)
    desc = (f"{done} x one sequence of {n} tokens ({fmt}), numpy oracle"
            + ("" if fmt == "fp16" else " incl. numpy dequantization")
            + " (numpy BLAS threads = host cores)")
    return nbytes / dt / 1e9, dt, nbytes, desc


def run_reference(args):
    """--impl reference: the reference's CPU algorithm (numpy port) on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    wl = WORKLOADS[args.workload]
    lens = workload_lens(wl, 0, args.seed)
    from bpt.roofline import decode_call_bytes
    bs, fmt = wl["block_size"], wl["fmt"]
    # a pool of 2 sequences; each step processes one whole sequence (rotating), capped at 32k
    sample = [min(int(x), 32768) for x in (lens[:2] if len(lens) > 1 else lens * 2)]
    pools = [oracle_sample_inputs(n, bs, fmt, args.seed + i) for i, n in enumerate(sample)]
    for i in range(args.warmup):
        oracle_step(*pools[i % len(pools)], fmt)
    t0 = time.perf_counter()
    nbytes = 0
    for i in range(args.steps):
        p = pools[i % len(pools)]
        oracle_step(*p, fmt)
        nbytes += decode_call_bytes([int(p[3][0])], bs, HQ, HKV, D, fmt)
    dt = time.perf_counter() - t0
    tbps = nbytes / dt / 1e12
    cores = os.cpu_count()
    line = {
        "impl": "reference", "metric": metric_name(wl), "value": tbps, "unit": "TB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(args.workload, wl, args.gpus),
        "cpu_baseline": {"value": tbps, "unit": "TB/s", "cores": cores, "kind": "port",
                         "sample": f"each step = one whole sequence of the workload "
                                   f"({sample} tokens, rotating; capped at 32k), numpy oracle"},
        "e2e": {"value": tbps, "unit": "TB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def metric_name(wl):
    return (f"achieved HBM TB/s of {wl['fmt']} paged-KV GQA decode "
            f"(Llama-3-8B layer; % of B200 peak and us/decode step in extra keys)")


# ----------------------------------------------------------------------------- bpt arm

def run_bpt(args):
    import torch
    import torch.distributed as dist
    from bpt import decode as dec
    from bpt.cache import random_paged_workload
    from bpt.roofline import decode_call_bytes, KIVI_FORMATS

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        with quiet_stdout():
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=dev)
            dist.barrier(device_ids=[local])  # creates the communicator

    wl = WORKLOADS[args.workload]
    bs, fmt = wl["block_size"], wl["fmt"]
    seqshard = args.seqshard and world > 1
    if seqshard:
        from bpt.dist import decode_sequence_sharded, token_shards
        full_lens = workload_lens(wl, 0, args.seed)          # same sequences on every rank
        lens = [hi - lo for lo, hi in (token_shards(n, bs, world)[rank] for n in full_lens)]
    else:
        lens = workload_lens(wl, rank, args.seed)
        full_lens = lens
    if fmt == "fp16":
        w = random_paged_workload(lens, HQ, HKV, D, bs, dev, seed=args.seed + rank,
                                  spare_blocks=64)
        kc, vc = w["k_cache"], w["v_cache"]
    else:
        from bpt.quant import random_kivi_workload
        w = random_kivi_workload(lens, HQ, HKV, D, bs, fmt, dev, seed=args.seed + rank,
                                 spare_blocks=64)
        kvcache = w["cache"]
    q, bt, sl = w["q"], w["block_table"], w["seq_lens"]
    L = max(1, args.layers)
    if L > 1 and seqshard:
        raise SystemExit("--layers > 1 is not combined with --seqshard")
    extra = []   # layers 1 .. L-1: their own caches, queries, tables and outputs
    for li in range(1, L):
        if fmt == "fp16":
            wx = random_paged_workload(lens, HQ, HKV, D, bs, dev, seed=args.seed + rank + 1009 * li,
                                       spare_blocks=64)
        else:
            wx = random_kivi_workload(lens, HQ, HKV, D, bs, fmt, dev,
                                      seed=args.seed + rank + 1009 * li, spare_blocks=64)
        wx["out"] = torch.empty_like(wx["q"])
        extra.append(wx)
    if seqshard:  # every rank decodes the same queries against its own token shard
        q = torch.randn(q.shape, generator=torch.Generator(device=dev).manual_seed(args.seed),
                        device=dev).to(torch.float16)
    B = len(lens)
    max_blocks = bt.shape[1]
    sms = dec._sm_count(local)
    if wl["fmt"] == "fp16":
        S = dec.effective_splits(B, HKV, bs, max_blocks, args.splits or None, sms)
    else:
        from bpt.quant import effective_splits_kivi
        S = effective_splits_kivi(kvcache, B, HQ, max_blocks, args.splits or None, sms)
    # algorithmic bytes of this rank's share of the job (seqshard: its tokens of the sequences,
    # plus q/out once on rank 0 so the job total counts them once)
    step_bytes = decode_call_bytes(lens, bs, HQ, HKV, D, wl["fmt"]) * L
    if seqshard and rank != 0:
        step_bytes -= len(lens) * HQ * D * 2 * 2
    f = KIVI_FORMATS[wl["fmt"]]
    kernel_bytes = step_bytes
    out = torch.empty_like(q)
    ws = torch.empty(dec.workspace_bytes(B, HQ, D, S), dtype=torch.uint8, device=dev)
    ex = None
    if seqshard and args.exchange == "nvlink":
        from bpt.dist import SequenceShardExchange
        ex = SequenceShardExchange(B, HQ, D)
    # split kernel (+ PDL merge); sequence sharding: split + fused exchange, or split + state
    # merge + NCCL all-gather + rank merge
    launches_per_step = ((2 if ex is not None else 4) if seqshard else (2 if S > 1 else 1)) * L
    stream = torch.cuda.current_stream(dev)

    def call():
        # one product call: split-KV kernel (+ its programmatically dependent merge)
        if seqshard:
            decode_sequence_sharded(q, kc if fmt == "fp16" else None,
                                    vc if fmt == "fp16" else None, bt, sl, out=out,
                                    kivi_cache=None if fmt == "fp16" else kvcache, exchange=ex)
        elif fmt == "fp16":
            dec.paged_decode_attention(q, kc, vc, bt, sl, num_splits=S, out=out, workspace=ws)
            for wx in extra:   # the layers run in order on one stream and share the workspace
                dec.paged_decode_attention(wx["q"], wx["k_cache"], wx["v_cache"],
                                           wx["block_table"], wx["seq_lens"], num_splits=S,
                                           out=wx["out"], workspace=ws)
        else:
            from bpt.quant import paged_decode_attention_kivi
            paged_decode_attention_kivi(q, kvcache, bt, sl, num_splits=S, out=out, workspace=ws)
            for wx in extra:
                paged_decode_attention_kivi(wx["q"], wx["cache"], wx["block_table"],
                                            wx["seq_lens"], num_splits=S, out=wx["out"],
                                            workspace=ws)

    # The device-timed leg replays the call as a CUDA graph (what a serving engine does with a
    # decode step), so host-side Python cost does not leak into small workloads' timing.
    graph = None
    if not args.eager and not (seqshard and ex is None):  # an NCCL all-gather step: eager
        call()
        torch.cuda.synchronize()
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            call()
        stream.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            call()

    graph_used = graph is not None

    def step(ev_a=None, ev_b=None):
        if ev_a is not None:
            ev_a.record(stream)
        if graph is not None:
            graph.replay()
        else:
            call()
        if ev_b is not None:
            ev_b.record(stream)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for _ in range(max(args.warmup, 0)):
        step()
    torch.cuda.synchronize()

    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    with sampler:
        t_start.record(stream)
        for _ in range(args.steps):
            step()
        t_end.record(stream)
        torch.cuda.synchronize()
    barrier()
    elapsed_ms = t_start.elapsed_time(t_end)
    # Per-call times come from a second pass of the same K steps with an event pair around each
    # call, outside the timed region above (whose loop has nothing between the calls).
    barrier()
    torch.cuda.synchronize()
    for i in range(args.steps):
        step(*evs[i])
    torch.cuda.synchronize()
    barrier()
    call_ms = [a.elapsed_time(b) for a, b in evs]
    kern_ms = sum(call_ms) / max(args.steps, 1)

    tot = torch.tensor([elapsed_ms, step_bytes * args.steps], dtype=torch.float64, device=dev)
    if world > 1:
        t_max = tot[:1].clone()
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
        b_sum = tot[1:].clone()
        dist.all_reduce(b_sum, op=dist.ReduceOp.SUM)
        elapsed_max, bytes_all = float(t_max.item()), float(b_sum.item())
    else:
        elapsed_max, bytes_all = elapsed_ms, float(step_bytes * args.steps)
    value_tbps = bytes_all / (elapsed_max * 1e-3) / 1e12

    # ---- e2e through the public API, host buffers, copies inside the timed region. One step =
    # upload of the step's inputs from pinned host memory, the public-API call, and the read-
    # back of its result into pinned host memory. Like a serving engine, the step is captured
    # once as a CUDA graph and replayed (the copies run on every replay); the NCCL
    # sequence-sharding path, which is not captured, runs it eagerly.
    e2e = None
    if not args.no_e2e:
        live_in = [(q, bt, sl)] + [(wx["q"], wx["block_table"], wx["seq_lens"]) for wx in extra]
        live_out = [out] + [wx["out"] for wx in extra]
        host_in = [tuple(t.cpu().pin_memory() for t in trio) for trio in live_in]
        host_out = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in live_out]

        def e2e_step():
            for lv, hs in zip(live_in, host_in):
                for d, h in zip(lv, hs):
                    d.copy_(h, non_blocking=True)
            call()
            for ho, lo in zip(host_out, live_out):
                ho.copy_(lo, non_blocking=True)

        e2e_step()
        torch.cuda.synchronize()
        e2e_graph = None
        if not (seqshard and ex is None):
            side = torch.cuda.Stream(dev)
            side.wait_stream(stream)
            with torch.cuda.stream(side):
                e2e_step()
            stream.wait_stream(side)
            e2e_graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(e2e_graph):
                e2e_step()
        run_e2e = e2e_graph.replay if e2e_graph is not None else e2e_step
        for _ in range(max(args.warmup, 1)):
            run_e2e()
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            run_e2e()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        # the result really came back: the last read-back equals the device output
        assert torch.equal(host_out[0], out.cpu()), "e2e read-back mismatch"
        e_ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
        e2e = {"value": bytes_all / (float(e_ms.item()) * 1e-3) / 1e12, "unit": "TB/s",
               "h2d_bytes_per_step": sum(t.nbytes for trio in live_in for t in trio),
               "d2h_bytes_per_step": sum(o.nbytes for o in live_out),
               "ms_per_step": float(e_ms.item()) / args.steps,
               "note": ("public API bpt.paged_decode_attention with the step's input upload "
                        "from pinned host memory and result read-back, "
                        + ("captured as one CUDA graph replayed per step"
                           if e2e_graph is not None else "eager calls")
                        + "; KV cache resident in HBM")}
        del e2e_graph

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbps, secs, nbytes, desc = cpu_oracle_sample(lens, bs, fmt, args.seed, args.cpu_seconds)
        cpu = {"value": gbps / 1e3, "unit": "TB/s", "cores": os.cpu_count(), "kind": "port",
               "sample": desc, "seconds": round(secs, 2)}

    graph = None
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier(device_ids=[local])
        if ex is not None:
            ex.close()
        dist.destroy_process_group()
    if rank != 0:
        return 0

    peak, peak_src = measured_peaks()
    achieved_gbs = kernel_bytes / (kern_ms * 1e-3) / 1e9
    traffic, traffic_note = ncu_traffic(split_kernel_name(fmt, bs), kernel_bytes)
    ms_per_step = elapsed_max / args.steps
    line = {
        "metric": metric_name(wl),
        "value": value_tbps, "unit": "TB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong" if seqshard else "weak",
        "vs_baseline": value_tbps / REFERENCE_PUBLISHED_TBPS,
        "vs_baseline_ref": "reference's best published Triton FP16 figure, 1.638 TB/s "
                           "(A100-80GB, B=32 ctx=16k, docs/NOTES.md:99)",
        "dtype": "f16" if fmt == "fp16" else f"{fmt} KV codes, f16 q/out, f32 math",
        "data": "synthetic (seeded N(0,1) fp16 q/K/V, random block tables)",
        "config": dict(config_dict(args.workload, wl, world, seqshard, args.exchange),
                       layers_per_step=L),
        "pct_of_b200_spec_peak": 100.0 * value_tbps * 1e3 / (B200_SPEC_GBS * world),
        "us_per_decode_step": {"one_layer": ms_per_step * 1e3 / L,
                               "llama3_8b_32_layers": ms_per_step * 1e3 * 32 / L,
                               "layers_per_step": L,
                               "32_layers": "measured" if L == 32 else f"{L} measured x {32 / L:g}"},
        "splits": S,
        "timing": ("eager calls" if graph_used is False
                   else "CUDA-graph replay of one product call per step"),
        "roofline": {"bound": "hbm",
                     "kernel": split_kernel_name(fmt, bs)
                               + " (+ PDL-chained merge_splits_kernel; timed together per call)",
                     "achieved": achieved_gbs, "peak": peak, "unit": "GB/s",
                     "frac": achieved_gbs / peak, "peak_source": peak_src,
                     "traffic": traffic, "traffic_note": traffic_note,
                     "algorithmic_bytes_per_launch": kernel_bytes,
                     "kernel_ms_per_launch": kern_ms,
                     # this rank's per-call CUDA-event times over the timed steps
                     "call_us": {"mean": kern_ms * 1e3,
                                 "median": statistics.median(call_ms) * 1e3 if call_ms else None,
                                 "min": min(call_ms) * 1e3 if call_ms else None}},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": args.steps * launches_per_step,
        "clocks": sampler.summary(),
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- reference Triton arm

def load_reference_triton():
    """The reference's src/bpt/triton_fp16.py from its offline install under baseline/_ref,
    loaded as a standalone module (the installed package is also called `bpt`)."""
    import importlib.util
    path = os.path.join(ROOT, "baseline", "_ref", "bpt", "triton_fp16.py")
    if not os.path.exists(path):
        return None, "reference not installed under baseline/_ref"
    spec = importlib.util.spec_from_file_location("bpt_reference_triton_fp16", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod, None


def run_reference_triton(args):
    """--impl reference-triton: the reference's paged_decode_attention_triton
    (src/bpt/triton_fp16.py:183-247) on this GPU over the same seeded workload as the bpt arm,
    timed per call with CUDA events (eager: the reference syncs on seq_lens.min() every call,
    so it cannot be captured in a CUDA graph). Single GPU; FP16 only (the reference has no
    quantized path). Also reports the best fixed num_splits and the max abs difference between
    its output and bpt's on the same inputs."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    wl = WORKLOADS[args.workload]
    base = {"impl": "reference-triton", "metric": metric_name(wl),
            "config": config_dict(args.workload, wl, 1)}
    if wl["fmt"] != "fp16":
        print(json.dumps({**base, "unavailable": "the reference has no quantized KV kernel"}))
        return 0
    import torch
    ref, why = load_reference_triton()
    if ref is None:
        print(json.dumps({**base, "unavailable": why}))
        return 0
    from bpt import decode as dec
    from bpt.cache import random_paged_workload
    from bpt.roofline import decode_call_bytes
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    bs = wl["block_size"]
    lens = workload_lens(wl, 0, args.seed)
    w = random_paged_workload(lens, HQ, HKV, D, bs, dev, seed=args.seed, spare_blocks=64)
    q, kc, vc, bt, sl = w["q"], w["k_cache"], w["v_cache"], w["block_table"], w["seq_lens"]
    nbytes = decode_call_bytes(lens, bs, HQ, HKV, D, "fp16")
    stream = torch.cuda.current_stream(dev)

    def timed(num_splits, steps, warmup):
        f = lambda: ref.paged_decode_attention_triton(q, kc, vc, bt, sl, num_splits=num_splits)
        for _ in range(warmup):
            f()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            f()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    ms = timed(None, args.steps, args.warmup)
    best = None
    for s in (1, 2, 4, 8, 16, 32, 64, 128):
        m = timed(s, max(3, args.steps // 4), 2)
        if best is None or m < best[1]:
            best = (s, m)
    out_ref = ref.paged_decode_attention_triton(q, kc, vc, bt, sl)
    out_bpt = dec.paged_decode_attention(q, kc, vc, bt, sl)
    torch.cuda.synchronize()
    diff = (out_ref.float() - out_bpt.float()).abs().max().item()
    peak, peak_src = measured_peaks()
    tbps = nbytes / (ms * 1e-3) / 1e12
    line = {
        **base, "value": tbps, "unit": "TB/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic (same seeded inputs as bpt)",
        "timing": "eager calls, CUDA events around K calls (the reference host-syncs per call)",
        "splits": "reference heuristic choose_num_splits",
        "frac_of_measured_hbm": tbps * 1e3 / peak, "peak_source": peak_src,
        "best_fixed_split": {"num_splits": best[0], "ms_per_step": best[1],
                             "value": nbytes / (best[1] * 1e-3) / 1e12},
        "max_abs_diff_vs_bpt": diff,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_flashinfer(args):
    """--impl flashinfer: FlashInfer's BatchDecodeWithPagedKVCacheWrapper (NHD, planned once)
    over the same seeded workload, timed per call with CUDA events over CUDA-graph replays
    like the bpt arm. A comparison point (the decode kernel a serving stack would otherwise
    call), not part of bpt. FP16, single GPU."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    wl = WORKLOADS[args.workload]
    base = {"impl": "flashinfer", "metric": metric_name(wl),
            "config": config_dict(args.workload, wl, 1)}
    if wl["fmt"] != "fp16":
        print(json.dumps({**base, "unavailable": "FlashInfer has no KIVI format"}))
        return 0
    import torch
    try:
        import flashinfer
    except Exception as e:  # noqa: BLE001
        print(json.dumps({**base, "unavailable": f"flashinfer import failed: {e}"}))
        return 0
    from bpt import decode as dec
    from bpt.cache import random_paged_workload
    from bpt.roofline import decode_call_bytes
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    bs = wl["block_size"]
    lens = workload_lens(wl, 0, args.seed)
    w = random_paged_workload(lens, HQ, HKV, D, bs, dev, seed=args.seed, spare_blocks=64)
    q, kc, vc, bt, sl = w["q"], w["k_cache"], w["v_cache"], w["block_table"], w["seq_lens"]
    pages = [(n + bs - 1) // bs for n in lens]
    indices = torch.cat([bt[b, :p] for b, p in enumerate(pages)]).to(torch.int32)
    indptr = torch.tensor([0] + list(torch.tensor(pages).cumsum(0)), dtype=torch.int32,
                          device=dev)
    last = torch.tensor([(n - 1) % bs + 1 for n in lens], dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream(dev)

    def time_mode(tensor_cores):
        """ms per call of FlashInfer's decode wrapper in one mode (CUDA-graph replays)."""
        fi = flashinfer.BatchDecodeWithPagedKVCacheWrapper(
            torch.empty(256 << 20, dtype=torch.uint8, device=dev), "NHD",
            use_tensor_cores=tensor_cores)
        fi.plan(indptr, indices, last, HQ, HKV, D, bs, q_data_type=torch.float16,
                kv_data_type=torch.float16)
        call = lambda: fi.run(q, (kc, vc), out=out)  # noqa: E731
        call()
        torch.cuda.synchronize()
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            call()
        stream.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(graph):
                call()
            step, how = graph.replay, "CUDA-graph replay of one call per step"
        except Exception:  # noqa: BLE001
            graph, step, how = None, call, "eager calls"
        for _ in range(max(args.warmup, 1)):
            step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        del graph
        return e0.elapsed_time(e1) / args.steps, how

    modes = {}
    for tc in (False, True):
        try:
            modes["tensor_cores" if tc else "cuda_cores"] = time_mode(tc)
        except Exception as e:  # noqa: BLE001
            modes["tensor_cores" if tc else "cuda_cores"] = (None, f"failed: {e}"[:200])
    best = min((v for v in modes.values() if v[0] is not None), key=lambda v: v[0])
    ms, timing = best
    nbytes = decode_call_bytes(lens, bs, HQ, HKV, D, "fp16")
    mine = dec.paged_decode_attention(q, kc, vc, bt, sl)
    torch.cuda.synchronize()
    peak, peak_src = measured_peaks()
    tbps = nbytes / (ms * 1e-3) / 1e12
    print(json.dumps({**base, "value": tbps, "unit": "TB/s", "n_gpus": 1, "steps": args.steps,
                      "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                      "scaling": "weak", "vs_baseline": None, "dtype": "f16",
                      "data": "synthetic (same seeded inputs as bpt)", "timing": timing,
                      "flashinfer_version": getattr(flashinfer, "__version__", "?"),
                      "modes_ms_per_step": {k: v[0] for k, v in modes.items()},
                      "frac_of_measured_hbm": tbps * 1e3 / peak, "peak_source": peak_src,
                      "max_abs_diff_vs_bpt": (out.float() - mine.float()).abs().max().item()}),
          flush=True)
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.impl == "reference-triton":
        return run_reference_triton(args)
    if args.impl == "flashinfer":
        return run_flashinfer(args)
    return run_bpt(args)


if __name__ == "__main__":
    sys.exit(main())
