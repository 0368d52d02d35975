#!/usr/bin/env python
"""bpt benchmark: achieved HBM bandwidth of paged-KV GQA decode on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl bpt|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU, NCCL)

A step is one single-layer decode call over one batch (Llama-3-8B layer: Hq=32, Hkv=8, D=128)
of synthetic paged KV with seeded ragged lengths and a random-permutation block table, inputs
resident in HBM. Multi-GPU runs shard by batch (each rank owns its own batch and KV pool, no
collective on the data path): weak scaling; the time is the max over ranks.

Prints ONE JSON line (rank 0). `value` is the whole-job achieved bandwidth in TB/s:
algorithmic bytes of all ranks' calls / max-over-ranks device time. Besides the contract keys:

* `parity`: after timing, sampled sequences (every q head) of the timed call's own output are
  checked against the reference's paged_decode_attention_ref (src/bpt/reference.py:20-49, from
  the offline install under baseline/_ref, run on the GPU in fp32; a torch restatement of it
  when the install is absent) at max abs 2e-3 / max rel 1e-2. A miss makes the exit status 1.
* `roofline`: the dominant kernel (the split-KV decode kernel + its merge) against the
  measured HBM copy peak.
* `e2e`: the same metric through the public API with per-step host->device copies of the
  step's inputs (q, block table, sequence lengths) from pinned memory and a device->host read
  of the output (the KV cache is resident state, like weights), replayed as a CUDA graph;
  `e2e_eager` is the same step as plain eager Python calls of the public API.
* `sweep` (N=1): the other BASELINE points (batch 1 at 4k-128k, B=8/16k, INT8/FP8/INT4 at
  B=1/128k and B=32/32k). Each is a decode step over L independent layers (own cache, q and
  table; L=32 = a whole Llama-3-8B step where it fits in memory) replayed as one CUDA graph,
  so the working set of a step is >= 1 GB and L2 never holds it; each point is parity-checked
  like the headline.
* `seqshard` (N>1): batch-1 / 128k-token sequences sharded over the ranks (FP16 and INT4
  through the fused NVLink exchange, FP16 through one NCCL all-gather), with the split kernel
  timed alone beside the whole call.
* `cpu_baseline` and `--impl reference`: the reference's own CPU path (its
  paged_decode_attention_ref on CPU torch tensors, all host threads) on whole sequences of the
  workload at their true lengths; the numpy oracle port when the reference is not installed.
"""
import argparse
import importlib.util
import json
import math
import os
import random
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
# BASELINE tolerance on fp16 outputs; rel as the reference computes it
# (tests/test_triton_fp16.py:39 of the reference: diff / ref.abs().clamp_min(1e-3))
ATOL, RTOL = 2e-3, 1e-2

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
# the default line's sweep (N=1): every other BASELINE configuration family's points
SWEEP = ["fp16_b1_ctx4k", "fp16_b1_ctx16k", "fp16_b1_ctx64k", "fp16_b1_ctx128k",
         "fp16_b8_ctx16k", "int8_b1_ctx128k", "fp8_b1_ctx128k", "int4_b1_ctx128k",
         "int8_b32_ctx32k", "fp8_b32_ctx32k", "int4_b32_ctx32k"]
# the multi-GPU line's sequence-sharding points (workload, exchange)
SEQSHARD = [("fp16_b1_ctx128k", "nvlink"), ("int4_b1_ctx128k", "nvlink"),
            ("fp16_b1_ctx128k", "nccl")]
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
                    help="reference: the reference's CPU path (its torch oracle, installed "
                         "under baseline/_ref; the numpy port when absent) on the host cores; "
                         "reference-triton: the reference's own Triton FP16 kernel on this "
                         "GPU, same inputs; flashinfer: FlashInfer's paged decode (the library "
                         "in this image) on this GPU, same inputs")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=DEFAULT_WORKLOAD)
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-sweep", action="store_true",
                    help="skip the sweep (N=1) / sequence-sharding (N>1) sub-benchmarks")
    ap.add_argument("--sweep", default=",".join(SWEEP),
                    help="comma-separated sweep workloads (N=1)")
    ap.add_argument("--parity-seqs", type=int, default=8,
                    help="sequences of the headline output checked against the reference")
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
        "l2": l2_note(wl),
    }


def l2_note(wl, layers=1):
    """How the timing keeps L2 (126 MB) from holding the step's working set."""
    from bpt.roofline import KIVI_FORMATS
    f = KIVI_FORMATS[wl["fmt"]]
    per_token = HKV * (2 * D * f.elem_bytes + D * f.k_group_bytes / wl["block_size"]
                       + f.v_token_bytes)
    gb = wl["batch"] * wl["ctx"] * per_token * layers / 1e9
    if gb >= 1.0:
        return (f"no flush: the per-step working set (~{gb:.1f} GB of KV) far exceeds the "
                "126 MB L2")
    return (f"no flush, per-step working set ~{gb * 1e3:.0f} MB: use --layers to rotate over "
            "distinct caches (the sweep's B=1 points do)")


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
            self._stop.clear()
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


def metric_name(wl):
    return (f"achieved HBM TB/s of {wl['fmt']} paged-KV GQA decode "
            f"(Llama-3-8B layer; % of B200 peak and us/decode step in extra keys)")


# ----------------------------------------------------------------------------- the reference

def load_reference_module(name):
    """src/bpt/<name>.py of the reference from its offline install under baseline/_ref, loaded
    as a standalone module (the installed package is also called `bpt`). (module, None) or
    (None, why)."""
    path = os.path.join(ROOT, "baseline", "_ref", "bpt", name + ".py")
    if not os.path.exists(path):
        return None, "reference not installed under baseline/_ref"
    try:
        spec = importlib.util.spec_from_file_location(f"bpt_reference_{name}", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        return mod, None
    except Exception as e:  # noqa: BLE001
        return None, f"loading the reference's {name}.py failed: {e}"[:200]


# ----------------------------------------------------------------------------- GPU parity checker

def torch_reference(q, k_cache, v_cache, block_table, seq_lens, scale=None):
    """fp32 torch restatement of the reference's paged_decode_attention_ref
    (src/bpt/reference.py:20-49): per sequence, gather its pages, fp32 softmax attention of
    each q head over its kv head. The checker when the reference is not installed."""
    import torch
    B, Hq, Dh = q.shape
    _, bs, Hkv, _ = k_cache.shape
    group = Hq // Hkv
    scale = scale or Dh ** -0.5
    out = torch.empty(B, Hq, Dh, dtype=torch.float32, device=q.device)
    for b in range(B):
        n = int(seq_lens[b])
        blocks = block_table[b, :(n + bs - 1) // bs].long()
        k = k_cache[blocks].reshape(-1, Hkv, Dh)[:n].float()
        v = v_cache[blocks].reshape(-1, Hkv, Dh)[:n].float()
        s = torch.einsum("hgd,nhd->hgn", q[b].float().reshape(Hkv, group, Dh), k) * scale
        out[b] = torch.einsum("hgn,nhd->hgd", torch.softmax(s, dim=-1), v).reshape(Hq, Dh)
    return out


def reference_checker():
    """(fn, description): the reference's own oracle when installed, else the restatement."""
    mod, _ = load_reference_module("reference")
    if mod is not None:
        return (mod.paged_decode_attention_ref,
                "the reference's paged_decode_attention_ref (src/bpt/reference.py:20-49, "
                "installed under baseline/_ref), fp32 math on the GPU")
    return (torch_reference, "fp32 torch restatement of src/bpt/reference.py:20-49 on the GPU "
                             "(reference not installed)")


def dequant_pages(cache, pages):
    """fp32 K and V pages [P, bs, H, D] of a KIVI cache, x = code * scale + zero (FP8:
    e4m3 * scale): the dequantized cache the fused kernels must match."""
    import torch
    kc, vc = cache.k_codes[pages], cache.v_codes[pages]
    if cache.fmt == "int4":   # keys: low nibble = even channel; values: low nibble = even token
        kc = torch.stack([kc & 0xF, kc >> 4], dim=-1).reshape(*kc.shape[:3], -1)
        vc = torch.stack([vc & 0xF, vc >> 4], dim=2).reshape(vc.shape[0], -1, *vc.shape[2:])
    ks = cache.k_scale[pages].float()[:, None]
    vs = cache.v_scale[pages].float()[..., None]
    if cache.fmt == "fp8":
        return (kc.view(torch.float8_e4m3fn).float() * ks,
                vc.view(torch.float8_e4m3fn).float() * vs)
    return (kc.float() * ks + cache.k_zero[pages].float()[:, None],
            vc.float() * vs + cache.v_zero[pages].float()[..., None])


def sequence_kv(layer, fmt, b, lo=0, hi=None):
    """fp32 K, V [n, Hkv, D] of tokens [lo, hi) of sequence b of a layer (gathered pages)."""
    import torch
    n = int(layer["seq_lens"][b])
    hi = n if hi is None else min(hi, n)
    if fmt == "fp16":
        bs = layer["k_cache"].shape[1]
        blocks = layer["block_table"][b, :(n + bs - 1) // bs].long()
        k = layer["k_cache"][blocks].reshape(-1, HKV, D)[lo:hi].float()
        v = layer["v_cache"][blocks].reshape(-1, HKV, D)[lo:hi].float()
        return k, v
    cache = layer["cache"]
    bs = cache.block_size
    kd, vd = dequant_pages(cache, layer["block_table"][b, :(n + bs - 1) // bs].long())
    return kd.reshape(-1, HKV, D)[lo:hi], vd.reshape(-1, HKV, D)[lo:hi]


def check_outputs(fmt, layer, out, seqs, checker):
    """max abs / max rel of out[seqs] (all q heads) against the checker, for a decode over a
    FP16 cache or a KIVI cache (the checker then runs on the dequantized pages)."""
    import torch
    fn, _ = checker
    q, bt, sl = layer["q"], layer["block_table"], layer["seq_lens"]
    max_abs = max_rel = 0.0
    finite = True
    for b in seqs:
        if fmt == "fp16":
            ref = fn(q[b:b + 1].float(), layer["k_cache"], layer["v_cache"], bt[b:b + 1],
                     sl[b:b + 1])
        else:
            n = int(sl[b])
            bs = layer["cache"].block_size
            kd, vd = dequant_pages(layer["cache"], bt[b, :(n + bs - 1) // bs].long())
            local = torch.arange(kd.shape[0], dtype=torch.int32, device=q.device)[None]
            ref = fn(q[b:b + 1].float(), kd, vd, local, sl[b:b + 1])
            del kd, vd
        o = out[b:b + 1].float()
        finite = finite and bool(torch.isfinite(o).all())
        d = (o - ref.float()).abs()
        max_abs = max(max_abs, d.max().item())
        max_rel = max(max_rel, (d / ref.float().abs().clamp_min(1e-3)).max().item())
    return {"max_abs": max_abs, "max_rel": max_rel, "sequences": len(seqs),
            "rows": len(seqs) * q.shape[1], "atol": ATOL, "rtol": RTOL,
            "ok": bool(finite and max_abs < ATOL and max_rel < RTOL)}


def merge_parity(*ps):
    return {"max_abs": max(p["max_abs"] for p in ps), "max_rel": max(p["max_rel"] for p in ps),
            "sequences": sum(p["sequences"] for p in ps), "rows": sum(p["rows"] for p in ps),
            "atol": ATOL, "rtol": RTOL, "ok": all(p["ok"] for p in ps)}


def sample_seqs(batch, k, seed):
    """k distinct sequence indices (seeded), always including the first and the last."""
    if batch <= k:
        return list(range(batch))
    rest = random.Random(seed).sample(range(1, batch - 1), k - 2)
    return sorted([0, batch - 1] + rest)


# ----------------------------------------------------------------------------- CPU baselines

def oracle_sample_inputs(n, block_size, fmt, seed):
    """One sequence of n tokens for the CPU paths (numpy): (q, kv, bt, sl). FP16 gives fp16
    pages; quantized formats give the KIVI *codes* cache (the timed step dequantizes it)."""
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


def cpu_path():
    """The CPU implementation timed as the reference: (kind, step(q, kv, bt, sl, fmt), what,
    threads). 'reference' = the reference's paged_decode_attention_ref on CPU torch tensors
    with every host thread; 'port' = the numpy oracle (when the reference is not installed)."""
    import numpy as np
    from oracle import kivi
    mod, _ = load_reference_module("reference")
    if mod is not None:
        import torch
        threads = os.cpu_count()
        torch.set_num_threads(threads)

        def step(q, kv, bt, sl, fmt):
            if fmt == "fp16":
                kc, vc = torch.from_numpy(kv[0]), torch.from_numpy(kv[1])
            else:
                kd, vd = kivi.dequantize_cache(kv, fmt)
                kc, vc = torch.from_numpy(kd), torch.from_numpy(vd)
            return mod.paged_decode_attention_ref(torch.from_numpy(q), kc, vc,
                                                  torch.from_numpy(bt), torch.from_numpy(sl))
        what = ("the reference's paged_decode_attention_ref (src/bpt/reference.py:20-49, "
                f"installed under baseline/_ref) on CPU torch tensors, {threads} threads")
        return "reference", step, what, threads

    from oracle import attention as oa

    def step(q, kv, bt, sl, fmt):
        if fmt == "fp16":
            return oa.paged_decode_attention_ref(q, kv[0], kv[1], bt, sl)
        kd, vd = kivi.dequantize_cache(kv, fmt)
        return oa.paged_decode_attention_ref(q, kd, vd, bt, sl, out_dtype=np.float16)
    return ("port", step, "numpy port of src/bpt/reference.py:20-49 (oracle/, the reference is "
            "not installed under baseline/_ref), numpy BLAS threads = host cores",
            os.cpu_count())


def cpu_pool(wl, lens, seed):
    """The sampled sequences of the workload, whole, at their true lengths: up to two
    distinct sequences (rotated through by the timed steps)."""
    bs, fmt = wl["block_size"], wl["fmt"]
    picks = [int(n) for n in lens[:2]]
    return [oracle_sample_inputs(n, bs, fmt, seed + i) for i, n in enumerate(picks)]


def cpu_sample_desc(pool, fmt, what):
    ns = [int(p[3][0]) for p in pool]
    return (f"each step = one whole sequence of the workload at its true length ({ns} tokens, "
            f"rotating), {what}" + ("" if fmt == "fp16" else
                                    "; KIVI: the numpy dequantization of the spec first"))


def cpu_reference_sample(wl, lens, seed, budget_s):
    """cpu_baseline of the bpt arm: the CPU path on whole sequences until ~budget_s seconds.
    Returns (TB/s, seconds, kind, cores, sample)."""
    from bpt.roofline import decode_call_bytes
    kind, step, what, threads = cpu_path()
    bs, fmt = wl["block_size"], wl["fmt"]
    pool = cpu_pool(wl, lens, seed)
    step(*pool[0], fmt)  # warm-up
    done, nbytes, t0 = 0, 0, time.perf_counter()
    while True:
        p = pool[done % len(pool)]
        step(*p, fmt)
        nbytes += decode_call_bytes([int(p[3][0])], bs, HQ, HKV, D, fmt)
        done += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return (nbytes / dt / 1e12, dt, kind, threads,
            f"{done} steps; " + cpu_sample_desc(pool, fmt, what))


def run_reference(args):
    """--impl reference: the reference's CPU path on the host cores (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    wl = WORKLOADS[args.workload]
    lens = workload_lens(wl, 0, args.seed)
    from bpt.roofline import decode_call_bytes
    bs, fmt = wl["block_size"], wl["fmt"]
    kind, step, what, threads = cpu_path()
    pool = cpu_pool(wl, lens, args.seed)
    for i in range(args.warmup):
        step(*pool[i % len(pool)], fmt)
    t0 = time.perf_counter()
    nbytes = 0
    for i in range(args.steps):
        p = pool[i % len(pool)]
        step(*p, fmt)
        nbytes += decode_call_bytes([int(p[3][0])], bs, HQ, HKV, D, fmt)
    dt = time.perf_counter() - t0
    tbps = nbytes / dt / 1e12
    line = {
        "impl": "reference", "metric": metric_name(wl), "value": tbps, "unit": "TB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / max(args.steps, 1) * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(args.workload, wl, args.gpus),
        "cpu_baseline": {"value": tbps, "unit": "TB/s", "cores": threads, "kind": kind,
                         "sample": cpu_sample_desc(pool, fmt, what)},
        "e2e": {"value": tbps, "unit": "TB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- bpt helpers

def build_layer(wl, lens, seed, dev):
    """One layer's decode inputs on the device (random-permutation table, 64 spare blocks)."""
    import torch
    from bpt.cache import random_paged_workload
    from bpt.quant import random_kivi_workload
    if wl["fmt"] == "fp16":
        w = random_paged_workload(lens, HQ, HKV, D, wl["block_size"], dev, seed=seed,
                                  spare_blocks=64)
    else:
        w = random_kivi_workload(lens, HQ, HKV, D, wl["block_size"], wl["fmt"], dev, seed=seed,
                                 spare_blocks=64)
    w["out"] = torch.empty_like(w["q"])
    return w


def layer_splits(wl, layer, forced, sms):
    from bpt import decode as dec
    B, max_blocks = layer["block_table"].shape
    if wl["fmt"] == "fp16":
        return dec.effective_splits(B, HKV, wl["block_size"], max_blocks, forced or None, sms)
    from bpt.quant import effective_splits_kivi
    return effective_splits_kivi(layer["cache"], B, HQ, max_blocks, forced or None, sms)


def layer_call(fmt, layer, S, ws):
    """One product call into layer['out'] (split-KV kernel + its PDL-chained merge)."""
    from bpt import decode as dec
    from bpt.quant import paged_decode_attention_kivi
    if fmt == "fp16":
        return lambda: dec.paged_decode_attention(
            layer["q"], layer["k_cache"], layer["v_cache"], layer["block_table"],
            layer["seq_lens"], num_splits=S, out=layer["out"], workspace=ws)
    return lambda: paged_decode_attention_kivi(layer["q"], layer["cache"], layer["block_table"],
                                               layer["seq_lens"], num_splits=S,
                                               out=layer["out"], workspace=ws)


def plain_call(fmt, layer):
    """The plainest public-API call a drop-in caller makes (fresh output and workspace)."""
    from bpt import paged_decode_attention
    from bpt.quant import paged_decode_attention_kivi
    if fmt == "fp16":
        return lambda: paged_decode_attention(layer["q"], layer["k_cache"], layer["v_cache"],
                                              layer["block_table"], layer["seq_lens"])
    return lambda: paged_decode_attention_kivi(layer["q"], layer["cache"], layer["block_table"],
                                               layer["seq_lens"])


def capture(fn, dev):
    """A CUDA graph of fn(), after one eager call and one warm-up on a side stream."""
    import torch
    stream = torch.cuda.current_stream(dev)
    fn()
    torch.cuda.synchronize()
    side = torch.cuda.Stream(dev)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        fn()
    stream.wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


def time_steps(step, steps, warmup, dev, barrier=lambda: None):
    """ms of `steps` back-to-back steps between two CUDA events on the launch stream, after
    `warmup` untimed steps; barrier + synchronize on both sides."""
    import torch
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(warmup, 0)):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    return e0.elapsed_time(e1)


def e2e_measure(layers, fmt, calls, steps, warmup, dev, nbytes, graph, barrier=lambda: None,
                reduce_max=lambda x: x):
    """End to end through the public API: every step uploads each layer's q, block table and
    sequence lengths from pinned host memory, makes the calls, and reads each output back into
    pinned host memory. graph=True replays the whole step as one CUDA graph (a serving
    engine's decode step); graph=False makes plain eager calls (`calls` are then the plainest
    public-API calls, fresh output each). Checks that the last read-back equals the device
    output."""
    import torch
    live_in = [(w["q"], w["block_table"], w["seq_lens"]) for w in layers]
    host_in = [tuple(t.cpu().pin_memory() for t in trio) for trio in live_in]
    host_out = [torch.empty(w["q"].shape, dtype=torch.float16).pin_memory() for w in layers]
    last = [None] * len(layers)

    def e2e_step():
        for lv, hs in zip(live_in, host_in):
            for d, h in zip(lv, hs):
                d.copy_(h, non_blocking=True)
        for i, c in enumerate(calls):
            o = c()
            last[i] = o
            host_out[i].copy_(o, non_blocking=True)

    run = capture(e2e_step, dev).replay if graph else e2e_step
    ms = reduce_max(time_steps(run, steps, max(warmup, 1), dev, barrier))
    assert torch.equal(host_out[0], last[0].cpu()), "e2e read-back mismatch"
    return {"value": nbytes * steps / (ms * 1e-3) / 1e12, "unit": "TB/s",
            "h2d_bytes_per_step": sum(t.nbytes for trio in live_in for t in trio),
            "d2h_bytes_per_step": sum(h.nbytes for h in host_out),
            "ms_per_step": ms / steps,
            "note": ("public API (bpt.paged_decode_attention / paged_decode_attention_kivi) "
                     "with each step's input upload from pinned host memory and result "
                     "read-back, " + ("captured as one CUDA graph replayed per step"
                                      if graph else "plain eager Python calls")
                     + "; KV cache resident in HBM")}


def sweep_layers(step_bytes):
    """Layers per sweep step: 32 (a whole Llama-3-8B decode step) when they fit in ~24 GB,
    raised to reach a >= 1 GB working set for the smallest layers; layers too large for 32 of
    them get enough for a >= 4 GB working set."""
    if 32 * step_bytes <= 24e9:
        return max(32, math.ceil(1e9 / step_bytes))
    return max(1, math.ceil(4e9 / step_bytes))


def run_sweep_point(name, args, dev, sms, checker, peak):
    """One sweep point: L independent layers replayed as one CUDA graph per step."""
    import torch
    from bpt import decode as dec
    from bpt.roofline import decode_call_bytes
    wl = WORKLOADS[name]
    fmt = wl["fmt"]
    lens = workload_lens(wl, 0, args.seed)
    one = decode_call_bytes(lens, wl["block_size"], HQ, HKV, D, fmt)
    L = sweep_layers(one)
    layers = [build_layer(wl, lens, args.seed + 1009 * i, dev) for i in range(L)]
    S = layer_splits(wl, layers[0], 0, sms)
    ws = torch.empty(dec.workspace_bytes(len(lens), HQ, D, S), dtype=torch.uint8, device=dev)
    calls = [layer_call(fmt, w, S, ws) for w in layers]

    def step():
        for c in calls:
            c()
    g = capture(step, dev)
    ms = time_steps(g.replay, args.steps, args.warmup, dev)
    us_layer = ms * 1e3 / args.steps / L
    tbps = one / (us_layer * 1e-6) / 1e12
    seqs = sample_seqs(len(lens), 2, args.seed)
    parity = merge_parity(check_outputs(fmt, layers[0], layers[0]["out"], seqs, checker),
                          check_outputs(fmt, layers[-1], layers[-1]["out"], seqs, checker))
    res = {"layers": L, "splits": S, "us_per_step": us_layer * L, "us_per_layer": us_layer,
           "tbps": tbps, "frac_of_measured_hbm": tbps * 1e3 / peak,
           "pct_of_b200_spec_peak": 100.0 * tbps * 1e3 / B200_SPEC_GBS,
           "bytes_per_layer": one, "working_set_gb": one * L / 1e9,
           "kernel": split_kernel_name(fmt, wl["block_size"]), "parity": parity}
    del g
    if name == "fp16_b1_ctx64k" and not args.no_e2e:
        res["e2e"] = e2e_measure(layers, fmt, [layer_call(fmt, w, S, ws) for w in layers],
                                 args.steps, args.warmup, dev, one * L, graph=True)
        res["e2e_eager"] = e2e_measure(layers, fmt, [plain_call(fmt, w) for w in layers],
                                       args.steps, args.warmup, dev, one * L, graph=False)
    del layers, calls, ws
    torch.cuda.empty_cache()
    return res


def run_sweep(args, dev, sms, checker, peak, local):
    names = [n for n in args.sweep.split(",") if n]
    out, t0 = {}, time.perf_counter()
    sampler = ClockSampler(local)
    with sampler:
        for n in names:
            out[n] = run_sweep_point(n, args, dev, sms, checker, peak)
    res = {"method": "per point: L independent layers (own KV cache, q, block table) per step, "
                     "one CUDA graph per step replayed back to back; working set >= 1 GB per "
                     "step, so L2 (126 MB) never holds it; us_per_layer = step time / L",
           "points": out, "clocks": sampler.summary(), "seconds": time.perf_counter() - t0}
    if "fp16_b1_ctx128k" in out and "int4_b1_ctx128k" in out:
        res["int4_vs_fp16_latency_128k"] = (out["fp16_b1_ctx128k"]["us_per_layer"]
                                            / out["int4_b1_ctx128k"]["us_per_layer"])
    res["accuracy"] = run_accuracy(args, dev)
    return res


def run_accuracy(args, dev, ctx=131072):
    """The KIVI formats' accuracy at 128k tokens through the decode kernels (bpt.accuracy):
    needle weight recovered per q head, and output error against the fp16 cache."""
    import torch
    from bpt.accuracy import needle_inputs, needle_study, summarize
    inputs = needle_inputs(ctx, seed=args.seed, device=dev)
    out = {"method": "needle in a BASELINE-distribution haystack (4 x10 outlier key channels "
                     "per kv head), one sequence of 131072 tokens, block_size 64; weights "
                     "measured through the kernels (two decodes differing only in the needle's "
                     "value); output error of each format against bpt's fp16 decode"}
    for fmt in ("int8", "fp8", "int4"):
        out[fmt] = summarize(needle_study(fmt, ctx, inputs=inputs))
    del inputs
    torch.cuda.empty_cache()
    return out


def torch_partial_state(q_b, k, v):
    """fp32 normalised partial attention of q_b [Hq, D] over k, v [n, Hkv, D]: (o [Hq, D],
    lse [Hq], natural log). Empty -> o = 0, lse = -inf (the reference split kernel's state,
    src/bpt/triton_fp16.py:138-144)."""
    import torch
    if k.shape[0] == 0:
        return (torch.zeros(HQ, D, device=q_b.device),
                torch.full((HQ,), float("-inf"), device=q_b.device))
    s = torch.einsum("hgd,nhd->hgn", q_b.float().reshape(HKV, HQ // HKV, D), k) * D ** -0.5
    m = s.amax(dim=-1, keepdim=True)
    e = torch.exp(s - m)
    l = e.sum(dim=-1, keepdim=True)
    o = torch.einsum("hgn,nhd->hgd", e, v) / l
    return o.reshape(HQ, D), (m + torch.log(l)).reshape(HQ)


def run_seqshard_point(name, exchange, args, world, rank, local, dev, sms):
    """Sequence sharding at this world size: rank r decodes its page-aligned token range of
    each sequence; the states merge through the fused NVLink exchange (one kernel, graph
    replays) or one NCCL all-gather (eager). Also times the split kernel alone, and checks the
    output against fp32 partial states of every rank's tokens merged in float64."""
    import torch
    import torch.distributed as dist
    from bpt import decode as dec
    from bpt.dist import SequenceShardExchange, decode_sequence_sharded, token_shards
    from bpt.quant import paged_decode_attention_kivi_partial
    from bpt.roofline import decode_call_bytes
    wl = WORKLOADS[name]
    fmt, bs = wl["fmt"], wl["block_size"]
    full = workload_lens(wl, 0, args.seed)
    ranges = [token_shards(n, bs, world)[rank] for n in full]
    lens = [hi - lo for lo, hi in ranges]
    L = 32
    layers = []
    for i in range(L):
        w = build_layer(wl, lens, args.seed + rank + 1009 * i, dev)
        g = torch.Generator(device=dev).manual_seed(args.seed + 1009 * i)   # same q on all ranks
        w["q"] = torch.randn(w["q"].shape, generator=g, device=dev).to(torch.float16)
        layers.append(w)
    S = layer_splits(wl, layers[0], 0, sms)
    ex = SequenceShardExchange(len(lens), HQ, D) if exchange == "nvlink" else None

    def barrier():
        dist.barrier(device_ids=[local])

    def reduce_max(x):
        t = torch.tensor([float(x)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def call(w):
        return decode_sequence_sharded(w["q"], w.get("k_cache"), w.get("v_cache"),
                                       w["block_table"], w["seq_lens"], num_splits=S,
                                       out=w["out"], kivi_cache=w.get("cache"), exchange=ex)

    def partial(w):
        if fmt == "fp16":
            return dec.paged_decode_attention_partial(w["q"], w["k_cache"], w["v_cache"],
                                                      w["block_table"], w["seq_lens"],
                                                      num_splits=S)
        return paged_decode_attention_kivi_partial(w["q"], w["cache"], w["block_table"],
                                                   w["seq_lens"], num_splits=S)

    def step():
        for w in layers:
            call(w)

    def split_step():
        for w in layers:
            partial(w)
    graphs = []
    if ex is not None:
        graphs.append(capture(step, dev))
        run = graphs[-1].replay
    else:
        step()
        run = step
    ms = reduce_max(time_steps(run, args.steps, args.warmup, dev, barrier))
    graphs.append(capture(split_step, dev))
    ms_split = reduce_max(time_steps(graphs[-1].replay, args.steps, args.warmup, dev, barrier))
    # parity: every rank's fp32 state of its own tokens (layer 0), gathered, merged in float64
    w0 = layers[0]
    states = []
    for b in range(len(lens)):
        k, v = sequence_kv(w0, fmt, b)
        o, lse = torch_partial_state(w0["q"][b], k, v)
        states.append(torch.cat([o.reshape(-1), lse]))
    mine = torch.stack(states).reshape(-1).contiguous()
    allst = torch.empty(world * mine.numel(), dtype=torch.float32, device=dev)
    dist.all_gather_into_tensor(allst, mine)
    allst = allst.view(world, len(lens), HQ * D + HQ).double()
    o_r, lse_r = allst[..., :HQ * D].view(world, len(lens), HQ, D), allst[..., HQ * D:]
    mx = lse_r.amax(dim=0, keepdim=True)
    wts = torch.exp(lse_r - mx)
    ref = (wts[..., None] * o_r).sum(0) / wts.sum(0)[..., None]
    d = (w0["out"].double() - ref).abs()
    max_abs = reduce_max(d.max().item())
    max_rel = reduce_max((d / ref.abs().clamp_min(1e-3)).max().item())
    nonfinite = reduce_max(0.0 if bool(torch.isfinite(w0["out"]).all()) else 1.0)
    parity = {"max_abs": max_abs, "max_rel": max_rel, "rows": len(lens) * HQ, "atol": ATOL,
              "rtol": RTOL, "ok": bool(nonfinite == 0 and max_abs < ATOL and max_rel < RTOL),
              "checker": "fp32 torch partial states of each rank's tokens (the reference "
                         "split kernel's (o, lse), src/bpt/triton_fp16.py:138-144), gathered "
                         "and merged in float64"}
    one = decode_call_bytes(full, bs, HQ, HKV, D, fmt)
    us = ms * 1e3 / args.steps / L
    us_split = ms_split * 1e3 / args.steps / L
    torch.cuda.synchronize()
    barrier()
    del graphs
    if ex is not None:
        ex.close()
    del layers
    torch.cuda.empty_cache()
    return {"exchange": exchange, "ranks": world, "layers": L, "splits_per_rank": S,
            "tokens_per_rank": max(lens), "us_per_layer": us, "tbps": one / (us * 1e-6) / 1e12,
            "split_kernel_us_per_layer": us_split,
            "exchange_us_per_layer": us - us_split,
            "timing": ("CUDA-graph replays of 32 layers (split kernel + fused exchange kernel "
                       "each)" if exchange == "nvlink" else
                       "eager: 32 layers of split + state merge + NCCL all-gather + rank merge"),
            "parity": parity}


# ----------------------------------------------------------------------------- bpt arm

def run_bpt(args):
    import torch
    import torch.distributed as dist
    from bpt import decode as dec
    from bpt.roofline import decode_call_bytes

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

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def reduce_max(x):
        if world == 1:
            return x
        t = torch.tensor([float(x)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

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
    L = max(1, args.layers)
    if L > 1 and seqshard:
        raise SystemExit("--layers > 1 is not combined with --seqshard")
    # layer 0 is the headline's; layers 1 .. L-1 have their own caches, queries and tables
    layers = [build_layer(wl, lens, args.seed + rank + 1009 * li, dev) for li in range(L)]
    w = layers[0]
    if seqshard:  # every rank decodes the same queries against its own token shard
        w["q"] = torch.randn(w["q"].shape,
                             generator=torch.Generator(device=dev).manual_seed(args.seed),
                             device=dev).to(torch.float16)
    q, bt, sl, out = w["q"], w["block_table"], w["seq_lens"], w["out"]
    B = len(lens)
    sms = dec._sm_count(local)
    S = layer_splits(wl, w, args.splits, sms)
    # algorithmic bytes of this rank's share of the job (seqshard: its tokens of the sequences,
    # plus q/out once on rank 0 so the job total counts them once)
    step_bytes = decode_call_bytes(lens, bs, HQ, HKV, D, fmt) * L
    if seqshard and rank != 0:
        step_bytes -= len(lens) * HQ * D * 2 * 2
    kernel_bytes = step_bytes
    ws = torch.empty(dec.workspace_bytes(B, HQ, D, S), dtype=torch.uint8, device=dev)
    ex = None
    if seqshard and args.exchange == "nvlink":
        from bpt.dist import SequenceShardExchange
        ex = SequenceShardExchange(B, HQ, D)
    # split kernel (+ PDL merge); sequence sharding: split + fused exchange, or split + state
    # merge + NCCL all-gather + rank merge
    launches_per_step = ((2 if ex is not None else 4) if seqshard else (2 if S > 1 else 1)) * L
    stream = torch.cuda.current_stream(dev)
    calls = [layer_call(fmt, lw, S, ws) for lw in layers]
    if seqshard:
        calls = [lambda: decode_sequence_sharded(
            q, w.get("k_cache"), w.get("v_cache"), bt, sl, num_splits=S, out=out,
            kivi_cache=w.get("cache"), exchange=ex)]

    def call():
        # the layers run in order on one stream and share the workspace
        for c in calls:
            c()

    # The device-timed leg replays the call as a CUDA graph (what a serving engine does with a
    # decode step), so host-side Python cost does not leak into small workloads' timing.
    graph = None
    if not args.eager and not (seqshard and ex is None):  # an NCCL all-gather step: eager
        graph = capture(call, dev)
    graph_used = graph is not None
    step = graph.replay if graph is not None else call

    for _ in range(max(args.warmup, 0)):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
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
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    for a, b in evs:
        a.record(stream)
        step()
        b.record(stream)
    torch.cuda.synchronize()
    barrier()
    call_ms = [a.elapsed_time(b) for a, b in evs]
    kern_ms = sum(call_ms) / max(args.steps, 1)

    elapsed_max = reduce_max(elapsed_ms)
    if world > 1:
        b_sum = torch.tensor([float(step_bytes * args.steps)], dtype=torch.float64, device=dev)
        dist.all_reduce(b_sum, op=dist.ReduceOp.SUM)
        bytes_all = float(b_sum.item())
    else:
        bytes_all = float(step_bytes * args.steps)
    value_tbps = bytes_all / (elapsed_max * 1e-3) / 1e12

    # ---- parity of the timed call's own output (the last replay wrote every layer's out)
    checker = reference_checker()
    if seqshard:
        parity = None   # the sequence-sharded headline is checked by the seqshard suite's code
    else:
        seqs = sample_seqs(B, args.parity_seqs, args.seed + rank)
        parity = check_outputs(fmt, w, out, seqs, checker)
        if L > 1:
            parity = merge_parity(parity, check_outputs(fmt, layers[-1], layers[-1]["out"],
                                                        seqs, checker))
        if world > 1:
            parity["max_abs"] = reduce_max(parity["max_abs"])
            parity["max_rel"] = reduce_max(parity["max_rel"])
            parity["ok"] = reduce_max(0.0 if parity["ok"] else 1.0) == 0.0
            parity["sequences"] *= world
            parity["rows"] *= world
        parity["checker"] = checker[1]
        parity["sampled"] = (f"{len(seqs)} sequences x all {HQ} q heads per rank (seeded "
                             "sample incl. the first and last sequence)")

    # ---- e2e through the public API, host buffers, copies inside the timed region
    e2e = e2e_eager = None
    if not args.no_e2e:
        nbytes_step = bytes_all / args.steps
        if seqshard:
            e2e = e2e_measure([w], fmt, calls, args.steps, args.warmup, dev, nbytes_step,
                              graph=ex is not None, barrier=barrier, reduce_max=reduce_max)
        else:
            e2e = e2e_measure(layers, fmt, [layer_call(fmt, lw, S, ws) for lw in layers],
                              args.steps, args.warmup, dev, nbytes_step, graph=True,
                              barrier=barrier, reduce_max=reduce_max)
            e2e_eager = e2e_measure(layers, fmt, [plain_call(fmt, lw) for lw in layers],
                                    args.steps, args.warmup, dev, nbytes_step, graph=False,
                                    barrier=barrier, reduce_max=reduce_max)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tbps, secs, kind, cores, desc = cpu_reference_sample(wl, lens, args.seed,
                                                             args.cpu_seconds)
        cpu = {"value": tbps, "unit": "TB/s", "cores": cores, "kind": kind, "sample": desc,
               "seconds": round(secs, 2)}

    peak, peak_src = measured_peaks()
    graph = None
    sweep = seqshard_suite = None
    if not args.no_sweep:
        del layers, calls, w, q, bt, sl, ws, step
        torch.cuda.empty_cache()
        if world == 1:
            sweep = run_sweep(args, dev, sms, checker, peak, local)
        elif not seqshard:
            seqshard_suite = {}
            for n, x in SEQSHARD:
                try:
                    seqshard_suite[f"{n}_{x}"] = run_seqshard_point(n, x, args, world, rank,
                                                                    local, dev, sms)
                except Exception as e:  # noqa: BLE001 - recorded in the line, headline kept
                    seqshard_suite[f"{n}_{x}"] = {"error": f"{type(e).__name__}: {e}"[:300]}
                    torch.cuda.synchronize()
                    torch.cuda.empty_cache()

    if world > 1:
        torch.cuda.synchronize()
        dist.barrier(device_ids=[local])
        if ex is not None:
            ex.close()
        dist.destroy_process_group()
    if rank != 0:
        return 0

    achieved_gbs = kernel_bytes / (kern_ms * 1e-3) / 1e9
    traffic, traffic_note = ncu_traffic(split_kernel_name(fmt, bs), kernel_bytes)
    ms_per_step = elapsed_max / args.steps
    measured_32 = {}
    if sweep:
        measured_32 = {n: p["us_per_step"] for n, p in sweep["points"].items()
                       if p["layers"] == 32}
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
                       layers_per_step=L, l2=l2_note(wl, L)),
        "pct_of_b200_spec_peak": 100.0 * value_tbps * 1e3 / (B200_SPEC_GBS * world),
        "us_per_decode_step": {
            "one_layer": ms_per_step * 1e3 / L, "layers_per_step": L,
            "llama3_8b_32_layers": ms_per_step * 1e3 if L == 32 else None,
            "llama3_8b_32_layers_note": (
                "measured: 32 layers in one graph" if L == 32 else
                "32 layers of this workload do not fit in HBM (one layer's KV is "
                f"{step_bytes / L / 1e9:.1f} GB per GPU); measured 32-layer steps of the "
                "sweep workloads are in llama3_8b_32_layers_measured"),
            "llama3_8b_32_layers_measured": measured_32},
        "splits": S,
        "timing": ("eager calls" if graph_used is False
                   else "CUDA-graph replay of one product call per step"),
        "parity": parity,
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
        "e2e_eager": e2e_eager,
        "gpu_launches": args.steps * launches_per_step,
        "clocks": sampler.summary(),
    }
    if sweep is not None:
        line["sweep"] = sweep
    if seqshard_suite is not None:
        line["seqshard"] = seqshard_suite
    print(json.dumps(line), flush=True)
    oks = [parity] + ([p["parity"] for p in sweep["points"].values()] if sweep else []) + \
          ([p["parity"] for p in seqshard_suite.values() if "parity" in p]
           if seqshard_suite else [])
    if any(p is not None and not p["ok"] for p in oks):
        print("bench: parity check failed (see the parity keys of the JSON line)",
              file=sys.stderr)
        return 1
    return 0


# ----------------------------------------------------------------------------- reference Triton arm

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
    ref, why = load_reference_module("triton_fp16")
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

    def timed(num_splits, steps, warmup):
        f = lambda: ref.paged_decode_attention_triton(q, kc, vc, bt, sl, num_splits=num_splits)
        return time_steps(f, steps, warmup, dev) / steps

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

    def time_mode(tensor_cores):
        """ms per call of FlashInfer's decode wrapper in one mode (CUDA-graph replays)."""
        fi = flashinfer.BatchDecodeWithPagedKVCacheWrapper(
            torch.empty(256 << 20, dtype=torch.uint8, device=dev), "NHD",
            use_tensor_cores=tensor_cores)
        fi.plan(indptr, indices, last, HQ, HKV, D, bs, q_data_type=torch.float16,
                kv_data_type=torch.float16)
        call = lambda: fi.run(q, (kc, vc), out=out)  # noqa: E731
        try:
            graph = capture(call, dev)
            step, how = graph.replay, "CUDA-graph replay of one call per step"
        except Exception:  # noqa: BLE001
            graph, step, how = None, call, "eager calls"
        ms = time_steps(step, args.steps, max(args.warmup, 1), dev)
        del graph
        return ms / args.steps, how

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
