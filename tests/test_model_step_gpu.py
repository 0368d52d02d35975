"""A whole Llama-3-8B decode step's attention as one CUDA graph (GPU).

A model decode step calls the attention once per layer: 32 layers, each with its own KV cache,
query and block table. The step is captured once as a CUDA graph of 32 product calls (split
kernel + PDL-chained merge each, one shared workspace) and replayed; every layer's output must
match the numpy oracle (a restatement of src/bpt/reference.py:20-49; for KIVI caches run on
the identically dequantized cache) at the BASELINE tolerance. The queries are then overwritten
in place and the graph replayed again, so a graph that replayed stale results would fail.
"""
import numpy as np
import pytest
import torch

from helpers import assert_close
from oracle import attention as oa
from oracle import cache as oc
from oracle import kivi

pytestmark = pytest.mark.gpu

LAYERS = 32
HQ, HKV, D = 32, 8, 128


def _layer(fmt, i):
    lens = [1500 + 97 * i, 513, 64 * (i % 5) + 1]
    if fmt == "fp16":
        c = oc.fp16_case(300 + i, lens, HQ, HKV, D, 16, "spare", 8)
        dev = {k: torch.from_numpy(c[k]).cuda() for k in
               ("q", "k_cache", "v_cache", "block_table", "seq_lens")}
        kd, vd = c["k_cache"], c["v_cache"]
    else:
        from bpt.quant import KiviCache
        c = kivi.quant_case(300 + i, lens, HQ, HKV, D, 64, fmt, "spare", 4)
        dev = {k: torch.from_numpy(c[k]).cuda() for k in ("q", "block_table", "seq_lens")}
        dev["cache"] = KiviCache(fmt=fmt, block_size=64,
                                 **{k: torch.from_numpy(v.copy()).cuda()
                                    for k, v in c["cache"].items()})
        kd, vd = kivi.dequantize_cache(c["cache"], fmt)
    dev["out"] = torch.empty_like(dev["q"])
    return dev, (kd, vd, c["block_table"], c["seq_lens"])


def _oracle(q, host):
    kd, vd, bt, sl = host
    return oa.paged_decode_attention_ref(q, kd, vd, bt, sl, out_dtype=np.float16)


@pytest.mark.parametrize("fmt", ["fp16", "int8", "int4"])
def test_32_layer_step_in_one_graph(fmt):
    from bpt import decode as dec
    from bpt.quant import effective_splits_kivi, paged_decode_attention_kivi
    layers = [_layer(fmt, i) for i in range(LAYERS)]
    sms = dec._sm_count(0)
    splits, need = [], 0
    for dv, _ in layers:
        B, mb = dv["block_table"].shape
        S = (dec.effective_splits(B, HKV, 16, mb, None, sms) if fmt == "fp16" else
             effective_splits_kivi(dv["cache"], B, HQ, mb, None, sms))
        splits.append(S)
        need = max(need, dec.workspace_bytes(B, HQ, D, S))
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")

    def step():
        for (dv, _), S in zip(layers, splits):
            if fmt == "fp16":
                dec.paged_decode_attention(dv["q"], dv["k_cache"], dv["v_cache"],
                                           dv["block_table"], dv["seq_lens"], num_splits=S,
                                           out=dv["out"], workspace=ws)
            else:
                paged_decode_attention_kivi(dv["q"], dv["cache"], dv["block_table"],
                                            dv["seq_lens"], num_splits=S, out=dv["out"],
                                            workspace=ws)

    step()
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for round_ in range(2):
        if round_:
            g = np.random.Generator(np.random.PCG64(77))
            for dv, _ in layers:   # new queries, written in place into the graph's inputs
                dv["q"].copy_(torch.from_numpy(
                    g.standard_normal(tuple(dv["q"].shape), dtype=np.float32)
                    .astype(np.float16)))
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize()
        for i, (dv, host) in enumerate(layers):
            ref = _oracle(dv["q"].cpu().numpy(), host)
            assert_close(dv["out"].float().cpu().numpy(), ref,
                         what=f"{fmt} layer {i} replay round {round_}")
    del graph
