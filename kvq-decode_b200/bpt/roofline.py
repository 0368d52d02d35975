"""Roofline: KV bytes read per decode step and the bandwidth-bound minimum time.

Keeps the reference module's names and semantics (src/bpt/roofline.py:1-67): ``GPUS``,
``KV_DTYPES``, ``SCALE_BYTES``, ``ZP_PER_SCALE``, ``ModelShape``, ``MODELS``,
``kv_bytes_per_token``, ``bytes_per_step``, ``min_time_ms``. The reference counts K/V payload
plus KIVI scale/zero overhead with keys grouped every ``group_size`` tokens and treats fp8 as
a plain cast.

Extensions for the formats bpt actually stores:
  * ``KIVI_FORMATS`` / ``kivi_bytes_per_token``: keys carry fp16 scale(+zero) per (page,
    kv head, channel), i.e. group = block_size; values per (token, kv head); FP8 is
    symmetric (scale only, no zero).
  * ``decode_call_bytes``: the algorithmic bytes one decode call must move for a concrete
    batch (K/V payload + scale/zero + block-table entries + q + out), the numerator of the
    achieved-bandwidth figure the benchmark reports.
"""
import argparse
from dataclasses import dataclass
from typing import Dict, Sequence

# Peak HBM/GDDR bandwidth, GB/s (1e9 B/s); spec-sheet values (reference: roofline.py:15-20)
GPUS: Dict[str, float] = {
    "T4": 320.0,
    "A100-80GB": 2039.0,
    "H100-SXM": 3350.0,
    "B200": 8000.0,
}

# (bytes per element, has scale/zero) -- reference semantics (roofline.py:23-28)
KV_DTYPES: Dict[str, tuple] = {
    "fp16": (2.0, False),
    "fp8": (1.0, False),
    "int8": (1.0, True),
    "int4": (0.5, True),
}

SCALE_BYTES = 2  # fp16
ZP_PER_SCALE = 2  # scale + zero


@dataclass(frozen=True)
class KiviFormat:
    elem_bytes: float       # payload bytes per element
    k_group_bytes: int      # fp16 bytes per key (page, head, channel) group: scale (+ zero)
    v_token_bytes: int      # fp16 bytes per value (token, head): scale (+ zero)


KIVI_FORMATS: Dict[str, KiviFormat] = {
    "fp16": KiviFormat(2.0, 0, 0),
    "int8": KiviFormat(1.0, 4, 4),
    "fp8": KiviFormat(1.0, 2, 2),
    "int4": KiviFormat(0.5, 4, 4),
}


@dataclass(frozen=True)
class ModelShape:
    layers: int
    q_heads: int
    kv_heads: int
    head_dim: int


MODELS: Dict[str, ModelShape] = {
    "llama3-8b": ModelShape(32, 32, 8, 128),
    "llama3-70b": ModelShape(80, 64, 8, 128),
    "llama2-7b": ModelShape(32, 32, 32, 128),
    "qwen2.5-7b": ModelShape(28, 28, 4, 128),
}


def kv_bytes_per_token(shape: ModelShape, kv_dtype: str, group_size: int = 128) -> float:
    """KV bytes per context token per decode step, all layers (reference roofline.py:50-58)."""
    elem, quant = KV_DTYPES[kv_dtype]
    per_head = 2 * shape.head_dim * elem
    if quant:
        k_scales = shape.head_dim * SCALE_BYTES * ZP_PER_SCALE / group_size
        v_scales = SCALE_BYTES * ZP_PER_SCALE
        per_head += k_scales + v_scales
    return shape.layers * shape.kv_heads * per_head


def kivi_bytes_per_token(shape: ModelShape, fmt: str, block_size: int) -> float:
    """Bytes per context token for the stored bpt formats (key group = one page)."""
    f = KIVI_FORMATS[fmt]
    per_head = 2 * shape.head_dim * f.elem_bytes
    per_head += shape.head_dim * f.k_group_bytes / block_size + f.v_token_bytes
    return shape.layers * shape.kv_heads * per_head


def bytes_per_step(shape: ModelShape, ctx: int, batch: int, kv_dtype: str,
                   group_size: int = 128) -> float:
    return kv_bytes_per_token(shape, kv_dtype, group_size) * ctx * batch


def min_time_ms(nbytes: float, gpu: str) -> float:
    return nbytes / (GPUS[gpu] * 1e9) * 1e3


def decode_call_bytes(seq_lens: Sequence[int], block_size: int, q_heads: int, kv_heads: int,
                      head_dim: int, fmt: str = "fp16") -> int:
    """Algorithmic bytes of one single-layer decode call over a concrete batch.

    sum_b [ n_b*Hkv*2*D*e + ceil(n_b/bs)*Hkv*D*k_group + n_b*Hkv*v_token ]
      + B*Hq*D*2*2 (q in, out) + sum_b ceil(n_b/bs)*4 (block-table entries)
    """
    f = KIVI_FORMATS[fmt]
    total = 0.0
    for n in seq_lens:
        n = int(n)
        pages = (n + block_size - 1) // block_size
        total += n * kv_heads * 2 * head_dim * f.elem_bytes
        total += pages * kv_heads * head_dim * f.k_group_bytes
        total += n * kv_heads * f.v_token_bytes
        total += pages * 4
    total += len(seq_lens) * q_heads * head_dim * 2 * 2
    return int(total)


def main(argv=None):
    """CLI (reference: bench/roofline.py:11-45), plus the bpt-stored formats."""
    p = argparse.ArgumentParser(description="KV bytes per decode step and minimum time")
    p.add_argument("--model", choices=sorted(MODELS), default="llama3-8b")
    p.add_argument("--layers", type=int, help="override (1 gives per-layer numbers)")
    p.add_argument("--q-heads", type=int)
    p.add_argument("--kv-heads", type=int)
    p.add_argument("--head-dim", type=int)
    p.add_argument("--ctx", type=int, default=32768)
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--kv-dtype", choices=sorted(KV_DTYPES), default="fp16")
    p.add_argument("--group-size", type=int, default=128,
                   help="tokens per key-scale group (quantized dtypes, reference model)")
    p.add_argument("--block-size", type=int, default=64,
                   help="page size of the bpt KIVI layout (key group = one page)")
    p.add_argument("--measured-gbps", type=float, default=None,
                   help="add a row for a measured peak (e.g. a STREAM copy on this GPU)")
    a = p.parse_args(argv)

    m = MODELS[a.model]
    shape = ModelShape(a.layers or m.layers, a.q_heads or m.q_heads,
                       a.kv_heads or m.kv_heads, a.head_dim or m.head_dim)
    tok = kv_bytes_per_token(shape, a.kv_dtype, a.group_size)
    step = bytes_per_step(shape, a.ctx, a.batch, a.kv_dtype, a.group_size)
    fp16_step = bytes_per_step(shape, a.ctx, a.batch, "fp16", a.group_size)
    kivi_tok = kivi_bytes_per_token(shape, a.kv_dtype, a.block_size)

    print(f"shape: {shape.layers}L, {shape.q_heads}q/{shape.kv_heads}kv heads, "
          f"D={shape.head_dim} | ctx={a.ctx} batch={a.batch} kv={a.kv_dtype}")
    print(f"bytes per context token (all layers): {tok:,.0f} B ({tok / 1024:.2f} KiB)")
    print(f"  bpt layout (key group = {a.block_size}-token page"
          f"{', fp8 scale-only' if a.kv_dtype == 'fp8' else ''}): {kivi_tok:,.0f} B")
    print(f"bytes per sequence per step:          {step / a.batch / 2**20:,.1f} MiB")
    print(f"bytes per decode step (batch):        {step / 2**30:,.3f} GiB")
    print("(KV-cache reads only; weights, q and output excluded)\n")
    gpus = dict(GPUS)
    if a.measured_gbps:
        gpus["measured"] = a.measured_gbps
    print(f"{'GPU':<10}{'peak GB/s':>10}{'min time ms':>13}{'min us/seq':>12}"
          f"{'max steps/s':>13}{'vs fp16':>9}")
    for gpu, bw in gpus.items():
        t = step / (bw * 1e9) * 1e3
        print(f"{gpu:<10}{bw:>10.0f}{t:>13.3f}{t * 1e3 / a.batch:>12.1f}"
              f"{1e3 / t:>13.1f}{fp16_step / step:>8.2f}x")


if __name__ == "__main__":
    main()
