"""numpy KIVI quantizer/dequantizer: the bit-exact specification. TEST INFRASTRUCTURE ONLY.

The reference has no quantized path (its README lists fused-dequant KV as "not started"), so
this module is the specification the CUDA cache-append kernel must match bit for bit, and the
dequantizer that turns a quantized cache into the fp32 cache the attention oracle
(``oracle.attention``) consumes ("fp32 math on the identically dequantized cache").
Parity of the quantizer is therefore *unpinned by the reference*; it is pinned by this spec
and by the golden codes committed under tests/golden/.

Granularity (KIVI): keys per (page, kv head, channel) over the page's valid tokens; values
per (token, kv head) over the D channels.

INT8 / INT4, asymmetric, unsigned codes in [0, Q], Q = 2**bits - 1:
    mn, mx  = min / max of the group (fp16 values, exact in fp32)
    scale   = fp16( fp32(mx - mn) / Q )          fp32 ops correctly rounded, then RNE to fp16
    zero    = fp16(mn)                            exact
    code    = clamp(rint((x - zero) / scale), 0, Q)   with the fp16-rounded scale/zero,
                                                      fp32 sub/div, round-half-even
    scale == 0 (constant group or underflow)  ->  code 0
    x_hat   = code * scale + zero                 fp32 (the product is exact; one rounding)

FP8-E4M3, symmetric, scale only:
    scale   = fp16( fp32(amax) / 448 )
    code    = e4m3_rne( clamp(x / scale, -448, 448) )   (clamped first: an unclamped cast of
                                                           a value past 448 can give NaN)
    scale == 0 -> code 0 (+0.0)
    x_hat   = fp32(code) * scale                  exact in fp32

Storage (block_size = bs, kv heads = H, head dim = D, num_blocks = nb):
    INT8 / FP8:  k_codes, v_codes [nb, bs, H, D] uint8 (FP8 codes are e4m3 bit patterns)
    INT4:        k_codes [nb, bs, H, D/2] uint8, low nibble = even channel
                 v_codes [nb, bs/2, H, D] uint8, low nibble = even token
    k_scale, k_zero [nb, H, D] fp16;  v_scale, v_zero [nb, bs, H] fp16 (FP8: no zeros)
Slots past a sequence's length inside its last page get code 0, v_scale 0, v_zero 0.
"""
from typing import Sequence

import numpy as np

try:
    import ml_dtypes
    _E4M3 = ml_dtypes.float8_e4m3fn
except ImportError:  # pragma: no cover - ml_dtypes ships with this image
    _E4M3 = None

FORMATS = ("int8", "fp8", "int4")
FP8_MAX = np.float32(448.0)


def _bits(fmt: str) -> int:
    return {"int8": 8, "int4": 4}[fmt]


# --------------------------------------------------------------------------- parameters

def int_params(mn: np.ndarray, mx: np.ndarray, bits: int):
    q = np.float32(2 ** bits - 1)
    scale = ((mx.astype(np.float32) - mn.astype(np.float32)) / q).astype(np.float16)
    zero = mn.astype(np.float16)
    return scale, zero


def int_codes(x: np.ndarray, scale: np.ndarray, zero: np.ndarray, bits: int) -> np.ndarray:
    """x, scale, zero broadcastable; fp32 (x - zero) / scale, RNE, clamp."""
    q = np.float32(2 ** bits - 1)
    s = scale.astype(np.float32)
    z = zero.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        t = (x.astype(np.float32) - z) / s
    t = np.where(s == 0, np.float32(0), t)
    c = np.clip(np.rint(t), 0, q)
    return c.astype(np.uint8)


def fp8_params(amax: np.ndarray):
    return (amax.astype(np.float32) / FP8_MAX).astype(np.float16)


def fp8_codes(x: np.ndarray, scale: np.ndarray) -> np.ndarray:
    if _E4M3 is None:
        raise RuntimeError("ml_dtypes is required for the FP8 specification")
    s = scale.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        t = x.astype(np.float32) / s
    t = np.where(s == 0, np.float32(0), t)
    t = np.clip(t, -FP8_MAX, FP8_MAX).astype(np.float32)
    return t.astype(_E4M3).view(np.uint8)


def fp8_decode(codes: np.ndarray) -> np.ndarray:
    return codes.view(_E4M3).astype(np.float32)


# --------------------------------------------------------------------------- packing

def pack_low_high(c: np.ndarray, axis: int) -> np.ndarray:
    """Two 4-bit codes per byte along ``axis``: low nibble = even index."""
    c = np.moveaxis(c, axis, -1)
    packed = (c[..., 0::2] & 0xF) | ((c[..., 1::2] & 0xF) << 4)
    return np.moveaxis(packed.astype(np.uint8), -1, axis)


def unpack_low_high(p: np.ndarray, axis: int) -> np.ndarray:
    p = np.moveaxis(p, axis, -1)
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), dtype=np.uint8)
    out[..., 0::2] = p & 0xF
    out[..., 1::2] = p >> 4
    return np.moveaxis(out, -1, axis)


# --------------------------------------------------------------------------- one page

def quantize_page(k: np.ndarray, v: np.ndarray, block_size: int, fmt: str):
    """Quantize the valid tokens of ONE page.

    k, v: [n_valid, H, D] fp16 with 1 <= n_valid <= block_size.
    Returns dict with k_codes [bs, H, D] (unpacked codes), k_scale/k_zero [H, D],
    v_codes [bs, H, D], v_scale/v_zero [bs, H]; slots >= n_valid are zero.
    """
    n, H, D = k.shape
    assert 1 <= n <= block_size
    kc = np.zeros((block_size, H, D), np.uint8)
    vc = np.zeros((block_size, H, D), np.uint8)
    vs = np.zeros((block_size, H), np.float16)
    vz = np.zeros((block_size, H), np.float16)
    if fmt == "fp8":
        ks = fp8_params(np.abs(k.astype(np.float32)).max(axis=0))          # [H, D]
        kz = None
        kc[:n] = fp8_codes(k, ks[None])
        vs[:n] = fp8_params(np.abs(v.astype(np.float32)).max(axis=2))     # [n, H]
        vc[:n] = fp8_codes(v, vs[:n, :, None])
        vz = None
    else:
        bits = _bits(fmt)
        ks, kz = int_params(k.min(axis=0), k.max(axis=0), bits)           # [H, D]
        kc[:n] = int_codes(k, ks[None], kz[None], bits)
        s, z = int_params(v.min(axis=2), v.max(axis=2), bits)             # [n, H]
        vs[:n], vz[:n] = s, z
        vc[:n] = int_codes(v, s[:, :, None], z[:, :, None], bits)
    return dict(k_codes=kc, k_scale=ks, k_zero=kz, v_codes=vc, v_scale=vs, v_zero=vz)


# --------------------------------------------------------------------------- whole caches

def empty_cache(num_blocks: int, block_size: int, H: int, D: int, fmt: str):
    kd = D // 2 if fmt == "int4" else D
    vt = block_size // 2 if fmt == "int4" else block_size
    c = dict(
        k_codes=np.zeros((num_blocks, block_size, H, kd), np.uint8),
        v_codes=np.zeros((num_blocks, vt, H, D), np.uint8),
        k_scale=np.zeros((num_blocks, H, D), np.float16),
        v_scale=np.zeros((num_blocks, block_size, H), np.float16),
    )
    if fmt != "fp8":
        c["k_zero"] = np.zeros((num_blocks, H, D), np.float16)
        c["v_zero"] = np.zeros((num_blocks, block_size, H), np.float16)
    return c


def store_page(cache: dict, phys: int, page: dict, fmt: str):
    kc, vc = page["k_codes"], page["v_codes"]
    if fmt == "int4":
        kc = pack_low_high(kc, axis=2)
        vc = pack_low_high(vc, axis=0)
    cache["k_codes"][phys] = kc
    cache["v_codes"][phys] = vc
    cache["k_scale"][phys] = page["k_scale"]
    cache["v_scale"][phys] = page["v_scale"]
    if fmt != "fp8":
        cache["k_zero"][phys] = page["k_zero"]
        cache["v_zero"][phys] = page["v_zero"]


def quantize_append(cache: dict, k_new: np.ndarray, v_new: np.ndarray,
                    new_lens: Sequence[int], start_pos: Sequence[int],
                    block_table: np.ndarray, block_size: int, fmt: str) -> dict:
    """Write tokens [start_pos[b], start_pos[b] + new_lens[b]) of every sequence.

    k_new/v_new [B, S, H, D] fp16 hold the new tokens from index 0. start_pos must be a
    multiple of block_size (key statistics are per page, so a page is always written whole
    from fp16 source rows). Mirrors the CUDA cache-append kernel.
    """
    for b, n in enumerate(new_lens):
        n, st = int(n), int(start_pos[b])
        assert st % block_size == 0
        for j in range((n + block_size - 1) // block_size):
            lo, hi = j * block_size, min((j + 1) * block_size, n)
            page = quantize_page(k_new[b, lo:hi], v_new[b, lo:hi], block_size, fmt)
            phys = int(block_table[b, st // block_size + j])
            store_page(cache, phys, page, fmt)
    return cache


def dequantize_cache(cache: dict, fmt: str):
    """Quantized cache -> fp32 (k_cache, v_cache) [nb, bs, H, D] (x_hat per the spec)."""
    kc, vc = cache["k_codes"], cache["v_codes"]
    if fmt == "int4":
        kc = unpack_low_high(kc, axis=3)
        vc = unpack_low_high(vc, axis=1)
    ks = cache["k_scale"].astype(np.float32)[:, None]        # [nb, 1, H, D]
    vs = cache["v_scale"].astype(np.float32)[..., None]       # [nb, bs, H, 1]
    if fmt == "fp8":
        k = fp8_decode(kc) * ks
        v = fp8_decode(vc) * vs
    else:
        kz = cache["k_zero"].astype(np.float32)[:, None]
        vz = cache["v_zero"].astype(np.float32)[..., None]
        k = kc.astype(np.float32) * ks + kz
        v = vc.astype(np.float32) * vs + vz
    return k.astype(np.float32), v.astype(np.float32)


def fill_garbage(cache: dict, g: np.random.Generator, used_pages: Sequence[int],
                 partial: Sequence[tuple], fmt: str, block_size: int):
    """Random codes/scales in every page no sequence owns and in the unused slots of partial
    pages, so a kernel that reads past seq_len or through a wrong block id is caught."""
    nb = cache["k_codes"].shape[0]
    unused = np.setdiff1d(np.arange(nb), np.asarray(used_pages, dtype=np.int64))
    for name, arr in cache.items():
        if unused.size:
            if arr.dtype == np.uint8:
                arr[unused] = g.integers(0, 256, size=(unused.size,) + arr.shape[1:],
                                         dtype=np.uint8)
            else:
                arr[unused] = (g.standard_normal((unused.size,) + arr.shape[1:]) * 4
                               ).astype(np.float16)
    for phys, n_valid in partial:
        if fmt == "int4":
            # keys: whole token rows past n_valid
            cache["k_codes"][phys, n_valid:] = g.integers(
                0, 256, size=cache["k_codes"][phys, n_valid:].shape, dtype=np.uint8)
            # values: token pairs; keep the valid nibble of a shared byte intact
            first = (n_valid + 1) // 2
            cache["v_codes"][phys, first:] = g.integers(
                0, 256, size=cache["v_codes"][phys, first:].shape, dtype=np.uint8)
            if n_valid % 2 == 1:
                keep = cache["v_codes"][phys, n_valid // 2] & 0xF
                junk = g.integers(0, 16, size=keep.shape, dtype=np.uint8)
                cache["v_codes"][phys, n_valid // 2] = keep | (junk << 4)
        else:
            for name in ("k_codes", "v_codes"):
                cache[name][phys, n_valid:] = g.integers(
                    0, 256, size=cache[name][phys, n_valid:].shape, dtype=np.uint8)
            if fmt == "fp8":
                # avoid NaN patterns (0x7F / 0xFF) so garbage stays finite for the oracle
                for name in ("k_codes", "v_codes"):
                    sl = cache[name][phys, n_valid:]
                    sl[(sl & 0x7F) == 0x7F] = 0x7E
        cache["v_scale"][phys, n_valid:] = (g.standard_normal(
            cache["v_scale"][phys, n_valid:].shape) * 4).astype(np.float16)
        if fmt != "fp8":
            cache["v_zero"][phys, n_valid:] = (g.standard_normal(
                cache["v_zero"][phys, n_valid:].shape) * 4).astype(np.float16)
    if fmt == "fp8" and unused.size:
        for name in ("k_codes", "v_codes"):
            sl = cache[name][unused]
            sl[(sl & 0x7F) == 0x7F] = 0x7E
            cache[name][unused] = sl
    return cache


def quant_case(seed: int, lens: Sequence[int], Hq: int, Hkv: int, D: int, block_size: int,
               fmt: str, mode: str = "spare", spare: int = 8, outliers: int = 4,
               garbage: bool = True):
    """A seeded KIVI parity case: quantize fresh N(0,1) K (with outlier channels) / V."""
    from oracle.cache import block_table_for, make_qkv, rng
    g = rng(seed)
    q, k, v = make_qkv(g, lens, Hq, Hkv, D, outlier_channels=outliers)
    bt, nb = block_table_for(g, lens, block_size, mode, spare)
    cache = empty_cache(nb, block_size, Hkv, D, fmt)
    quantize_append(cache, k, v, lens, [0] * len(lens), bt, block_size, fmt)
    if garbage:
        used, partial = [], []
        for b, n in enumerate(lens):
            p = (int(n) + block_size - 1) // block_size
            used += [int(x) for x in bt[b, :p]]
            if n % block_size:
                partial.append((int(bt[b, p - 1]), int(n) % block_size))
        fill_garbage(cache, g, used, partial, fmt, block_size)
    return dict(q=q, k=k, v=v, cache=cache, block_table=bt,
                seq_lens=np.asarray(lens, dtype=np.int32), num_blocks=nb)
