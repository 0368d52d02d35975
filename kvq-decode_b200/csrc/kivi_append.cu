// KIVI cache-append quantizer: fp16 K/V rows -> INT8 / FP8-E4M3 / INT4 paged codes.
//
// No reference counterpart (the reference lists quantized KV as "not started"); the
// arithmetic is the specification in oracle/kivi.py, step for step, so the codes and fp16
// scale/zero-points match numpy bit for bit:
//   INT (Q = 2^bits - 1):  scale = fp16((mx - mn) / Q), zero = fp16(mn),
//                          code  = clamp(rint((x - zero) / scale), 0, Q), scale == 0 -> 0
//   FP8:                   scale = fp16(amax / 448),
//                          code  = e4m3_rne(clamp(x / scale, -448, 448)), scale == 0 -> 0
// with every fp32 operation correctly rounded (__fsub_rn / __fdiv_rn: no contraction, no
// fast-math reciprocal) and round-half-even for rint and the fp16 / e4m3 conversions.
//
// One CTA per (new page j of sequence b, kv head h): keys are quantized per channel over the
// page's valid tokens (a thread per channel pair), values per token over the channels (a warp
// per token, or per token pair for INT4, whose value bytes pack two tokens).
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <math.h>

#include "common.cuh"
#include "decode_common.h"

namespace bpt {
namespace {

constexpr int kAppendThreads = 128;

__device__ __forceinline__ void int_params(float mn, float mx, float q, __half& s, __half& z) {
  s = __float2half_rn(__fdiv_rn(__fsub_rn(mx, mn), q));
  z = __float2half_rn(mn);
}

__device__ __forceinline__ uint32_t int_code(float x, float s, float z, float q) {
  if (s == 0.f) return 0u;
  float r = rintf(__fdiv_rn(__fsub_rn(x, z), s));
  r = fminf(fmaxf(r, 0.f), q);
  return uint32_t(r);
}

__device__ __forceinline__ uint32_t fp8_code(float x, float s) {
  if (s == 0.f) return 0u;
  float t = __fdiv_rn(x, s);
  t = fminf(fmaxf(t, -448.f), 448.f);
  return uint32_t(__nv_cvt_float_to_fp8(t, __NV_SATFINITE, __NV_E4M3));
}

struct AppendArgs {
  bpt_kivi_cache c;
  const __half* k_new;
  int64_t kn_sb, kn_st, kn_sh;
  const __half* v_new;
  int64_t vn_sb, vn_st, vn_sh;
  const int32_t* new_lens;
  const int32_t* start_pos;
  const int32_t* block_table;
  int64_t bt_sb;
  int max_blocks;
};

template <int FMT>
__global__ void __launch_bounds__(kAppendThreads) kivi_append_kernel(const AppendArgs a) {
  constexpr bool kFp8 = FMT == BPT_KV_FP8_E4M3;
  constexpr bool kInt4 = FMT == BPT_KV_INT4;
  constexpr float kQ = kInt4 ? 15.f : 255.f;
  const bpt_kivi_cache& c = a.c;
  const int j = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int bs = c.block_size, D = c.head_dim;
  const int n = __ldg(a.new_lens + b);
  if (n <= j * bs) return;
  const int n_valid = min(bs, n - j * bs);
  const int page = __ldg(a.start_pos + b) / bs + j;
  if (page < 0 || page >= a.max_blocks) return;
  const int phys = __ldg(a.block_table + int64_t(b) * a.bt_sb + page);
  if (phys < 0 || int64_t(phys) >= c.num_blocks) return;

  const __half* kr = a.k_new + int64_t(b) * a.kn_sb + int64_t(j) * bs * a.kn_st +
                     int64_t(h) * a.kn_sh;
  const __half* vr = a.v_new + int64_t(b) * a.vn_sb + int64_t(j) * bs * a.vn_st +
                     int64_t(h) * a.vn_sh;
  uint8_t* kc = static_cast<uint8_t*>(c.k_codes) + int64_t(phys) * c.k_codes_stride[0] +
                int64_t(h) * c.k_codes_stride[2];
  uint8_t* vc = static_cast<uint8_t*>(c.v_codes) + int64_t(phys) * c.v_codes_stride[0] +
                int64_t(h) * c.v_codes_stride[2];
  __half* ks = static_cast<__half*>(c.k_scale) + int64_t(phys) * c.k_param_stride[0] +
               int64_t(h) * c.k_param_stride[1];
  __half* kz = kFp8 ? nullptr
                    : static_cast<__half*>(c.k_zero) + int64_t(phys) * c.k_param_stride[0] +
                          int64_t(h) * c.k_param_stride[1];
  __half* vs = static_cast<__half*>(c.v_scale) + int64_t(phys) * c.v_param_stride[0] + h;
  __half* vz = kFp8 ? nullptr
                    : static_cast<__half*>(c.v_zero) + int64_t(phys) * c.v_param_stride[0] + h;

  // ---------------------------------------------------------------- keys: per channel
  for (int d0 = 2 * threadIdx.x; d0 < D; d0 += 2 * blockDim.x) {
    float lo[2], hi[2];
    lo[0] = lo[1] = INFINITY;
    hi[0] = hi[1] = -INFINITY;
    for (int i = 0; i < n_valid; ++i) {
      const __half2 x2 = *reinterpret_cast<const __half2*>(kr + int64_t(i) * a.kn_st + d0);
      const float2 x = __half22float2(x2);
      if (kFp8) {
        hi[0] = fmaxf(hi[0], fabsf(x.x));
        hi[1] = fmaxf(hi[1], fabsf(x.y));
      } else {
        lo[0] = fminf(lo[0], x.x); hi[0] = fmaxf(hi[0], x.x);
        lo[1] = fminf(lo[1], x.y); hi[1] = fmaxf(hi[1], x.y);
      }
    }
    __half s[2], z[2];
    float sf[2], zf[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      if (kFp8) {
        s[e] = __float2half_rn(__fdiv_rn(hi[e], 448.f));
        z[e] = __float2half_rn(0.f);
      } else {
        int_params(lo[e], hi[e], kQ, s[e], z[e]);
      }
      sf[e] = __half2float(s[e]);
      zf[e] = __half2float(z[e]);
      ks[d0 + e] = s[e];
      if (!kFp8) kz[d0 + e] = z[e];
    }
    for (int i = 0; i < bs; ++i) {
      uint32_t q0 = 0u, q1 = 0u;
      if (i < n_valid) {
        const float2 x =
            __half22float2(*reinterpret_cast<const __half2*>(kr + int64_t(i) * a.kn_st + d0));
        q0 = kFp8 ? fp8_code(x.x, sf[0]) : int_code(x.x, sf[0], zf[0], kQ);
        q1 = kFp8 ? fp8_code(x.y, sf[1]) : int_code(x.y, sf[1], zf[1], kQ);
      }
      uint8_t* row = kc + int64_t(i) * c.k_codes_stride[1];
      if (kInt4) {
        row[d0 >> 1] = uint8_t((q0 & 0xFu) | ((q1 & 0xFu) << 4));
      } else {
        row[d0] = uint8_t(q0);
        row[d0 + 1] = uint8_t(q1);
      }
    }
  }

  // ---------------------------------------------------------------- values: per token
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int tok_per_item = kInt4 ? 2 : 1;
  for (int item = warp; item * tok_per_item < bs; item += nwarps) {
    uint32_t codes_lo_tok[8], codes_hi_tok[8];  // up to D = 256: 8 channels per lane
#pragma unroll
    for (int k = 0; k < 8; ++k) codes_lo_tok[k] = codes_hi_tok[k] = 0u;
    for (int tt = 0; tt < tok_per_item; ++tt) {
      const int i = item * tok_per_item + tt;
      float sf = 0.f, zf = 0.f;
      __half s = __float2half_rn(0.f), z = __float2half_rn(0.f);
      if (i < n_valid) {
        float lo = INFINITY, hi = -INFINITY;
        for (int d = lane; d < D; d += 32) {
          const float x = __half2float(vr[int64_t(i) * a.vn_st + d]);
          if (kFp8) {
            hi = fmaxf(hi, fabsf(x));
          } else {
            lo = fminf(lo, x);
            hi = fmaxf(hi, x);
          }
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
          hi = fmaxf(hi, __shfl_xor_sync(kFullMask, hi, off));
          if (!kFp8) lo = fminf(lo, __shfl_xor_sync(kFullMask, lo, off));
        }
        if (kFp8) {
          s = __float2half_rn(__fdiv_rn(hi, 448.f));
        } else {
          int_params(lo, hi, kQ, s, z);
        }
        sf = __half2float(s);
        zf = __half2float(z);
      }
      if (lane == 0) {
        vs[int64_t(i) * c.v_param_stride[1]] = s;
        if (!kFp8) vz[int64_t(i) * c.v_param_stride[1]] = z;
      }
      int k = 0;
      for (int d = lane; d < D; d += 32, ++k) {
        uint32_t q = 0u;
        if (i < n_valid) {
          const float x = __half2float(vr[int64_t(i) * a.vn_st + d]);
          q = kFp8 ? fp8_code(x, sf) : int_code(x, sf, zf, kQ);
        }
        if (tt == 0) codes_lo_tok[k] = q; else codes_hi_tok[k] = q;
      }
    }
    int k = 0;
    for (int d = lane; d < D; d += 32, ++k) {
      if (kInt4) {
        vc[int64_t(item) * c.v_codes_stride[1] + d] =
            uint8_t((codes_lo_tok[k] & 0xFu) | ((codes_hi_tok[k] & 0xFu) << 4));
      } else {
        vc[int64_t(item) * c.v_codes_stride[1] + d] = uint8_t(codes_lo_tok[k]);
      }
    }
  }
}

}  // namespace
}  // namespace bpt

using namespace bpt;

extern "C" int bpt_kivi_append(const bpt_kivi_cache* cache, const void* k_new, int64_t kn_sb,
                               int64_t kn_st, int64_t kn_sh, const void* v_new, int64_t vn_sb,
                               int64_t vn_st, int64_t vn_sh, const int32_t* new_lens,
                               const int32_t* start_pos, const int32_t* block_table,
                               int64_t bt_sb, int max_blocks, int batch, int max_new,
                               void* stream) {
  if (!cache || batch < 0 || max_new < 0 || max_blocks < 0) return BPT_ERR_INVALID_ARGUMENT;
  const bpt_kivi_cache& c = *cache;
  if (c.format != BPT_KV_INT8 && c.format != BPT_KV_FP8_E4M3 && c.format != BPT_KV_INT4)
    return BPT_ERR_INVALID_ARGUMENT;
  if (c.block_size < 16 || c.block_size > 256 || (c.block_size & (c.block_size - 1)))
    return BPT_ERR_UNSUPPORTED_SHAPE;
  if (c.head_dim <= 0 || c.head_dim > 256 || (c.head_dim % 2) || c.kv_heads <= 0)
    return BPT_ERR_UNSUPPORTED_SHAPE;
  if (batch == 0 || max_new == 0) return BPT_OK;
  if (!k_new || !v_new || !new_lens || !start_pos || !block_table || !c.k_codes ||
      !c.v_codes || !c.k_scale || !c.v_scale)
    return BPT_ERR_INVALID_ARGUMENT;
  if (c.format != BPT_KV_FP8_E4M3 && (!c.k_zero || !c.v_zero)) return BPT_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new)) & 3)
    return BPT_ERR_ALIGNMENT;
  if ((kn_st | kn_sh | kn_sb) & 1) return BPT_ERR_ALIGNMENT;  // half2 loads along D
  AppendArgs a;
  a.c = c;
  a.k_new = static_cast<const __half*>(k_new);
  a.kn_sb = kn_sb; a.kn_st = kn_st; a.kn_sh = kn_sh;
  a.v_new = static_cast<const __half*>(v_new);
  a.vn_sb = vn_sb; a.vn_st = vn_st; a.vn_sh = vn_sh;
  a.new_lens = new_lens;
  a.start_pos = start_pos;
  a.block_table = block_table;
  a.bt_sb = bt_sb;
  a.max_blocks = max_blocks;
  dim3 grid((max_new + c.block_size - 1) / c.block_size, c.kv_heads, batch);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (c.format) {
    case BPT_KV_INT8: kivi_append_kernel<BPT_KV_INT8><<<grid, kAppendThreads, 0, st>>>(a); break;
    case BPT_KV_FP8_E4M3:
      kivi_append_kernel<BPT_KV_FP8_E4M3><<<grid, kAppendThreads, 0, st>>>(a);
      break;
    default: kivi_append_kernel<BPT_KV_INT4><<<grid, kAppendThreads, 0, st>>>(a); break;
  }
  return cudaGetLastError() == cudaSuccess ? BPT_OK : BPT_ERR_LAUNCH;
}
