// The end of a split, shared by the split kernels: the per-warp online-softmax states of one
// CTA (max m_w, sum l_w and the unnormalised accumulator A_w of every q head, left in shared
// memory by the warps) combined into the split's normalised partial state (o_part row and
// lse in log2 units) or, for a one-split call, the fp16 output. The combination is the
// reference's split merge (src/bpt/triton_fp16.py:152-162) applied to the warps of one CTA.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "common.cuh"
#include "decode_common.h"

namespace bpt {

// sM, sL [NW][8] and sAcc [NW][8][D] (16-byte aligned) as the warps left them; sF: 8 * NW floats
// of scratch. Threads [0, nthreads) of the CTA call this together and sync() is a barrier over
// exactly them. The per-head weights 2^(m_w - M) / L are computed once per head and every
// element is then one fma chain and one vector store per 4 channels: the epilogue of the split
// that ends last is on the call's critical path, while the SM's other CTAs still stream, and
// the per-element form (max, exp2 and a division for every element) took ~1.7 us there.
template <int NW, int D, typename Sync>
__device__ __forceinline__ void write_split_state(const float* sM, const float* sL,
                                                  const float* sAcc, float* sF,
                                                  const DecodeParams& p, int b, int qh0,
                                                  int split, int tid, int nthreads, Sync sync) {
  constexpr float kNegInfS = -INFINITY;
  const int S = p.splits;
  const bool to_out = S == 1 && p.final_out;
  if (tid < p.group) {
    const int hg = tid;
    float M = kNegInfS;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, sM[w * 8 + hg]);
    float f[NW], L = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      f[w] = M != kNegInfS ? fast_exp2(sM[w * 8 + hg] - M) : 0.f;
      L = fmaf(sL[w * 8 + hg], f[w], L);
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) sF[hg * NW + w] = f[w] * inv;
    if (!to_out)
      p.lse[(int64_t(b) * p.q_heads + qh0 + hg) * S + split] =
          L > 0.f ? M + __log2f(L) : kNegInfS;
  }
  sync();
  // caller partial buffers may be offset views: vector stores only where aligned
  const bool out_vec = (reinterpret_cast<uintptr_t>(p.out) & 7) == 0 && p.o_sb % 4 == 0 &&
                       p.o_sh % 4 == 0;
  const bool part_vec = (reinterpret_cast<uintptr_t>(p.o_part) & 15) == 0;
  for (int idx = 4 * tid; idx < p.group * D; idx += 4 * nthreads) {
    const int hg = idx / D, d = idx % D;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float fw = sF[hg * NW + w];
      const float4 a = *reinterpret_cast<const float4*>(sAcc + (w * 8 + hg) * D + d);
      o.x = fmaf(a.x, fw, o.x);
      o.y = fmaf(a.y, fw, o.y);
      o.z = fmaf(a.z, fw, o.z);
      o.w = fmaf(a.w, fw, o.w);
    }
    if (to_out) {
      __half* dst = p.out + int64_t(b) * p.o_sb + int64_t(qh0 + hg) * p.o_sh + d;
      const __half2 h01 = __floats2half2_rn(o.x, o.y), h23 = __floats2half2_rn(o.z, o.w);
      if (out_vec) {
        uint2 pk;
        pk.x = *reinterpret_cast<const uint32_t*>(&h01);
        pk.y = *reinterpret_cast<const uint32_t*>(&h23);
        *reinterpret_cast<uint2*>(dst) = pk;
      } else {
        dst[0] = __low2half(h01);
        dst[1] = __high2half(h01);
        dst[2] = __low2half(h23);
        dst[3] = __high2half(h23);
      }
    } else {
      float* dst = p.o_part + ((int64_t(b) * p.q_heads + qh0 + hg) * S + split) * D + d;
      if (part_vec) {
        *reinterpret_cast<float4*>(dst) = o;
      } else {
        dst[0] = o.x;
        dst[1] = o.y;
        dst[2] = o.z;
        dst[3] = o.w;
      }
    }
  }
}

}  // namespace bpt
