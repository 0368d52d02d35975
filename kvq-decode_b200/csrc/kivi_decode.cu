// Fused-dequant split-KV decode over KIVI-quantized paged caches (INT8, FP8-E4M3, INT4).
//
// No reference counterpart (the reference lists quantized KV as "not started"). The result
// must match the reference oracle run in fp32 on the identically dequantized cache
// (x_hat = code * scale + zero, oracle/kivi.py), so the kernel never rounds a dequantized
// value to fp16. Instead the scales are folded into the other operand:
//
//   keys (per page, head, channel d):  q . k_hat = sum_d (q_d s_d) c_d + sum_d q_d z_d
//       q' = q * s is split into fp16 hi + lo and fed as MMA rows 0-7 (hi) and 8-15 (lo);
//       codes enter the MMA exactly as fp16 integers; the bias sum_d q_d z_d is fp32.
//   values (per token t, head):       sum_t p_t v_hat_t = sum_t (p_t s_t) c_t + sum_t p_t z_t
//       p' = p * s_t is split into fp16 hi/lo exactly like the fp16 kernel's P; the zero-point
//       term is accumulated in fp32 per head.
//
// Work decomposition, TMA producer, split partial states and merge are those of the fp16
// tensor-core kernel (mma_decode.cuh). Per chunk of 16*NCW tokens the producer loads, with
// one mbarrier transaction: the K and V code rows (4-D TMA boxes, page indirection = box
// coordinate; INT8/FP8 rows 128 B with the 128-byte swizzle, INT4 key rows 64 B with the
// 64-byte swizzle, INT4 value pair-rows 128 B), the page's k_scale / k_zero rows (TMA),
// and each token's v_scale / v_zero (cp.async, 4-byte granules, tracked by the same barrier).
//
// Fragment layouts (mma.sync m16n8k16, lane = 4 g + t):
//   QK^T  B = K^T via ldmatrix on the code rows: lane gets 4 code bytes (INT8/FP8: channels
//         16 c + 4 t + {0..3}) or 8 nibbles (INT4: channels 32 c + 8 t + {0..7}) of token g;
//         the k-slot -> channel mapping is chosen so each 32-bit word converts with 2-4
//         instructions, and q' is laid out with the same mapping (any consistent permutation
//         of the reduction dimension is exact).
//   P.V   A = V^T: lane loads 16 channels of 4 tokens (LDS.128) and transposes bytes with
//         prmt (INT8/FP8) or pairs nibbles of a token-pair byte (INT4) into fp16x2 fragments.
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <math.h>

#include "common.cuh"
#include "decode_common.h"
#include "mma_decode.cuh"
#include "split_state.cuh"

namespace bpt {
namespace kivi {

using mma::kNegInf;
using mma::ldsm_x4;
using mma::mma_16816;
using mma::pack_half2;

constexpr int D = 128;                  // KIVI kernels are built for head_dim 128
constexpr uint32_t kMagic = 0x64006400u;  // fp16 1024.0 in both halves
constexpr uint32_t kMagicBytes = 0x64646464u;
constexpr int kC0Int8 = 128;   // code centre, INT8
constexpr int kC0Int4 = 8;     // code centre, INT4

template <int FMT, int NCW, int STAGES, bool G8>
struct Cfg {
  static constexpr bool INT4 = FMT == BPT_KV_INT4;
  static constexpr bool FP8 = FMT == BPT_KV_FP8_E4M3;
  static constexpr int CHUNK = 16 * NCW;
  static constexpr int THREADS = (NCW + 1) * 32;
  static constexpr int K_ROW = INT4 ? 64 : 128;          // bytes per token row of K codes
  static constexpr int V_ROWS = INT4 ? CHUNK / 2 : CHUNK;  // V code rows per chunk (128 B)
  static constexpr int K_BYTES = CHUNK * K_ROW;
  static constexpr int V_BYTES = V_ROWS * 128;
  static constexpr int MAXPG = CHUNK / 16;                 // pages (boxes) per chunk at most
  static constexpr int KP_BYTES = MAXPG * 512;             // k_scale + k_zero rows (fp16 x 128)
  static constexpr int VP_BYTES = CHUNK * 8;               // v_scale, v_zero 4-byte granules
  static constexpr int STAGE_RAW = K_BYTES + V_BYTES + KP_BYTES + VP_BYTES;
  static constexpr int STAGE_BYTES = (STAGE_RAW + 1023) & ~1023;
  static constexpr int NACC = G8 ? 2 : 1;
  static constexpr size_t RING_BYTES = size_t(STAGES) * STAGE_BYTES;
  static constexpr size_t Q_BYTES = 8 * D * 4;             // fp32 q of the group's heads
  static constexpr size_t MERGE_BYTES = size_t(NCW) * 8 * (D + 3) * 4;
  static constexpr size_t BODY_BYTES = RING_BYTES > MERGE_BYTES ? RING_BYTES : MERGE_BYTES;
  static constexpr size_t SMEM_BYTES = 1024 + BODY_BYTES + Q_BYTES + 2 * STAGES * 8 + 64;
};

struct KiviParams {
  DecodeParams d;           // q / block table / seq_lens / out / partials / shape
  const uint8_t* v_scale;   // v_scale / v_zero base (element 0 is 4-byte aligned)
  const uint8_t* v_zero;
  int64_t vps0, vps1;       // element strides (block, token); head stride 1
  int lbs, lbox;            // log2 of block_size and of the TMA box rows
};

// Integer codes enter the MMA centred (code - C0), so the fp32 accumulator sums
// mean-zero terms instead of growing linearly and cancelling against the zero-point term at the
// end (the tensor-core accumulation rounds each step, so a large running sum loses the small
// terms); C0 * scale is moved into the fp32 bias / zero-point sums. The magic-number fp16
// (1024 + code, or 1024 + 16 * code for a high nibble left in place) minus (1024 + C0) or
// (1024 + 16 * C0) is exact: every operand is an integer below 2048.
template <int OFF>
__device__ __forceinline__ uint32_t hsub_const(uint32_t x) {
  __half2 h = *reinterpret_cast<__half2*>(&x);
  h = __hsub2(h, __float2half2_rn(float(OFF)));
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t cvt_e4m3x2(uint32_t lo16) {
  uint32_t r;
  const unsigned short v = static_cast<unsigned short>(lo16 & 0xFFFFu);
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}

__device__ __forceinline__ void cp_async_4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// 2^e as an exact fp32 (e in [-126, 127]).
__device__ __forceinline__ float exp2i(int e) {
  e = max(-126, min(127, e));
  return __int_as_float((127 + e) << 23);
}

// Power-of-two exponent E with x * 2^E in [2^14, 2^15) (x > 0 finite): keeps an fp16 operand
// in the normal range with headroom, so its hi/lo split stays exact to ~22 bits.
__device__ __forceinline__ int norm_exponent(float x) {
  const int ex = ((__float_as_int(x) >> 23) & 0xFF) - 127;
  return 14 - ex;
}

// Channel (and scale multiplier) of q' k-slot element e (0,1 = a0 lo/hi, 2,3 = a2 lo/hi) at
// k-step ks for thread-in-group t; must mirror the key-word conversion below.
template <bool INT4>
__device__ __forceinline__ int q_channel(int ks, int e, int t, float& mult) {
  if constexpr (INT4) {
    const int c = ks >> 1, r = ks & 1;
    const int base = 32 * c + 8 * t;
    mult = r ? 0.0625f : 1.f;
    const int off0[4] = {0, 4, 2, 6};
    return base + off0[e] + r;
  } else {
    mult = 1.f;
    return 16 * ks + 4 * t + e;
  }
}

template <int FMT, int NCW, int STAGES, int MINB, bool G8>
__global__ void __launch_bounds__((NCW + 1) * 32, MINB)
kivi_decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                   const __grid_constant__ CUtensorMap tmKS,
                   const __grid_constant__ CUtensorMap tmKZ, const KiviParams kp) {
  using C = Cfg<FMT, NCW, STAGES, G8>;
  constexpr int CHUNK = C::CHUNK;
  constexpr bool INT4 = C::INT4, FP8 = C::FP8;
  const DecodeParams& p = kp.d;
  constexpr float kC0 = INT4 ? float(kC0Int4) : float(kC0Int8);  // unused for FP8
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* sQ = reinterpret_cast<float*>(smem + C::BODY_BYTES);              // [8][D]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BODY_BYTES + C::Q_BYTES);
  uint64_t* empty = full + STAGES;
  float* sM = reinterpret_cast<float*>(smem);   // merge scratch aliases the ring at the end
  float* sL = sM + NCW * 8;
  float* sAcc = sL + NCW * 8;

  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.splits;

  // the tensor maps are kernel parameters, not written by the previous kernel: their fetch
  // overlaps the wait
  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
    prefetch_tensormap(&tmKS);
    if (!FP8) prefetch_tensormap(&tmKZ);
  }
  // launched as a programmatic dependent of the previous kernel in the stream: nothing that
  // kernel may write (q, the cache, the table, the lengths, the workspace) is read before
  // it completed
  pdl_wait();
  int n = __ldg(p.seq_lens + b);
  if (n < 0) {
    if (threadIdx.x == 0) flag_device_error(p.status, BPT_DEV_NEG_SEQ_LEN);
    n = 0;
  }
  const int64_t cap = int64_t(p.max_blocks) * p.block_size;
  if (n > cap) {
    if (threadIdx.x == 0) flag_device_error(p.status, BPT_DEV_SEQ_TOO_LONG);
    n = int(cap);
  }
  const int n_units = cdiv(n, CHUNK);
  const int span = p.balance ? cdiv(batch_max_len(p.seq_lens, p.batch, cap), CHUNK) : n_units;
  int u0, u1;
  split_range(split, S, n_units, span, &u0, &u1);
  const int t_begin = u0 * CHUNK;
  const int t_end = min(u1 * CHUNK, n);
  const int nchunks = u1 - u0;
  const int qh0 = h * p.group;

  if (nchunks <= 0 || t_begin >= t_end) {
    for (int idx = threadIdx.x; idx < p.group * D; idx += blockDim.x) {
      const int g = idx / D, d = idx % D;
      if (S == 1 && p.final_out) {
        p.out[int64_t(b) * p.o_sb + int64_t(qh0 + g) * p.o_sh + d] = __float2half_rn(0.f);
      } else {
        const int64_t row = (int64_t(b) * p.q_heads + qh0 + g) * S + split;
        p.o_part[row * D + d] = 0.f;
        if (d == 0) p.lse[row] = kNegInf;
      }
    }
    return;
  }

  // fp32 q of the group's heads (padding heads zero), for q' = q * k_scale
  for (int idx = threadIdx.x; idx < 8 * D; idx += blockDim.x) {
    const int g = idx / D, d = idx % D;
    sQ[idx] = g < p.group
                  ? __half2float(p.q[int64_t(b) * p.q_sb + int64_t(qh0 + g) * p.q_sh + d])
                  : 0.f;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1 + 32);  // producer's expect_tx arrive + 32 cp.async arrivals
      mbar_init(&empty[s], NCW);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();   // the merge grid may launch now; it waits for this grid's end

  if (warp == NCW) {
    // ------------------------------------------------------------------ producer warp
    const uint64_t pol = l2_evict_first_policy();
    const int32_t* bt = p.block_table + int64_t(b) * p.bt_sb;
    const int R = p.box_rows;                 // min(block_size, CHUNK)
    const int bs = p.block_size;
    const uint32_t box_bytes =
        uint32_t(R) * C::K_ROW + uint32_t(INT4 ? R / 2 : R) * 128u + (FP8 ? 256u : 512u);
    const int last_page = (t_end - 1) / bs;
    int win_base = t_begin / bs;
    int win = (win_base + lane <= last_page) ? __ldg(bt + win_base + lane) : 0;
    int issued = 0;
    for (int c = 0; c < nchunks; ++c) {
      const int stage = c % STAGES;
      const uint32_t par = uint32_t(c / STAGES) & 1u;
      bool w_ok = (lane == 0) ? mbar_wait(&empty[stage], par ^ 1u) : true;
      w_ok = __shfl_sync(kFullMask, w_ok, 0);
      if (!w_ok) {
        if (lane == 0) flag_device_error(p.status, BPT_DEV_WAIT_TIMEOUT);
        break;
      }
      uint8_t* st = smem + stage * C::STAGE_BYTES;
      uint8_t* kbuf = st;
      uint8_t* vbuf = st + C::K_BYTES;
      uint8_t* kpar = vbuf + C::V_BYTES;
      uint8_t* vpar = kpar + C::KP_BYTES;
      const int tok0 = (u0 + c) * CHUNK;
      const int tok_last = min(tok0 + CHUNK, t_end) - 1;
      if (tok_last / bs - win_base >= 32) {     // re-anchor the block-table window
        win_base = tok0 / bs;
        win = (win_base + lane <= last_page) ? __ldg(bt + win_base + lane) : 0;
      }
      const int nbox = min(CHUNK / R, cdiv(t_end - tok0, R));
      if (lane == 0) mbar_arrive_expect_tx(&full[stage], uint32_t(nbox) * box_bytes);
      for (int j = 0; j < nbox; ++j) {
        const int t = tok0 + j * R;
        const int pg = t / bs;
        int phys = __shfl_sync(kFullMask, win, pg - win_base);
        if (lane == 0) {
          if (phys < 0 || int64_t(phys) >= p.num_blocks) {
            flag_device_error(p.status, BPT_DEV_BAD_BLOCK_ID);
            phys = 0;
          }
          const int row = t - pg * bs;
          tma_load_4d(kbuf + j * R * C::K_ROW, &tmK, &full[stage], 0, p.k_c1 ? row : h,
                      p.k_c1 ? h : row, phys, pol);
          const int vrow = INT4 ? row / 2 : row;
          tma_load_4d(vbuf + j * (INT4 ? R / 2 : R) * 128, &tmV, &full[stage], 0,
                      p.v_c1 ? vrow : h, p.v_c1 ? h : vrow, phys, pol);
          // k_scale / k_zero rows [D] of (page, head): 3-D maps {D, H, blocks}
          tma_load_3d(kpar + j * 512, &tmKS, &full[stage], 0, h, phys);
          if (!FP8) tma_load_3d(kpar + j * 512 + 256, &tmKZ, &full[stage], 0, h, phys);
        }
      }
      // per-token value scale / zero (4-byte granules holding the head's fp16)
      for (int i = lane; i < CHUNK; i += 32) {
        const int t = tok0 + i;
        const int pg = min(t, tok_last) / bs;
        const int ph = __shfl_sync(kFullMask, win, pg - win_base);
        if (t <= tok_last && ph >= 0 && int64_t(ph) < p.num_blocks) {
          const int64_t el = int64_t(ph) * kp.vps0 + int64_t(t - pg * bs) * kp.vps1 + h;
          const int64_t off = (el * 2) & ~int64_t(3);
          cp_async_4(smem_u32(vpar + 4 * i), kp.v_scale + off);
          if (!FP8) cp_async_4(smem_u32(vpar + 4 * CHUNK + 4 * i), kp.v_zero + off);
        }
      }
      cp_async_arrive_noinc(&full[stage]);
      ++issued;
    }
    pdl_launch_dependents();
    if (lane == 0) {
      for (int c = max(0, issued - STAGES); c < issued; ++c)
        if (!mbar_wait(&full[c % STAGES], uint32_t(c / STAGES) & 1u))
          flag_device_error(p.status, BPT_DEV_WAIT_TIMEOUT);
    }
    return;
  }

  // -------------------------------------------------------------------- consumer warps
  const int g = lane >> 2, t4 = lane & 3;
  const int qhead = G8 ? g : (g & 3);
  const int mj = lane >> 3, mr = lane & 7;
  // ldmatrix rows for K: matrices (nb0, chunk c), (nb0, c+1), (nb1, c), (nb1, c+1) for
  // INT8/FP8; (nb0, c), (nb1, c), (nb0, c+1), (nb1, c+1) for INT4
  const int k_tok = INT4 ? (warp * 16 + 8 * (mj & 1) + mr) : (warp * 16 + 8 * (mj >> 1) + mr);
  const int k_csel = INT4 ? (mj >> 1) : (mj & 1);
  const uint32_t k_row_off = uint32_t(k_tok) * C::K_ROW;
  const uint32_t k_swz = INT4 ? uint32_t((k_tok >> 1) & 3) : uint32_t(k_tok & 7);
  // V rows this lane reads
  const int vc_chunk = INT4 ? (((g & 1) << 2) | (g >> 1)) : g;   // logical 16-byte chunk
  const float inv_group16 = 0.0625f;

  uint32_t qa0[8], qa1[8], qa2[8], qa3[8];   // q' hi (rows g) / lo (rows g+8) fragments
  float bias = 0.f;                          // sum_d q_d z_d for head qhead (INT formats)
  float kdown = 1.f;                         // 2^-kexp: undoes the q' normalisation
  int cur_page = -1;
  int vexp = 0x7fffffff;                     // running p' exponent of this warp (unset)

  float acc[C::NACC][8][4];
#pragma unroll
  for (int a = 0; a < C::NACC; ++a)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[a][i][0] = acc[a][i][1] = acc[a][i][2] = acc[a][i][3] = 0.f;
  float m_run = kNegInf, l_run = 0.f, z_run = 0.f;
  const float sl2 = p.scale_log2;
  const int colA = 2 * t4, colB = 2 * t4 + 1;
  const int srcA = (G8 ? colA : (colA & 3)) * 4, srcB = (G8 ? colB : (colB & 3)) * 4;

  for (int c = 0; c < nchunks; ++c) {
    const int stage = c % STAGES;
    const uint32_t par = uint32_t(c / STAGES) & 1u;
    const bool w_ok = __all_sync(kFullMask, mbar_wait(&full[stage], par));
    if (!w_ok) {
      if (lane == 0) flag_device_error(p.status, BPT_DEV_WAIT_TIMEOUT);
      break;
    }
    uint8_t* st = smem + stage * C::STAGE_BYTES;
    const uint32_t kbase = smem_u32(st);
    uint8_t* vbuf = st + C::K_BYTES;
    const __half* kpar = reinterpret_cast<const __half*>(vbuf + C::V_BYTES);
    const uint32_t* vpar = reinterpret_cast<const uint32_t*>(vbuf + C::V_BYTES + C::KP_BYTES);
    const int tok0 = (u0 + c) * CHUNK;
    const int lim = t_end - tok0 - warp * 16;       // valid rows of this warp's 16
    const int R = p.box_rows;
    const int slot = (warp * 16) / R;              // box (page) holding this warp's rows
    const int page = (tok0 + warp * 16) / p.block_size;

    // ---- q' = q * k_scale (hi / lo fp16, normalised by 2^kexp) and the zero-point bias,
    //      once per page
    if (page != cur_page) {
      cur_page = page;
      const __half* ks = kpar + slot * 256;
      const __half* kz = ks + 128;
      float bsum = 0.f, qmax = 0.f;
#pragma unroll
      for (int ks_i = 0; ks_i < 8; ++ks_i)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float mult;
          const int ch = q_channel<INT4>(ks_i, e, t4, mult);
          const float qv = sQ[qhead * D + ch];
          const float sk = __half2float(ks[ch]);
          qmax = fmaxf(qmax, fabsf(qv * sk * mult));
          if (!FP8) bsum = fmaf(qv, fmaf(kC0, sk, __half2float(kz[ch])), bsum);
        }
      qmax = fmaxf(qmax, __shfl_xor_sync(kFullMask, qmax, 1));
      qmax = fmaxf(qmax, __shfl_xor_sync(kFullMask, qmax, 2));
      const int kexp = (qmax > 0.f && qmax < INFINITY) ? norm_exponent(qmax) : 0;
      const float kup = exp2i(kexp);
      kdown = exp2i(-kexp);
#pragma unroll
      for (int ks_i = 0; ks_i < 8; ++ks_i) {
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float mult;
          const int ch = q_channel<INT4>(ks_i, e, t4, mult);
          v[e] = sQ[qhead * D + ch] * __half2float(ks[ch]) * (mult * kup);
        }
        uint32_t h01, l01, h23, l23;
        mma::split_hi_lo(v[0], v[1], h01, l01);
        mma::split_hi_lo(v[2], v[3], h23, l23);
        qa0[ks_i] = h01; qa1[ks_i] = l01; qa2[ks_i] = h23; qa3[ks_i] = l23;
      }
      if (!FP8) {
        bsum += __shfl_xor_sync(kFullMask, bsum, 1);
        bsum += __shfl_xor_sync(kFullMask, bsum, 2);
        bias = bsum;
      }
    }

    // ---- S = q' . codes (rows g: hi, rows g+8: lo; total = sum of both)
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
    if constexpr (INT4) {
#pragma unroll
      for (int cc = 0; cc < 4; cc += 2) {
        const uint32_t ch = uint32_t(cc + k_csel) ^ k_swz;
        uint32_t w0, w1, w2, w3;  // (nb0, cc), (nb1, cc), (nb0, cc+1), (nb1, cc+1)
        ldsm_x4(kbase + k_row_off + (ch << 4), w0, w1, w2, w3);
        const uint32_t ws[4] = {w0, w1, w2, w3};
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const int chunk = cc + (m >> 1);
          float* sacc = (m & 1) ? s1 : s0;
          const uint32_t w = ws[m], w8 = ws[m] >> 8;
          const uint32_t h0 = hsub_const<1024 + kC0Int4>((w & 0x000F000Fu) | kMagic);
          const uint32_t h1 = hsub_const<1024 + 16 * kC0Int4>((w & 0x00F000F0u) | kMagic);
          const uint32_t h2 = hsub_const<1024 + kC0Int4>((w8 & 0x000F000Fu) | kMagic);
          const uint32_t h3 = hsub_const<1024 + 16 * kC0Int4>((w8 & 0x00F000F0u) | kMagic);
          const int k0 = 2 * chunk, k1 = 2 * chunk + 1;
          float t0[4] = {sacc[0], sacc[1], sacc[2], sacc[3]};
          mma_16816(t0, qa0[k0], qa1[k0], qa2[k0], qa3[k0], h0, h2);
          mma_16816(t0, qa0[k1], qa1[k1], qa2[k1], qa3[k1], h1, h3);
          sacc[0] = t0[0]; sacc[1] = t0[1]; sacc[2] = t0[2]; sacc[3] = t0[3];
        }
      }
    } else {
#pragma unroll
      for (int kk = 0; kk < 8; kk += 2) {
        const uint32_t ch = uint32_t(kk + k_csel) ^ k_swz;
        uint32_t w0, w1, w2, w3;  // (nb0, kk), (nb0, kk+1), (nb1, kk), (nb1, kk+1)
        ldsm_x4(kbase + k_row_off + (ch << 4), w0, w1, w2, w3);
        const uint32_t ws[4] = {w0, w1, w2, w3};
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const int ks_i = kk + (m & 1);
          float* sacc = (m >> 1) ? s1 : s0;
          uint32_t b0, b1;
          if constexpr (FP8) {
            b0 = cvt_e4m3x2(ws[m]);
            b1 = cvt_e4m3x2(ws[m] >> 16);
          } else {
            b0 = hsub_const<1024 + kC0Int8>(__byte_perm(ws[m], kMagicBytes, 0x4140));
            b1 = hsub_const<1024 + kC0Int8>(__byte_perm(ws[m], kMagicBytes, 0x4342));
          }
          float t0[4] = {sacc[0], sacc[1], sacc[2], sacc[3]};
          mma_16816(t0, qa0[ks_i], qa1[ks_i], qa2[ks_i], qa3[ks_i], b0, b1);
          sacc[0] = t0[0]; sacc[1] = t0[1]; sacc[2] = t0[2]; sacc[3] = t0[3];
        }
      }
    }

    // ---- online softmax; this lane owns q head `qhead`, tokens 2t, 2t+1, 2t+8, 2t+9
    const int tk = 2 * t4;
    const float bsc = FP8 ? 0.f : bias;
    const float x0 = (tk < lim) ? fmaf(s0[0] + s0[2], kdown, bsc) * sl2 : kNegInf;
    const float x1 = (tk + 1 < lim) ? fmaf(s0[1] + s0[3], kdown, bsc) * sl2 : kNegInf;
    const float x2 = (tk + 8 < lim) ? fmaf(s1[0] + s1[2], kdown, bsc) * sl2 : kNegInf;
    const float x3 = (tk + 9 < lim) ? fmaf(s1[1] + s1[3], kdown, bsc) * sl2 : kNegInf;
    float mx = fmaxf(fmaxf(x0, x1), fmaxf(x2, x3));
    mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, 2));
    const float m_new = fmaxf(m_run, mx);
    if (__any_sync(kFullMask, m_new > m_run)) {
      const float alpha = fast_exp2(m_run - (m_new == kNegInf ? 0.f : m_new));
      l_run *= alpha;
      z_run *= alpha;
      const float aA = __shfl_sync(kFullMask, alpha, srcA);
      const float aB = __shfl_sync(kFullMask, alpha, srcB);
#pragma unroll
      for (int a = 0; a < C::NACC; ++a)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          acc[a][i][0] *= aA; acc[a][i][1] *= aB; acc[a][i][2] *= aA; acc[a][i][3] *= aB;
        }
      m_run = m_new;
    }
    const float m_use = (m_run == kNegInf) ? 0.f : m_run;
    const float p0 = fast_exp2(x0 - m_use), p1 = fast_exp2(x1 - m_use);
    const float p2 = fast_exp2(x2 - m_use), p3 = fast_exp2(x3 - m_use);
    l_run += (p0 + p1) + (p2 + p3);

    // value scale / zero of the four tokens (invalid tokens: p = 0 and never touch the data)
    const int trow = warp * 16 + tk;
    float vsv[4], vzv[4];
    const int trows[4] = {trow, trow + 1, trow + 8, trow + 9};
    const float pv[4] = {p0, p1, p2, p3};
    float pp[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const bool ok = pv[e] > 0.f;
      // the 4-byte granule holding this (token, head) element; block strides are even, so
      // the element's half is the parity of (row in page) * token stride + head
      const int rowp = (tok0 + trows[e]) & (p.block_size - 1);
      const int half_sel = int((int64_t(rowp) * kp.vps1 + h) & 1);
      uint32_t gs = vpar[trows[e]];
      const __half2 hs = *reinterpret_cast<__half2*>(&gs);
      vsv[e] = half_sel ? __high2float(hs) : __low2float(hs);
      if (!FP8) {
        uint32_t gz = vpar[CHUNK + trows[e]];
        const __half2 hz = *reinterpret_cast<__half2*>(&gz);
        vzv[e] = half_sel ? __high2float(hz) : __low2float(hz);
        z_run = ok ? fmaf(pv[e], fmaf(kC0, vsv[e], vzv[e]), z_run) : z_run;
      }
      pp[e] = ok ? pv[e] * vsv[e] : 0.f;
    }
    // keep p' = p * v_scale * 2^vexp in fp16's normal range: vexp follows the largest value
    // scale seen by this warp (it only decreases; acc is rescaled by an exact power of two)
    {
      float vmx = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (pv[e] > 0.f) vmx = fmaxf(vmx, fabsf(vsv[e]));
      vmx = fmaxf(vmx, __shfl_xor_sync(kFullMask, vmx, 1));
      vmx = fmaxf(vmx, __shfl_xor_sync(kFullMask, vmx, 2));
      if (vmx > 0.f && vmx < INFINITY) {
        const int ve = norm_exponent(vmx);
        if (vexp == 0x7fffffff) {
          vexp = ve;
        } else if (ve < vexp) {
          const float f = exp2i(ve - vexp);
#pragma unroll
          for (int a = 0; a < C::NACC; ++a)
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              acc[a][i][0] *= f; acc[a][i][1] *= f; acc[a][i][2] *= f; acc[a][i][3] *= f;
            }
          vexp = ve;
        }
      }
      const float vup = exp2i(vexp == 0x7fffffff ? 0 : vexp);
#pragma unroll
      for (int e = 0; e < 4; ++e) pp[e] *= vup;
    }
    uint32_t pb0, pb1, lo0, lo1;
    if constexpr (INT4) {
      // k-slots: 2t <- token 2t, 2t+1 <- 2t+8 (low nibbles); 2t+8 <- 2t+1, 2t+9 <- 2t+9
      // (high nibbles, stored x16)
      uint32_t h02, l02, h13, l13;
      mma::split_hi_lo(pp[0], pp[2], h02, l02);
      mma::split_hi_lo(pp[1] * inv_group16, pp[3] * inv_group16, h13, l13);
      pb0 = G8 ? h02 : (g < 4 ? h02 : l02);
      pb1 = G8 ? h13 : (g < 4 ? h13 : l13);
      lo0 = l02;
      lo1 = l13;
    } else {
      uint32_t h01, l01, h23, l23;
      mma::split_hi_lo(pp[0], pp[1], h01, l01);
      mma::split_hi_lo(pp[2], pp[3], h23, l23);
      pb0 = G8 ? h01 : (g < 4 ? h01 : l01);
      pb1 = G8 ? h23 : (g < 4 ? h23 : l23);
      lo0 = l01;
      lo1 = l23;
    }

    // FP8 codes can encode NaN: zero the V rows of invalid tokens (INT codes are finite)
    if (FP8 && lim < 16) {
      for (int idx = lane; idx < 16 * 8; idx += 32) {
        const int r = idx >> 3, ch = idx & 7;
        if (r >= lim)
          *reinterpret_cast<uint4*>(vbuf + (warp * 16 + r) * 128 + ch * 16) =
              make_uint4(0u, 0u, 0u, 0u);
      }
      __syncwarp();
    }

    // ---- O^T += V^T P'^T
    uint4 va, vb, vcw, vd;
    if constexpr (INT4) {
      const int pr0 = warp * 8 + t4, pr1 = warp * 8 + t4 + 4;
      va = *reinterpret_cast<const uint4*>(vbuf + pr0 * 128 + ((vc_chunk ^ (pr0 & 7)) << 4));
      vb = *reinterpret_cast<const uint4*>(vbuf + pr1 * 128 + ((vc_chunk ^ (pr1 & 7)) << 4));
      const uint32_t P[4] = {va.x, va.y, va.z, va.w}, Q[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const uint32_t r = __byte_perm(P[m >> 1], Q[m >> 1], (m & 1) ? 0x7632 : 0x5410);
        const uint32_t r8 = r >> 8;
        const uint32_t a0 = hsub_const<1024 + kC0Int4>((r & 0x000F000Fu) | kMagic);
        const uint32_t a1 = hsub_const<1024 + kC0Int4>((r8 & 0x000F000Fu) | kMagic);
        const uint32_t a2 = hsub_const<1024 + 16 * kC0Int4>((r & 0x00F000F0u) | kMagic);
        const uint32_t a3 = hsub_const<1024 + 16 * kC0Int4>((r8 & 0x00F000F0u) | kMagic);
        mma::mma_16816_acc(acc[0][m], a0, a1, a2, a3, pb0, pb1);
        if constexpr (G8) mma::mma_16816_acc(acc[C::NACC - 1][m], a0, a1, a2, a3, lo0, lo1);
      }
    } else {
      const int r0 = warp * 16 + tk, r1 = r0 + 1, r2 = r0 + 8, r3 = r0 + 9;
      va = *reinterpret_cast<const uint4*>(vbuf + r0 * 128 + ((vc_chunk ^ (r0 & 7)) << 4));
      vb = *reinterpret_cast<const uint4*>(vbuf + r1 * 128 + ((vc_chunk ^ (r1 & 7)) << 4));
      vcw = *reinterpret_cast<const uint4*>(vbuf + r2 * 128 + ((vc_chunk ^ (r2 & 7)) << 4));
      vd = *reinterpret_cast<const uint4*>(vbuf + r3 * 128 + ((vc_chunk ^ (r3 & 7)) << 4));
      const uint32_t A[4] = {va.x, va.y, va.z, va.w}, B[4] = {vb.x, vb.y, vb.z, vb.w};
      const uint32_t Cw[4] = {vcw.x, vcw.y, vcw.z, vcw.w}, Dw[4] = {vd.x, vd.y, vd.z, vd.w};
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const uint32_t sel = (m & 1) ? 0x7362u : 0x5140u;
        const uint32_t X = __byte_perm(A[m >> 1], B[m >> 1], sel);
        const uint32_t Y = __byte_perm(Cw[m >> 1], Dw[m >> 1], sel);
        uint32_t a0, a1, a2, a3;
        if constexpr (FP8) {
          a0 = cvt_e4m3x2(X); a1 = cvt_e4m3x2(X >> 16);
          a2 = cvt_e4m3x2(Y); a3 = cvt_e4m3x2(Y >> 16);
        } else {
          a0 = hsub_const<1024 + kC0Int8>(__byte_perm(X, kMagicBytes, 0x4140));
          a1 = hsub_const<1024 + kC0Int8>(__byte_perm(X, kMagicBytes, 0x4342));
          a2 = hsub_const<1024 + kC0Int8>(__byte_perm(Y, kMagicBytes, 0x4140));
          a3 = hsub_const<1024 + kC0Int8>(__byte_perm(Y, kMagicBytes, 0x4342));
        }
        mma::mma_16816_acc(acc[0][m], a0, a1, a2, a3, pb0, pb1);
        if constexpr (G8) mma::mma_16816_acc(acc[C::NACC - 1][m], a0, a1, a2, a3, lo0, lo1);
      }
    }
    if (FP8 && lim < 16) mma::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
  }

  pdl_launch_dependents();
  l_run += __shfl_xor_sync(kFullMask, l_run, 1);
  l_run += __shfl_xor_sync(kFullMask, l_run, 2);
  z_run += __shfl_xor_sync(kFullMask, z_run, 1);
  z_run += __shfl_xor_sync(kFullMask, z_run, 2);
  // per-head zero-point term for this lane's output columns (heads colA, colB)
  const float zA = __shfl_sync(kFullMask, z_run, srcA);
  const float zB = __shfl_sync(kFullMask, z_run, srcB);
  const float vdown = exp2i(vexp == 0x7fffffff ? 0 : -vexp);
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if constexpr (G8) {
        acc[0][i][e] += acc[C::NACC - 1][i][e];
      } else {
        acc[0][i][e] += __shfl_xor_sync(kFullMask, acc[0][i][e], 2);
      }
      acc[0][i][e] *= vdown;
    }
  named_barrier_sync(1, NCW * 32);
  if (t4 == 0 && (G8 || g < 4)) {
    sM[warp * 8 + qhead] = m_run;
    sL[warp * 8 + qhead] = l_run;
  }
  if (G8 || t4 < 2) {
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      const int d0 = 16 * vc_chunk + 2 * m;   // row g of MMA m; row g+8 is d0 + 1
      sAcc[(warp * 8 + colA) * D + d0] = acc[0][m][0] + (FP8 ? 0.f : zA);
      sAcc[(warp * 8 + colB) * D + d0] = acc[0][m][1] + (FP8 ? 0.f : zB);
      sAcc[(warp * 8 + colA) * D + d0 + 1] = acc[0][m][2] + (FP8 ? 0.f : zA);
      sAcc[(warp * 8 + colB) * D + d0 + 1] = acc[0][m][3] + (FP8 ? 0.f : zB);
    }
  }
  named_barrier_sync(1, NCW * 32);
  write_split_state<NCW, D>(sM, sL, sAcc, sAcc + NCW * 8 * D, p, b, qh0, split,
                            int(threadIdx.x), NCW * 32,
                            [] { named_barrier_sync(1, NCW * 32); });
}

#ifndef BPT_KIVI_NCW
#define BPT_KIVI_NCW 2
#endif
#ifndef BPT_KIVI_STAGES
#define BPT_KIVI_STAGES 4
#endif
#ifndef BPT_KIVI_MINB
#define BPT_KIVI_MINB 4
#endif

constexpr int kNcw = BPT_KIVI_NCW;

template <int FMT, bool G8>
int launch(const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tks,
           const CUtensorMap& tkz, const KiviParams& kp, cudaStream_t st) {
  using C = Cfg<FMT, kNcw, BPT_KIVI_STAGES, G8>;
  auto kern = kivi_decode_kernel<FMT, kNcw, BPT_KIVI_STAGES, BPT_KIVI_MINB, G8>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           int(C::SMEM_BYTES)) != cudaSuccess)
    return BPT_ERR_LAUNCH;
  dim3 grid(kp.d.splits, kp.d.kv_heads, kp.d.batch);
  return launch_dependent(kern, grid, dim3(C::THREADS), C::SMEM_BYTES, st, tk, tv, tks, tkz,
                          kp) == cudaSuccess
             ? BPT_OK
             : BPT_ERR_LAUNCH;
}

#include "kivi_int.cuh"

#ifndef BPT_KIVI_INT8_STAGES
#define BPT_KIVI_INT8_STAGES 3
#endif
#ifndef BPT_KIVI_INT4_STAGES
#define BPT_KIVI_INT4_STAGES 3
#endif
#ifndef BPT_KIVI_INT_MINB
#define BPT_KIVI_INT_MINB 3
#endif

#include "kivi_tc.cuh"

#ifndef BPT_KIVI_TC_KSLOTS
#define BPT_KIVI_TC_KSLOTS 2
#endif
#ifndef BPT_KIVI_TC_VSLOTS
#define BPT_KIVI_TC_VSLOTS 3
#endif
#ifndef BPT_KIVI_TC_MINB
#define BPT_KIVI_TC_MINB 2
#endif
// INT4 at large batch and long context uses a second tcgen05 shape: a 2-slot value ring, which
// fits 3 CTAs per SM. Measured on one B200: INT4 B=64/32k 929 -> 882 us, B=32/32k 506 ->
// 490 us; but B=1/128k 64.9 -> 67.6 us and B=32/8k ~181 -> 209 us (more splits, so fewer
// chunks per CTA to amortise its setup). It serves calls with batch * kv_heads >= MIN_CTAS
// and a block table of at least MIN_TOKENS tokens.
#ifndef BPT_KIVI_TC_WIDE_MIN_CTAS
#define BPT_KIVI_TC_WIDE_MIN_CTAS 256
#endif
#ifndef BPT_KIVI_TC_WIDE_MIN_TOKENS
#define BPT_KIVI_TC_WIDE_MIN_TOKENS 32768
#endif

template <int FMT, bool WIDE = false>
using TcCfg = TCfg<FMT, BPT_KIVI_TC_KSLOTS, WIDE ? 2 : BPT_KIVI_TC_VSLOTS>;
template <bool WIDE>
constexpr int tc_minb() {
  return WIDE ? 3 : BPT_KIVI_TC_MINB;
}

inline bool tc_wide(int format, int batch, int kv_heads, int block_size, int max_blocks) {
  return format == BPT_KV_INT4 && int64_t(batch) * kv_heads >= BPT_KIVI_TC_WIDE_MIN_CTAS &&
         int64_t(max_blocks) * block_size >= BPT_KIVI_TC_WIDE_MIN_TOKENS;
}

template <int FMT>
using IntCfg =
    ICfg<FMT, FMT == BPT_KV_INT4 ? BPT_KIVI_INT4_STAGES : BPT_KIVI_INT8_STAGES>;

constexpr int kSmemPerSm = 228 * 1024;   // shared memory of one B200 SM
constexpr int kSmemPerCtaReserved = 1024;

template <int FMT>
int int_resident_ctas(int block_size) {
  using C = IntCfg<FMT>;
  const int box = block_size < C::CHUNK ? block_size : C::CHUNK;
  const int per = int(C::smem_bytes(C::CHUNK / box)) + kSmemPerCtaReserved;
  int r = kSmemPerSm / per;
  if (r > BPT_KIVI_INT_MINB) r = BPT_KIVI_INT_MINB;
  return r < 1 ? 1 : r;
}

template <int FMT, bool WIDE = false>
int tc_resident_ctas(int block_size) {
  using C = TcCfg<FMT, WIDE>;
  const int box = block_size < C::CHUNK ? block_size : C::CHUNK;
  const int per = int(C::smem_bytes(C::CHUNK / box)) + kSmemPerCtaReserved;
  int r = kSmemPerSm / per;
  if (r > tc_minb<WIDE>()) r = tc_minb<WIDE>();
  return r < 1 ? 1 : r;
}

template <int FMT, bool WIDE = false>
int launch_tc(const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tks,
              const CUtensorMap& tkz, const CUtensorMap& tvs, const CUtensorMap& tvz,
              const KiviParams& kp, cudaStream_t st) {
  using C = TcCfg<FMT, WIDE>;
  auto kern = kivi_tc_decode_kernel<FMT, BPT_KIVI_TC_KSLOTS, WIDE ? 2 : BPT_KIVI_TC_VSLOTS,
                                    tc_minb<WIDE>()>;
  const size_t smem = C::smem_bytes(C::CHUNK / kp.d.box_rows);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) !=
      cudaSuccess)
    return BPT_ERR_LAUNCH;
  dim3 grid(kp.d.splits, kp.d.kv_heads, kp.d.batch);
  return launch_dependent(kern, grid, dim3(C::THREADS), smem, st, tk, tv, tks, tkz, tvs, tvz,
                          kp) == cudaSuccess
             ? BPT_OK
             : BPT_ERR_LAUNCH;
}

template <int FMT>
int launch_int(const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tks,
               const CUtensorMap& tkz, const KiviParams& kp, cudaStream_t st) {
  using C = IntCfg<FMT>;
  constexpr int kStages = FMT == BPT_KV_INT4 ? BPT_KIVI_INT4_STAGES : BPT_KIVI_INT8_STAGES;
  auto kern = kivi_int_decode_kernel<FMT, kStages, BPT_KIVI_INT_MINB>;
  const size_t smem = C::smem_bytes(C::CHUNK / kp.d.box_rows);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) !=
      cudaSuccess)
    return BPT_ERR_LAUNCH;
  dim3 grid(kp.d.splits, kp.d.kv_heads, kp.d.batch);
  return launch_dependent(kern, grid, dim3(C::THREADS), smem, st, tk, tv, tks, tkz, kp) ==
                 cudaSuccess
             ? BPT_OK
             : BPT_ERR_LAUNCH;
}

}  // namespace kivi

// 3-D tiled map over a [num_blocks, H, 128] fp16 parameter array (unit inner stride), box =
// one (block, head) row of 128 values.
int encode_param_map(CUtensorMap* map, const void* base, int kv_heads, int64_t num_blocks,
                     int64_t s_blk, int64_t s_head) {
  auto enc = tensor_map_encoder_fn();
  if (!enc) return BPT_ERR_DRIVER;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((s_blk * 2) % 16) || ((s_head * 2) % 16))
    return BPT_ERR_ALIGNMENT;
  cuuint64_t dims[3] = {cuuint64_t(kivi::D), cuuint64_t(kv_heads),
                        cuuint64_t(num_blocks > 0 ? num_blocks : 1)};
  cuuint64_t strides[2] = {cuuint64_t(s_head * 2), cuuint64_t(s_blk * 2)};
  cuuint32_t box[3] = {cuuint32_t(kivi::D), 1u, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? BPT_OK : BPT_ERR_TENSOR_MAP;
}

// 3-D tiled map over a [num_blocks, block_size, H] fp16 per-token parameter array (v_scale /
// v_zero), box = 8 heads x box_rows tokens of one block.
int encode_vparam_map(CUtensorMap* map, const void* base, int kv_heads, int block_size,
                      int64_t num_blocks, int64_t s_blk, int64_t s_tok, int box_rows) {
  auto enc = tensor_map_encoder_fn();
  if (!enc) return BPT_ERR_DRIVER;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((s_blk * 2) % 16) || ((s_tok * 2) % 16))
    return BPT_ERR_ALIGNMENT;
  cuuint64_t dims[3] = {cuuint64_t(kv_heads), cuuint64_t(block_size),
                        cuuint64_t(num_blocks > 0 ? num_blocks : 1)};
  cuuint64_t strides[2] = {cuuint64_t(s_tok * 2), cuuint64_t(s_blk * 2)};
  cuuint32_t box[3] = {8u, cuuint32_t(box_rows), 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? BPT_OK : BPT_ERR_TENSOR_MAP;
}

namespace {

int ilog2(int x) {
  int r = 0;
  while ((1 << (r + 1)) <= x) ++r;
  return r;
}

// Which KIVI kernel serves a (format, group, block_size, kv_heads):
//   TC   INT8 / INT4, group <= 4, block_size >= 32, kv_heads a multiple of 8 (the per-token
//        value parameters arrive as TMA boxes of 8 heads): tcgen05 integer MMAs (kivi_tc.cuh)
//   INT  other INT8 / INT4 with group <= 4: mma.sync integer MMAs (kivi_int.cuh)
//   F16  FP8, or group > 4: fp16 mma.sync with hi / lo operand pairs (this file)
// TC and INT share the 128-token chunk, so the split count does not depend on the choice.
enum class KiviKernel { TC, INT, F16 };

KiviKernel kivi_kernel_for(int format, int group, int block_size, int kv_heads) {
  if ((format == BPT_KV_INT8 || format == BPT_KV_INT4) && group <= 4)
    return (block_size >= 32 && kv_heads % 8 == 0) ? KiviKernel::TC : KiviKernel::INT;
  return KiviKernel::F16;
}

// tokens per pipeline stage and CTAs per SM of the kernel serving (format, group)
void kivi_kernel_shape(int format, int group, int block_size, int kv_heads, int batch,
                       int max_blocks, int* chunk, int* resident) {
  using namespace kivi;
  const bool int4 = format == BPT_KV_INT4;
  switch (kivi_kernel_for(format, group, block_size, kv_heads)) {
    case KiviKernel::TC:
      *chunk = TcCfg<BPT_KV_INT8>::CHUNK;
      *resident = !int4 ? tc_resident_ctas<BPT_KV_INT8>(block_size)
                  : tc_wide(format, batch, kv_heads, block_size, max_blocks)
                      ? tc_resident_ctas<BPT_KV_INT4, true>(block_size)
                      : tc_resident_ctas<BPT_KV_INT4>(block_size);
      break;
    case KiviKernel::INT:
      *chunk = IntCfg<BPT_KV_INT8>::CHUNK;
      *resident = int4 ? int_resident_ctas<BPT_KV_INT4>(block_size)
                       : int_resident_ctas<BPT_KV_INT8>(block_size);
      break;
    default:
      *chunk = 16 * kNcw;
      *resident = BPT_KIVI_MINB;
  }
}

}  // namespace

int effective_splits_kivi(int format, int batch, int kv_heads, int q_heads, int block_size,
                          int max_blocks, int num_splits, int sm_count) {
  const int group = (kv_heads > 0 && q_heads > 0) ? q_heads / kv_heads : 1;
  int chunk, resident;
  kivi_kernel_shape(format, group, block_size, kv_heads, batch, max_blocks, &chunk, &resident);
  const int s = num_splits > 0 ? num_splits
                               : plan_splits(batch, kv_heads, block_size, max_blocks, sm_count,
                                             resident, chunk);
  return clamp_splits(s, block_size, max_blocks, chunk);
}

// Launch the KIVI split kernel (final_out: one split writes fp16 out directly).
int run_split_kivi(const bpt_kivi_cache& c, const void* q, int64_t q_sb, int64_t q_sh,
                   const int32_t* block_table, int64_t bt_sb, const int32_t* seq_lens,
                   void* out, int64_t o_sb, int64_t o_sh, int batch, int q_heads,
                   int max_blocks, float scale, int splits, int final_out, float* o_part,
                   float* lse, unsigned* status, cudaStream_t st) {
  using namespace kivi;
  if (batch < 0 || q_heads <= 0 || c.kv_heads <= 0 || q_heads % c.kv_heads || splits < 1 ||
      max_blocks < 0)
    return BPT_ERR_INVALID_ARGUMENT;
  if (batch == 0) return BPT_OK;
  if (c.format != BPT_KV_INT8 && c.format != BPT_KV_FP8_E4M3 && c.format != BPT_KV_INT4)
    return BPT_ERR_INVALID_ARGUMENT;
  if (c.head_dim != D) return BPT_ERR_UNSUPPORTED_SHAPE;
  const int group = q_heads / c.kv_heads;
  if (group > 8) return BPT_ERR_UNSUPPORTED_SHAPE;
  const int bs = c.block_size;
  if (bs < 16 || bs > 256 || (bs & (bs - 1))) return BPT_ERR_UNSUPPORTED_SHAPE;
  if (!q || !block_table || !seq_lens || !c.k_codes || !c.v_codes || !c.k_scale || !c.v_scale)
    return BPT_ERR_INVALID_ARGUMENT;
  const bool fp8 = c.format == BPT_KV_FP8_E4M3;
  if (!fp8 && (!c.k_zero || !c.v_zero)) return BPT_ERR_INVALID_ARGUMENT;
  if (final_out ? !out : (!o_part || !lse)) return BPT_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(q) & 15) || ((q_sb * 2) % 16) || ((q_sh * 2) % 16))
    return BPT_ERR_ALIGNMENT;
  if ((reinterpret_cast<uintptr_t>(c.v_scale) & 3) ||
      (!fp8 && (reinterpret_cast<uintptr_t>(c.v_zero) & 3)) || (c.v_param_stride[0] & 1))
    return BPT_ERR_ALIGNMENT;

  KiviParams kp{};
  DecodeParams& p = kp.d;
  KiviKernel which = kivi_kernel_for(c.format, group, bs, c.kv_heads);
  // the value-parameter TMA boxes need 16-byte aligned bases and strides
  if (which == KiviKernel::TC &&
      ((reinterpret_cast<uintptr_t>(c.v_scale) & 15) ||
       (reinterpret_cast<uintptr_t>(c.v_zero) & 15) || ((c.v_param_stride[0] * 2) % 16) ||
       ((c.v_param_stride[1] * 2) % 16)))
    which = KiviKernel::INT;
  const int chunk = which == KiviKernel::TC    ? TcCfg<BPT_KV_INT8>::CHUNK
                    : which == KiviKernel::INT ? IntCfg<BPT_KV_INT8>::CHUNK
                                               : 16 * kNcw;
  const int box_rows = bs < chunk ? bs : chunk;
  const bool int4 = c.format == BPT_KV_INT4;
  CUtensorMap tk, tv, tks, tkz;
  int rc = encode_kv_map(&tk, c.k_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, int4 ? D / 2 : D,
                         c.kv_heads, bs, c.num_blocks, c.k_codes_stride[2], c.k_codes_stride[1],
                         c.k_codes_stride[0], int4 ? D / 2 : D, box_rows, &p.k_c1,
                         int4 ? 64 : 128);
  if (rc) return rc;
  rc = encode_kv_map(&tv, c.v_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, D, c.kv_heads,
                     int4 ? bs / 2 : bs, c.num_blocks, c.v_codes_stride[2], c.v_codes_stride[1],
                     c.v_codes_stride[0], D, int4 ? box_rows / 2 : box_rows, &p.v_c1, 128);
  if (rc) return rc;
  rc = encode_param_map(&tks, c.k_scale, c.kv_heads, c.num_blocks, c.k_param_stride[0],
                        c.k_param_stride[1]);
  if (rc) return rc;
  rc = encode_param_map(&tkz, fp8 ? c.k_scale : c.k_zero, c.kv_heads, c.num_blocks,
                        c.k_param_stride[0], c.k_param_stride[1]);
  if (rc) return rc;
  p.q = static_cast<const __half*>(q);
  p.q_sb = q_sb;
  p.q_sh = q_sh;
  p.block_table = block_table;
  p.bt_sb = bt_sb;
  p.seq_lens = seq_lens;
  p.out = static_cast<__half*>(out);
  p.o_sb = o_sb;
  p.o_sh = o_sh;
  p.o_part = o_part;
  p.lse = lse;
  p.status = status;
  p.batch = batch;
  p.q_heads = q_heads;
  p.kv_heads = c.kv_heads;
  p.group = group;
  p.splits = splits;
  p.final_out = final_out;
  {
    int kchunk = 0, kresident = 1;
    kivi_kernel_shape(c.format, group, bs, c.kv_heads, batch, max_blocks, &kchunk, &kresident);
    p.balance = balanced_splits(batch, c.kv_heads, splits, kresident) ? 1 : 0;
  }
  p.block_size = bs;
  p.max_blocks = max_blocks;
  p.box_rows = box_rows;
  p.num_blocks = c.num_blocks;
  const float sc = scale > 0.f ? scale : 1.0f / sqrtf(float(D));
  p.scale_log2 = sc * 1.4426950408889634f;
  kp.v_scale = static_cast<const uint8_t*>(c.v_scale);
  kp.v_zero = static_cast<const uint8_t*>(fp8 ? c.v_scale : c.v_zero);
  kp.vps0 = c.v_param_stride[0];
  kp.vps1 = c.v_param_stride[1];
  kp.lbs = ilog2(bs);
  kp.lbox = ilog2(box_rows);
  const bool g8 = group > 4;
  if (which != KiviKernel::F16) {
    if (which == KiviKernel::TC) {
      CUtensorMap tvs, tvz;
      rc = encode_vparam_map(&tvs, c.v_scale, c.kv_heads, bs, c.num_blocks, c.v_param_stride[0],
                             c.v_param_stride[1], box_rows);
      if (rc) return rc;
      rc = encode_vparam_map(&tvz, c.v_zero, c.kv_heads, bs, c.num_blocks, c.v_param_stride[0],
                             c.v_param_stride[1], box_rows);
      if (rc) return rc;
      if (!int4)
        rc = launch_tc<BPT_KV_INT8>(tk, tv, tks, tkz, tvs, tvz, kp, st);
      else if (tc_wide(c.format, batch, c.kv_heads, bs, max_blocks))
        rc = launch_tc<BPT_KV_INT4, true>(tk, tv, tks, tkz, tvs, tvz, kp, st);
      else
        rc = launch_tc<BPT_KV_INT4>(tk, tv, tks, tkz, tvs, tvz, kp, st);
    } else
      rc = int4 ? launch_int<BPT_KV_INT4>(tk, tv, tks, tkz, kp, st)
                : launch_int<BPT_KV_INT8>(tk, tv, tks, tkz, kp, st);
    if (rc) return rc;
    return cudaGetLastError() == cudaSuccess ? BPT_OK : BPT_ERR_LAUNCH;
  }
  switch (c.format) {
    case BPT_KV_INT8:
      rc = g8 ? launch<BPT_KV_INT8, true>(tk, tv, tks, tkz, kp, st)
              : launch<BPT_KV_INT8, false>(tk, tv, tks, tkz, kp, st);
      break;
    case BPT_KV_FP8_E4M3:
      rc = g8 ? launch<BPT_KV_FP8_E4M3, true>(tk, tv, tks, tkz, kp, st)
              : launch<BPT_KV_FP8_E4M3, false>(tk, tv, tks, tkz, kp, st);
      break;
    default:
      rc = g8 ? launch<BPT_KV_INT4, true>(tk, tv, tks, tkz, kp, st)
              : launch<BPT_KV_INT4, false>(tk, tv, tks, tkz, kp, st);
  }
  if (rc) return rc;
  return cudaGetLastError() == cudaSuccess ? BPT_OK : BPT_ERR_LAUNCH;
}

}  // namespace bpt

using namespace bpt;

extern "C" int bpt_decode_kivi(const bpt_kivi_cache* cache, const void* q, int64_t q_sb,
                               int64_t q_sh, const int32_t* block_table, int64_t bt_sb,
                               const int32_t* seq_lens, void* out, int64_t o_sb, int64_t o_sh,
                               int batch, int q_heads, int max_blocks, float scale,
                               int num_splits, int sm_count, void* workspace,
                               size_t workspace_bytes, void* stream) {
  if (!cache) return BPT_ERR_INVALID_ARGUMENT;
  if (batch < 0 || q_heads <= 0) return BPT_ERR_INVALID_ARGUMENT;
  if (batch == 0) return BPT_OK;
  if (!workspace || !out) return BPT_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(out) & 15) || ((o_sb * 2) % 16) || ((o_sh * 2) % 16))
    return BPT_ERR_ALIGNMENT;
  const int S = effective_splits_kivi(cache->format, batch, cache->kv_heads, q_heads,
                                      cache->block_size, max_blocks, num_splits, sm_count);
  if (workspace_bytes < bpt_decode_workspace_bytes(batch, q_heads, cache->head_dim, S))
    return BPT_ERR_WORKSPACE_TOO_SMALL;
  WorkspaceView ws = workspace_view(workspace, batch, q_heads, cache->head_dim, S);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = run_split_kivi(*cache, q, q_sb, q_sh, block_table, bt_sb, seq_lens, out, o_sb, o_sh,
                          batch, q_heads, max_blocks, scale, S, 1, ws.o_part, ws.lse, ws.status,
                          st);
  if (rc || S == 1) return rc;
  return launch_merge(ws.o_part, ws.lse, batch, q_heads, S, cache->head_dim,
                      static_cast<__half*>(out), o_sb, o_sh, nullptr, nullptr, st, true);
}

extern "C" int bpt_effective_splits_kivi(int format, int batch, int kv_heads, int q_heads,
                                         int block_size, int max_blocks, int num_splits,
                                         int sm_count) {
  return effective_splits_kivi(format, batch, kv_heads, q_heads, block_size, max_blocks,
                               num_splits, sm_count);
}

extern "C" int bpt_decode_kivi_partial(const bpt_kivi_cache* cache, const void* q, int64_t q_sb,
                                       int64_t q_sh, const int32_t* block_table, int64_t bt_sb,
                                       const int32_t* seq_lens, int batch, int q_heads,
                                       int max_blocks, float scale, int splits, float* o_part,
                                       float* lse, unsigned* status, void* stream) {
  if (!cache) return BPT_ERR_INVALID_ARGUMENT;
  return run_split_kivi(*cache, q, q_sb, q_sh, block_table, bt_sb, seq_lens, nullptr, 0, 0,
                        batch, q_heads, max_blocks, scale, splits, 0, o_part, lse, status,
                        static_cast<cudaStream_t>(stream));
}
