// Tensor-core split-KV decode kernel for fp16 paged KV (head_dim a multiple of 64).
//
// Work decomposition (same as the CUDA-core kernel in decode_fp16.cu): one CTA owns one
// (sequence b, kv head h, split s); a split is a contiguous range of CHUNK-token chunks of the
// sequence; a producer warp streams each chunk's K and V pages into a STAGES-deep shared-memory
// ring with 4-D TMA boxes (page indirection = box coordinate); NCW consumer warps take 16 tokens
// of each chunk and keep their own online-softmax state, merged once per split.
//
// Consumer math, per warp and chunk, on warp-level tensor-core MMAs (mma.sync m16n8k16,
// fp16 x fp16 -> fp32, register fragments):
//
//   QK^T   S[16 rows x 8 tok] = Q[16 x 16 d] . K^T            (2 n-blocks = 16 tokens)
//          A = Q fragments, constant for the split (registers); B = K via ldmatrix.
//          group <= 4: rows 0-3 and 4-7 both hold q heads 0-3 ("hi" and "lo" copies);
//          group 5-8: rows 0-7 hold q heads 0-7. Rows 8-15 are zero.
//   P.V    O^T[16 d x 8 col] = V^T[16 d x 16 tok] . P^T[16 tok x 8 col]
//          A = V^T via ldmatrix.trans; B = P^T straight from the S accumulator the same lane
//          owns. P is split into fp16 hi = fp16(p) and lo = fp16(p - hi); group <= 4 puts hi in
//          columns 0-3 and lo in columns 4-7 of ONE MMA (rows 0-3 feed hi, rows 4-7 feed lo),
//          group 5-8 uses a second MMA for lo. O = hi + lo carries ~22 bits of P, so the result
//          matches fp32 math (an fp16 P alone costs ~1e-4 absolute error).
//
// K/V stage buffers are 64-column blocks written by TMA with the 128-byte swizzle (16-byte
// chunk c of token row r lands at chunk c ^ (r % 8)); every ldmatrix phase then reads 8
// distinct bank groups.
#pragma once

#include "common.cuh"
#include "split_state.cuh"
#include "decode_common.h"

namespace bpt {
namespace mma {

constexpr float kNegInf = -INFINITY;

template <int D, int NCW, int STAGES, bool G8>
struct Cfg {
  static constexpr int CHUNK = 16 * NCW;              // tokens per stage
  static constexpr int THREADS = (NCW + 1) * 32;      // + 1 producer warp
  static constexpr int NCB = D / 64;                  // 64-column (128-byte) blocks
  static constexpr int BLOCK_ELEMS = CHUNK * 64;
  static constexpr int BLOCK_BYTES = BLOCK_ELEMS * 2;
  static constexpr int STAGE_ELEMS = CHUNK * D;
  static constexpr int KSTEPS = D / 16;
  static constexpr int DB16 = D / 16;                 // 16-row d blocks of O^T
  static constexpr int NACC = G8 ? 2 : 1;
  static constexpr size_t MERGE_BYTES = size_t(NCW) * 8 * (D + 3) * 4;
  static constexpr size_t RING_BYTES = size_t(STAGES) * STAGE_ELEMS * 2 * 2;
  static constexpr size_t BODY_BYTES = RING_BYTES > MERGE_BYTES ? RING_BYTES : MERGE_BYTES;
  static constexpr size_t SMEM_BYTES = 1024 + BODY_BYTES + 2 * STAGES * 8 + 64;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                              uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// d = A.B with a zero accumulator (a fresh partial product).
__device__ __forceinline__ void mma_16816_zc(float (&d)[4], uint32_t a0, uint32_t a1,
                                             uint32_t a2, uint32_t a3, uint32_t b0,
                                             uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

// acc += A.B, with the product formed by the tensor core from a zero accumulator and added
// in fp32 round-to-nearest: a long-running accumulator never passes through the tensor
// core's own accumulation, whose per-step rounding would otherwise build up over thousands
// of tokens on a large running sum.
__device__ __forceinline__ void mma_16816_acc(float (&acc)[4], uint32_t a0, uint32_t a1,
                                              uint32_t a2, uint32_t a3, uint32_t b0,
                                              uint32_t b1) {
  float t[4];
  mma_16816_zc(t, a0, a1, a2, a3, b0, b1);
  acc[0] += t[0]; acc[1] += t[1]; acc[2] += t[2]; acc[3] += t[3];
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// fp16 hi = fp16(p) and lo = fp16(p - hi) for two adjacent tokens, packed as half2.
__device__ __forceinline__ void split_hi_lo(float p0, float p1, uint32_t& hi, uint32_t& lo) {
  __half2 h = __floats2half2_rn(p0, p1);
  const float2 hf = __half22float2(h);
  hi = *reinterpret_cast<uint32_t*>(&h);
  lo = pack_half2(p0 - hf.x, p1 - hf.y);
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <int D, int NCW, int STAGES, int MINB, bool G8>
__global__ void __launch_bounds__((NCW + 1) * 32, MINB)
split_kv_fp16_mma_kernel(const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const DecodeParams p) {
  using C = Cfg<D, NCW, STAGES, G8>;
  constexpr int CHUNK = C::CHUNK;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __half* sK = reinterpret_cast<__half*>(smem);
  __half* sV = sK + STAGES * C::STAGE_ELEMS;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BODY_BYTES);
  uint64_t* empty = full + STAGES;
  // per-warp states for the end-of-split merge, aliased onto the ring once it is drained
  float* sM = reinterpret_cast<float*>(smem);
  float* sL = sM + NCW * 8;
  float* sAcc = sL + NCW * 8;

  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.splits;

  // the tensor maps are kernel parameters, not written by the previous kernel: their fetch
  // overlaps the wait
  if (warp == NCW && lane == 0) {
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
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

  if (nchunks <= 0 || t_begin >= t_end) {  // empty split (CTA-uniform)
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

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NCW);
    }
    fence_mbar_init();
  }
  __syncthreads();
  // the merge grid may start launching now (it waits in griddepcontrol.wait for this whole
  // grid to complete), which takes its launch latency off the end of the call
  pdl_launch_dependents();

  if (warp == NCW) {
    // ------------------------------------------------------------------ producer warp
    const uint64_t pol = l2_evict_first_policy();
    const int32_t* bt = p.block_table + int64_t(b) * p.bt_sb;
    const int R = p.box_rows;                     // min(block_size, CHUNK)
    const int bs = p.block_size;
    const uint32_t box_bytes = uint32_t(R) * 64 * 2;
    const int last_page = (t_end - 1) / bs;
    int win_base = t_begin / bs;                  // lane i caches block_table[win_base + i]
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
      const int tok0 = (u0 + c) * CHUNK;
      const int nbox = min(CHUNK / R, cdiv(t_end - tok0, R));
      if (lane == 0)
        mbar_arrive_expect_tx(&full[stage], uint32_t(nbox) * C::NCB * box_bytes * 2u);
      for (int j = 0; j < nbox; ++j) {
        const int t = tok0 + j * R;
        const int pg = t / bs;
        while (pg - win_base >= 32) {            // warp-uniform window advance
          win_base += 32;
          win = (win_base + lane <= last_page) ? __ldg(bt + win_base + lane) : 0;
        }
        int phys = __shfl_sync(kFullMask, win, pg - win_base);
        if (lane == 0) {
          if (phys < 0 || int64_t(phys) >= p.num_blocks) {
            flag_device_error(p.status, BPT_DEV_BAD_BLOCK_ID);
            phys = 0;
          }
          const int row = t - pg * bs;
#pragma unroll
          for (int cb = 0; cb < C::NCB; ++cb) {
            const int so = stage * C::STAGE_ELEMS + cb * C::BLOCK_ELEMS + j * R * 64;
            tma_load_4d(sK + so, &tmK, &full[stage], cb * 64, p.k_c1 ? row : h,
                        p.k_c1 ? h : row, phys, pol);
            tma_load_4d(sV + so, &tmV, &full[stage], cb * 64, p.v_c1 ? row : h,
                        p.v_c1 ? h : row, phys, pol);
          }
        }
      }
      ++issued;
    }
    pdl_launch_dependents();
    // never let the CTA exit while a bulk copy still writes its shared memory
    if (lane == 0) {
      for (int c = max(0, issued - STAGES); c < issued; ++c)
        if (!mbar_wait(&full[c % STAGES], uint32_t(c / STAGES) & 1u))
          flag_device_error(p.status, BPT_DEV_WAIT_TIMEOUT);
    }
    return;
  }

  // -------------------------------------------------------------------- consumer warps
  const int g = lane >> 2;          // fragment row group
  const int t4 = lane & 3;          // thread in group
  const int qhead = G8 ? g : (g & 3);
  const bool qvalid = qhead < p.group;

  uint32_t qa0[C::KSTEPS], qa2[C::KSTEPS];
  {
    const __half* qrow =
        p.q + int64_t(b) * p.q_sb + int64_t(qh0 + (qvalid ? qhead : 0)) * p.q_sh;
#pragma unroll
    for (int ks = 0; ks < C::KSTEPS; ++ks) {
      qa0[ks] = qvalid ? *reinterpret_cast<const uint32_t*>(qrow + 16 * ks + 2 * t4) : 0u;
      qa2[ks] = qvalid ? *reinterpret_cast<const uint32_t*>(qrow + 16 * ks + 8 + 2 * t4) : 0u;
    }
  }

  // ldmatrix addressing: matrix j = lane >> 3, row r = lane & 7. For K (QK^T B operand) the
  // four matrices are (tok 0-7, d lo8), (tok 0-7, d hi8), (tok 8-15, lo8), (tok 8-15, hi8);
  // for V^T (P.V A operand, .trans) they are (tok 0-7, d lo8), (tok 0-7, d hi8),
  // (tok 8-15, d lo8), (tok 8-15, d hi8) of one 16-wide d block: the same pattern.
  const int mj = lane >> 3, mr = lane & 7;
  const int ld_tok = warp * 16 + 8 * (mj >> 1) + mr;
  const uint32_t ld_sel = uint32_t(mj & 1);
  const uint32_t ld_row = uint32_t(ld_tok) * 128u;
  const uint32_t ld_swz = uint32_t(ld_tok & 7);

  float acc[C::NACC][C::DB16][4];
#pragma unroll
  for (int a = 0; a < C::NACC; ++a)
#pragma unroll
    for (int i = 0; i < C::DB16; ++i) acc[a][i][0] = acc[a][i][1] = acc[a][i][2] = acc[a][i][3] = 0.f;
  float m_run = kNegInf, l_run = 0.f;
  const float sl2 = p.scale_log2;
  // lanes whose alpha (per q head) each accumulator column needs
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
    const uint32_t kbase = smem_u32(sK + stage * C::STAGE_ELEMS);
    const uint32_t vbase = smem_u32(sV + stage * C::STAGE_ELEMS);
    const int lim = t_end - (u0 + c) * CHUNK - warp * 16;  // valid rows of this warp's 16

    // ---- S = Q K^T
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < C::KSTEPS; ++ks) {
      const uint32_t chunk = (uint32_t((ks & 3) << 1) | ld_sel) ^ ld_swz;
      const uint32_t addr = kbase + uint32_t(ks >> 2) * C::BLOCK_BYTES + ld_row + (chunk << 4);
      uint32_t b0, b1, b2, b3;
      ldsm_x4(addr, b0, b1, b2, b3);
      mma_16816(s0, qa0[ks], 0u, qa2[ks], 0u, b0, b1);
      mma_16816(s1, qa0[ks], 0u, qa2[ks], 0u, b2, b3);
    }

    // ---- online softmax (log2 domain): this lane owns q head `qhead`, tokens 2t, 2t+1, +8
    const int tk = 2 * t4;
    const float x0 = (tk < lim) ? s0[0] * sl2 : kNegInf;
    const float x1 = (tk + 1 < lim) ? s0[1] * sl2 : kNegInf;
    const float x2 = (tk + 8 < lim) ? s1[0] * sl2 : kNegInf;
    const float x3 = (tk + 9 < lim) ? s1[1] * sl2 : kNegInf;
    float mx = fmaxf(fmaxf(x0, x1), fmaxf(x2, x3));
    mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, 2));
    const float m_new = fmaxf(m_run, mx);
    if (__any_sync(kFullMask, m_new > m_run)) {
      const float alpha = fast_exp2(m_run - (m_new == kNegInf ? 0.f : m_new));
      l_run *= alpha;
      const float aA = __shfl_sync(kFullMask, alpha, srcA);
      const float aB = __shfl_sync(kFullMask, alpha, srcB);
#pragma unroll
      for (int a = 0; a < C::NACC; ++a)
#pragma unroll
        for (int i = 0; i < C::DB16; ++i) {
          acc[a][i][0] *= aA; acc[a][i][1] *= aB; acc[a][i][2] *= aA; acc[a][i][3] *= aB;
        }
      m_run = m_new;
    }
    const float m_use = (m_run == kNegInf) ? 0.f : m_run;
    const float p0 = fast_exp2(x0 - m_use), p1 = fast_exp2(x1 - m_use);
    const float p2 = fast_exp2(x2 - m_use), p3 = fast_exp2(x3 - m_use);
    l_run += (p0 + p1) + (p2 + p3);
    uint32_t hi0, lo0, hi1, lo1;
    split_hi_lo(p0, p1, hi0, lo0);
    split_hi_lo(p2, p3, hi1, lo1);

    // ---- rows past the end of the split: zero V so stale or NaN bytes cannot reach O
    if (lim < 16) {
      uint8_t* vst = reinterpret_cast<uint8_t*>(sV + stage * C::STAGE_ELEMS);
      for (int idx = lane; idx < 16 * C::NCB * 8; idx += 32) {
        const int r = idx / (C::NCB * 8), rest = idx % (C::NCB * 8);
        if (r >= lim)
          *reinterpret_cast<uint4*>(vst + (rest >> 3) * C::BLOCK_BYTES + (warp * 16 + r) * 128 +
                                    (rest & 7) * 16) = make_uint4(0u, 0u, 0u, 0u);
      }
      __syncwarp();
    }

    // ---- O^T += V^T P^T
    const uint32_t pb0 = G8 ? hi0 : (g < 4 ? hi0 : lo0);
    const uint32_t pb1 = G8 ? hi1 : (g < 4 ? hi1 : lo1);
#pragma unroll
    for (int db = 0; db < C::DB16; ++db) {
      const uint32_t chunk = (uint32_t((2 * db) & 7) | ld_sel) ^ ld_swz;
      const uint32_t addr = vbase + uint32_t(db >> 2) * C::BLOCK_BYTES + ld_row + (chunk << 4);
      uint32_t a0, a1, a2, a3;
      ldsm_x4_trans(addr, a0, a1, a2, a3);
      mma_16816_acc(acc[0][db], a0, a1, a2, a3, pb0, pb1);
      if constexpr (G8) mma_16816_acc(acc[C::NACC - 1][db], a0, a1, a2, a3, lo0, lo1);
    }
    if (lim < 16) fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
  }

  pdl_launch_dependents();
  // ---- per-warp state -> shared memory
  l_run += __shfl_xor_sync(kFullMask, l_run, 1);
  l_run += __shfl_xor_sync(kFullMask, l_run, 2);
  // O = hi + lo: G8 keeps lo in the second accumulator; otherwise lo sits in columns 4-7,
  // i.e. in lane t4 ^ 2 of the same row group.
#pragma unroll
  for (int i = 0; i < C::DB16; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if constexpr (G8) {
        acc[0][i][e] += acc[C::NACC - 1][i][e];
      } else {
        acc[0][i][e] += __shfl_xor_sync(kFullMask, acc[0][i][e], 2);
      }
    }
  named_barrier_sync(1, NCW * 32);  // every consumer warp is done reading the ring
  if (t4 == 0 && (G8 || g < 4)) {
    sM[warp * 8 + qhead] = m_run;
    sL[warp * 8 + qhead] = l_run;
  }
  if (G8 || t4 < 2) {
#pragma unroll
    for (int i = 0; i < C::DB16; ++i) {
      const int d = 16 * i + g;
      sAcc[(warp * 8 + colA) * D + d] = acc[0][i][0];
      sAcc[(warp * 8 + colB) * D + d] = acc[0][i][1];
      sAcc[(warp * 8 + colA) * D + d + 8] = acc[0][i][2];
      sAcc[(warp * 8 + colB) * D + d + 8] = acc[0][i][3];
    }
  }
  named_barrier_sync(1, NCW * 32);
  write_split_state<NCW, D>(sM, sL, sAcc, sAcc + NCW * 8 * D, p, b, qh0, split,
                            int(threadIdx.x), NCW * 32,
                            [] { named_barrier_sync(1, NCW * 32); });
}

template <int D, int NCW, int STAGES, int MINB, bool G8>
int launch(const CUtensorMap& tk, const CUtensorMap& tv, const DecodeParams& p,
           cudaStream_t st) {
  using C = Cfg<D, NCW, STAGES, G8>;
  auto kern = split_kv_fp16_mma_kernel<D, NCW, STAGES, MINB, G8>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           int(C::SMEM_BYTES)) != cudaSuccess)
    return BPT_ERR_LAUNCH;
  dim3 grid(p.splits, p.kv_heads, p.batch);
  return launch_dependent(kern, grid, dim3(C::THREADS), C::SMEM_BYTES, st, tk, tv, p) ==
                 cudaSuccess
             ? BPT_OK
             : BPT_ERR_LAUNCH;
}

}  // namespace mma
}  // namespace bpt
