// FP16 paged-KV GQA decode for sm_100a: split-KV kernel + split merge kernel + C entry.
//
// Replaces the reference's Triton path (src/bpt/triton_fp16.py): _split_kernel (:83-144),
// _paged_decode_kernel (:25-80, here the same kernel with one split) and _merge_kernel
// (:147-163).
//
// Work decomposition. One CTA owns one (sequence b, kv head h, split s) and serves all
// `group` q heads that share kv head h from a single read of K/V. A split is a contiguous
// range of 64-token chunks of the sequence (chunks are split as evenly as possible per
// sequence, so ragged batches stay balanced). Per chunk the producer warp issues one 4-D TMA
// box per page (or per 64-row slice of a page larger than 64 tokens) for K and for V straight
// from the paged cache into a STAGES-deep shared-memory ring; the page indirection is only the
// box coordinate. Four consumer warps each take 16 tokens of the chunk and keep their own
// online-softmax state (m, l, acc); the four states are merged through shared memory once per
// split. QK^T uses fma.rn.f32.f16 (fp16 operands, exact products, fp32 accumulation); P stays
// fp32 for P.V. Scores are kept in the log2 domain (q.k * scale * log2 e).
//
// Output: one split -> normalised fp16 out directly; several -> normalised fp32 partial o and
// its log2-sum-exp per (b, q head, split) in the workspace, then merge_splits.
#include <cudaTypedefs.h>

#include <math.h>
#include <mutex>

#include "common.cuh"
#include "decode_common.h"
#include "mma_decode.cuh"

namespace bpt {

namespace {

constexpr int kChunk = 64;          // tokens per pipeline stage
constexpr int kResidentFp16 = 4;    // tensor-core split CTAs resident per SM (the planner's)
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr float kNegInf = -INFINITY;

constexpr int ilog2(int x) { return x <= 1 ? 0 : 1 + ilog2(x / 2); }

// Lane geometry for head_dim D and padded group GP: a token's D elements are spread over LPT
// lanes (EPL elements each), so one warp covers TPP tokens per pass.
template <int D, int GP>
struct Geo {
  static constexpr int EPL0 = (64 / GP) < (D / 8) ? (64 / GP) : (D / 8);
  static constexpr int EPL = EPL0 < 2 ? 2 : EPL0;
  static constexpr int LPT = D / EPL;
  static_assert(LPT <= 32 && LPT >= GP, "unsupported head_dim / group combination");
  static constexpr int TPP = 32 / LPT;
  static constexpr int TPW = kChunk / kConsumerWarps;
  static constexpr int PASSES = TPW / TPP;
  static constexpr int VEC = EPL >= 8 ? 8 : EPL;  // fp16 elements per shared-memory load
  static constexpr int NVEC = EPL / VEC;
  static constexpr int W = VEC / 2;               // 32-bit words per load
  static constexpr int LOG_LPT = ilog2(LPT);
  static constexpr int LOG_GP = ilog2(GP);
  static constexpr int DUP = LPT / GP;            // lanes holding the same reduced score
  static constexpr int STAGES = D <= 64 ? 4 : (D <= 128 ? 3 : 2);
  static constexpr int STAGE_ELEMS = kChunk * D;  // per K (or V) stage buffer
  static constexpr size_t MERGE_BYTES = size_t(kConsumerWarps) * GP * (D + 2) * 4;
  static constexpr size_t SMEM_BYTES =
      1024 + size_t(STAGES) * STAGE_ELEMS * 2 * 2 + MERGE_BYTES + 2 * STAGES * 8 + 64;
};

// Transpose-reduce NV partial sums over the lanes of a token group: each level halves the
// number of values per lane (send half, keep half), then plain butterflies. Afterwards the
// lane holds the full sum for head (lane % LPT) >> (LOG_LPT - LOG_GP).
template <int NV, int OFF>
struct TransposeReduce {
  __device__ __forceinline__ static void run(float* v, int lane) {
    if constexpr (OFF >= 1) {
      if constexpr (NV > 1) {
        constexpr int H = NV / 2;
        const bool upper = (lane & OFF) != 0;
#pragma unroll
        for (int i = 0; i < H; ++i) {
          const float send = upper ? v[i] : v[i + H];
          const float keep = upper ? v[i + H] : v[i];
          v[i] = keep + __shfl_xor_sync(kFullMask, send, OFF);
        }
        TransposeReduce<H, OFF / 2>::run(v, lane);
      } else {
        v[0] += __shfl_xor_sync(kFullMask, v[0], OFF);
        TransposeReduce<1, OFF / 2>::run(v, lane);
      }
    }
  }
};

template <int W>
__device__ __forceinline__ void load_words(uint32_t (&w)[W], const __half* p) {
  if constexpr (W == 4) {
    const uint4 t = *reinterpret_cast<const uint4*>(p);
    w[0] = t.x; w[1] = t.y; w[2] = t.z; w[3] = t.w;
  } else if constexpr (W == 2) {
    const uint2 t = *reinterpret_cast<const uint2*>(p);
    w[0] = t.x; w[1] = t.y;
  } else {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  }
}

template <int D, int GP>
__global__ void __launch_bounds__(kThreads)
split_kv_fp16_kernel(const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const DecodeParams p) {
  using G = Geo<D, GP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __half* sK = reinterpret_cast<__half*>(smem);
  __half* sV = sK + G::STAGES * G::STAGE_ELEMS;
  float* sM = reinterpret_cast<float*>(sV + G::STAGES * G::STAGE_ELEMS);  // [NCW][GP]
  float* sL = sM + kConsumerWarps * GP;                                    // [NCW][GP]
  float* sAcc = sL + kConsumerWarps * GP;                                  // [NCW][GP][D]
  uint64_t* full = reinterpret_cast<uint64_t*>(sAcc + kConsumerWarps * GP * D);
  uint64_t* empty = full + G::STAGES;

  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.splits;

  // the tensor maps are kernel parameters, not written by the previous kernel: their fetch
  // overlaps the wait
  if (threadIdx.x == 0) {
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
  const int n_units = cdiv(n, kChunk);
  const int span = p.balance ? cdiv(batch_max_len(p.seq_lens, p.batch, cap), kChunk) : n_units;
  int u0, u1;
  split_range(split, S, n_units, span, &u0, &u1);
  const int t_begin = u0 * kChunk;
  const int t_end = min(u1 * kChunk, n);
  const int nchunks = u1 - u0;
  const int qh0 = h * p.group;

  if (nchunks <= 0 || t_begin >= t_end) {  // empty split: o = 0, lse = -inf (CTA-uniform)
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
    for (int s = 0; s < G::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();   // the merge grid may launch now; it waits for this grid's end

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------------ producer warp
    const uint64_t pol = l2_evict_first_policy();
    const int32_t* bt = p.block_table + int64_t(b) * p.bt_sb;
    const int R = p.box_rows;                  // rows per TMA box = min(block_size, 64)
    const int bs = p.block_size;
    const uint32_t box_bytes = uint32_t(R) * D * 2;
    const int last_page = (t_end - 1) / bs;
    int win_base = t_begin / bs;               // lane i caches block_table[win_base + i]
    int win = (win_base + lane <= last_page) ? __ldg(bt + win_base + lane) : 0;
    int issued = 0;
    bool ok = true;
    for (int c = 0; c < nchunks; ++c) {
      const int stage = c % G::STAGES;
      const uint32_t par = uint32_t(c / G::STAGES) & 1u;
      bool w_ok = (lane == 0) ? mbar_wait(&empty[stage], par ^ 1u) : true;
      w_ok = __shfl_sync(kFullMask, w_ok, 0);
      if (!w_ok) {
        if (lane == 0) flag_device_error(p.status, BPT_DEV_WAIT_TIMEOUT);
        ok = false;
        break;
      }
      const int tok0 = (u0 + c) * kChunk;
      const int nbox = min(kChunk / R, cdiv(t_end - tok0, R));
      if (lane == 0) mbar_arrive_expect_tx(&full[stage], uint32_t(nbox) * box_bytes * 2u);
      for (int j = 0; j < nbox; ++j) {
        const int t = tok0 + j * R;
        const int pg = t / bs;
        while (pg - win_base >= 32) {          // warp-uniform window advance
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
          const int so = stage * G::STAGE_ELEMS + j * R * D;
          tma_load_4d(sK + so, &tmK, &full[stage], 0, p.k_c1 ? row : h, p.k_c1 ? h : row,
                      phys, pol);
          tma_load_4d(sV + so, &tmV, &full[stage], 0, p.v_c1 ? row : h, p.v_c1 ? h : row,
                      phys, pol);
        }
      }
      ++issued;
    }
    (void)ok;
    pdl_launch_dependents();
    // Drain: never leave the CTA with a bulk copy still writing its shared memory.
    if (lane == 0) {
      for (int c = max(0, issued - G::STAGES); c < issued; ++c)
        if (!mbar_wait(&full[c % G::STAGES], uint32_t(c / G::STAGES) & 1u))
          flag_device_error(p.status, BPT_DEV_WAIT_TIMEOUT);
    }
    return;
  }

  // -------------------------------------------------------------------- consumer warps
  const int j = lane % G::LPT;        // sub-lane inside the token group
  const int tg = lane / G::LPT;       // token group
  const int hl = j >> (G::LOG_LPT - G::LOG_GP);

  // q of the group's heads, packed fp16 pairs; padded heads are zero.
  uint32_t qw[GP][G::EPL / 2];
#pragma unroll
  for (int g = 0; g < GP; ++g) {
#pragma unroll
    for (int i = 0; i < G::NVEC; ++i) {
      uint32_t w[G::W];
      if (g < p.group) {
        load_words<G::W>(w, p.q + int64_t(b) * p.q_sb + int64_t(qh0 + g) * p.q_sh +
                                (i * G::LPT + j) * G::VEC);
      } else {
#pragma unroll
        for (int e = 0; e < G::W; ++e) w[e] = 0u;
      }
#pragma unroll
      for (int e = 0; e < G::W; ++e) qw[g][i * G::W + e] = w[e];
    }
  }

  float acc[GP][G::EPL];
#pragma unroll
  for (int g = 0; g < GP; ++g)
#pragma unroll
    for (int e = 0; e < G::EPL; ++e) acc[g][e] = 0.f;
  float m_run = kNegInf, l_run = 0.f;
  const float sl2 = p.scale_log2;

  for (int c = 0; c < nchunks; ++c) {
    const int stage = c % G::STAGES;
    const uint32_t par = uint32_t(c / G::STAGES) & 1u;
    const bool w_ok = __all_sync(kFullMask, mbar_wait(&full[stage], par));
    if (!w_ok) {
      if (lane == 0) flag_device_error(p.status, BPT_DEV_WAIT_TIMEOUT);
      break;
    }
    const __half* kS = sK + stage * G::STAGE_ELEMS;
    const __half* vS = sV + stage * G::STAGE_ELEMS;
    const int tok_base = (u0 + c) * kChunk;
    const bool last = (c == nchunks - 1);

    float sc[G::PASSES];
#pragma unroll
    for (int ps = 0; ps < G::PASSES; ++ps) {
      const int row = warp * G::TPW + ps * G::TPP + tg;
      float s[GP];
#pragma unroll
      for (int g = 0; g < GP; ++g) s[g] = 0.f;
#pragma unroll
      for (int i = 0; i < G::NVEC; ++i) {
        uint32_t w[G::W];
        load_words<G::W>(w, kS + row * D + (i * G::LPT + j) * G::VEC);
#pragma unroll
        for (int e = 0; e < G::W; ++e)
#pragma unroll
          for (int g = 0; g < GP; ++g) s[g] = fma_f16x2_f32(qw[g][i * G::W + e], w[e], s[g]);
      }
      TransposeReduce<GP, G::LPT / 2>::run(s, lane);
      const bool valid = tok_base + row < t_end;
      sc[ps] = valid ? s[0] * sl2 : kNegInf;
    }

    float mx = sc[0];
#pragma unroll
    for (int ps = 1; ps < G::PASSES; ++ps) mx = fmaxf(mx, sc[ps]);
#pragma unroll
    for (int off = G::LPT; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, off));
    const float m_new = fmaxf(m_run, mx);
    if (__any_sync(kFullMask, m_new > m_run)) {
      const float alpha = fast_exp2(m_run - (m_new == kNegInf ? 0.f : m_new));
      l_run *= alpha;
#pragma unroll
      for (int g = 0; g < GP; ++g) {
        const float ag = __shfl_sync(kFullMask, alpha, g * G::DUP);
#pragma unroll
        for (int e = 0; e < G::EPL; ++e) acc[g][e] *= ag;
      }
      m_run = m_new;
    }
    const float m_use = (m_run == kNegInf) ? 0.f : m_run;

    float pr[G::PASSES];
#pragma unroll
    for (int ps = 0; ps < G::PASSES; ++ps) {
      pr[ps] = fast_exp2(sc[ps] - m_use);
      l_run += pr[ps];
    }

#pragma unroll
    for (int ps = 0; ps < G::PASSES; ++ps) {
      const int row = warp * G::TPW + ps * G::TPP + tg;
      const bool valid = tok_base + row < t_end;
      float pg[GP];
#pragma unroll
      for (int g = 0; g < GP; ++g)
        pg[g] = __shfl_sync(kFullMask, pr[ps], tg * G::LPT + g * G::DUP);
#pragma unroll
      for (int i = 0; i < G::NVEC; ++i) {
        uint32_t w[G::W];
        load_words<G::W>(w, vS + row * D + (i * G::LPT + j) * G::VEC);
        if (last && !valid) {
#pragma unroll
          for (int e = 0; e < G::W; ++e) w[e] = 0u;  // stale / garbage rows never reach acc
        }
#pragma unroll
        for (int e = 0; e < G::W; ++e) {
          const float2 f = half2_bits_to_float2(w[e]);
#pragma unroll
          for (int g = 0; g < GP; ++g) {
            acc[g][i * G::VEC + 2 * e] = fmaf(pg[g], f.x, acc[g][i * G::VEC + 2 * e]);
            acc[g][i * G::VEC + 2 * e + 1] = fmaf(pg[g], f.y, acc[g][i * G::VEC + 2 * e + 1]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
  }

  pdl_launch_dependents();
  // Reduce over the token groups of the warp.
#pragma unroll
  for (int off = G::LPT; off < 32; off <<= 1) {
    l_run += __shfl_xor_sync(kFullMask, l_run, off);
#pragma unroll
    for (int g = 0; g < GP; ++g)
#pragma unroll
      for (int e = 0; e < G::EPL; ++e) acc[g][e] += __shfl_xor_sync(kFullMask, acc[g][e], off);
  }
  if (tg == 0) {
    if (j % G::DUP == 0) {
      sM[warp * GP + hl] = m_run;
      sL[warp * GP + hl] = l_run;
    }
#pragma unroll
    for (int g = 0; g < GP; ++g)
#pragma unroll
      for (int i = 0; i < G::NVEC; ++i)
#pragma unroll
        for (int e = 0; e < G::VEC; ++e)
          sAcc[(warp * GP + g) * D + (i * G::LPT + j) * G::VEC + e] = acc[g][i * G::VEC + e];
  }
  named_barrier_sync(1, kConsumerWarps * 32);

  // Merge the four warp states and write this split's result.
  for (int idx = threadIdx.x; idx < p.group * D; idx += kConsumerWarps * 32) {
    const int g = idx / D, d = idx % D;
    float M = kNegInf;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, sM[w * GP + g]);
    float L = 0.f, O = 0.f;
    if (M != kNegInf) {
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float f = fast_exp2(sM[w * GP + g] - M);
        L = fmaf(sL[w * GP + g], f, L);
        O = fmaf(sAcc[(w * GP + g) * D + d], f, O);
      }
    }
    const float o = L > 0.f ? O / L : 0.f;
    if (S == 1 && p.final_out) {
      p.out[int64_t(b) * p.o_sb + int64_t(qh0 + g) * p.o_sh + d] = __float2half_rn(o);
    } else {
      const int64_t row = (int64_t(b) * p.q_heads + qh0 + g) * S + split;
      p.o_part[row * D + d] = o;
      if (d == 0) p.lse[row] = L > 0.f ? M + __log2f(L) : kNegInf;
    }
  }
}

// Stage 2: out = sum_s w_s o_s / sum_s w_s, w_s = 2^(lse_s - max lse) (lse in log2 units).
// The partial states are addressed through strides (elements) so the same kernel merges the
// split partials [B, Hq, S, D] of one call and rank states gathered as [S ranks, B, Hq, ...].
// F16OUT: write the normalised fp16 output; otherwise write the merged fp32 state (o, lse),
// which is what a cross-GPU merge of sequence shards consumes.
struct MergeLayout {
  int64_t o_ss, o_sb, o_sh;   // partial o: split, batch, head strides (d stride 1)
  int64_t l_ss, l_sb, l_sh;   // partial lse strides
};

// Each warp's online merge is a serial chain per row (exp2, 4 fma), so a warp takes few rows:
// 4 rows per warp and up to 32 warps cover 128 split rows in one memory round trip. Measured
// on one B200 at B=1 (74 splits): 8 warps x 16 rows 2.27 us from the release of the merge grid
// to its end, 10 x 8 2.07 us, 19 x 4 2.02 us (then the combine over 19 warp states dominates).
constexpr int kMergeWarps = 32;   // most warps per merge CTA
constexpr int kMergeRows = 4;     // partial rows a warp loads before using any

// 4 consecutive channels 4c .. 4c + 3 of one partial row (zero past D)
template <bool VEC>
__device__ __forceinline__ float4 load_row4(const float* row, int c, int D) {
  if constexpr (VEC) return __ldg(reinterpret_cast<const float4*>(row) + c);
  const int d = 4 * c;
  return make_float4(row[d], d + 1 < D ? row[d + 1] : 0.f, d + 2 < D ? row[d + 2] : 0.f,
                     d + 3 < D ? row[d + 3] : 0.f);
}

template <bool F16OUT, bool VEC>
__global__ void __launch_bounds__(kMergeWarps * 32)
merge_splits_kernel(const float* __restrict__ o_part, const float* __restrict__ lse,
                    const MergeLayout lay, int q_heads, int splits, int D,
                    __half* __restrict__ out16, int64_t o_sb, int64_t o_sh,
                    float* __restrict__ o32, float* __restrict__ lse32) {
  // One CTA per (q head, sequence) of W = ceil(S / 4) <= 32 warps. Warp w owns splits w,
  // w + W, w + 2W, ... and merges them online in batches of kMergeRows rows: every load of a
  // batch (each row's lse and this lane's 4 channels of its o row) is issued before any is
  // used, so up to 128 partial rows cost one memory round trip. Lane l holds channels
  // 4 (32 g + l) .. + 3 of channel group g (one group for D <= 128). The W warp states
  // (max, sum, o) are then combined through shared memory in warp order, so the result does
  // not depend on timing: lane w of warp 0 turns state w into its weight 2^(m_w - M) / L once,
  // then every lane sums the weighted o of the W states. VEC: o rows are 16-byte aligned with
  // D % 4 == 0 (float4 loads).
  constexpr int R = kMergeRows;
  const int W = int(blockDim.x) >> 5;
  __shared__ float s_m[kMergeWarps], s_l[kMergeWarps], s_f[kMergeWarps];
  __shared__ float4 s_o[kMergeWarps][32];
  const int hq = blockIdx.x, b = blockIdx.y;
  const float* l = lse + int64_t(b) * lay.l_sb + int64_t(hq) * lay.l_sh;
  const float* o = o_part + int64_t(b) * lay.o_sb + int64_t(hq) * lay.o_sh;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nd4 = (D + 3) >> 2;
  pdl_wait();
  // the next kernel in the stream (the next call's split kernel) may start launching: its CTAs
  // take the SM slots this merge leaves free and wait for its completion
  pdl_launch_dependents();

  for (int c0 = 0; c0 < nd4; c0 += 32) {
    const int c = c0 + lane;
    const bool c_in = c < nd4;
    float m = kNegInf, wsum = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = warp; s0 < splits; s0 += W * R) {
      float ls[R];
      float4 v[R];
#pragma unroll
      for (int u = 0; u < R; ++u) {
        const int s = s0 + W * u;
        const bool in = s < splits;
        ls[u] = in ? l[int64_t(s) * lay.l_ss] : kNegInf;
        v[u] = (in && c_in) ? load_row4<VEC>(o + int64_t(s) * lay.o_ss, c, D)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      float mb = m;
#pragma unroll
      for (int u = 0; u < R; ++u) mb = fmaxf(mb, ls[u]);
      if (mb != kNegInf) {   // warp-uniform: every lane holds the same lse values
        const float f = fast_exp2(m - mb);   // 0 while m is -inf
        wsum *= f;
        acc.x *= f; acc.y *= f; acc.z *= f; acc.w *= f;
#pragma unroll
        for (int u = 0; u < R; ++u) {
          // a split of weight 0 contributes nothing even if its row holds garbage (select,
          // not branch, so the loads stay independent)
          const float w = fast_exp2(ls[u] - mb);
          const bool on = w != 0.f;
          wsum += w;
          acc.x = fmaf(w, on ? v[u].x : 0.f, acc.x);
          acc.y = fmaf(w, on ? v[u].y : 0.f, acc.y);
          acc.z = fmaf(w, on ? v[u].z : 0.f, acc.z);
          acc.w = fmaf(w, on ? v[u].w : 0.f, acc.w);
        }
        m = mb;
      }
    }
    if (lane == 0) {
      s_m[warp] = m;
      s_l[warp] = wsum;
    }
    s_o[warp][lane] = acc;
    __syncthreads();
    if (warp == 0) {
      // lane w: state w's weight; the max and the sum run over the lanes in a fixed order
      const float mw = lane < W ? s_m[lane] : kNegInf;
      float M = mw;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(kFullMask, M, off));
      const float fw = (lane < W && M != kNegInf) ? fast_exp2(mw - M) : 0.f;
      float L = lane < W ? s_l[lane] * fw : 0.f;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(kFullMask, L, off);
      const float inv = L > 0.f ? 1.f / L : 0.f;
      s_f[lane] = fw * inv;
      __syncwarp();
      float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
      for (int w = 0; w < W; ++w) {
        const float f = s_f[w];
        const float4 a = s_o[w][lane];
        O.x = fmaf(a.x, f, O.x);
        O.y = fmaf(a.y, f, O.y);
        O.z = fmaf(a.z, f, O.z);
        O.w = fmaf(a.w, f, O.w);
      }
      const float r[4] = {O.x, O.y, O.z, O.w};
      if (c_in) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int d = 4 * c + e;
          if (d < D) {
            if constexpr (F16OUT) {
              out16[int64_t(b) * o_sb + int64_t(hq) * o_sh + d] = __float2half_rn(r[e]);
            } else {
              o32[(int64_t(b) * q_heads + hq) * D + d] = r[e];
            }
          }
        }
      }
      if constexpr (!F16OUT) {
        if (c0 == 0 && lane == 0)
          lse32[int64_t(b) * q_heads + hq] = L > 0.f ? M + __log2f(L) : kNegInf;
      }
    }
    __syncthreads();   // s_m / s_l / s_o are rewritten by the next channel group
  }
}

template <int D, int GP>
int launch_split(const CUtensorMap& tk, const CUtensorMap& tv, const DecodeParams& p,
                 cudaStream_t st) {
  using G = Geo<D, GP>;
  auto kern = split_kv_fp16_kernel<D, GP>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           int(G::SMEM_BYTES)) != cudaSuccess)
    return BPT_ERR_LAUNCH;
  dim3 grid(p.splits, p.kv_heads, p.batch);
  return launch_dependent(kern, grid, dim3(kThreads), G::SMEM_BYTES, st, tk, tv, p) ==
                 cudaSuccess
             ? BPT_OK
             : BPT_ERR_LAUNCH;
}

template <int D>
int dispatch_group(int gp, const CUtensorMap& tk, const CUtensorMap& tv, const DecodeParams& p,
                   cudaStream_t st) {
  switch (gp) {
    case 1: return launch_split<D, 1>(tk, tv, p, st);
    case 2: return launch_split<D, 2>(tk, tv, p, st);
    case 4: return launch_split<D, 4>(tk, tv, p, st);
    case 8: return launch_split<D, 8>(tk, tv, p, st);
    default: return BPT_ERR_UNSUPPORTED_SHAPE;
  }
}


#ifndef BPT_FP16_NCW
#define BPT_FP16_NCW 2      // consumer warps per CTA (chunk = 16 * NCW tokens)
#endif
#ifndef BPT_FP16_STAGES
#define BPT_FP16_STAGES 3   // shared-memory ring depth
#endif
#ifndef BPT_FP16_MINB
#define BPT_FP16_MINB 4     // CTAs per SM the register budget is sized for
#endif

// Tensor-core kernel configuration for head_dim D. Many resident CTAs (independent TMA
// streams) per SM matter more than a deep ring: for D <= 128 a CTA is 2 consumer warps + 1
// producer warp streaming 32-token chunks through a 3-stage ring (48 KB at D=128), 4 CTAs
// per SM. Measured on B200 against 2-4 consumer warps, 2-4 stages, 2-6 CTAs/SM.
template <int D>
struct Fp16Tc {
  static constexpr int NCW = D >= 256 ? 4 : BPT_FP16_NCW;
  static constexpr int STAGES = D >= 256 ? 2 : BPT_FP16_STAGES;
  static constexpr int MINB = D >= 256 ? 1 : BPT_FP16_MINB;
  static constexpr int CHUNK = 16 * NCW;
};

template <int D>
int launch_split_mma(bool g8, const CUtensorMap& tk, const CUtensorMap& tv,
                     const DecodeParams& p, cudaStream_t st) {
  using T = Fp16Tc<D>;
  return g8 ? mma::launch<D, T::NCW, T::STAGES, T::MINB, true>(tk, tv, p, st)
            : mma::launch<D, T::NCW, T::STAGES, T::MINB, false>(tk, tv, p, st);
}

int tc_chunk_tokens(int head_dim) {
  switch (head_dim) {
    case 64: return Fp16Tc<64>::CHUNK;
    case 128: return Fp16Tc<128>::CHUNK;
    case 256: return Fp16Tc<256>::CHUNK;
    default: return kChunk;
  }
}

}  // namespace

static int launch_merge_layout(const float* o_part, const float* lse, const MergeLayout& lay,
                               int batch, int q_heads, int splits, int D, __half* out16,
                               int64_t o_sb, int64_t o_sh, float* o32, float* lse32,
                               cudaStream_t st, bool pdl) {
  if (batch <= 0) return BPT_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(q_heads, batch);
  const int warps = splits >= kMergeWarps * kMergeRows ? kMergeWarps
                                                        : (splits + kMergeRows - 1) / kMergeRows;
  cfg.blockDim = dim3(32 * (warps < 1 ? 1 : warps));
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  // float4 loads when every (b, head, split) row starts on a 16-byte boundary
  const bool vec = (D % 4 == 0) && (lay.o_ss % 4 == 0) && (lay.o_sb % 4 == 0) &&
                   (lay.o_sh % 4 == 0) && ((reinterpret_cast<uintptr_t>(o_part) & 15) == 0);
  float* const no32 = nullptr;
  __half* const no16 = nullptr;
  cudaError_t e;
  if (out16) {
    e = vec ? cudaLaunchKernelEx(&cfg, merge_splits_kernel<true, true>, o_part, lse, lay,
                                 q_heads, splits, D, out16, o_sb, o_sh, no32, no32)
            : cudaLaunchKernelEx(&cfg, merge_splits_kernel<true, false>, o_part, lse, lay,
                                 q_heads, splits, D, out16, o_sb, o_sh, no32, no32);
  } else {
    e = vec ? cudaLaunchKernelEx(&cfg, merge_splits_kernel<false, true>, o_part, lse, lay,
                                 q_heads, splits, D, no16, int64_t(0), int64_t(0), o32, lse32)
            : cudaLaunchKernelEx(&cfg, merge_splits_kernel<false, false>, o_part, lse, lay,
                                 q_heads, splits, D, no16, int64_t(0), int64_t(0), o32, lse32);
  }
  return e == cudaSuccess ? BPT_OK : BPT_ERR_LAUNCH;
}

int launch_merge(const float* o_part, const float* lse, int batch, int q_heads, int splits,
                 int D, __half* out16, int64_t o_sb, int64_t o_sh, float* o32, float* lse32,
                 cudaStream_t st, bool pdl) {
  MergeLayout lay;  // [B, Hq, S, D] partials of one call
  lay.o_ss = D;
  lay.o_sh = int64_t(splits) * D;
  lay.o_sb = int64_t(q_heads) * splits * D;
  lay.l_ss = 1;
  lay.l_sh = splits;
  lay.l_sb = int64_t(q_heads) * splits;
  return launch_merge_layout(o_part, lse, lay, batch, q_heads, splits, D, out16, o_sb, o_sh, o32,
                             lse32, st, pdl);
}

// Validate, encode the tensor maps and launch the split kernel. `final_out` selects the
// one-split fast path that writes fp16 `out`; otherwise partial states go to o_part/lse.
int run_split_fp16(const void* q, int64_t q_sb, int64_t q_sh, const void* k_cache, int64_t k_sb,
                   int64_t k_st, int64_t k_sh, const void* v_cache, int64_t v_sb, int64_t v_st,
                   int64_t v_sh, int64_t num_blocks, const int32_t* block_table, int64_t bt_sb,
                   const int32_t* seq_lens, void* out, int64_t o_sb, int64_t o_sh, int batch,
                   int q_heads, int kv_heads, int head_dim, int block_size, int max_blocks,
                   float scale, int splits, int final_out, float* o_part, float* lse,
                   unsigned* status, cudaStream_t st) {
  if (batch < 0 || q_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || block_size <= 0 ||
      max_blocks < 0 || num_blocks < 0 || splits < 1)
    return BPT_ERR_INVALID_ARGUMENT;
  if (q_heads % kv_heads != 0) return BPT_ERR_INVALID_ARGUMENT;
  if (batch == 0) return BPT_OK;
  if (!q || !k_cache || !v_cache || !block_table || !seq_lens) return BPT_ERR_INVALID_ARGUMENT;
  if (final_out ? !out : (!o_part || !lse)) return BPT_ERR_INVALID_ARGUMENT;
  const int group = q_heads / kv_heads;
  const int gp = group <= 1 ? 1 : group <= 2 ? 2 : group <= 4 ? 4 : group <= 8 ? 8 : 16;
  if (gp > 8) return BPT_ERR_UNSUPPORTED_SHAPE;
  if (!(head_dim == 16 || head_dim == 32 || head_dim == 64 || head_dim == 128 ||
        head_dim == 256))
    return BPT_ERR_UNSUPPORTED_SHAPE;
  if (block_size < 16 || block_size > 256 || (block_size & (block_size - 1)))
    return BPT_ERR_UNSUPPORTED_SHAPE;
  if (reinterpret_cast<uintptr_t>(q) & 15) return BPT_ERR_ALIGNMENT;
  if (((q_sb * 2) % 16) || ((q_sh * 2) % 16)) return BPT_ERR_ALIGNMENT;

  DecodeParams p{};
  // head_dim a multiple of 64: tensor-core kernel over 64-column swizzled boxes;
  // head_dim 16 / 32: CUDA-core kernel over whole rows.
  const bool mma_path = head_dim % 64 == 0;
  const int chunk = mma_path ? tc_chunk_tokens(head_dim) : kChunk;
  const int box_rows = block_size < chunk ? block_size : chunk;
  const int box_inner = mma_path ? 64 : head_dim;
  const int swizzle = mma_path ? 128 : 0;
  CUtensorMap tk, tv;
  int rc = encode_kv_map(&tk, k_cache, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, head_dim, kv_heads,
                         block_size, num_blocks, k_sh, k_st, k_sb, box_inner, box_rows, &p.k_c1,
                         swizzle);
  if (rc) return rc;
  rc = encode_kv_map(&tv, v_cache, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, head_dim, kv_heads,
                     block_size, num_blocks, v_sh, v_st, v_sb, box_inner, box_rows, &p.v_c1,
                     swizzle);
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
  p.kv_heads = kv_heads;
  p.group = group;
  p.splits = splits;
  p.final_out = final_out;
  p.balance = balanced_splits(batch, kv_heads, splits, kResidentFp16) ? 1 : 0;
  p.block_size = block_size;
  p.max_blocks = max_blocks;
  p.box_rows = box_rows;
  p.num_blocks = num_blocks;
  const float sc = scale > 0.f ? scale : 1.0f / sqrtf(float(head_dim));
  p.scale_log2 = sc * 1.4426950408889634f;
  switch (head_dim) {
    case 16: rc = dispatch_group<16>(gp, tk, tv, p, st); break;
    case 32: rc = dispatch_group<32>(gp, tk, tv, p, st); break;
    case 64: rc = launch_split_mma<64>(gp > 4, tk, tv, p, st); break;
    case 128: rc = launch_split_mma<128>(gp > 4, tk, tv, p, st); break;
    case 256: rc = launch_split_mma<256>(gp > 4, tk, tv, p, st); break;
    default: rc = BPT_ERR_UNSUPPORTED_SHAPE;
  }
  if (rc) return rc;
  return cudaGetLastError() == cudaSuccess ? BPT_OK : BPT_ERR_LAUNCH;
}

}  // namespace bpt

using namespace bpt;

extern "C" int bpt_decode_fp16(const void* q, int64_t q_sb, int64_t q_sh, const void* k_cache,
                               int64_t k_sb, int64_t k_st, int64_t k_sh, const void* v_cache,
                               int64_t v_sb, int64_t v_st, int64_t v_sh, int64_t num_blocks,
                               const int32_t* block_table, int64_t bt_sb,
                               const int32_t* seq_lens, void* out, int64_t o_sb, int64_t o_sh,
                               int batch, int q_heads, int kv_heads, int head_dim,
                               int block_size, int max_blocks, float scale, int num_splits,
                               int sm_count, void* workspace, size_t workspace_bytes,
                               void* stream) {
  if (batch < 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads != 0)
    return BPT_ERR_INVALID_ARGUMENT;
  if (batch == 0) return BPT_OK;
  if (!workspace || !out) return BPT_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(out) & 15) || ((o_sb * 2) % 16) || ((o_sh * 2) % 16))
    return BPT_ERR_ALIGNMENT;
  const int S = bpt_effective_splits(batch, kv_heads, block_size, max_blocks, num_splits,
                                     sm_count);
  if (workspace_bytes < bpt_decode_workspace_bytes(batch, q_heads, head_dim, S))
    return BPT_ERR_WORKSPACE_TOO_SMALL;
  WorkspaceView ws = workspace_view(workspace, batch, q_heads, head_dim, S);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = run_split_fp16(q, q_sb, q_sh, k_cache, k_sb, k_st, k_sh, v_cache, v_sb, v_st, v_sh,
                          num_blocks, block_table, bt_sb, seq_lens, out, o_sb, o_sh, batch,
                          q_heads, kv_heads, head_dim, block_size, max_blocks, scale, S, 1,
                          ws.o_part, ws.lse, ws.status, st);
  if (rc || S == 1) return rc;
  return launch_merge(ws.o_part, ws.lse, batch, q_heads, S, head_dim,
                      static_cast<__half*>(out), o_sb, o_sh, nullptr, nullptr, st, true);
}

extern "C" int bpt_decode_fp16_partial(const void* q, int64_t q_sb, int64_t q_sh,
                                       const void* k_cache, int64_t k_sb, int64_t k_st,
                                       int64_t k_sh, const void* v_cache, int64_t v_sb,
                                       int64_t v_st, int64_t v_sh, int64_t num_blocks,
                                       const int32_t* block_table, int64_t bt_sb,
                                       const int32_t* seq_lens, int batch, int q_heads,
                                       int kv_heads, int head_dim, int block_size,
                                       int max_blocks, float scale, int splits, float* o_part,
                                       float* lse, unsigned* status, void* stream) {
  return run_split_fp16(q, q_sb, q_sh, k_cache, k_sb, k_st, k_sh, v_cache, v_sb, v_st, v_sh,
                        num_blocks, block_table, bt_sb, seq_lens, nullptr, 0, 0, batch,
                        q_heads, kv_heads, head_dim, block_size, max_blocks, scale, splits, 0,
                        o_part, lse, status, static_cast<cudaStream_t>(stream));
}

extern "C" int bpt_merge_partials(const float* o_part, const float* lse, int batch, int q_heads,
                                  int head_dim, int splits, void* out, int64_t o_sb,
                                  int64_t o_sh, void* stream) {
  if (batch < 0 || q_heads <= 0 || head_dim <= 0 || splits < 1) return BPT_ERR_INVALID_ARGUMENT;
  if (batch == 0) return BPT_OK;
  if (!o_part || !lse || !out) return BPT_ERR_INVALID_ARGUMENT;
  return launch_merge(o_part, lse, batch, q_heads, splits, head_dim, static_cast<__half*>(out),
                      o_sb, o_sh, nullptr, nullptr, static_cast<cudaStream_t>(stream), false);
}

extern "C" int bpt_merge_states(const float* o_part, const float* lse, int batch, int q_heads,
                                int head_dim, int splits, float* o_out, float* lse_out,
                                void* stream) {
  if (batch < 0 || q_heads <= 0 || head_dim <= 0 || splits < 1) return BPT_ERR_INVALID_ARGUMENT;
  if (batch == 0) return BPT_OK;
  if (!o_part || !lse || !o_out || !lse_out) return BPT_ERR_INVALID_ARGUMENT;
  return launch_merge(o_part, lse, batch, q_heads, splits, head_dim, nullptr, 0, 0, o_out,
                      lse_out, static_cast<cudaStream_t>(stream), false);
}

extern "C" int bpt_merge_rank_states(const float* states, int ranks, int batch, int q_heads,
                                     int head_dim, void* out, int64_t o_sb, int64_t o_sh,
                                     void* stream) {
  if (ranks < 1 || batch < 0 || q_heads <= 0 || head_dim <= 0) return BPT_ERR_INVALID_ARGUMENT;
  if (batch == 0) return BPT_OK;
  if (!states || !out) return BPT_ERR_INVALID_ARGUMENT;
  // each rank's block: o [B, Hq, D] then lse [B, Hq]
  const int64_t block = int64_t(batch) * q_heads * (head_dim + 1);
  MergeLayout lay;
  lay.o_ss = block;
  lay.o_sb = int64_t(q_heads) * head_dim;
  lay.o_sh = head_dim;
  lay.l_ss = block;
  lay.l_sb = q_heads;
  lay.l_sh = 1;
  const float* lse = states + int64_t(batch) * q_heads * head_dim;
  return launch_merge_layout(states, lse, lay, batch, q_heads, ranks, head_dim,
                             static_cast<__half*>(out), o_sb, o_sh, nullptr, nullptr,
                             static_cast<cudaStream_t>(stream), false);
}
