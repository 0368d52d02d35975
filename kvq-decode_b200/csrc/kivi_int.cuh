// INT8 / INT4 KIVI decode on integer tensor-core MMAs (mma.sync m16n8k32, 8-bit operands,
// exact 32-bit integer accumulation). Included by kivi_decode.cu inside namespace
// bpt::kivi; used for group <= 4 (the fp16-MMA kernel in kivi_decode.cu serves FP8 and larger
// groups).
//
// Why integers: the codes ARE small integers, so they enter the MMA with no per-value
// conversion (INT8 keys: none at all; INT4 keys: one mask or shift-and-mask per 4 codes), and
// integer accumulation is exact. The fp operands become fixed point instead:
//
//   QK^T   q'_d = q_d * k_scale_d (per page, q head, channel) -> x = round(q' * 2^Ek),
//          |x| < 2^30, split into four balanced signed bytes (x = sum_k l_k 256^k). Every
//          token of a page shares the rounding of x, so x keeps all the bits the limbs hold.
//          MMA rows: 0-3 = limb 0 of heads 0-3, 8-11 = limb 1, 4-7 = limb 2, 12-15 = limb 3.
//          S = (L0 + 256 L1 + 65536 (L2 + 256 L3)) * 2^-Ek + sum_d q_d k_zero_d  (fp32 after)
//   P.V    p'_t = p_t * v_scale_t -> round(p' * 2^Ev) < 2^32, four unsigned bytes. MMA_a
//          columns = limb 0 | limb 1 (heads 0-3 each), MMA_b = limb 2 | limb 3; A = value
//          codes transposed to (channel rows, 4 tokens per register).
//          O = sum_t p'_t c_t (exact int) * 2^-Ev + sum_t p_t v_zero_t        (fp32)
//
// p is taken relative to a per-head reference m_ref that trails the running max by up to 4
// (log2 units): p <= 16, so p' keeps at least 26 significant bits for the largest terms and
// the int32 accumulators are converted to fp32 ("flushed") only when a score exceeds
// m_ref + 4, when a value scale outgrows the fixed-point exponent, or every 1024 chunks (32
// tokens x 255 x 255 per chunk keeps 1024 chunks inside int32).
//
// CTA = 4 warps, no producer warp: 128 tokens per pipeline stage, 32 per warp. Thread 0 issues
// the TMA loads of a stage (key / value code boxes, the page's k_scale / k_zero rows); every
// thread copies its own token's v_scale / v_zero granules with cp.async, tracked by the same
// mbarrier. Per stage, warp w quantizes q head w against the stage's k_scale rows into a
// double-buffered fragment-ordered block; a consumer mbarrier (bounded wait) publishes it,
// and at that point every warp is done with the previous stage, which is refilled.

constexpr float kSoftmaxHeadroom = 4.f;   // log2 units
constexpr int kValueHeadroom = 1;         // bits
constexpr int kExpUnset = 0x7fffffff;

template <int FMT, int STAGES>
struct ICfg {
  static constexpr bool INT4 = FMT == BPT_KV_INT4;
  static constexpr int NW = 4;
  static constexpr int CHUNK = 32 * NW;                    // tokens per stage
  static constexpr int THREADS = 32 * NW;
  static constexpr int K_ROW = INT4 ? 64 : 128;
  static constexpr int K_BYTES = CHUNK * K_ROW;
  static constexpr int V_BYTES = (INT4 ? CHUNK / 2 : CHUNK) * 128;
  static constexpr int VP_BYTES = CHUNK * 8;               // [token][scale granule, zero granule]
  // stage = [K codes][V codes][v params][k_scale | k_zero rows of the chunk's nslot boxes];
  // nslot = CHUNK / box_rows is a launch-time value (1 for block_size >= CHUNK)
  static constexpr int STAGE_FIXED = K_BYTES + V_BYTES + VP_BYTES;
  static constexpr int FQ_ROW = 144;                       // 128 B of limbs + bank padding
  static constexpr int FQ_SLOT = 16 * FQ_ROW;              // 16 limb rows
  static constexpr size_t MERGE_BYTES = size_t(NW) * 8 * (D + 3) * 4;
  __host__ __device__ static constexpr int stage_bytes(int nslot) {
    return (STAGE_FIXED + nslot * 512 + 1023) & ~1023;
  }
  __host__ __device__ static constexpr size_t body_bytes(int nslot) {
    return size_t(STAGES) * stage_bytes(nslot) > MERGE_BYTES
               ? size_t(STAGES) * stage_bytes(nslot)
               : MERGE_BYTES;
  }
  // q limbs [buf 2][slot][row 16][FQ_ROW], then {bias', kdown'} [buf 2][slot][head 4]
  __host__ __device__ static constexpr size_t fq_bytes(int nslot) {
    return size_t(2) * nslot * (FQ_SLOT + 32);
  }
  __host__ __device__ static constexpr size_t smem_bytes(int nslot) {
    return 1024 + body_bytes(nslot) + fq_bytes(nslot) + (STAGES + 1) * 8;
  }
};

__device__ __forceinline__ void mma_s8u8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_u8u8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t redux_max_u32(uint32_t v) {
  uint32_t r;
  asm volatile("redux.sync.max.u32 %0, %1, 0xffffffff;" : "=r"(r) : "r"(v));
  return r;
}

__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// [x0.byte k, x1.byte k, x2.byte k, x3.byte k]
__device__ __forceinline__ uint32_t byte_sel(uint32_t x0, uint32_t x1, uint32_t x2, uint32_t x3,
                                             uint32_t k) {
  const uint32_t s = k | ((4 + k) << 4);
  return __byte_perm(__byte_perm(x0, x1, s), __byte_perm(x2, x3, s), 0x5410);
}

// floor(log2(x)) of a positive finite fp32 given by its bits (subnormals count as -127)
__device__ __forceinline__ int exponent_of_bits(uint32_t bits) {
  return int(bits >> 23) - 127;
}

template <int FMT, int STAGES, int MINB>
__global__ void __launch_bounds__(128, MINB)
kivi_int_decode_kernel(const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV,
                       const __grid_constant__ CUtensorMap tmKS,
                       const __grid_constant__ CUtensorMap tmKZ, const KiviParams kp) {
  using C = ICfg<FMT, STAGES>;
  constexpr int CHUNK = C::CHUNK;
  constexpr int NW = C::NW;
  constexpr bool INT4 = C::INT4;
  const DecodeParams& p = kp.d;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int lR = kp.lbox, R = 1 << lR;          // rows per TMA box (min(block_size, CHUNK))
  const int lbs = kp.lbs, bs = 1 << lbs;
  const int nslot = CHUNK >> lR;
  const int stage_bytes = C::stage_bytes(nslot);
  uint8_t* fq_base = smem + C::body_bytes(nslot);
  float* qp_base = reinterpret_cast<float*>(fq_base + 2 * nslot * C::FQ_SLOT);
  uint64_t* full = reinterpret_cast<uint64_t*>(fq_base + C::fq_bytes(nslot));
  uint64_t* prep = full + STAGES;
  float* sM = reinterpret_cast<float*>(smem);   // merge scratch aliases the ring at the end
  float* sL = sM + NW * 8;
  float* sAcc = sL + NW * 8;

  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.splits;

  // the tensor maps are kernel parameters, not written by the previous kernel: their fetch
  // overlaps the wait
  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
    prefetch_tensormap(&tmKS);
    prefetch_tensormap(&tmKZ);
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

  // q-limb blocks and page constants start at zero: rows of heads >= group stay zero
  for (int i = threadIdx.x; i < int(C::fq_bytes(nslot) / 16); i += blockDim.x)
    reinterpret_cast<uint4*>(fq_base)[i] = make_uint4(0u, 0u, 0u, 0u);
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&full[s], 1 + C::THREADS);
    mbar_init(prep, NW);
    fence_mbar_init();
  }

  // q of this warp's head for the 4 channels this lane quantizes (fragment order: lane
  // lambda = 8 t + 2 ks + half owns byte lanes 4 lambda .. 4 lambda + 3 of every limb row)
  const bool prep_warp = warp < p.group;
  const int pt = lane >> 3, pks = (lane >> 1) & 3, phalf = lane & 1;
  const int pch0 = INT4 ? 32 * pks + 8 * pt : 32 * pks + 16 * phalf + 4 * pt;
  const uint32_t psel = phalf ? 0x7632u : 0x5410u;   // INT4: odd / even channel of each pair
  float qv[4] = {0.f, 0.f, 0.f, 0.f};
  if (prep_warp) {
    const __half* qrow = p.q + int64_t(b) * p.q_sb + int64_t(qh0 + warp) * p.q_sh + pch0;
    uint32_t w01, w23;
    if constexpr (INT4) {
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(qrow));
      w01 = __byte_perm(raw.x, raw.y, psel);
      w23 = __byte_perm(raw.z, raw.w, psel);
    } else {
      const uint2 raw = __ldg(reinterpret_cast<const uint2*>(qrow));
      w01 = raw.x;
      w23 = raw.y;
    }
    const float2 f01 = half2_bits_to_float2(w01), f23 = half2_bits_to_float2(w23);
    qv[0] = f01.x; qv[1] = f01.y; qv[2] = f23.x; qv[3] = f23.y;
  }
  __syncthreads();
  pdl_launch_dependents();   // the merge grid may launch now; it waits for this grid's end

  // ------------------------------------------------------------------ loads of one stage
  const int32_t* bt = p.block_table + int64_t(b) * p.bt_sb;
  const int last_page = (t_end - 1) >> lbs;
  int win_base = t_begin >> lbs;   // block-table window: lane i holds entry win_base + i
  int win = (win_base + lane <= last_page) ? __ldg(bt + win_base + lane) : 0;
  const uint64_t pol = l2_evict_first_policy();
  const uint32_t box_bytes = uint32_t(R) * C::K_ROW + uint32_t(INT4 ? R / 2 : R) * 128u + 512u;

  // every thread calls issue() for the same chunks in the same order (identical windows)
  auto issue = [&](int cc) {
    const int stg = cc % STAGES;
    uint8_t* sb = smem + stg * stage_bytes;
    uint8_t* vbuf = sb + C::K_BYTES;
    uint8_t* vpar = vbuf + C::V_BYTES;
    uint8_t* kpar = vpar + C::VP_BYTES;
    const int tok0 = (u0 + cc) * CHUNK;
    const int tok_last = min(tok0 + CHUNK, t_end) - 1;
    if ((tok_last >> lbs) - win_base >= 32) {
      win_base = tok0 >> lbs;
      win = (win_base + lane <= last_page) ? __ldg(bt + win_base + lane) : 0;
    }
    if (warp == 0) {
      const int nbox = (tok_last - tok0 + R) >> lR;
      if (lane == 0) mbar_arrive_expect_tx(&full[stg], uint32_t(nbox) * box_bytes);
      for (int j = 0; j < nbox; ++j) {
        const int t = tok0 + (j << lR);
        int phys = __shfl_sync(kFullMask, win, (t >> lbs) - win_base);
        if (lane == 0) {
          if (phys < 0 || int64_t(phys) >= p.num_blocks) {
            flag_device_error(p.status, BPT_DEV_BAD_BLOCK_ID);
            phys = 0;
          }
          const int row = t & (bs - 1);
          tma_load_4d(sb + j * R * C::K_ROW, &tmK, &full[stg], 0, p.k_c1 ? row : h,
                      p.k_c1 ? h : row, phys, pol);
          const int vrow = INT4 ? row / 2 : row;
          tma_load_4d(vbuf + j * (INT4 ? R / 2 : R) * 128, &tmV, &full[stg], 0,
                      p.v_c1 ? vrow : h, p.v_c1 ? h : vrow, phys, pol);
          tma_load_3d(kpar + j * 512, &tmKS, &full[stg], 0, h, phys);
          tma_load_3d(kpar + j * 512 + 256, &tmKZ, &full[stg], 0, h, phys);
        }
      }
    }
    // this thread's token: the 4-byte granules holding its v_scale / v_zero
    const int t = tok0 + 32 * warp + lane;
    const int ph = __shfl_sync(kFullMask, win, (min(t, tok_last) >> lbs) - win_base);
    if (t <= tok_last && ph >= 0 && int64_t(ph) < p.num_blocks) {
      const int64_t el = int64_t(ph) * kp.vps0 + int64_t(t & (bs - 1)) * kp.vps1 + h;
      const int64_t off = (el * 2) & ~int64_t(3);
      cp_async_4(smem_u32(vpar + 8 * (t - tok0)), kp.v_scale + off);
      cp_async_4(smem_u32(vpar + 8 * (t - tok0) + 4), kp.v_zero + off);
    }
    cp_async_arrive_noinc(&full[stg]);
  };

  int issued = 0;
  for (; issued < STAGES - 1 && issued < nchunks; ++issued) issue(issued);

  // ------------------------------------------------------------------ consumer state
  const int g = lane >> 2, t4 = lane & 3;
  const bool upper = g >= 4;                 // keeps n-blocks 2, 3 (lower lanes: 0, 1)
  const int mj = lane >> 3, mr = lane & 7;
  const int vc = INT4 ? (((g & 1) << 2) | (g >> 1)) : g;   // logical V chunk of this lane
  const uint32_t la = upper ? 1u : 0u, lb = 2u + la;        // p' limbs of column g
  const float mA = upper ? 65536.f : 1.f;                   // rows g: limb 0 or limb 2
  // half of each v-param granule: (row * token stride + head) & 1, row even / odd
  const int hs0 = h & 1, hs1 = int((kp.vps1 + h) & 1);
  const uint32_t vsel = (hs0 ? 0x32u : 0x10u) | ((hs1 ? 0x76u : 0x54u) << 8);
  const int srcA = ((2 * t4) & 3) * 4, srcB = ((2 * t4 + 1) & 3) * 4;

  int ia[8][4], ib[8][4];
  float master[8][4];
#pragma unroll
  for (int m = 0; m < 8; ++m)
#pragma unroll
    for (int e = 0; e < 4; ++e) { ia[m][e] = 0; ib[m][e] = 0; master[m][e] = 0.f; }
  float m_ref = kNegInf, l_run = 0.f, z_run = 0.f;
  int vexp = kExpUnset;
  int since_flush = 0;      // chunks accumulated in ia / ib since the last flush
  int consumed = 0;

  // int32 accumulators -> fp32: this lane's columns hold limbs (0, 2) or (1, 3) of a head
  auto flush = [&]() {
    const float vdown = exp2i(vexp == kExpUnset ? 0 : -vexp);
#pragma unroll
    for (int m = 0; m < 8; ++m)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        master[m][e] =
            fmaf(fmaf(65536.f, float(ib[m][e]), float(ia[m][e])), vdown, master[m][e]);
        ia[m][e] = 0;
        ib[m][e] = 0;
      }
    since_flush = 0;
  };

  for (int c = 0; c < nchunks; ++c) {
    const int stg = c % STAGES;
    if (!__all_sync(kFullMask, mbar_wait(&full[stg], uint32_t(c / STAGES) & 1u))) {
      if (lane == 0) flag_device_error(p.status, BPT_DEV_WAIT_TIMEOUT);
      break;
    }
    consumed = c + 1;
    uint8_t* st = smem + stg * stage_bytes;
    const uint32_t kbase = smem_u32(st);
    const uint8_t* vbuf = st + C::K_BYTES;
    const uint8_t* vpar = vbuf + C::V_BYTES;
    const __half* kpar = reinterpret_cast<const __half*>(vpar + C::VP_BYTES);
    const int tok0 = (u0 + c) * CHUNK;
    const int nbox = min(nslot, (t_end - tok0 + R - 1) >> lR);
    uint8_t* fq = fq_base + (c & 1) * nslot * C::FQ_SLOT;
    float* qp = qp_base + (c & 1) * nslot * 8;

    // ---- q' limbs of head `warp` for every box of the chunk
    if (prep_warp) {
      for (int j = 0; j < nbox; ++j) {
        const __half* ks = kpar + j * 256 + pch0;
        uint32_t s01, s23, z01, z23;
        if constexpr (INT4) {
          const uint4 rs = *reinterpret_cast<const uint4*>(ks);
          const uint4 rz = *reinterpret_cast<const uint4*>(ks + 128);
          s01 = __byte_perm(rs.x, rs.y, psel); s23 = __byte_perm(rs.z, rs.w, psel);
          z01 = __byte_perm(rz.x, rz.y, psel); z23 = __byte_perm(rz.z, rz.w, psel);
        } else {
          const uint2 rs = *reinterpret_cast<const uint2*>(ks);
          const uint2 rz = *reinterpret_cast<const uint2*>(ks + 128);
          s01 = rs.x; s23 = rs.y; z01 = rz.x; z23 = rz.y;
        }
        const float2 sa = half2_bits_to_float2(s01), sb = half2_bits_to_float2(s23);
        const float2 za = half2_bits_to_float2(z01), zb = half2_bits_to_float2(z23);
        const float qs0 = qv[0] * sa.x, qs1 = qv[1] * sa.y, qs2 = qv[2] * sb.x,
                    qs3 = qv[3] * sb.y;
        float bsum = fmaf(qv[3], zb.y, fmaf(qv[2], zb.x, fmaf(qv[1], za.y, qv[0] * za.x)));
        const float lm = fmaxf(fmaxf(fabsf(qs0), fabsf(qs1)), fmaxf(fabsf(qs2), fabsf(qs3)));
        const uint32_t qm = redux_max_u32(__float_as_uint(lm));
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) bsum += __shfl_xor_sync(kFullMask, bsum, off);
        // |q' 2^ek| < 2^30 keeps the top of four balanced limbs inside int8
        const int ek = qm ? min(126, 29 - exponent_of_bits(qm)) : 0;
        const float kup = exp2i(ek);
        const uint32_t y0 = uint32_t(__float2int_rn(qs0 * kup)) + 0x80808080u;
        const uint32_t y1 = uint32_t(__float2int_rn(qs1 * kup)) + 0x80808080u;
        const uint32_t y2 = uint32_t(__float2int_rn(qs2 * kup)) + 0x80808080u;
        const uint32_t y3 = uint32_t(__float2int_rn(qs3 * kup)) + 0x80808080u;
        // x + 0x80808080 = sum_k (l_k + 128) 256^k: byte k ^ 0x80 is the signed limb l_k
        uint8_t* slot = fq + j * C::FQ_SLOT + 4 * lane;
        *reinterpret_cast<uint32_t*>(slot + warp * C::FQ_ROW) =
            byte_sel(y0, y1, y2, y3, 0u) ^ 0x80808080u;
        *reinterpret_cast<uint32_t*>(slot + (8 + warp) * C::FQ_ROW) =
            byte_sel(y0, y1, y2, y3, 1u) ^ 0x80808080u;
        *reinterpret_cast<uint32_t*>(slot + (4 + warp) * C::FQ_ROW) =
            byte_sel(y0, y1, y2, y3, 2u) ^ 0x80808080u;
        *reinterpret_cast<uint32_t*>(slot + (12 + warp) * C::FQ_ROW) =
            byte_sel(y0, y1, y2, y3, 3u) ^ 0x80808080u;
        if (lane == 0)
          *reinterpret_cast<float2*>(qp + j * 8 + warp * 2) =
              make_float2(bsum * p.scale_log2, exp2i(-ek) * p.scale_log2);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(prep);
    if (!__all_sync(kFullMask, mbar_wait(prep, uint32_t(c) & 1u))) {
      if (lane == 0) flag_device_error(p.status, BPT_DEV_WAIT_TIMEOUT);
      break;
    }
    // every warp is past chunk c - 1: its stage takes chunk c + STAGES - 1
    if (issued < nchunks) {
      issue(issued);
      ++issued;
    }

    // ---- S = q'_int . codes: lanes g < 4 hold limbs 0 (rows g) and 1 (rows g + 8),
    //      lanes g >= 4 limbs 2 (rows g) and 3 (rows g + 8); own = their share of head g & 3
    float own[4][2];
    uint32_t A[8], Bq[8];
#pragma unroll
    for (int hb = 0; hb < 2; ++hb) {
      if (hb == 0 || lR == 4) {
        const uint8_t* fr = fq + ((32 * warp + 16 * hb) >> lR) * C::FQ_SLOT + t4 * 32;
        const uint4 ra0 = *reinterpret_cast<const uint4*>(fr + g * C::FQ_ROW);
        const uint4 ra1 = *reinterpret_cast<const uint4*>(fr + g * C::FQ_ROW + 16);
        A[0] = ra0.x; A[1] = ra0.y; A[2] = ra0.z; A[3] = ra0.w;
        A[4] = ra1.x; A[5] = ra1.y; A[6] = ra1.z; A[7] = ra1.w;
        const uint4 rb0 = *reinterpret_cast<const uint4*>(fr + (g + 8) * C::FQ_ROW);
        const uint4 rb1 = *reinterpret_cast<const uint4*>(fr + (g + 8) * C::FQ_ROW + 16);
        Bq[0] = rb0.x; Bq[1] = rb0.y; Bq[2] = rb0.z; Bq[3] = rb0.w;
        Bq[4] = rb1.x; Bq[5] = rb1.y; Bq[6] = rb1.z; Bq[7] = rb1.w;
      }
#pragma unroll
      for (int nbi = 0; nbi < 2; ++nbi) {
        const int nb = 2 * hb + nbi;
        const int row = 32 * warp + 8 * nb + mr;   // token row this lane addresses
        int sacc[4] = {0, 0, 0, 0};
        if constexpr (INT4) {
          uint32_t w0, w1, w2, w3;   // 16-byte chunks 0..3 = k-steps 0..3
          ldsm_x4(kbase + uint32_t(row) * 64u + ((uint32_t(mj) ^ uint32_t((row >> 1) & 3)) << 4),
                  w0, w1, w2, w3);
          const uint32_t ws[4] = {w0, w1, w2, w3};
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            mma_s8u8(sacc, A[2 * ks], Bq[2 * ks], A[2 * ks + 1], Bq[2 * ks + 1],
                     ws[ks] & 0x0F0F0F0Fu, (ws[ks] >> 4) & 0x0F0F0F0Fu);
        } else {
          uint32_t w[8];             // chunks 0..7: k-step ks uses chunks 2 ks, 2 ks + 1
          const uint32_t rb = kbase + uint32_t(row) * 128u;
          const uint32_t swz = uint32_t(row & 7);
          ldsm_x4(rb + ((uint32_t(mj) ^ swz) << 4), w[0], w[1], w[2], w[3]);
          ldsm_x4(rb + ((uint32_t(mj + 4) ^ swz) << 4), w[4], w[5], w[6], w[7]);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            mma_s8u8(sacc, A[2 * ks], Bq[2 * ks], A[2 * ks + 1], Bq[2 * ks + 1], w[2 * ks],
                     w[2 * ks + 1]);
        }
        // lower lanes: L0 + 256 L1; upper lanes: 65536 (L2 + 256 L3)
        own[nb][0] = mA * fmaf(256.f, float(sacc[2]), float(sacc[0]));
        own[nb][1] = mA * fmaf(256.f, float(sacc[3]), float(sacc[1]));
      }
    }

    // ---- reduce-scatter with lane g ^ 4: this lane keeps n-blocks kb, kb + 1 of head g & 3
    const int kb = upper ? 2 : 0;
    const float2 qpv =
        *reinterpret_cast<const float2*>(qp + ((32 * warp + 16 * (kb >> 1)) >> lR) * 8 +
                                         (g & 3) * 2);
    float x[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int nbk = k >> 1, e = k & 1;
      const float keep = upper ? own[2 + nbk][e] : own[nbk][e];
      const float send = upper ? own[nbk][e] : own[2 + nbk][e];
      x[k] = fmaf(keep + __shfl_xor_sync(kFullMask, send, 16), qpv.y, qpv.x);
    }
    // value scale / zero of the kept tokens (32 w + 8 (kb + nbk) + 2 t4 + e)
    float vs[4], vz[4];
#pragma unroll
    for (int nbk = 0; nbk < 2; ++nbk) {
      const uint4 gr =
          *reinterpret_cast<const uint4*>(vpar + 8 * (32 * warp + 8 * (kb + nbk) + 2 * t4));
      const float2 s2 = half2_bits_to_float2(__byte_perm(gr.x, gr.z, vsel));
      const float2 z2 = half2_bits_to_float2(__byte_perm(gr.y, gr.w, vsel));
      vs[2 * nbk] = s2.x; vs[2 * nbk + 1] = s2.y;
      vz[2 * nbk] = z2.x; vz[2 * nbk + 1] = z2.y;
    }
    if (tok0 + CHUNK > t_end) {   // last chunk of the split: mask tokens past the end
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int tok = tok0 + 32 * warp + 8 * (kb + (k >> 1)) + 2 * t4 + (k & 1);
        if (tok >= t_end) {
          x[k] = kNegInf;
          vs[k] = 0.f;
          vz[k] = 0.f;
        }
      }
    }

    // ---- reference max (per head) and value exponent (per warp)
    float mx = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
    mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, 2));
    mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, 16));
    const bool need = mx > m_ref + kSoftmaxHeadroom;
    const bool m_rebase = __any_sync(kFullMask, need);
    const uint32_t vmb = redux_max_u32(__float_as_uint(
        fmaxf(fmaxf(fabsf(vs[0]), fabsf(vs[1])), fmaxf(fabsf(vs[2]), fabsf(vs[3])))));
    // p' = p v_scale 2^vexp < 2^32 with p <= 2^4 needs v_scale < 2^(28 - vexp)
    int vexp_new = vexp;
    bool v_rebase = false;
    if (vmb != 0u) {
      const int ve = 31 - int(kSoftmaxHeadroom) - exponent_of_bits(vmb);
      if (vexp == kExpUnset || ve < vexp) {
        v_rebase = vexp != kExpUnset;
        vexp_new = max(-126, min(126, ve - kValueHeadroom));
      }
    }
    if (since_flush > 0 && (m_rebase || v_rebase || since_flush >= 1024)) flush();
    vexp = vexp_new;
    if (m_rebase) {
      const float m_new = need ? mx : m_ref;
      const float alpha = need ? fast_exp2(m_ref - m_new) : 1.f;
      l_run *= alpha;
      z_run *= alpha;
      const float aA = __shfl_sync(kFullMask, alpha, srcA);
      const float aB = __shfl_sync(kFullMask, alpha, srcB);
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        master[m][0] *= aA; master[m][1] *= aB; master[m][2] *= aA; master[m][3] *= aB;
      }
      m_ref = m_new;
    }
    const float m_use = (m_ref == kNegInf) ? 0.f : m_ref;
    const float vup = exp2i(vexp == kExpUnset ? 0 : vexp);

    // ---- p' (32-bit fixed point) of the kept tokens; exchange with lane g ^ 4
    uint32_t pm[4], po[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float pe = fast_exp2(x[k] - m_use);
      const float vsup = vs[k] * vup;
      pm[k] = __float2uint_rn(pe * vsup);   // saturates at 2^32 - 1
      // l and z take the weight the token enters the MMA with, p' / (v_scale 2^vexp), so a
      // token whose p' rounds to 0 drops out whole instead of leaving its v_zero behind
      const float pw = vsup > 0.f ? float(pm[k]) * __frcp_rn(vsup) : pe;
      l_run += pw;
      z_run = fmaf(pw, vz[k], z_run);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) po[k] = __shfl_xor_sync(kFullMask, pm[k], 16);
    const uint32_t own_a = byte_sel(pm[0], pm[1], pm[2], pm[3], la);
    const uint32_t oth_a = byte_sel(po[0], po[1], po[2], po[3], la);
    const uint32_t own_b = byte_sel(pm[0], pm[1], pm[2], pm[3], lb);
    const uint32_t oth_b = byte_sel(po[0], po[1], po[2], po[3], lb);
    // k-slots 4 t .. 4 t + 3 = n-blocks 0, 1 (tokens 2t, 2t+1); 16 + 4 t .. = n-blocks 2, 3
    const uint32_t ba0 = upper ? oth_a : own_a, ba1 = upper ? own_a : oth_a;
    const uint32_t bb0 = upper ? oth_b : own_b, bb1 = upper ? own_b : oth_b;

    // ---- O^T += codes^T . p'^T (exact int32); A rows = channels of this lane's V chunk
    if constexpr (INT4) {
      // pair-rows (tokens 2p, 2p+1 per byte): k-slots 4t..4t+3 <- pairs t, 4+t;
      // 16+4t.. <- pairs 8+t, 12+t
      uint4 P4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int pr = 16 * warp + 4 * i + t4;
        P4[i] = *reinterpret_cast<const uint4*>(vbuf + pr * 128 + ((vc ^ (pr & 7)) << 4));
      }
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const uint32_t Pw[4] = {(&P4[0].x)[w], (&P4[1].x)[w], (&P4[2].x)[w], (&P4[3].x)[w]};
        uint32_t Rl[4], Rh[4];   // token-set 1 (pairs 0,1 of Pw) and 2 (pairs 2,3)
#pragma unroll
        for (int sset = 0; sset < 2; ++sset) {
          const uint32_t X = Pw[2 * sset], Y = Pw[2 * sset + 1];
          const uint32_t u = __byte_perm(X, Y, 0x5140), v = __byte_perm(X, Y, 0x7362);
          const uint32_t ul = u & 0x0F0F0F0Fu, uh = (u >> 4) & 0x0F0F0F0Fu;
          const uint32_t vl = v & 0x0F0F0F0Fu, vh = (v >> 4) & 0x0F0F0F0Fu;
          uint32_t* Rr = sset ? Rh : Rl;
          Rr[0] = __byte_perm(ul, uh, 0x5140);
          Rr[1] = __byte_perm(ul, uh, 0x7362);
          Rr[2] = __byte_perm(vl, vh, 0x5140);
          Rr[3] = __byte_perm(vl, vh, 0x7362);
        }
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int m = 2 * w + jj;
          mma_u8u8(ia[m], Rl[2 * jj], Rl[2 * jj + 1], Rh[2 * jj], Rh[2 * jj + 1], ba0, ba1);
          mma_u8u8(ib[m], Rl[2 * jj], Rl[2 * jj + 1], Rh[2 * jj], Rh[2 * jj + 1], bb0, bb1);
        }
      }
    } else {
      uint4 V8[8];   // rows 2t, 2t+1, 8+2t, 9+2t, 16+2t, 17+2t, 24+2t, 25+2t
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int r = 32 * warp + 8 * (i >> 1) + 2 * t4 + (i & 1);
        V8[i] = *reinterpret_cast<const uint4*>(vbuf + r * 128 + ((vc ^ (r & 7)) << 4));
      }
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        uint32_t Rl[4], Rh[4];
#pragma unroll
        for (int sset = 0; sset < 2; ++sset) {
          const uint32_t r0 = (&V8[4 * sset + 0].x)[w], r1 = (&V8[4 * sset + 1].x)[w];
          const uint32_t r2 = (&V8[4 * sset + 2].x)[w], r3 = (&V8[4 * sset + 3].x)[w];
          const uint32_t x01 = __byte_perm(r0, r1, 0x5140), x01b = __byte_perm(r0, r1, 0x7362);
          const uint32_t x23 = __byte_perm(r2, r3, 0x5140), x23b = __byte_perm(r2, r3, 0x7362);
          uint32_t* Rr = sset ? Rh : Rl;
          Rr[0] = __byte_perm(x01, x23, 0x5410);
          Rr[1] = __byte_perm(x01, x23, 0x7632);
          Rr[2] = __byte_perm(x01b, x23b, 0x5410);
          Rr[3] = __byte_perm(x01b, x23b, 0x7632);
        }
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int m = 2 * w + jj;
          mma_u8u8(ia[m], Rl[2 * jj], Rl[2 * jj + 1], Rh[2 * jj], Rh[2 * jj + 1], ba0, ba1);
          mma_u8u8(ib[m], Rl[2 * jj], Rl[2 * jj + 1], Rh[2 * jj], Rh[2 * jj + 1], bb0, bb1);
        }
      }
    }
    ++since_flush;
  }

  if (since_flush > 0) flush();
  // nothing may still be writing this CTA's shared memory when it exits
  cp_async_wait_all();
  if (threadIdx.x == 0) {
    for (int cc = consumed; cc < issued; ++cc)
      if (!mbar_wait(&full[cc % STAGES], uint32_t(cc / STAGES) & 1u))
        flag_device_error(p.status, BPT_DEV_WAIT_TIMEOUT);
  }
  pdl_launch_dependents();
#pragma unroll
  for (int off = 1; off <= 16; off <<= 1) {
    if (off == 4 || off == 8) continue;
    l_run += __shfl_xor_sync(kFullMask, l_run, off);
    z_run += __shfl_xor_sync(kFullMask, z_run, off);
  }
  const float zA = __shfl_sync(kFullMask, z_run, srcA);
  const float zB = __shfl_sync(kFullMask, z_run, srcB);
  // columns 2 t4, 2 t4 + 1 of lanes t4 < 2 hold limbs (0, 2); lane t4 ^ 2 holds (1, 3)
#pragma unroll
  for (int m = 0; m < 8; ++m)
#pragma unroll
    for (int e = 0; e < 4; ++e)
      master[m][e] = fmaf(256.f, __shfl_xor_sync(kFullMask, master[m][e], 2), master[m][e]);
  __syncthreads();   // every warp is done with the ring
  if (t4 == 0 && g < 4) {
    sM[warp * 8 + g] = m_ref;
    sL[warp * 8 + g] = l_run;
  }
  if (t4 < 2) {
    const int colA = 2 * t4, colB = 2 * t4 + 1;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      const int d0 = 16 * vc + 2 * m;   // row g of MMA m; row g + 8 is d0 + 1
      sAcc[(warp * 8 + colA) * D + d0] = master[m][0] + zA;
      sAcc[(warp * 8 + colB) * D + d0] = master[m][1] + zB;
      sAcc[(warp * 8 + colA) * D + d0 + 1] = master[m][2] + zA;
      sAcc[(warp * 8 + colB) * D + d0 + 1] = master[m][3] + zB;
    }
  }
  __syncthreads();
  write_split_state<NW, D>(sM, sL, sAcc, sAcc + NW * 8 * D, p, b, qh0, split, int(threadIdx.x),
                           int(blockDim.x), [] { __syncthreads(); });
}
