// INT8 / INT4 KIVI decode on the 5th-generation tensor cores (tcgen05.mma kind::i8, operands
// in shared memory, exact int32 accumulators in tensor memory). Included by kivi_decode.cu
// inside namespace bpt::kivi; serves group <= 4 and block_size >= 32.
//
// Per 128-token chunk of one (sequence, kv head, split), with 4 warps / 128 threads:
//
//   QK^T   D_qk[token][16 j + 4 h + limb] = sum_k K[token][k] * B_qk[16 j + 4 h + limb][k]
//          M = 128 tokens, N = 16 per page slot j, K = 128 channel bytes (4 MMAs of 32).
//          A = the key code tile exactly as TMA stored it (K-major, 128-byte swizzle). B = the
//          q' limbs: x = round(q * k_scale * 2^Ek) (|x| < 2^30) as four balanced signed
//          bytes, written by the warps in the same K-major swizzled layout.
//          INT4: a packed byte is lo + 16 hi (lo = even channel), so
//            16 sum_k (lo_k x_2k + hi_k x_2k+1) = sum_k byte_k x_2k+1 + lo_k (16 x_2k - x_2k+1)
//          (|x| < 2^26, so 16 x_2k - x_2k+1 fits four limbs). Two MMAs read the packed tile as
//          TMA stored it (64-byte rows, 64-byte swizzle) against B rows of x_2k+1, two read a
//          low-nibble copy (one AND per word, same layout) against rows of 16 x_2k - x_2k+1.
//          S_h = (L0 + 256 L1 + 65536 L2 + 2^24 L3) * 2^-Ek [/ 16, INT4] + sum_d q_d k_zero_d
//   P.V    D_pv[channel][4 h + limb] += sum_t V[t][channel] * P'[t][4 h + limb]
//          M = 128 channels, N = 16, K = 128 tokens. A = the value code tile read MN-major
//          (token rows of 128 channel bytes, as TMA stored it), B = P' rows of 16 bytes: the
//          four little-endian bytes of p'_h = round(p_h * v_scale_t * 2^Ev) < 2^32.
//          INT4: value bytes pack tokens 2p (lo) and 2p + 1 (hi). The compute warps split the
//          tile into a low-nibble copy (even tokens) and a high-nibble copy (odd tokens), same
//          layout; two MMAs read each against the P' rows of its tokens, so every token's p'
//          keeps all 32 bits (a packed-byte form would round the odd tokens' p' to multiples
//          of 16, and in very peaked softmaxes the many small weights near that step are lost).
//          O_h = D_pv combined over limbs * 2^-Ev + sum_t p~_h v_zero_t          (fp32)
//          The normaliser and the zero-point sum use the weight each token actually entered
//          the MMA with, p~ = p' / (v_scale_t 2^Ev) (p itself for a token whose v_scale is 0).
//          With the exact p there, a token whose p' rounds to 0 would still add its v_zero
//          (the minimum of its values) while its v_scale * code part is dropped: a bias that
//          grows with the tokens of a split and that the cancellation between the two sums
//          amplifies wherever the output is small.
//
// Thread t owns token t for the softmax (no redundancy: its 4 heads are 4 registers) and
// channel t when D_pv is read back. The softmax reference m_ref (per head) and the value
// exponent Ev are uniform over the CTA (chunk maxima exchanged through shared memory); D_pv
// is read back into fp32 ("flushed") only when a chunk max exceeds m_ref + 4, when a value
// scale outgrows Ev, or every 256 chunks (int32 headroom).
//
// Warp roles (192 threads): warps 0-3 compute (thread t = token t for the softmax, channel t
// when D_pv is read back), warp 4 loads (TMA: code tiles, k_scale / k_zero rows, and the
// [token][8 heads] v_scale / v_zero rows around this head), warp 5 issues the MMAs. Keys and
// values have separate TMA rings (SK / SV slots); a slot is refilled when the MMA that read it
// committed (tcgen05.commit on the slot's "empty" barrier). Per chunk c the compute warps read
// S(c) from TMEM, quantize q for chunk c + 1 (INT4: and copy its keys' low nibbles) and
// publish it (QK(c + 1) overlaps the rest of the chunk), exchange chunk maxima, then
// (PV(c - 1) done) write P'(c) (INT4: and chunk c's value nibble tiles) for PV(c). INT4 calls
// at large batch and long context use a 2-slot value ring (3 CTAs per SM). Every wait on
// TMA / MMA completion or on another warp is time-bounded; a failed wait raises a shared
// abort flag.

namespace tc {

__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
  return uint64_t((addr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (uint64_t(layout) << 61);
}
constexpr uint32_t kSw128 = 2, kSw64 = 4, kSwNone = 0;

// instruction descriptor of kind::i8 with an s32 accumulator
constexpr uint32_t idesc_i8(int m, int n, bool a_signed, bool b_signed, bool a_mn, bool b_mn) {
  return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | ((b_signed ? 1u : 0u) << 10) |
         ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) | (uint32_t(n >> 3) << 17) |
         (uint32_t(m >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 16 consecutive 32-bit TMEM columns of this warp's 32 lanes
__device__ __forceinline__ void ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];\n\ttcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_free(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// total order on fp32 as unsigned ints (for a max through integer reductions / atomics)
__device__ __forceinline__ uint32_t ord_f32(float x) {
  const uint32_t b = __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float unord_f32(uint32_t u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u);
}
constexpr uint32_t kOrdNegInf = 0x007FFFFFu;   // ord_f32(-inf)

}  // namespace tc

template <int FMT, int SK, int SV>
struct TCfg {
  static constexpr bool INT4 = FMT == BPT_KV_INT4;
  static constexpr int CHUNK = 128;
  static constexpr int CONSUMERS = 128;                     // warps 0-3
  static constexpr int THREADS = CONSUMERS + 64;            // + producer warp 4, MMA warp 5
  static constexpr int K_ROW = INT4 ? 64 : 128;             // key bytes per token in a K slot
  static constexpr int K_TILE = CHUNK * K_ROW;
  static constexpr int V_TILE = (INT4 ? CHUNK / 2 : CHUNK) * 128;
  static constexpr int VS_BYTES = CHUNK * 16;               // v_scale [token][8 heads] fp16
  static constexpr int KX_BYTES = INT4 ? CHUNK * 64 : 0;        // low nibbles of the keys
  static constexpr int VX_BYTES = INT4 ? CHUNK / 2 * 128 : 0;   // low nibbles of the values
  static constexpr int VH_BYTES = VX_BYTES;                     // high nibbles of the values
  static constexpr int P_BYTES = CHUNK * 16;                // P' [token][16 B]
  // K slot = key tile + the chunk's k_scale | k_zero rows (nslot x 512 B); V slot = value
  // tile + v_scale and v_zero of the chunk's tokens for the 8 heads around this one
  __host__ __device__ static constexpr int kslot_bytes(int nslot) {
    return (K_TILE + nslot * 512 + 1023) & ~1023;
  }
  __host__ __device__ static constexpr int vslot_bytes() {
    return (V_TILE + 2 * VS_BYTES + 1023) & ~1023;
  }
  __host__ __device__ static constexpr int bqk_bytes(int nslot) { return nslot * 16 * 128; }
  // misc: qp [chunk parity][slot][head] float2 | xchg [3][8] | reduce [4][8] | tmem slot,
  // abort flags, pv reset flag | mbarriers
  __host__ __device__ static constexpr int misc_bytes(int nslot) {
    return 2 * nslot * 32 + 96 + 128 + 32 + (2 * SK + 2 * SV + 4) * 8;
  }
  __host__ __device__ static constexpr size_t smem_bytes(int nslot) {
    return 1024 + size_t(SK) * kslot_bytes(nslot) + size_t(SV) * vslot_bytes() + KX_BYTES +
           VX_BYTES + VH_BYTES + bqk_bytes(nslot) + P_BYTES + misc_bytes(nslot);
  }
  // TMEM: D_qk at columns [0, 16 nslot), D_pv (16 columns) at pv_col
  __host__ __device__ static constexpr uint32_t pv_col(int nslot) {
    return nslot <= 2 ? 32u : 64u;
  }
  __host__ __device__ static constexpr uint32_t tmem_cols(int nslot) {
    return nslot <= 2 ? 64u : 128u;
  }
};

__device__ __forceinline__ int redux_add_s32(int v) {
  int r;
  asm("redux.sync.add.s32 %0, %1, 0xffffffff;" : "=r"(r) : "r"(v));
  return r;
}
__device__ __forceinline__ uint32_t redux_max_nv(uint32_t v) {
  uint32_t r;
  asm("redux.sync.max.u32 %0, %1, 0xffffffff;" : "=r"(r) : "r"(v));
  return r;
}

template <int FMT, int SK, int SV, int MINB>
__global__ void __launch_bounds__(192, MINB)
kivi_tc_decode_kernel(const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV,
                      const __grid_constant__ CUtensorMap tmKS,
                      const __grid_constant__ CUtensorMap tmKZ,
                      const __grid_constant__ CUtensorMap tmVS,
                      const __grid_constant__ CUtensorMap tmVZ, const KiviParams kp) {
  using C = TCfg<FMT, SK, SV>;
  constexpr int CHUNK = C::CHUNK;
  constexpr bool INT4 = C::INT4;
  const DecodeParams& p = kp.d;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int lR = kp.lbox, R = 1 << lR;          // rows per TMA box (min(block_size, CHUNK))
  const int lbs = kp.lbs, bs = 1 << lbs;
  const int nslot = CHUNK >> lR;
  const int kslot = C::kslot_bytes(nslot);
  constexpr int vslot = C::vslot_bytes();
  uint8_t* kring = smem;
  uint8_t* vring = kring + SK * kslot;
  uint8_t* kx = vring + SV * vslot;                        // INT4 low-nibble key tile
  uint8_t* vx = kx + C::KX_BYTES;                          // INT4 low-nibble value tile
  uint8_t* vh = vx + C::VX_BYTES;                          // INT4 high-nibble value tile
  // q' limb rows (K-major; INT8 128-byte rows, 128-byte swizzle; INT4 two sets of 64-byte
  // rows, 64-byte swizzle: v rows for the packed tile, then x - v rows for the low nibbles)
  uint8_t* bqk = vh + C::VH_BYTES;
  // P' [token][16 B] (INT4: [pair][16 B] of v for the packed tile, then of p' - v)
  uint8_t* pbuf = bqk + C::bqk_bytes(nslot);
  uint8_t* misc = pbuf + C::P_BYTES;
  // {bias', kdown'} per [chunk parity][slot][head]: every compute warp reads all heads' entries
  // of chunk c for its scores while a faster warp may already write chunk c + 1's, so the two
  // chunks use different halves (a warp reaches chunk c + 2 only after the named barrier that
  // every warp passes after its chunk-c score read)
  float2* qp = reinterpret_cast<float2*>(misc);
  const int qp_bytes = 2 * nslot * 32;
  uint32_t* xchg = reinterpret_cast<uint32_t*>(misc + qp_bytes);          // [3][8]
  float* red = reinterpret_cast<float*>(misc + qp_bytes + 96);             // [4 warps][8]
  uint32_t* tslot = reinterpret_cast<uint32_t*>(misc + qp_bytes + 224);
  // abort_flag: any role gave up waiting (producer and MMA warp stop); cabort: written by the
  // compute warps only, read by them right after their named barrier
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + qp_bytes + 228);
  volatile int* cabort = reinterpret_cast<volatile int*>(misc + qp_bytes + 232);
  volatile int* pv_reset = reinterpret_cast<volatile int*>(misc + qp_bytes + 236);
  uint64_t* bars = reinterpret_cast<uint64_t*>(misc + qp_bytes + 256);
  uint64_t* kfull = bars;                 // producer -> consumers / MMA (TMA bytes)
  uint64_t* kempty = kfull + SK;          // QK committed -> producer
  uint64_t* vfull = kempty + SK;          // TMA bytes
  uint64_t* vempty = vfull + SV;          // PV committed -> producer
  uint64_t* opready = vempty + SV;        // consumers wrote q' limbs (+ INT4 keys)
  uint64_t* pready = opready + 1;         // consumers wrote P' (+ INT4 values)
  uint64_t* qk_bar = pready + 1;          // QK committed -> consumers
  uint64_t* pv_bar = qk_bar + 1;          // PV committed -> consumers

  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = p.splits;

  // launched as a programmatic dependent of the previous kernel in the stream: nothing that
  // kernel may write (q, the cache, the table, the lengths, the workspace) is read before
  // it completed
  pdl_wait();
  int n = __ldg(p.seq_lens + b);
  if (n < 0) {
    if (tid == 0) flag_device_error(p.status, BPT_DEV_NEG_SEQ_LEN);
    n = 0;
  }
  const int64_t cap = int64_t(p.max_blocks) * p.block_size;
  if (n > cap) {
    if (tid == 0) flag_device_error(p.status, BPT_DEV_SEQ_TOO_LONG);
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
    for (int idx = tid; idx < p.group * D; idx += blockDim.x) {
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

  // ---------------------------------------------------------------------------- setup
  // q' limb rows start at zero (rows of heads >= group and limb row 3 stay zero)
  for (int i = tid; i < C::bqk_bytes(nslot) / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(bqk)[i] = make_uint4(0u, 0u, 0u, 0u);
  for (int i = tid; i < 2 * nslot * 4; i += blockDim.x) qp[i] = make_float2(0.f, 0.f);
  if (tid < 24) xchg[tid] = (tid & 7) < 4 ? tc::kOrdNegInf : 0u;
  if (tid == 0) {
    *abort_flag = 0;
    *cabort = 0;
    *pv_reset = 0;
    for (int s = 0; s < SK; ++s) {
      mbar_init(&kfull[s], 1);
      mbar_init(&kempty[s], 1);
    }
    for (int s = 0; s < SV; ++s) {
      mbar_init(&vfull[s], 1);
      mbar_init(&vempty[s], 1);
    }
    mbar_init(opready, C::CONSUMERS);
    mbar_init(pready, C::CONSUMERS);
    mbar_init(qk_bar, 1);
    mbar_init(pv_bar, 1);
    fence_mbar_init();
  }
  const uint32_t ncols = C::tmem_cols(nslot);
  if (warp == 0) tc::tmem_alloc(tslot, ncols);
  tc::fence_async_smem();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  // the merge grid may start launching now; it waits for this whole grid to complete
  pdl_launch_dependents();
  const uint32_t tmem = *tslot;
  const uint32_t pv_col = C::pv_col(nslot);
  int qk_issued = 0, pv_issued = 0;   // MMA warp

  if (warp == 4) {
    // ================================================================ producer warp
    const int32_t* bt = p.block_table + int64_t(b) * p.bt_sb;
    const int last_page = (t_end - 1) >> lbs;
    // block-table windows of the key and value streams: lane i holds entry base + i
    int kwin_base = t_begin >> lbs, vwin_base = kwin_base;
    int kwin = (kwin_base + lane <= last_page) ? __ldg(bt + kwin_base + lane) : 0;
    int vwin = kwin;
    const uint64_t pol = l2_evict_first_policy();
    if (lane == 0) {
      prefetch_tensormap(&tmK);
      prefetch_tensormap(&tmV);
      prefetch_tensormap(&tmKS);
      prefetch_tensormap(&tmKZ);
      prefetch_tensormap(&tmVS);
      prefetch_tensormap(&tmVZ);
    }
    auto page_of = [&](int t, int& wbase, int& w, int tok0, int tok_last) {
      if ((tok_last >> lbs) - wbase >= 32) {   // re-anchor the window at the chunk's first page
        wbase = tok0 >> lbs;
        w = (wbase + lane <= last_page) ? __ldg(bt + wbase + lane) : 0;
      }
      return __shfl_sync(kFullMask, w, (min(t, tok_last) >> lbs) - wbase);
    };
    auto wait_slot = [&](uint64_t* bar, int phase) {
      bool ok = (lane == 0) ? mbar_wait(bar, uint32_t(phase) & 1u) : true;
      ok = __shfl_sync(kFullMask, ok, 0);
      if (!ok && lane == 0) *abort_flag = 1;
      return ok;
    };
    for (int cc = 0; cc < nchunks; ++cc) {
      if (*abort_flag) break;
      const int tok0 = (u0 + cc) * CHUNK;
      const int tok_last = min(tok0 + CHUNK, t_end) - 1;
      const int nbox = (tok_last - tok0 + R) >> lR;
      // keys: the slot's previous chunk committed its QK
      const int ks = cc % SK;
      if (cc >= SK && !wait_slot(&kempty[ks], cc / SK - 1)) break;
      {
        uint8_t* kb = kring + ks * kslot;
        uint8_t* kpar = kb + C::K_TILE;
        if (lane == 0)
          mbar_arrive_expect_tx(&kfull[ks], uint32_t(nbox) * (uint32_t(R) * C::K_ROW + 512u));
        for (int j = 0; j < nbox; ++j) {
          const int t = tok0 + (j << lR);
          int phys = page_of(t, kwin_base, kwin, tok0, tok_last);
          if (lane == 0) {
            if (phys < 0 || int64_t(phys) >= p.num_blocks) {
              flag_device_error(p.status, BPT_DEV_BAD_BLOCK_ID);
              phys = 0;
            }
            const int row = t & (bs - 1);
            tma_load_4d(kb + j * R * C::K_ROW, &tmK, &kfull[ks], 0, p.k_c1 ? row : h,
                        p.k_c1 ? h : row, phys, pol);
            tma_load_3d(kpar + j * 512, &tmKS, &kfull[ks], 0, h, phys);
            tma_load_3d(kpar + j * 512 + 256, &tmKZ, &kfull[ks], 0, h, phys);
          }
        }
      }
      // values: the slot's previous chunk committed its PV
      const int vs_ = cc % SV;
      if (cc >= SV && !wait_slot(&vempty[vs_], cc / SV - 1)) break;
      {
        uint8_t* vb = vring + vs_ * vslot;
        uint8_t* vsc = vb + C::V_TILE;
        const uint32_t vbox = uint32_t(INT4 ? R / 2 : R) * 128u;
        if (lane == 0)
          mbar_arrive_expect_tx(&vfull[vs_], uint32_t(nbox) * (vbox + uint32_t(R) * 32u));
        for (int j = 0; j < nbox; ++j) {
          const int t = tok0 + (j << lR);
          int phys = page_of(t, vwin_base, vwin, tok0, tok_last);
          if (lane == 0) {
            if (phys < 0 || int64_t(phys) >= p.num_blocks) phys = 0;
            const int row = t & (bs - 1);
            const int vrow = INT4 ? row / 2 : row;
            tma_load_4d(vb + j * (INT4 ? R / 2 : R) * 128, &tmV, &vfull[vs_], 0,
                        p.v_c1 ? vrow : h, p.v_c1 ? h : vrow, phys, pol);
            // v_scale / v_zero [token][8 heads] of the box's tokens (3-D map {H, bs, blocks})
            tma_load_3d(vsc + (j << lR) * 16, &tmVS, &vfull[vs_], h & ~7, row, phys);
            tma_load_3d(vsc + C::VS_BYTES + (j << lR) * 16, &tmVZ, &vfull[vs_], h & ~7, row,
                        phys);
          }
        }
      }
    }
    if (*abort_flag && lane == 0) {   // loads of the last chunks may still be in flight
      for (int s = 0; s < SK; ++s) mbar_wait(&kfull[s], 0), mbar_wait(&kfull[s], 1);
      for (int s = 0; s < SV; ++s) mbar_wait(&vfull[s], 0), mbar_wait(&vfull[s], 1);
    }
  } else if (warp == 5) {
    // ================================================================ MMA warp (lane 0)
    if (lane == 0) {
      const uint32_t id_qk = tc::idesc_i8(128, 16 * nslot, false, true, false, false);
      const uint32_t id_pv = tc::idesc_i8(128, 16, false, false, true, true);
      auto issue_pv = [&](int cc) {
        if (!mbar_wait(pready, uint32_t(cc) & 1u)) {
          *abort_flag = 1;
          return false;
        }
        tc::fence_after();
        const uint32_t a0 = smem_u32(vring + (cc % SV) * vslot), b0 = smem_u32(pbuf);
        const uint32_t acc0 = *pv_reset ? 0u : 1u;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          // INT4: k = 0, 1 the high nibbles (odd tokens), k = 2, 3 the low nibbles (even
          // tokens), 32 pair rows each, against the P' rows of those tokens
          const uint32_t a = INT4 ? (k < 2 ? smem_u32(vh) : smem_u32(vx)) + 4096 * (k & 1)
                                  : a0 + 4096 * k;
          tc::mma_i8(tmem + pv_col, tc::smem_desc(a, 16384, 1024, tc::kSw128),
                     tc::smem_desc(b0 + 512 * k, 128, 256, tc::kSwNone), id_pv,
                     k == 0 ? acc0 : 1u);
        }
        tc::commit(pv_bar);
        tc::commit(&vempty[cc % SV]);
        ++pv_issued;
        return true;
      };
      for (int c = 0; c < nchunks; ++c) {
        if (*abort_flag) break;
        if (!mbar_wait(opready, uint32_t(c) & 1u)) {
          *abort_flag = 1;
          break;
        }
        tc::fence_after();
        const uint32_t a0 = smem_u32(kring + (c % SK) * kslot);
        const uint32_t b0 = smem_u32(bqk);
        if constexpr (INT4) {   // packed key bytes x v rows, then low nibbles x (x - v) rows
          const uint32_t a1 = smem_u32(kx), b1 = b0 + uint32_t(nslot) * 16u * 64u;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc::mma_i8(tmem, tc::smem_desc((k < 2 ? a0 : a1) + 32 * (k & 1), 16, 512, tc::kSw64),
                       tc::smem_desc((k < 2 ? b0 : b1) + 32 * (k & 1), 16, 512, tc::kSw64),
                       id_qk, k > 0);
        } else {
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc::mma_i8(tmem, tc::smem_desc(a0 + 32 * k, 16, 1024, tc::kSw128),
                       tc::smem_desc(b0 + 32 * k, 16, 1024, tc::kSw128), id_qk, k > 0);
        }
        tc::commit(qk_bar);
        tc::commit(&kempty[c % SK]);
        ++qk_issued;
        if (c >= 1 && !issue_pv(c - 1)) break;
      }
      if (!*abort_flag && pv_issued == nchunks - 1) issue_pv(nchunks - 1);
      // nothing may still be running when the CTA releases its tensor memory
      if (qk_issued > 0) mbar_wait(qk_bar, uint32_t(qk_issued - 1) & 1u);
      if (pv_issued > 0) mbar_wait(pv_bar, uint32_t(pv_issued - 1) & 1u);
    }
    __syncwarp();
  } else {
    // ================================================================ consumer warps 0-3
    // q of this warp's head for the 4 channels behind B_qk bytes 4 lane .. 4 lane + 3
    // (INT8: channel k = byte k; INT4: byte k < 64 is channel 2k, byte k >= 64 is 2(k-64)+1)
    const bool prep_warp = warp < p.group;
    const int pch0 = INT4 ? 8 * (lane & 15) : 4 * lane;
    const uint32_t psel = (INT4 && lane >= 16) ? 0x7632u : 0x5410u;
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
    const uint32_t tmem_warp = tmem + (uint32_t(32 * warp) << 16);

    // the q' limbs of one page slot: 4 channels per lane, this warp's head
    struct Limbs {
      uint32_t l0, l1, l2, l3;   // l3: INT4 only
      float bias, kdown;
    };
    auto quantize = [&](const __half* kpar_j) -> Limbs {
      const __half* ks = kpar_j + pch0;
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
      const float qs0 = qv[0] * sa.x, qs1 = qv[1] * sa.y, qs2 = qv[2] * sb.x, qs3 = qv[3] * sb.y;
      const float bp = fmaf(qv[3], zb.y, fmaf(qv[2], zb.x, fmaf(qv[1], za.y, qv[0] * za.x)));
      const float lm = fmaxf(fmaxf(fabsf(qs0), fabsf(qs1)), fmaxf(fabsf(qs2), fabsf(qs3)));
      const uint32_t qm = redux_max_nv(__float_as_uint(lm));
      // bias = sum over the warp of bp, as an exact integer sum in 2^-eb fixed point
      const uint32_t bm = redux_max_nv(__float_as_uint(fabsf(bp)));
      const int eb = bm ? min(126, 24 - exponent_of_bits(bm)) : 0;
      const float bsum = float(redux_add_s32(__float2int_rn(bp * exp2i(eb)))) * exp2i(-eb);
      // Four balanced limbs. INT8: |q' 2^ek| < 2^30 (a product of two fp16 values has 22
      // significant bits, so the largest channels' x is exact). Every token of a page shares
      // the rounding of x, weighted by its codes (about half their range on average), so x
      // carries all the bits the limbs hold: a coarser x shifts whole pages' scores together.
      // INT4: |q' 2^ek| < 2^26, so b = 16 x_even - x_odd below fits the four limbs.
      const int ek = qm ? min(122, (INT4 ? 25 : 29) - exponent_of_bits(qm)) : 0;
      const float kup = exp2i(ek);
      int x0 = __float2int_rn(qs0 * kup), x1 = __float2int_rn(qs1 * kup);
      int x2 = __float2int_rn(qs2 * kup), x3 = __float2int_rn(qs3 * kup);
      if constexpr (INT4) {
        // A packed byte is lo + 16 hi (lo = even channel). The packed tile meets a = x_odd
        // (lanes 16-31) and the low-nibble copy meets b = 16 x_even - x_odd (lanes 0-15, the
        // partner lane holds x_odd of the same pairs): sum byte a + lo b = 16 sum (lo x_even
        // + hi x_odd), every channel at full precision; kdown carries the 2^-4.
        const int w0 = __shfl_xor_sync(kFullMask, x0, 16), w1 = __shfl_xor_sync(kFullMask, x1, 16);
        const int w2 = __shfl_xor_sync(kFullMask, x2, 16), w3 = __shfl_xor_sync(kFullMask, x3, 16);
        const bool lo_lane = lane < 16;
        x0 = lo_lane ? 16 * x0 - w0 : x0;
        x1 = lo_lane ? 16 * x1 - w1 : x1;
        x2 = lo_lane ? 16 * x2 - w2 : x2;
        x3 = lo_lane ? 16 * x3 - w3 : x3;
      }
      // x + 0x80808080 = sum_k (l_k + 128) 256^k: byte k ^ 0x80 is the signed limb l_k
      constexpr uint32_t kBias = 0x80808080u;
      const uint32_t y0 = uint32_t(x0) + kBias, y1 = uint32_t(x1) + kBias;
      const uint32_t y2 = uint32_t(x2) + kBias, y3 = uint32_t(x3) + kBias;
      return Limbs{byte_sel(y0, y1, y2, y3, 0u) ^ 0x80808080u,
                   byte_sel(y0, y1, y2, y3, 1u) ^ 0x80808080u,
                   byte_sel(y0, y1, y2, y3, 2u) ^ 0x80808080u,
                   byte_sel(y0, y1, y2, y3, 3u) ^ 0x80808080u, bsum * p.scale_log2,
                   exp2i(-ek - (INT4 ? 4 : 0)) * p.scale_log2};
    };
    auto store_limbs = [&](int j, int cc, const Limbs& L) {
      const int row0 = 16 * j + 4 * warp;
      const uint32_t cofs = (uint32_t(lane) & 3u) << 2;
      const uint32_t lv[4] = {L.l0, L.l1, L.l2, L.l3};
#pragma unroll
      for (int limb = 0; limb < 4; ++limb) {
        const int row = row0 + limb;
        if constexpr (INT4) {   // pair bytes 4 (lane & 15) .. + 3 of a 64-byte swizzled row
          uint8_t* set = bqk + (lane < 16 ? nslot * 16 * 64 : 0);
          const uint32_t chunk = (uint32_t(lane) & 15u) >> 2;
          *reinterpret_cast<uint32_t*>(set + row * 64 + ((chunk ^ uint32_t((row >> 1) & 3)) << 4) +
                                       cofs) = lv[limb];
        } else {
          *reinterpret_cast<uint32_t*>(bqk + row * 128 +
                                       ((uint32_t((lane >> 2) ^ (row & 7))) << 4) + cofs) =
              lv[limb];
        }
      }
      if (lane == 0) qp[((cc & 1) * nslot + j) * 4 + warp] = make_float2(L.bias, L.kdown);
    };
    // low nibbles of a packed INT4 tile, word for word (the copy keeps the tile's layout)
    auto low_nibbles = [&](const uint8_t* src, uint8_t* dst, int bytes) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int o = 16 * (tid + i * C::CONSUMERS);
        if (o < bytes) {
          const uint4 w = *reinterpret_cast<const uint4*>(src + o);
          *reinterpret_cast<uint4*>(dst + o) = make_uint4(
              w.x & 0x0F0F0F0Fu, w.y & 0x0F0F0F0Fu, w.z & 0x0F0F0F0Fu, w.w & 0x0F0F0F0Fu);
        }
      }
    };
    // low and high nibbles of a packed INT4 value tile into two tiles of the same layout
    auto split_nibbles = [&](const uint8_t* src, uint8_t* lo, uint8_t* hi, int bytes) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int o = 16 * (tid + i * C::CONSUMERS);
        if (o < bytes) {
          const uint4 w = *reinterpret_cast<const uint4*>(src + o);
          *reinterpret_cast<uint4*>(lo + o) = make_uint4(
              w.x & 0x0F0F0F0Fu, w.y & 0x0F0F0F0Fu, w.z & 0x0F0F0F0Fu, w.w & 0x0F0F0F0Fu);
          *reinterpret_cast<uint4*>(hi + o) =
              make_uint4((w.x >> 4) & 0x0F0F0F0Fu, (w.y >> 4) & 0x0F0F0F0Fu,
                         (w.z >> 4) & 0x0F0F0F0Fu, (w.w >> 4) & 0x0F0F0F0Fu);
        }
      }
    };
    // q' limbs of chunk cc against its k_scale rows (INT4: and the keys' low-nibble tile)
    auto prep = [&](int cc) {
      const uint8_t* kb = kring + (cc % SK) * kslot;
      const __half* kpar = reinterpret_cast<const __half*>(kb + C::K_TILE);
      const int tok0 = (u0 + cc) * CHUNK;
      const int nbox = min(nslot, (t_end - tok0 + R - 1) >> lR);
      if constexpr (INT4) low_nibbles(kb, kx, C::KX_BYTES);
      if (!prep_warp) return;
      for (int j = 0; j < nbox; j += 2) {   // two page slots at a time (independent chains)
        const int j2 = min(j + 1, nbox - 1);
        const Limbs a = quantize(kpar + j * 256);
        const Limbs c2 = quantize(kpar + j2 * 256);
        store_limbs(j, cc, a);
        if (j2 != j) store_limbs(j2, cc, c2);
      }
    };

    const int hl = h & 7;   // this head within the 8-head v_scale / v_zero rows
    float m_ref[4] = {kNegInf, kNegInf, kNegInf, kNegInf};
    float l_run[4] = {0.f, 0.f, 0.f, 0.f}, z_run[4] = {0.f, 0.f, 0.f, 0.f};
    float master[4] = {0.f, 0.f, 0.f, 0.f};   // channel tid, heads 0-3 (relative to m_ref)
    int vexp = kExpUnset;
    int since_flush = 0;   // PV chunks accumulated in D_pv since it was last read back
    bool reset_pv = true;  // next PV MMA overwrites D_pv
    auto flush = [&]() {   // D_pv (this thread = channel tid) -> master
      uint32_t r[16];
      tc::ld16(tmem_warp + pv_col, r);
      const float vdown = exp2i(vexp == kExpUnset ? 0 : -vexp);
#pragma unroll
      for (int hh = 0; hh < 4; ++hh) {
        const float v = fmaf(16777216.f, float(int(r[4 * hh + 3])),
                             fmaf(65536.f, float(int(r[4 * hh + 2])),
                                  fmaf(256.f, float(int(r[4 * hh + 1])), float(int(r[4 * hh])))));
        master[hh] = fmaf(v, vdown, master[hh]);
      }
      since_flush = 0;
      reset_pv = true;
    };
    auto wait_or_abort = [&](uint64_t* bar, int phase) {
      if (!__all_sync(kFullMask, mbar_wait(bar, uint32_t(phase) & 1u)) && lane == 0) {
        *cabort = 1;
        *abort_flag = 1;
      }
    };
    auto consumers_sync = [&]() { named_barrier_sync(1, C::CONSUMERS); };

    // chunk 0's operands
    wait_or_abort(&kfull[0], 0);
    if (!*cabort) prep(0);
    tc::fence_async_smem();
    mbar_arrive(opready);

    for (int c = 0; c < nchunks; ++c) {
      // ---- scores of token tid (QK(c) reads the q' limbs and keys written last iteration)
      wait_or_abort(qk_bar, c);
      wait_or_abort(&vfull[c % SV], c / SV);
      const int tok0 = (u0 + c) * CHUNK;
      const uint8_t* vb = vring + (c % SV) * vslot;
      const __half* vsc = reinterpret_cast<const __half*>(vb + C::V_TILE);
      float x[4] = {kNegInf, kNegInf, kNegInf, kNegInf};
      float vs = 0.f, vz = 0.f;
      uint32_t* xc = xchg + (c % 3) * 8;
      if (!*cabort) {
        tc::fence_after();
        const int slot = (32 * warp) >> lR;      // warp-uniform (box rows >= 32)
        uint32_t r[16];
        tc::ld16(tmem_warp + 16u * uint32_t(slot), r);
        const bool valid = tok0 + tid < t_end;
        const float2* qpb = qp + ((c & 1) * nslot + slot) * 4;
#pragma unroll
        for (int hh = 0; hh < 4; ++hh) {
          float s = fmaf(65536.f, float(int(r[4 * hh + 2])),
                         fmaf(256.f, float(int(r[4 * hh + 1])), float(int(r[4 * hh]))));
          s = fmaf(16777216.f, float(int(r[4 * hh + 3])), s);
          const float2 q2 = qpb[hh];
          x[hh] = valid ? fmaf(s, q2.y, q2.x) : kNegInf;
        }
        if (valid) {
          vs = __half2float(vsc[tid * 8 + hl]);
          vz = __half2float(vsc[C::VS_BYTES / 2 + tid * 8 + hl]);
        }
        uint32_t m[5];
#pragma unroll
        for (int hh = 0; hh < 4; ++hh) m[hh] = redux_max_nv(tc::ord_f32(x[hh]));
        m[4] = redux_max_nv(__float_as_uint(fabsf(vs)));
        if (lane == 0) {
#pragma unroll
          for (int i = 0; i < 5; ++i) atomicMax(xc + i, m[i]);
        }
      }
      // ---- next chunk's operands: its key slot is loaded; QK(c) is done with the buffers
      if (c + 1 < nchunks) {
        wait_or_abort(&kfull[(c + 1) % SK], (c + 1) / SK);
        if (!*cabort) prep(c + 1);
        tc::fence_async_smem();
        tc::fence_before();
        mbar_arrive(opready);
      }
      consumers_sync();
      if (*cabort) break;
      float mx[4];
#pragma unroll
      for (int hh = 0; hh < 4; ++hh) mx[hh] = tc::unord_f32(xc[hh]);
      const uint32_t vmb = xc[4];
      if (tid < 8) xchg[((c + 2) % 3) * 8 + tid] = tid < 4 ? tc::kOrdNegInf : 0u;

      // ---- PV of chunk c - 1 done: P' / the values' nibble tiles are free, D_pv is final
      if (c >= 1) wait_or_abort(pv_bar, c - 1);
      if constexpr (INT4) split_nibbles(vb, vx, vh, C::VX_BYTES);

      // ---- reference max / value exponent (uniform over the CTA); read D_pv back if needed
      bool need[4], m_rebase = false;
#pragma unroll
      for (int hh = 0; hh < 4; ++hh) {
        need[hh] = mx[hh] > m_ref[hh] + kSoftmaxHeadroom;
        m_rebase |= need[hh];
      }
      int vexp_new = vexp;
      bool v_rebase = false;
      if (vmb != 0u) {
        const int ve = 31 - int(kSoftmaxHeadroom) - exponent_of_bits(vmb);
        if (vexp == kExpUnset || ve < vexp) {
          v_rebase = vexp != kExpUnset;
          vexp_new = max(-126, min(126, ve - kValueHeadroom));
        }
      }
      if (since_flush > 0 && (m_rebase || v_rebase || since_flush >= 256) && !*cabort) {
        tc::fence_after();
        flush();
      }
      vexp = vexp_new;
      if (m_rebase) {
#pragma unroll
        for (int hh = 0; hh < 4; ++hh) {
          if (need[hh]) {
            const float alpha = fast_exp2(m_ref[hh] - mx[hh]);
            master[hh] *= alpha;
            l_run[hh] *= alpha;
            z_run[hh] *= alpha;
            m_ref[hh] = mx[hh];
          }
        }
      }
      const float vsup = vs * exp2i(vexp == kExpUnset ? 0 : vexp);
      // 1 / (v_scale 2^Ev): turns a token's p' back into the weight the MMA gives it
      const float vinv = vsup > 0.f ? __frcp_rn(vsup) : 0.f;
      uint32_t pq[4];
#pragma unroll
      for (int hh = 0; hh < 4; ++hh) {
        const float pe = fast_exp2(x[hh] - (m_ref[hh] == kNegInf ? 0.f : m_ref[hh]));
        pq[hh] = __float2uint_rn(pe * vsup);   // saturates at 2^32 - 1
        // the token's weight as the MMA sees it, so l and z stay consistent with D_pv
        const float pw = vsup > 0.f ? float(pq[hh]) * vinv : pe;
        l_run[hh] += pw;
        z_run[hh] = fmaf(pw, vz, z_run[hh]);
      }
      // INT4: odd tokens' P' rows first (they meet the high-nibble tile), then even tokens'
      uint8_t* prow = INT4 ? pbuf + ((tid & 1) ? 0 : 1024) + 16 * (tid >> 1) : pbuf + 16 * tid;
      *reinterpret_cast<uint4*>(prow) = make_uint4(pq[0], pq[1], pq[2], pq[3]);
      if (tid == 0) *pv_reset = reset_pv ? 1 : 0;
      tc::fence_async_smem();
      tc::fence_before();
      mbar_arrive(pready);
      reset_pv = false;
      ++since_flush;
    }

    // ---- last PV done: read D_pv back
    if (!*cabort) {
      wait_or_abort(pv_bar, nchunks - 1);
      if (!*cabort) {
        tc::fence_after();
        flush();
      }
    }
    // l and z of every head, summed over the CTA's tokens
#pragma unroll
    for (int hh = 0; hh < 4; ++hh) {
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
        l_run[hh] += __shfl_xor_sync(kFullMask, l_run[hh], off);
        z_run[hh] += __shfl_xor_sync(kFullMask, z_run[hh], off);
      }
    }
    if (lane == 0) {
#pragma unroll
      for (int hh = 0; hh < 4; ++hh) {
        red[warp * 8 + hh] = l_run[hh];
        red[warp * 8 + 4 + hh] = z_run[hh];
      }
    }
    consumers_sync();
    const bool ok = !*cabort && !*abort_flag;
    for (int hh = 0; hh < p.group; ++hh) {
      const float L = red[hh] + red[8 + hh] + red[16 + hh] + red[24 + hh];
      const float Z = red[4 + hh] + red[12 + hh] + red[20 + hh] + red[28 + hh];
      const float o = (ok && L > 0.f) ? (master[hh] + Z) / L : 0.f;
      if (S == 1 && p.final_out) {
        p.out[int64_t(b) * p.o_sb + int64_t(qh0 + hh) * p.o_sh + tid] = __float2half_rn(o);
      } else {
        const int64_t row = (int64_t(b) * p.q_heads + qh0 + hh) * S + split;
        p.o_part[row * D + tid] = o;
        if (tid == 0) p.lse[row] = (ok && L > 0.f) ? m_ref[hh] + __log2f(L) : kNegInf;
      }
    }
    if (!ok && tid == 0) flag_device_error(p.status, BPT_DEV_WAIT_TIMEOUT);
  }

  // ---------------------------------------------------------------------------- teardown
  pdl_launch_dependents();
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_free(tmem, ncols);
}
