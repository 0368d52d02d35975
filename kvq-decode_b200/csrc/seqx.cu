// Sequence-sharded decode across the GPUs of one node: the split merge, the cross-GPU exchange
// of the per-(sequence, q head) softmax states and the merge of the ranks' states, fused into
// one kernel that stores into the peers' memory over NVLink. No reference counterpart (the
// reference is single-GPU); the merge formula is the reference's split merge
// (src/bpt/triton_fp16.py:152-162) in log2 units.
//
// Every rank owns one receive buffer, allocated here and mapped into the other ranks with CUDA
// IPC (plain peer mappings; no multicast object). Layout, in 8-byte words:
//   states [2][world][B * Hq][slot] set (epoch & 1); slot (r, item) is written by rank r:
//                                   o[0, D) then lse2,
//                                   each value in its own word as {fp32 bits, epoch}; a slot is
//                                   a whole number of 128-byte lines
//   ctl    [32]                     ctl[0] (u32): epoch of the last finished call,
//                                   ctl[1] (u32): CTAs done with the current call
//
// Exchange protocol (the "low-latency" pattern of flag-carrying words): a value and the call's
// epoch travel in ONE naturally aligned 8-byte store, which lands atomically, so a reader that
// sees the current epoch in a word also sees that word's value: no fence and no separate flag
// are needed, and each thread waits only for the words it reads itself. Consecutive calls
// alternate between two slot sets: a rank can only start call i + 2 after every peer finished
// call i (it needs their call-(i + 1) states, which they write after finishing call i), so a
// set is never overwritten while a peer may still read it.
//
// Per call, every CTA takes items (b, hq) = blockIdx.x, blockIdx.x + gridDim.x, ...:
//   phase 1: merge this rank's S split rows of the item into one state (o, lse2) and store it,
//            epoch-tagged, into slot (rank, item) of every rank's buffer (peer stores over
//            NVLink);
//   phase 2: each thread polls (time-bounded) the words it needs in the local buffer until they
//            carry the epoch -- one lse2 per rank, then its channels of every rank's o -- and the
//            CTA merges the world states into the fp16 output.
// A CTA finishes all its phase-1 stores before it waits, and the grid never exceeds what is
// resident at once, so no rank can wait on a CTA that cannot start. The epoch is
// ctl[0] + 1; the last CTA to finish bumps ctl[0], so consecutive calls (also graph replays)
// use fresh epochs and the buffer never needs clearing. A wait that runs out of its budget sets
// BPT_DEV_WAIT_TIMEOUT in the status word and the kernel continues (the output is then wrong,
// the GPU stays usable).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <string.h>

#include "common.cuh"
#include "decode_common.h"

namespace bpt {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kThreads = 128;
constexpr float kNegInf = -INFINITY;

struct RankBufs {
  float* p[kMaxRanks];
};

// 8-byte words per (rank, item) slot: D + 1 values, rounded up to 16 words (128 bytes)
__host__ __device__ constexpr size_t slot_words(int D) {
  return (size_t(D) + 1 + 15) & ~size_t(15);
}

__device__ __forceinline__ void st_tagged(uint64_t* p, float v, unsigned epoch) {
  const uint64_t w = (uint64_t(epoch) << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ uint64_t ld_tagged(const uint64_t* p) {
  uint64_t w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}

// Wait (time-bounded) until word p carries `epoch`; returns its value (0 after a timeout; once
// a thread timed out it stops waiting for later words).
__device__ __forceinline__ float wait_tagged(const uint64_t* p, unsigned epoch, uint64_t budget_ns,
                                             int* timed_out) {
  uint64_t w = ld_tagged(p);
  if (unsigned(w >> 32) != epoch) {
    if (*timed_out) return 0.f;
    const uint64_t t0 = global_timer_ns();
    do {
      if (global_timer_ns() - t0 > budget_ns) {
        *timed_out = 1;
        return 0.f;
      }
      w = ld_tagged(p);
    } while (unsigned(w >> 32) != epoch);
  }
  return __uint_as_float(unsigned(w));
}

__global__ void __launch_bounds__(kThreads)
seq_exchange_kernel(const float* __restrict__ o_part, const float* __restrict__ lse, int batch,
                    int q_heads, int splits, int D, RankBufs bufs, int world, int rank,
                    __half* __restrict__ out, int64_t o_sb, int64_t o_sh, unsigned* status,
                    uint64_t budget_ns) {
  extern __shared__ float w_s[];      // [splits]
  __shared__ float red[4];
  __shared__ float4 part[4][64];      // per-warp sums, D <= 256
  __shared__ float st_lse[kMaxRanks];
  __shared__ int timed_out;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int items = batch * q_heads;
  const int nd4 = D >> 2;
  uint64_t* const* slots = reinterpret_cast<uint64_t* const*>(bufs.p);
  const size_t set_words = size_t(world) * items * slot_words(D);
  unsigned* ctl = reinterpret_cast<unsigned*>(slots[rank] + 2 * set_words);
  pdl_wait();
  const unsigned epoch = *reinterpret_cast<volatile unsigned*>(ctl) + 1u;
  const size_t set0 = (epoch & 1u) * set_words;   // this call's slot set
  uint64_t* mine = slots[rank] + set0;
  int my_timeout = 0;
  if (tid == 0) timed_out = 0;

  // ---- phase 1: local split merge, epoch-tagged stores into every rank's slot (rank, item)
  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    const float* l = lse + int64_t(it) * splits;
    const float* o = o_part + int64_t(it) * splits * D;
    float m = kNegInf;
    for (int s = tid; s < splits; s += kThreads) m = fmaxf(m, l[s]);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(kFullMask, m, off));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    const float M = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    __syncthreads();
    float wsum = 0.f;
    for (int s = tid; s < splits; s += kThreads) {
      const float w = (M == kNegInf) ? 0.f : fast_exp2(l[s] - M);
      w_s[s] = w;
      wsum += w;
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) wsum += __shfl_xor_sync(kFullMask, wsum, off);
    if (lane == 0) red[warp] = wsum;
    __syncthreads();
    const float W = red[0] + red[1] + red[2] + red[3];
    for (int c = lane; c < nd4; c += 32) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int s = warp; s < splits; s += 4) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(o + int64_t(s) * D) + c);
        const float w = w_s[s];
        const bool on = w != 0.f;
        acc.x = fmaf(w, on ? v.x : 0.f, acc.x);
        acc.y = fmaf(w, on ? v.y : 0.f, acc.y);
        acc.z = fmaf(w, on ? v.z : 0.f, acc.z);
        acc.w = fmaf(w, on ? v.w : 0.f, acc.w);
      }
      part[warp][c] = acc;
    }
    __syncthreads();
    const float invW = W > 0.f ? 1.f / W : 0.f;
    const float* pf = reinterpret_cast<const float*>(&part[0][0]);
    const size_t base = set0 + (size_t(rank) * items + it) * slot_words(D);
    for (int d = tid; d < D; d += kThreads) {
      // channel d of the 4 warp sums: part[w][d / 4].{x,y,z,w}[d % 4]
      const float v = ((pf[d] + pf[256 + d]) + (pf[512 + d] + pf[768 + d])) * invW;
      for (int r = 0; r < world; ++r) st_tagged(slots[r] + base + d, v, epoch);
    }
    if (tid < world)
      st_tagged(slots[tid] + base + D, W > 0.f ? M + __log2f(W) : kNegInf, epoch);
    __syncthreads();   // part / w_s / red are reused by the next item
  }

  // ---- phase 2: wait for every rank's state of my items, merge them
  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    if (tid < world)
      st_lse[tid] = wait_tagged(mine + (size_t(tid) * items + it) * slot_words(D) + D, epoch,
                                budget_ns, &my_timeout);
    __syncthreads();
    float M = kNegInf;
    for (int r = 0; r < world; ++r) M = fmaxf(M, st_lse[r]);
    float wr[kMaxRanks];
    float W = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      wr[r] = (r < world && M != kNegInf) ? fast_exp2(st_lse[r] - M) : 0.f;
      W += wr[r];
    }
    const float invW = W > 0.f ? 1.f / W : 0.f;
    const int b = it / q_heads, hq = it % q_heads;
    for (int d = tid; d < D; d += kThreads) {
      float acc = 0.f;
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r) {
        if (r < world) {
          // every rank's word is awaited (even at weight 0) so no store of this call is
          // still in flight into the buffer when the next call starts
          const float v = wait_tagged(mine + (size_t(r) * items + it) * slot_words(D) + d,
                                      epoch, budget_ns, &my_timeout);
          if (wr[r] != 0.f) acc = fmaf(wr[r], v, acc);
        }
      }
      out[int64_t(b) * o_sb + int64_t(hq) * o_sh + d] = __float2half_rn(acc * invW);
    }
    __syncthreads();   // st_lse is reused by the next item
  }

  // ---- the last CTA to finish publishes this call's epoch
  if (my_timeout) timed_out = 1;
  __syncthreads();
  if (tid == 0) {
    if (timed_out) flag_device_error(status, BPT_DEV_WAIT_TIMEOUT);
    __threadfence();
    const unsigned done = atomicAdd(&ctl[1], 1u);
    if (done == gridDim.x - 1) {
      ctl[1] = 0u;
      __threadfence();
      *reinterpret_cast<volatile unsigned*>(ctl) = epoch;
    }
  }
}

int resident_grid() {
  static int cached = 0;
  if (cached) return cached;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, seq_exchange_kernel, kThreads,
                                                    4096) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  cached = per_sm * device_sm_count();
  return cached;
}

}  // namespace
}  // namespace bpt

using namespace bpt;

extern "C" size_t bpt_seqx_buffer_bytes(int world, int batch, int q_heads, int head_dim) {
  if (world < 1 || batch < 1 || q_heads < 1 || head_dim < 1) return 0;
  const size_t items = size_t(batch) * q_heads;
  return (2 * size_t(world) * items * slot_words(head_dim) + 32) * 8;
}

extern "C" int bpt_seqx_alloc(size_t bytes, void** buf, void* ipc_handle) {
  if (!buf || !ipc_handle || bytes == 0) return BPT_ERR_INVALID_ARGUMENT;
  *buf = nullptr;
  if (cudaMalloc(buf, bytes) != cudaSuccess) return BPT_ERR_LAUNCH;
  if (cudaMemset(*buf, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(*buf);
    *buf = nullptr;
    return BPT_ERR_LAUNCH;
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, *buf) != cudaSuccess) {
    cudaFree(*buf);
    *buf = nullptr;
    return BPT_ERR_LAUNCH;
  }
  static_assert(sizeof(h) == BPT_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(ipc_handle, &h, sizeof(h));
  return BPT_OK;
}

extern "C" int bpt_seqx_open(const void* ipc_handle, void** peer_buf) {
  if (!ipc_handle || !peer_buf) return BPT_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return cudaIpcOpenMemHandle(peer_buf, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess
             ? BPT_OK
             : BPT_ERR_LAUNCH;
}

extern "C" int bpt_seqx_close(void* peer_buf) {
  if (!peer_buf) return BPT_ERR_INVALID_ARGUMENT;
  return cudaIpcCloseMemHandle(peer_buf) == cudaSuccess ? BPT_OK : BPT_ERR_LAUNCH;
}

extern "C" int bpt_seqx_free(void* buf) {
  if (!buf) return BPT_ERR_INVALID_ARGUMENT;
  return cudaFree(buf) == cudaSuccess ? BPT_OK : BPT_ERR_LAUNCH;
}

extern "C" int bpt_seqx_merge_fp16(const float* o_part, const float* lse, int batch, int q_heads,
                                   int head_dim, int splits, void* const* bufs, int world,
                                   int rank, void* out, int64_t o_sb, int64_t o_sh,
                                   unsigned* status, unsigned budget_us, void* stream) {
  if (batch < 0 || q_heads < 1 || splits < 1 || world < 1 || world > kMaxRanks || rank < 0 ||
      rank >= world || !bufs || budget_us == 0)
    return BPT_ERR_INVALID_ARGUMENT;
  if (head_dim % 4 != 0 || head_dim > 256) return BPT_ERR_UNSUPPORTED_SHAPE;
  if (batch == 0) return BPT_OK;
  if (!o_part || !lse || !out) return BPT_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(o_part) & 15) || (head_dim * splits) % 4)
    return BPT_ERR_ALIGNMENT;
  RankBufs rb{};
  for (int r = 0; r < world; ++r) {
    if (!bufs[r] || (reinterpret_cast<uintptr_t>(bufs[r]) & 15)) return BPT_ERR_INVALID_ARGUMENT;
    rb.p[r] = static_cast<float*>(bufs[r]);
  }
  const size_t smem = size_t(splits) * sizeof(float);
  if (smem > 48 * 1024) return BPT_ERR_UNSUPPORTED_SHAPE;
  const int items = batch * q_heads;
  int grid = resident_grid();
  if (grid > items) grid = items;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(
      &cfg, seq_exchange_kernel, o_part, lse, batch, q_heads, splits, head_dim, rb, world, rank,
      static_cast<__half*>(out), o_sb, o_sh, status, uint64_t(budget_us) * 1000ull);
  return e == cudaSuccess ? BPT_OK : BPT_ERR_LAUNCH;
}
