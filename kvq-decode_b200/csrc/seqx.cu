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
//   ctl    [B * Hq] (u32)           ctl[c]: epoch of the last call CTA c of the exchange
//                                   kernel finished (the grid never exceeds B * Hq CTAs)
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
//   phase 1: merge this rank's S split rows of the item into one state (o, lse2), reading up
//            to 128 split rows in one memory round trip, and store it, epoch-tagged, into slot
//            (rank, item) of every rank's buffer (peer stores over NVLink);
//   phase 2: thread d reads the words it needs in the local buffer -- every rank's lse2 and
//            o[d] -- all at once, polls (time-bounded) those that do not carry the epoch yet,
//            and merges the world states into channel d of the fp16 output.
// A CTA finishes all its phase-1 stores before it waits, and the grid never exceeds what is
// resident at once, so no rank can wait on a CTA that cannot start. Each CTA keeps its own
// epoch: ctl[c] + 1, read together with its first split rows and written back when it is done,
// so consecutive calls (also graph replays) use fresh epochs, the buffer never needs clearing,
// and no CTA waits for another at the end. CTA c of every rank handles the same items and has
// run in the same calls (the grid, min(B * Hq, resident CTAs), is the same on every rank and in
// every call of one buffer), so writer and reader of a slot agree on its epoch. A wait that
// runs out of its budget sets BPT_DEV_WAIT_TIMEOUT in the status word and the kernel continues
// (the output is then wrong, the GPU stays usable).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <mutex>
#include <math.h>
#include <string.h>

#include "common.cuh"
#include "decode_common.h"

namespace bpt {
namespace {

constexpr int kMaxRanks = 8;
// few rows per warp: each warp's online merge is a serial chain per row (as in the split
// merge of decode_fp16.cu)
constexpr int kWarps = 16;   // 512 threads: the second phase keeps its words in registers
constexpr int kThreads = 32 * kWarps;
constexpr int kRows = 8;    // split rows a warp loads before using any
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

// The value of word p for this call, given a first read w of it: if w does not carry `epoch`
// yet, poll (time-bounded) until it does. Returns 0 after a timeout; once a thread timed out it
// stops waiting for later words.
__device__ __forceinline__ float finish_tagged(const uint64_t* p, uint64_t w, unsigned epoch,
                                               uint64_t budget_ns, int* timed_out) {
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
  __shared__ float s_m[kWarps], s_l[kWarps], s_f[kWarps];
  __shared__ float4 s_o[kWarps][32];
  __shared__ int timed_out;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int items = batch * q_heads;
  const int nd4 = D >> 2;
  uint64_t* const* slots = reinterpret_cast<uint64_t* const*>(bufs.p);
  const size_t set_words = size_t(world) * items * slot_words(D);
  unsigned* ctl = reinterpret_cast<unsigned*>(slots[rank] + 2 * set_words) + blockIdx.x;
  pdl_wait();
  // issued before the split rows' loads and first used after them: no extra round trip
  unsigned epoch;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(epoch) : "l"(ctl) : "memory");
  int my_timeout = 0;
  if (tid == 0) timed_out = 0;

  // ---- phase 1: local split merge, epoch-tagged stores into every rank's slot (rank, item).
  // Warp w owns splits w, w + 16, ... and merges them online in batches of kRows rows, every
  // load of a batch (the rows' lse and this lane's 4 channels of their o) issued before any is
  // used; the 16 warp states are combined in warp order through shared memory, lane w of
  // warp 0 turning state w into its weight 2^(m_w - M) / L once.
  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    const float* l = lse + int64_t(it) * splits;
    const float* o = o_part + int64_t(it) * splits * D;
    for (int c0 = 0; c0 < nd4; c0 += 32) {
      const int c = c0 + lane;
      const bool c_in = c < nd4;
      float m = kNegInf, wsum = 0.f;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int s0 = warp; s0 < splits; s0 += kWarps * kRows) {
        float ls[kRows];
        float4 v[kRows];
#pragma unroll
        for (int u = 0; u < kRows; ++u) {
          const int sp = s0 + kWarps * u;
          const bool in = sp < splits;
          ls[u] = in ? l[sp] : kNegInf;
          v[u] = (in && c_in) ? __ldg(reinterpret_cast<const float4*>(o + int64_t(sp) * D) + c)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float mb = m;
#pragma unroll
        for (int u = 0; u < kRows; ++u) mb = fmaxf(mb, ls[u]);
        if (mb != kNegInf) {   // warp-uniform
          const float f = fast_exp2(m - mb);
          wsum *= f;
          acc.x *= f; acc.y *= f; acc.z *= f; acc.w *= f;
#pragma unroll
          for (int u = 0; u < kRows; ++u) {
            // a split of weight 0 contributes nothing even if its row holds garbage
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
        const float mw = lane < kWarps ? s_m[lane] : kNegInf;   // lane w: state w
        float M = mw;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
          M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
        const float fw = (lane < kWarps && M != kNegInf) ? fast_exp2(mw - M) : 0.f;
        float L = lane < kWarps ? s_l[lane] * fw : 0.f;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
        if (lane < kWarps) s_f[lane] = L > 0.f ? fw / L : 0.f;
        __syncwarp();
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
        for (int w = 0; w < kWarps; ++w) {
          const float f = s_f[w];
          const float4 a4 = s_o[w][lane];
          O.x = fmaf(a4.x, f, O.x);
          O.y = fmaf(a4.y, f, O.y);
          O.z = fmaf(a4.z, f, O.z);
          O.w = fmaf(a4.w, f, O.w);
        }
        const size_t base =
            size_t((epoch + 1u) & 1u) * set_words + (size_t(rank) * items + it) * slot_words(D);
        if (c_in) {
          const float r4[4] = {O.x, O.y, O.z, O.w};
          for (int r = 0; r < world; ++r)
#pragma unroll
            for (int e = 0; e < 4; ++e)
              st_tagged(slots[r] + base + 4 * c + e, r4[e], epoch + 1u);
        }
        if (c0 == 0 && lane < world)
          st_tagged(slots[lane] + base + D, L > 0.f ? M + __log2f(L) : kNegInf, epoch + 1u);
      }
      __syncthreads();   // s_m / s_l / s_o are rewritten next
    }
  }

  // the next kernel in the stream may start launching; it waits for this grid's completion
  pdl_launch_dependents();
  epoch += 1u;   // this call's epoch
  const uint64_t* mine = slots[rank] + size_t(epoch & 1u) * set_words;

  // ---- phase 2: every rank's state of my items -> the merged fp16 output. Thread d reads
  // every rank's lse word and o word d at once, then polls (time-bounded) only the words that
  // do not carry this call's epoch yet. Every word is awaited, even at weight 0, so no store
  // of this call is still in flight into the buffer when the next call starts.
  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    const int b = it / q_heads, hq = it % q_heads;
    const uint64_t* item0 = mine + size_t(it) * slot_words(D);
    const size_t rstride = size_t(items) * slot_words(D);
    for (int d = tid; d < D; d += kThreads) {
      uint64_t lw[kMaxRanks], ow[kMaxRanks];
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r) {
        if (r < world) {
          lw[r] = ld_tagged(item0 + r * rstride + D);
          ow[r] = ld_tagged(item0 + r * rstride + d);
        }
      }
      float ls[kMaxRanks], ov[kMaxRanks];
      float M = kNegInf;
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r) {
        ls[r] = kNegInf;
        ov[r] = 0.f;
        if (r < world) {
          ls[r] = finish_tagged(item0 + r * rstride + D, lw[r], epoch, budget_ns, &my_timeout);
          ov[r] = finish_tagged(item0 + r * rstride + d, ow[r], epoch, budget_ns, &my_timeout);
          M = fmaxf(M, ls[r]);
        }
      }
      float W = 0.f, acc = 0.f;
      if (M != kNegInf) {
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r) {
          const float w = r < world ? fast_exp2(ls[r] - M) : 0.f;
          W += w;
          if (w != 0.f) acc = fmaf(w, ov[r], acc);
        }
      }
      out[int64_t(b) * o_sb + int64_t(hq) * o_sh + d] = __float2half_rn(W > 0.f ? acc / W : 0.f);
    }
  }

  // ---- this CTA is done with the call: its next call uses the next epoch (the next kernel
  // in the stream sees the store once this grid has completed)
  if (my_timeout) timed_out = 1;
  __syncthreads();
  if (tid == 0) {
    if (timed_out) flag_device_error(status, BPT_DEV_WAIT_TIMEOUT);
    *ctl = epoch;
  }
}

// CTAs of the exchange kernel that are resident at once on the current device, cached per
// device ordinal (GPUs of one process may differ in SM count). The first call on a device
// queries the occupancy API, so make it before any stream capture.
constexpr int kMaxGridDevices = 64;
int g_resident_grid[kMaxGridDevices];
std::mutex g_resident_mu;

int resident_grid() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxGridDevices) return 0;
  std::lock_guard<std::mutex> lock(g_resident_mu);
  if (g_resident_grid[dev]) return g_resident_grid[dev];
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, seq_exchange_kernel, kThreads,
                                                    0) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  g_resident_grid[dev] = per_sm * device_sm_count();
  return g_resident_grid[dev];
}

}  // namespace
}  // namespace bpt

using namespace bpt;

extern "C" size_t bpt_seqx_buffer_bytes(int world, int batch, int q_heads, int head_dim) {
  if (world < 1 || batch < 1 || q_heads < 1 || head_dim < 1) return 0;
  const size_t items = size_t(batch) * q_heads;
  return (2 * size_t(world) * items * slot_words(head_dim) + items) * 8;
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
  const int items = batch * q_heads;
  int grid = resident_grid();
  if (grid < 1) return BPT_ERR_NO_DEVICE;
  if (grid > items) grid = items;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 0;
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
