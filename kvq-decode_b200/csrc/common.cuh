// Device-side building blocks shared by the bpt kernels: mbarriers with time-bounded waits,
// TMA (cp.async.bulk.tensor) page loads, named barriers, warp reductions.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/bpt.h"

namespace bpt {

constexpr unsigned kFullMask = 0xffffffffu;
// A pipeline wait gives up after this long (ns of %globaltimer). A healthy wait lasts at most
// microseconds; the budget only bounds a kernel that would otherwise spin forever.
constexpr uint64_t kWaitBudgetNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ----------------------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that may suspend the thread for up to `hint_ns` (it resumes as soon as the phase
// completes), so a waiting warp sleeps instead of taking issue slots from working warps.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity,
                                                    uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete, giving up after budget_ns. Returns
// false if the budget ran out (the caller records BPT_DEV_WAIT_TIMEOUT and leaves the pipeline).
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, uint64_t budget_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, 1000000u)) return true;
    if (global_timer_ns() - t0 > budget_ns) return false;
  }
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  return mbar_wait_for(bar, parity, kWaitBudgetNs);
}

// ----------------------------------------------------------------------------- TMA

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 4-D tiled TMA load into this CTA's shared memory, completion signalled on `bar` as
// transaction bytes. Coordinates are element indices, innermost first. The innermost
// coordinate passed by the bpt kernels is always 0 (16-byte aligned by construction).
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ----------------------------------------------------------------------------- PDL

// Let a programmatically dependent grid (the split merge) start launching; it still waits
// for this grid's completion in pdl_wait() before reading anything this grid wrote.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Wait until the preceding grid in the stream has completed and its writes are visible
// (a no-op when the grid was not launched as a programmatic dependent).
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Launch `kern` as a programmatic dependent of the previous kernel in `st`: its CTAs may be
// scheduled once that kernel's CTAs have all called pdl_launch_dependents() (or exited), and
// they wait in pdl_wait() for its completion. After a kernel that never calls
// pdl_launch_dependents() this only saves the launch latency.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_dependent(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                    cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Args&&>(args)...);
}

// ----------------------------------------------------------------------------- misc

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// acc += q.lo * k.lo + q.hi * k.hi with fp16 operands and an fp32 accumulator
// (fma.rn.f32.f16: the fp16 product is exact in fp32, one rounding per fma).
__device__ __forceinline__ float fma_f16x2_f32(uint32_t q2, uint32_t k2, float acc) {
  asm("{\n\t.reg .f16 ql, qh, kl, kh;\n\t"
      "mov.b32 {ql, qh}, %1;\n\t"
      "mov.b32 {kl, kh}, %2;\n\t"
      "fma.rn.f32.f16 %0, ql, kl, %0;\n\t"
      "fma.rn.f32.f16 %0, qh, kh, %0;\n\t}"
      : "+f"(acc)
      : "r"(q2), "r"(k2));
  return acc;
}

__device__ __forceinline__ float2 half2_bits_to_float2(uint32_t v) {
  __half2 h = *reinterpret_cast<__half2*>(&v);
  return __half22float2(h);
}

__device__ __forceinline__ void flag_device_error(unsigned* status, unsigned flag) {
  if (status) atomicOr(status, flag);
}

template <typename T>
__host__ __device__ constexpr T cdiv(T a, T b) {
  return (a + b - 1) / b;
}

// Chunk range [*u0, *u1) of split `split` of S over a sequence of n_units chunks. Unbalanced:
// the sequence's own chunks are cut into S parts. Balanced: the batch's longest sequence
// (span_units chunks) is cut into S parts and a shorter sequence keeps the parts that cover
// it, so every non-empty split of the batch has about span_units / S chunks and a ragged
// batch launched as one wave has no long-sequence tail (the later splits of short sequences
// are empty).
__device__ __forceinline__ void split_range(int split, int S, int n_units, int span_units,
                                            int* u0, int* u1) {
  *u0 = min(n_units, int(int64_t(split) * span_units / S));
  *u1 = min(n_units, int(int64_t(split + 1) * span_units / S));
}

// Longest sequence of the batch, each length clamped to [0, cap] as the kernels clamp their
// own. Every warp computes it for itself (no barrier): lane l reads lengths l, l + 32, ...
__device__ __forceinline__ int batch_max_len(const int32_t* seq_lens, int batch, int64_t cap) {
  const int lane = threadIdx.x & 31;
  int m = 0;
  for (int i = lane; i < batch; i += 32) m = max(m, __ldg(seq_lens + i));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  return int(min(int64_t(m), cap));
}

}  // namespace bpt
