// FP16 paged decode for callers that cannot allocate device memory.
//
// bpt_decode_fp16 needs a caller-provided workspace for the split-KV partial states. Some
// callers cannot get one at call time: an engine that hands out all device memory at start-up
// and forbids cudaMalloc afterwards, a plugin whose host framework passes it only the input
// and output buffers, or code that runs where allocating is unsafe (inside an allocator hook
// or a callback that must not block on the allocator's locks). For them this entry point keeps
// the partial states in a fixed scratch array compiled into the library instead.
//
// The array (BPT_NOALLOC_SCRATCH_BYTES) is reserved on every GPU that loads this library's
// device code and stays there until the process exits. Host code cannot use the array's name
// as a device address, so each call made outside stream capture, with its device current, looks
// the address up with cudaGetSymbolAddress and keeps it for captured calls; make the first
// call on each device before any stream capture. Every call shares the one array per device, so two calls whose kernels overlap on
// the GPU (different streams, no ordering between them) race on it. Nothing in the array needs
// to start at zero: a call writes every partial-state row it later reads. This path records no
// device-side check flags (it has no status word to hand back).
#include <cuda_runtime.h>

#include <mutex>

#include "decode_common.h"

namespace bpt {
namespace {

// lse2 rows, then o_part rows: the same layout bpt_decode_fp16 uses after its status word.
static __device__ __align__(256) unsigned char g_noalloc_scratch[BPT_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices];
std::mutex g_scratch_mu;

size_t round256(size_t x) { return (x + 255) & ~size_t(255); }

// Device address of the current device's copy of the scratch array. Outside stream capture
// it is looked up on every call, so a reset device or another context made current on the
// same ordinal (both reload the module, which can move the array) gets its own address; a
// call being captured reuses the address the last uncaptured call on this device found.
int scratch_address(cudaStream_t stream, void** addr) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return BPT_ERR_NO_DEVICE;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  const bool capturing =
      cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!capturing) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr)
      return BPT_ERR_LAUNCH;
    g_scratch_addr[dev] = p;
  }
  if (!g_scratch_addr[dev]) return BPT_ERR_LAUNCH;  // first call on this device was captured
  *addr = g_scratch_addr[dev];
  return BPT_OK;
}

}  // namespace
}  // namespace bpt

using namespace bpt;

extern "C" int bpt_decode_fp16_noalloc(const void* q, int64_t q_sb, int64_t q_sh,
                                       const void* k_cache, int64_t k_sb, int64_t k_st,
                                       int64_t k_sh, const void* v_cache, int64_t v_sb,
                                       int64_t v_st, int64_t v_sh, int64_t num_blocks,
                                       const int32_t* block_table, int64_t bt_sb,
                                       const int32_t* seq_lens, void* out, int64_t o_sb,
                                       int64_t o_sh, int batch, int q_heads, int kv_heads,
                                       int head_dim, int block_size, int max_blocks,
                                       float scale, int num_splits, int sm_count,
                                       void* stream) {
  if (batch < 0 || q_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || q_heads % kv_heads != 0)
    return BPT_ERR_INVALID_ARGUMENT;
  if (batch == 0) return BPT_OK;
  if (!out) return BPT_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(out) & 15) || ((o_sb * 2) % 16) || ((o_sh * 2) % 16))
    return BPT_ERR_ALIGNMENT;
  const int S = bpt_effective_splits(batch, kv_heads, block_size, max_blocks, num_splits,
                                     sm_count);
  const size_t rows = size_t(batch) * q_heads * S;
  const size_t lse_bytes = round256(rows * sizeof(float));
  if (lse_bytes + rows * head_dim * sizeof(float) > BPT_NOALLOC_SCRATCH_BYTES)
    return BPT_ERR_WORKSPACE_TOO_SMALL;  // more partial state than the fixed array holds
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* base = nullptr;
  int rc = scratch_address(st, &base);
  if (rc) return rc;
  float* lse = static_cast<float*>(base);
  float* o_part = reinterpret_cast<float*>(static_cast<char*>(base) + lse_bytes);
  rc = run_split_fp16(q, q_sb, q_sh, k_cache, k_sb, k_st, k_sh, v_cache, v_sb, v_st, v_sh,
                      num_blocks, block_table, bt_sb, seq_lens, out, o_sb, o_sh, batch, q_heads,
                      kv_heads, head_dim, block_size, max_blocks, scale, S, 1, o_part, lse,
                      nullptr, st);
  if (rc || S == 1) return rc;
  return launch_merge(o_part, lse, batch, q_heads, S, head_dim, static_cast<__half*>(out), o_sb,
                      o_sh, nullptr, nullptr, st, true);
}
