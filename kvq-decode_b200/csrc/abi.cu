// C-ABI utilities: status strings, split planner, workspace sizing, tensor-map encoding.
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>

#include "decode_common.h"

namespace bpt {

namespace {

constexpr int kChunkTokens = 32;    // tokens per pipeline stage of the decode kernels
constexpr int kResidentCtas = 4;    // decode CTAs resident per SM
constexpr int kMinChunksPerSplit = 2;
constexpr int kMinSingleWaveSplits = 4;
constexpr int kWaves = 7;                      // several-wave plans: just under 7 full waves
constexpr int64_t kMaxSingleWaveTokens = 8192; // longest split of a one-wave plan
constexpr int64_t kMinMultiWaveTokens = 1024;  // shortest split of a several-wave plan

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

}  // namespace

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder_fn() { return tensor_map_encoder(); }

int device_sm_count() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 148;
  return sms;
}

WorkspaceView workspace_view(void* ws, int batch, int q_heads, int head_dim, int splits) {
  (void)head_dim;
  char* base = static_cast<char*>(ws);
  WorkspaceView v;
  v.status = reinterpret_cast<unsigned*>(base);
  v.lse = reinterpret_cast<float*>(base + 256);
  const size_t lse_bytes = align256(size_t(batch) * q_heads * splits * sizeof(float));
  v.o_part = reinterpret_cast<float*>(base + 256 + lse_bytes);
  return v;
}

int encode_kv_map(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                  int inner, int kv_heads, int block_size, int64_t num_blocks, int64_t s_head,
                  int64_t s_tok, int64_t s_blk, int box_inner, int box_rows,
                  int* token_is_dim1, int swizzle_bytes) {
  auto enc = tensor_map_encoder();
  if (!enc) return BPT_ERR_DRIVER;
  if (reinterpret_cast<uintptr_t>(base) & 15) return BPT_ERR_ALIGNMENT;
  if (num_blocks <= 0) num_blocks = 1;  // an empty cache is never read (no valid token)
  const int64_t sh = s_head * elem_bytes, st = s_tok * elem_bytes, sb = s_blk * elem_bytes;
  if ((sh % 16) || (st % 16) || (sb % 16)) return BPT_ERR_ALIGNMENT;
  const bool tok1 = st < sh;  // head-major page ([block, head, token, inner])
  *token_is_dim1 = tok1 ? 1 : 0;
  cuuint64_t dims[4] = {cuuint64_t(inner), cuuint64_t(tok1 ? block_size : kv_heads),
                        cuuint64_t(tok1 ? kv_heads : block_size), cuuint64_t(num_blocks)};
  cuuint64_t strides[3] = {cuuint64_t(tok1 ? st : sh), cuuint64_t(tok1 ? sh : st),
                           cuuint64_t(sb)};
  cuuint32_t box[4] = {cuuint32_t(box_inner), cuuint32_t(tok1 ? box_rows : 1),
                       cuuint32_t(tok1 ? 1 : box_rows), 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_NONE;
  if (swizzle_bytes == 128) sw = CU_TENSOR_MAP_SWIZZLE_128B;
  else if (swizzle_bytes == 64) sw = CU_TENSOR_MAP_SWIZZLE_64B;
  else if (swizzle_bytes == 32) sw = CU_TENSOR_MAP_SWIZZLE_32B;
  CUresult r = enc(map, dtype, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? BPT_OK : BPT_ERR_TENSOR_MAP;
}

}  // namespace bpt

using namespace bpt;

extern "C" const char* bpt_status_string(int status) {
  switch (status) {
    case BPT_OK: return "ok";
    case BPT_ERR_INVALID_ARGUMENT: return "invalid argument";
    case BPT_ERR_UNSUPPORTED_SHAPE: return "unsupported shape (head_dim/group/block_size)";
    case BPT_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
    case BPT_ERR_LAUNCH: return "CUDA launch error";
    case BPT_ERR_TENSOR_MAP: return "tensor map encoding rejected the cache view";
    case BPT_ERR_ALIGNMENT: return "pointer or stride not 16-byte aligned";
    case BPT_ERR_DRIVER: return "CUDA driver entry point unavailable";
    case BPT_ERR_DEVICE_CHECK: return "device-side check failed";
    case BPT_ERR_NO_DEVICE: return "no CUDA device";
    default: return "unknown status";
  }
}

extern "C" int bpt_version(void) { return 100; }

namespace bpt {

int plan_splits(int batch, int kv_heads, int block_size, int max_blocks, int sm_count,
                int resident_per_sm, int chunk_tokens) {
  // One CTA per (sequence, kv head, split); resident_per_sm of them fit on an SM at once.
  if (sm_count <= 0) sm_count = device_sm_count();
  const int64_t units = (int64_t(max_blocks) * block_size + chunk_tokens - 1) / chunk_tokens;
  const int64_t work = int64_t(batch > 0 ? batch : 1) * (kv_heads > 0 ? kv_heads : 1);
  const int64_t resident = int64_t(sm_count) * resident_per_sm;
  int64_t want = resident / work;
  // ONE wave when at least 4 splits fit in it and its splits stay at most 8192 tokens of the
  // table: every CTA starts together, and a ragged batch is balanced by cutting the longest
  // sequence (split_range), so no CTA runs much longer than the others. Otherwise just under
  // 7 full waves of shorter CTAs (floor, so the last wave is nearly full: a last wave of a
  // few CTAs cannot keep HBM busy), with splits of at least 1024 tokens. Measured on B200
  // (ragged FP16 batches, lengths U[0.75, 1] ctx): B=16/64k 4 splits 604 us vs 32 splits
  // 556 us; B=32/64k 19 splits 1135 us vs 16 splits 1102 us; B=64/64k 10 vs 8 splits
  // 2190 vs 2169 us (one box, the two planners alternated).
  const int64_t span_tokens = units * chunk_tokens;
  if (want < kMinSingleWaveSplits || span_tokens > kMaxSingleWaveTokens * want) {
    const int64_t one_wave = want;
    want = kWaves * resident / work;
    // a context too short for that many 1024-token splits: fewer, but never fewer than fill
    // one wave
    const int64_t most = span_tokens / kMinMultiWaveTokens;
    if (want > most) want = most > one_wave ? most : one_wave;
  }
  int64_t cap = units / kMinChunksPerSplit;
  if (cap < 1) cap = 1;
  if (want > cap) want = cap;
  if (want < 1) want = 1;
  return int(want);
}

// Balanced splits for a multi-sequence batch launched as one wave. Several-wave launches keep
// equal per-sequence splits (the block scheduler fills their tail; balancing them measured
// slower on B200: B=64/64k 2211 -> 2316 us).
bool balanced_splits(int batch, int kv_heads, int splits, int resident_per_sm) {
  if (batch < 2) return false;
  return int64_t(batch) * kv_heads * splits <= int64_t(device_sm_count()) * resident_per_sm;
}

int clamp_splits(int s, int block_size, int max_blocks, int chunk_tokens) {
  const int64_t units = (int64_t(max_blocks) * block_size + chunk_tokens - 1) / chunk_tokens;
  if (s > units) s = int(units);
  if (s < 1) s = 1;
  return s;
}

}  // namespace bpt

extern "C" int bpt_plan_splits(int batch, int kv_heads, int block_size, int max_blocks,
                               int sm_count) {
  return plan_splits(batch, kv_heads, block_size, max_blocks, sm_count, kResidentCtas,
                     kChunkTokens);
}

extern "C" int bpt_effective_splits(int batch, int kv_heads, int block_size, int max_blocks,
                                    int num_splits, int sm_count) {
  const int s = num_splits > 0
                    ? num_splits
                    : bpt_plan_splits(batch, kv_heads, block_size, max_blocks, sm_count);
  return clamp_splits(s, block_size, max_blocks, kChunkTokens);
}

extern "C" size_t bpt_decode_workspace_bytes(int batch, int q_heads, int head_dim, int splits) {
  if (batch <= 0 || q_heads <= 0 || head_dim <= 0 || splits <= 0) return 256;
  const size_t rows = size_t(batch) * q_heads * splits;
  return 256 + align256(rows * sizeof(float)) + rows * head_dim * sizeof(float);
}
