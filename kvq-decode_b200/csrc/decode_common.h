// Host+device declarations shared by the decode translation units.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/bpt.h"

namespace bpt {

struct DecodeParams {
  const __half* q;
  int64_t q_sb, q_sh;
  const int32_t* block_table;
  int64_t bt_sb;
  const int32_t* seq_lens;
  __half* out;
  int64_t o_sb, o_sh;
  float* o_part;    // [B, Hq, S, D] normalised partial outputs (fp32)
  float* lse;       // [B, Hq, S] log2-sum-exp of the partials
  unsigned* status; // device check flags
  int batch, q_heads, kv_heads, group, splits, block_size, max_blocks, box_rows;
  int k_c1, v_c1;   // 1: tensor-map dim 1 is the token dim (head-major cache), 0: the head dim
  int final_out;    // 1: a one-split call writes normalised fp16 `out` directly
  int balance;      // 1: splits sized by the batch's longest sequence (split_range)
  int64_t num_blocks;
  float scale_log2; // softmax scale * log2(e)
};

struct WorkspaceView {
  unsigned* status;
  float* lse;
  float* o_part;
};

// Workspace layout: [status word, padded to 256 B][lse, padded to 256 B][o_part].
WorkspaceView workspace_view(void* ws, int batch, int q_heads, int head_dim, int splits);

// 4-D tiled tensor map over a paged cache [num_blocks, block_size, Hkv, inner] whose inner
// dimension is contiguous; strides in elements. The two middle dimensions are ordered by
// stride; *token_is_dim1 tells the kernel which coordinate is which. The box is
// {box_inner, 1 head, box_rows tokens, 1 block}. swizzle_bytes: 0 (none), 32, 64 or 128 (the
// box's inner extent in bytes must not exceed it); a swizzled box lands in shared memory with
// 16-byte chunk c of row r stored at chunk c ^ (r % (swizzle_bytes / 16)).
int encode_kv_map(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                  int inner, int kv_heads, int block_size, int64_t num_blocks, int64_t s_head,
                  int64_t s_tok, int64_t s_blk, int box_inner, int box_rows, int* token_is_dim1,
                  int swizzle_bytes = 0);

// Merge `splits` partial states per (b, q head). Exactly one of out16 (fp16 [B, Hq, D] with
// strides o_sb/o_sh) or (o32 [B, Hq, D] contiguous fp32 + lse32 [B, Hq]) is written. pdl:
// launch as a programmatic dependent of the split kernel just enqueued on the same stream.
int launch_merge(const float* o_part, const float* lse, int batch, int q_heads, int splits,
                 int D, __half* out16, int64_t o_sb, int64_t o_sh, float* o32, float* lse32,
                 cudaStream_t st, bool pdl);

// Validate, encode the tensor maps and launch the FP16 split kernel (decode_fp16.cu).
int run_split_fp16(const void* q, int64_t q_sb, int64_t q_sh, const void* k_cache, int64_t k_sb,
                   int64_t k_st, int64_t k_sh, const void* v_cache, int64_t v_sb, int64_t v_st,
                   int64_t v_sh, int64_t num_blocks, const int32_t* block_table, int64_t bt_sb,
                   const int32_t* seq_lens, void* out, int64_t o_sb, int64_t o_sh, int batch,
                   int q_heads, int kv_heads, int head_dim, int block_size, int max_blocks,
                   float scale, int splits, int final_out, float* o_part, float* lse,
                   unsigned* status, cudaStream_t st);

int device_sm_count();
// Split planner for a kernel with `resident_per_sm` CTAs per SM and `chunk_tokens` tokens per
// pipeline stage (splits are whole chunks); clamp_splits bounds a requested count.
int plan_splits(int batch, int kv_heads, int block_size, int max_blocks, int sm_count,
                int resident_per_sm, int chunk_tokens);
int clamp_splits(int s, int block_size, int max_blocks, int chunk_tokens);
// Whether a call of batch * kv_heads * splits CTAs, resident_per_sm per SM, uses balanced
// splits: a batch of several sequences launched as one wave, where the ragged tail of equal
// per-sequence splits is not hidden by later waves.
bool balanced_splits(int batch, int kv_heads, int splits, int resident_per_sm);

// cuTensorMapEncodeTiled resolved through the runtime's driver entry-point query (no link
// dependency on libcuda); null if unavailable.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder_fn();

}  // namespace bpt
