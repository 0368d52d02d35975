/*
 * bpt — B200-native paged-KV GQA decode attention: the C ABI.
 *
 * Every entry point takes plain device pointers, element strides and sizes, a caller-owned
 * device workspace and a cudaStream_t passed as void*. Nothing here allocates, synchronises
 * the host or reads device memory from the host, so every call can be enqueued inside a
 * CUDA graph capture. Return value: 0 = success, negative = bpt_status (see below);
 * bpt_status_string() turns it into text.
 *
 * Layouts (vLLM-style paged cache, the reference's layout, src/bpt/reference.py:3-9):
 *   q            [B, Hq, D]                        fp16, inner stride 1
 *   k/v cache    [num_blocks, block_size, Hkv, D]  inner stride 1, other strides free
 *   block_table  [B, max_blocks] int32             logical page -> physical block
 *   seq_lens     [B] int32                         valid tokens per sequence (0 allowed)
 *   out          [B, Hq, D] fp16
 */
#ifndef BPT_H_
#define BPT_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum bpt_status {
  BPT_OK = 0,
  BPT_ERR_INVALID_ARGUMENT = -1,  /* null pointer, negative size, Hq % Hkv != 0, ... */
  BPT_ERR_UNSUPPORTED_SHAPE = -2, /* head_dim / group / block_size outside the built set */
  BPT_ERR_WORKSPACE_TOO_SMALL = -3,
  BPT_ERR_LAUNCH = -4,            /* CUDA launch or runtime error */
  BPT_ERR_TENSOR_MAP = -5,        /* cuTensorMapEncodeTiled rejected the cache view */
  BPT_ERR_ALIGNMENT = -6,         /* pointer / stride not 16-byte aligned */
  BPT_ERR_DRIVER = -7,            /* driver entry point unavailable */
  BPT_ERR_DEVICE_CHECK = -8,      /* device-side check tripped (see bpt_device_flags) */
  BPT_ERR_NO_DEVICE = -9
};

/* Device-side check flags, OR-ed into the first 4 bytes of the workspace by the kernels.
 * Reading them needs a device->host copy, so the host library never does it on its own;
 * the Python layer does it only in checked mode (BPT_CHECKS=1). */
enum bpt_device_flags {
  BPT_DEV_BAD_BLOCK_ID = 1,    /* block_table entry outside [0, num_blocks) */
  BPT_DEV_SEQ_TOO_LONG = 2,    /* seq_len > max_blocks * block_size (clamped) */
  BPT_DEV_WAIT_TIMEOUT = 4,    /* a pipeline wait gave up after its time budget */
  BPT_DEV_NEG_SEQ_LEN = 8      /* seq_len < 0 (treated as 0) */
};

const char* bpt_status_string(int status);
int bpt_version(void);

/* Number of KV splits the heuristic picks. Replaces choose_num_splits
 * (src/bpt/triton_fp16.py:175-180); B200 tuning: one wave of CTAs when at least 4 splits fit
 * in it and they stay at most 8192 tokens of the table long, otherwise just under 7 full
 * waves of splits of at least 1024 tokens. A multi-sequence batch launched as one wave cuts
 * its longest sequence into the splits and every other sequence keeps the splits that cover
 * it (its later splits are empty); otherwise each sequence's own tokens are cut evenly. */
int bpt_plan_splits(int batch, int kv_heads, int block_size, int max_blocks, int sm_count);

/* Split count a decode call actually uses for a requested num_splits (<= 0 = heuristic),
 * mirroring the clamping of src/bpt/triton_fp16.py:208-217. */
int bpt_effective_splits(int batch, int kv_heads, int block_size, int max_blocks,
                         int num_splits, int sm_count);

/* Workspace bytes a decode call with this many effective splits needs. */
size_t bpt_decode_workspace_bytes(int batch, int q_heads, int head_dim, int splits);

/* FP16 paged decode: replaces paged_decode_attention_triton
 * (src/bpt/triton_fp16.py:183-247) and its kernels _split_kernel (:83-144),
 * _paged_decode_kernel (:25-80) and _merge_kernel (:147-163).
 * Strides are in elements. scale <= 0 selects 1/sqrt(head_dim) (triton_fp16.py:203-204).
 * num_splits: <= 0 heuristic, 1 single pass, n n-way split (triton_fp16.py:192).
 * sm_count: SMs of the target device, used only by the heuristic (<= 0: query it). */
int bpt_decode_fp16(const void* q, int64_t q_sb, int64_t q_sh,
                    const void* k_cache, int64_t k_sb, int64_t k_st, int64_t k_sh,
                    const void* v_cache, int64_t v_sb, int64_t v_st, int64_t v_sh,
                    int64_t num_blocks,
                    const int32_t* block_table, int64_t bt_sb,
                    const int32_t* seq_lens,
                    void* out, int64_t o_sb, int64_t o_sh,
                    int batch, int q_heads, int kv_heads, int head_dim,
                    int block_size, int max_blocks,
                    float scale, int num_splits, int sm_count,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Stage 1 alone: the split kernel (src/bpt/triton_fp16.py:83-144) with exactly `splits`
 * splits, writing normalised fp32 partial outputs o_part [B, Hq, splits, D] and their
 * log2-sum-exp lse [B, Hq, splits] (log2 units: lse2 = ln-sum-exp * log2(e); -inf for an
 * empty split). Used for sequence sharding across GPUs, where each rank's states are merged
 * after an all-gather. status (nullable) receives bpt_device_flags. */
int bpt_decode_fp16_partial(const void* q, int64_t q_sb, int64_t q_sh,
                            const void* k_cache, int64_t k_sb, int64_t k_st, int64_t k_sh,
                            const void* v_cache, int64_t v_sb, int64_t v_st, int64_t v_sh,
                            int64_t num_blocks,
                            const int32_t* block_table, int64_t bt_sb,
                            const int32_t* seq_lens,
                            int batch, int q_heads, int kv_heads, int head_dim,
                            int block_size, int max_blocks, float scale, int splits,
                            float* o_part, float* lse, unsigned* status, void* stream);

/* Stage 2: merge `splits` partial states per (b, q head) into fp16 out [B, Hq, D]
 * (replaces _merge_kernel, src/bpt/triton_fp16.py:147-163). */
int bpt_merge_partials(const float* o_part, const float* lse, int batch, int q_heads,
                       int head_dim, int splits, void* out, int64_t o_sb, int64_t o_sh,
                       void* stream);

/* Stage 2 keeping fp32 state: merged o [B, Hq, D] (contiguous) and lse [B, Hq] (log2). */
int bpt_merge_states(const float* o_part, const float* lse, int batch, int q_heads,
                     int head_dim, int splits, float* o_out, float* lse_out, void* stream);

/* Cross-GPU merge of sequence-shard states. `states` holds `ranks` consecutive blocks (the
 * output of an all-gather), each laid out as o [B, Hq, D] fp32 followed by lse [B, Hq]
 * (log2 units) — exactly what bpt_merge_states writes for one rank's shard. The merged
 * fp16 result goes to out [B, Hq, D]. No reference counterpart (the reference is single-GPU);
 * the merge formula is the reference's split merge (src/bpt/triton_fp16.py:152-162). */
int bpt_merge_rank_states(const float* states, int ranks, int batch, int q_heads,
                          int head_dim, void* out, int64_t o_sb, int64_t o_sh, void* stream);

/* ---------------------------------------------------------------- KIVI-quantized caches
 *
 * No counterpart in the reference (its README lists quantized KV as "not started"); the
 * format follows the BASELINE KIVI description. Keys are quantized per (page, kv head,
 * channel) over the page's tokens, values per (token, kv head) over the channels; INT8/INT4
 * are asymmetric (unsigned codes, fp16 scale + zero-point, x ~= code * scale + zero), FP8-E4M3
 * is symmetric (x ~= e4m3(code) * scale). Codes are computed from the fp16-rounded scale/zero
 * with fp32 round-half-even arithmetic, bit-exact with the numpy specification in
 * oracle/kivi.py. Storage, block_size = bs, H kv heads, D head dim:
 *   INT8 / FP8  k_codes, v_codes [num_blocks, bs, H, D]   uint8
 *   INT4        k_codes [num_blocks, bs, H, D/2]  (low nibble = even channel)
 *               v_codes [num_blocks, bs/2, H, D]  (low nibble = even token)
 *   k_scale, k_zero [num_blocks, H, D] fp16;  v_scale, v_zero [num_blocks, bs, H] fp16
 *   (FP8: k_zero / v_zero unused, may be NULL).
 * Strides are in elements of each array (bytes for the uint8 code arrays). */
enum bpt_kv_format { BPT_KV_INT8 = 1, BPT_KV_FP8_E4M3 = 2, BPT_KV_INT4 = 3 };

typedef struct bpt_kivi_cache {
  int format;          /* enum bpt_kv_format */
  int block_size;      /* tokens per page (power of two, 16..256; even for INT4) */
  int kv_heads;
  int head_dim;
  int64_t num_blocks;
  void* k_codes;  int64_t k_codes_stride[3];  /* block, token, head (inner stride 1) */
  void* v_codes;  int64_t v_codes_stride[3];  /* block, token (INT4: token pair), head */
  void* k_scale;  void* k_zero;  int64_t k_param_stride[2];  /* block, head */
  void* v_scale;  void* v_zero;  int64_t v_param_stride[2];  /* block, token */
} bpt_kivi_cache;

/* Quantize and write new tokens into a KIVI cache (the cache-append step; no reference
 * counterpart). Sequence b receives tokens [start_pos[b], start_pos[b] + new_lens[b]) from
 * k_new / v_new [batch, max_new, H, D] fp16 (token t of the append at index t). start_pos[b]
 * must be a multiple of block_size: key statistics are per page, so a page is always
 * written whole from fp16 rows; slots past the appended tokens in the last page get code 0 and
 * value scale/zero 0. new_lens / start_pos / block_table are device arrays. */
int bpt_kivi_append(const bpt_kivi_cache* cache,
                    const void* k_new, int64_t kn_sb, int64_t kn_st, int64_t kn_sh,
                    const void* v_new, int64_t vn_sb, int64_t vn_st, int64_t vn_sh,
                    const int32_t* new_lens, const int32_t* start_pos,
                    const int32_t* block_table, int64_t bt_sb, int max_blocks,
                    int batch, int max_new, void* stream);

/* Split count a KIVI decode call uses for a requested num_splits (<= 0 = heuristic), as
 * bpt_effective_splits for the kernel that serves this format and group (its tokens per
 * pipeline stage and CTAs per SM differ from the fp16 kernel's). No reference counterpart. */
int bpt_effective_splits_kivi(int format, int batch, int kv_heads, int q_heads, int block_size,
                              int max_blocks, int num_splits, int sm_count);

/* Fused-dequant decode over a KIVI cache: same contract as bpt_decode_fp16 (split
 * semantics, workspace, status codes), with splits from bpt_effective_splits_kivi. The result
 * equals fp32 attention over the dequantized cache (x_hat in fp32, never rounded to fp16):
 * key scales are folded into q, value scales into the softmax weights, zero-points into fp32
 * bias terms. INT8 / INT4 with group <= 4 run on integer tensor-core MMAs (q * scale and
 * p * scale as exact-accumulated fixed point); FP8 and larger groups on fp16 MMAs (hi + lo
 * fp16 pairs). Built for head_dim 128 and group <= 8. No reference counterpart. */
int bpt_decode_kivi(const bpt_kivi_cache* cache,
                    const void* q, int64_t q_sb, int64_t q_sh,
                    const int32_t* block_table, int64_t bt_sb, const int32_t* seq_lens,
                    void* out, int64_t o_sb, int64_t o_sh,
                    int batch, int q_heads, int max_blocks,
                    float scale, int num_splits, int sm_count,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Stage 1 alone over a KIVI cache, as bpt_decode_fp16_partial. */
int bpt_decode_kivi_partial(const bpt_kivi_cache* cache,
                            const void* q, int64_t q_sb, int64_t q_sh,
                            const int32_t* block_table, int64_t bt_sb, const int32_t* seq_lens,
                            int batch, int q_heads, int max_blocks, float scale, int splits,
                            float* o_part, float* lse, unsigned* status, void* stream);

/* Size of the fixed scratch array behind bpt_decode_fp16_noalloc, per GPU. */
#define BPT_NOALLOC_SCRATCH_BYTES (8u * 1024u * 1024u)

/* bpt_decode_fp16 without a workspace argument, for callers that cannot allocate device
 * memory when they call (an engine that owns all device memory after start-up, a plugin
 * handed only its input and output buffers, code running where allocation is not allowed).
 * No counterpart in the reference. The split-KV partial states live in a fixed
 * BPT_NOALLOC_SCRATCH_BYTES array inside the library, reserved on each GPU that loads it until
 * the process exits; a call needing more (B * Hq * splits * (head_dim + 1) * 4 bytes, rounded)
 * returns BPT_ERR_WORKSPACE_TOO_SMALL without launching. Every call made outside stream
 * capture looks up the current device's array address (cudaGetSymbolAddress, with the device
 * current) and keeps it for calls being captured, so make the first call on a device before
 * any stream capture. All calls share the array: calls whose kernels overlap on the GPU race.
 * It allocates nothing and records no device-check flags: a block id outside [0, num_blocks)
 * reads page 0 instead and a too-long seq_len is cut at the table, with no error returned (the
 * kernels' own guards keep every access in bounds). Other arguments as bpt_decode_fp16. */
int bpt_decode_fp16_noalloc(const void* q, int64_t q_sb, int64_t q_sh,
                            const void* k_cache, int64_t k_sb, int64_t k_st, int64_t k_sh,
                            const void* v_cache, int64_t v_sb, int64_t v_st, int64_t v_sh,
                            int64_t num_blocks,
                            const int32_t* block_table, int64_t bt_sb,
                            const int32_t* seq_lens,
                            void* out, int64_t o_sb, int64_t o_sh,
                            int batch, int q_heads, int kv_heads, int head_dim,
                            int block_size, int max_blocks,
                            float scale, int num_splits, int sm_count, void* stream);

/* ---------------------------------------------------------------- sequence sharding
 *
 * Fused cross-GPU exchange for sequence-sharded decode (one process per GPU of one node; no
 * reference counterpart). Each rank allocates one receive buffer with bpt_seqx_alloc, sends
 * its IPC handle to the others (any out-of-band channel, e.g. an all-gather of the 64 bytes),
 * and maps theirs with bpt_seqx_open. Per call, after the split kernel wrote this rank's
 * partial states (bpt_decode_fp16_partial / bpt_decode_kivi_partial into o_part [B, Hq, S, D],
 * lse [B, Hq, S]), bpt_seqx_merge_fp16 merges the splits, stores the per-(sequence, q head)
 * state into every rank's buffer over NVLink (peer stores, no collective library), waits
 * (time-bounded, budget_us) for all ranks' states and writes the merged fp16 out [B, Hq, D] on
 * every rank. bufs[r] is rank r's buffer as mapped in this process (bufs[rank] = own). All
 * ranks must make the same sequence of calls with the same batch / q_heads / head_dim; a wait
 * that runs out sets BPT_DEV_WAIT_TIMEOUT in *status. head_dim % 4 == 0, <= 256; world <= 8.
 * A buffer serves one (world, batch, q_heads, head_dim). The first bpt_seqx_merge_fp16 call on
 * a device sizes the kernel's grid to what is resident on that device (an occupancy query);
 * make it before capturing the call in a CUDA graph. */
#define BPT_IPC_HANDLE_BYTES 64
size_t bpt_seqx_buffer_bytes(int world, int batch, int q_heads, int head_dim);
int bpt_seqx_alloc(size_t bytes, void** buf, void* ipc_handle);
int bpt_seqx_open(const void* ipc_handle, void** peer_buf);
int bpt_seqx_close(void* peer_buf);
int bpt_seqx_free(void* buf);
int bpt_seqx_merge_fp16(const float* o_part, const float* lse, int batch, int q_heads,
                        int head_dim, int splits, void* const* bufs, int world, int rank,
                        void* out, int64_t o_sb, int64_t o_sh, unsigned* status,
                        unsigned budget_us, void* stream);

/* Self-test of failure detection: launches one CTA that waits on a pipeline barrier nothing
 * completes, with a budget of budget_us microseconds (1 .. 1e6), on the decode kernels' own
 * bounded-wait code; it must give up and OR BPT_DEV_WAIT_TIMEOUT into *status (device
 * memory), leaving the CUDA context usable. No reference counterpart. */
int bpt_selftest_wait_timeout(unsigned* status, unsigned budget_us, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BPT_H_ */
