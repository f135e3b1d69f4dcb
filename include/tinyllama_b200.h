/*
 * tinyllama_b200.h — C ABI of the B200 (sm_100a) decode hot path.
 *
 * One shared library, libtinyllama_b200.so, exports every entry point below.
 * The signatures carry only plain pointers, sizes and enums: no torch or
 * pybind types cross this boundary, so the Python op modules (cscr.attention,
 * cscr.cache, cscr.pos_encoding), a ctypes/cffi binding or a C++ engine can
 * all bind it the same way.
 *
 * Conventions shared by every entry point
 *   - Device pointers belong to the device that is current on the calling
 *     thread; the caller selects it (cudaSetDevice / a device guard) first.
 *   - `stream` is a cudaStream_t passed as void*. NULL means the legacy
 *     default stream. All work is enqueued asynchronously on that stream;
 *     nothing synchronises the host.
 *   - The return value is a tlb_status. On failure tlb_last_error() returns
 *     a message for the calling thread (valid until its next call).
 *   - Element types are given by tlb_dtype. All tensors are dense row-major
 *     ("contiguous" in torch terms) unless a stride argument says otherwise.
 *   - Kernels never trap: inputs that the reference would read out of
 *     bounds (a block id outside the pool, a position beyond the cos/sin
 *     table, a slot outside the cache) are skipped and a bit is set in a
 *     per-device status word, readable with tlb_get_device_status().
 */
#ifndef TINYLLAMA_B200_H_
#define TINYLLAMA_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TLB_API __attribute__((visibility("default")))
#else
#define TLB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum tlb_status {
    TLB_OK = 0,
    TLB_ERR_INVALID_ARGUMENT = 1, /* shape / dtype / alignment check failed */
    TLB_ERR_UNSUPPORTED = 2,      /* valid request this build cannot serve */
    TLB_ERR_CUDA = 3,             /* a CUDA runtime call or launch failed */
    TLB_ERR_WORKSPACE = 4         /* workspace missing or too small */
} tlb_status;

typedef enum tlb_dtype {
    TLB_FLOAT32 = 0,
    TLB_FLOAT16 = 1,
    TLB_BFLOAT16 = 2,
    TLB_INT32 = 3,
    TLB_INT64 = 4
} tlb_dtype;

/* Bits of the per-device status word (tlb_get_device_status). */
#define TLB_STATUS_BAD_BLOCK_ID     0x1u  /* block id >= num_blocks in a block table */
#define TLB_STATUS_SEQ_TOO_LONG     0x2u  /* seq_len > max_blocks_per_seq * block_size */
#define TLB_STATUS_BAD_POSITION     0x4u  /* RoPE position outside the cos/sin table */
#define TLB_STATUS_BAD_SLOT         0x8u  /* slot / logical block outside the cache */
#define TLB_STATUS_WAIT_TIMEOUT     0x10u /* a bounded pipeline wait gave up */

/* Message describing the last failure on the calling thread ("" if none). */
TLB_API const char* tlb_last_error(void);

/* Library version string. */
TLB_API const char* tlb_version(void);

/* Reads (and, if clear != 0, resets) the status word of the current device.
 * Enqueued on `stream` and waits for it: a debugging aid, not a hot-path
 * call. When it reports TLB_STATUS_WAIT_TIMEOUT, the static scratch of
 * tlb_paged_attention_no_alloc on this device is cleared again before its next
 * use; a caller that owns an attention workspace must re-zero its counter
 * prefix itself (a kernel that gave up a wait may leave counters set). */
TLB_API int tlb_get_device_status(uint32_t* status_out, int clear, void* stream);

/* Bounded waits of the tensor-core attention kernels. Every wait of the
 * kernel's pipeline (a stage's data, a free stage, a hand-off between warps,
 * a phase of the merge) gives up after `tries` mbarrier probes, sets
 * TLB_STATUS_WAIT_TIMEOUT, lets the copies it already issued land and
 * returns; no kernel waits without bound. TLB_WAIT_LIMIT_DEFAULT (the value
 * in force until this is called) is far above any legitimate wait. Smaller
 * values are a failure-injection aid for tests (0: every such wait gives up
 * at once). Process-wide; applies to launches issued after the call. No
 * reference counterpart (the reference kernels do not wait). */
#define TLB_WAIT_LIMIT_DEFAULT (1u << 22)
TLB_API int tlb_attention_set_wait_limit(uint32_t tries);

/* ------------------------------------------------------------------------
 * Paged attention (decode: one query token per sequence).
 *
 * Replaces the pybind op `paged_attention(query, key_cache, value_cache,
 * block_tables, seq_lens, scale)` of cscr/attention.cpp:7-48 and its kernel
 * launch cscr/attention_kernel.cu:111-150.
 *
 *   out, query   : [num_seqs, num_heads, head_dim]            dtype
 *   key_cache    : [num_blocks, num_kv_heads, block_size, head_dim]  dtype
 *   value_cache  : same shape as key_cache                     dtype
 *   block_tables : [num_seqs, max_blocks_per_seq] int32 (entries < 0 skipped)
 *   seq_lens     : [num_seqs] int32
 *   dtype        : TLB_FLOAT32, TLB_FLOAT16 or TLB_BFLOAT16
 *
 * Query head h attends to KV head h / (num_heads / num_kv_heads). A sequence
 * whose length is <= 0, or whose blocks are all skipped, yields zeros.
 *
 * `workspace` is device scratch of at least the size that
 * tlb_paged_attention_workspace_size() returns for the same arguments
 * (256-byte aligned). Its first tlb_paged_attention_workspace_zeroed_bytes()
 * bytes (arrival counters) must be zero when the call starts; the call
 * leaves exactly that prefix zero again and writes partial results after it.
 * Successive calls on one stream can therefore share a buffer, re-zeroing
 * only when a call's prefix is longer than the previous call's (more
 * sequences * kv heads). Calls that overlap in time need separate buffers.
 * ---------------------------------------------------------------------- */
TLB_API int tlb_paged_attention_workspace_size(int64_t num_seqs, int64_t num_heads,
                                       int64_t num_kv_heads, int64_t head_dim,
                                       int dtype, size_t* bytes_out);

TLB_API int tlb_paged_attention_workspace_zeroed_bytes(int64_t num_seqs,
                                               int64_t num_kv_heads,
                                               size_t* bytes_out);

/* Flags of tlb_paged_attention. */
/* The kernel launched just before on `stream` writes neither block_tables
 * nor seq_lens (nor reads the output buffer): the attention kernel may then
 * start while that kernel finishes and read this metadata early
 * (programmatic dependent launch); query and cache are still read only after
 * it completes. Leave unset when the predecessor is unknown. */
#define TLB_ATTN_OVERLAP_PROLOGUE 0x1u

TLB_API int tlb_paged_attention(void* out, const void* query, const void* key_cache,
                        const void* value_cache, const int32_t* block_tables,
                        const int32_t* seq_lens, int64_t num_seqs,
                        int64_t num_heads, int64_t num_kv_heads,
                        int64_t head_dim, int64_t num_blocks,
                        int64_t block_size, int64_t max_blocks_per_seq,
                        float scale, int dtype, void* workspace,
                        size_t workspace_bytes, unsigned flags, void* stream);

/* ------------------------------------------------------------------------
 * Paged attention with no caller-provided workspace (no counterpart in the
 * reference, whose kernel needs no scratch).
 *
 * For callers that cannot allocate device memory: an engine that hands all
 * free memory to its KV pool after profiling (as the reference's worker sizes
 * the cache, src/worker/worker.py:31-81) has nothing left to allocate per
 * call, and a host that binds only this header may have no CUDA allocator.
 * Same arguments and results as tlb_paged_attention without the workspace:
 * the scratch is a fixed __device__ array of TLB_NO_ALLOC_SCRATCH_BYTES inside
 * the library, held by every GPU that loads it until the process exits.
 * Batches whose scratch would not fit are rejected (TLB_ERR_WORKSPACE).
 * The first call on a device looks the array up (cudaGetSymbolAddress) and
 * clears it with an async memset; make that first call outside any stream
 * capture. Calls share the array: calls whose kernels can overlap on the GPU
 * (unordered streams) race and must not be issued. Allocates nothing.
 * ---------------------------------------------------------------------- */
#define TLB_NO_ALLOC_SCRATCH_BYTES (16u << 20)

TLB_API int tlb_paged_attention_no_alloc(void* out, const void* query, const void* key_cache,
                        const void* value_cache, const int32_t* block_tables,
                        const int32_t* seq_lens, int64_t num_seqs,
                        int64_t num_heads, int64_t num_kv_heads,
                        int64_t head_dim, int64_t num_blocks,
                        int64_t block_size, int64_t max_blocks_per_seq,
                        float scale, int dtype, unsigned flags, void* stream);

/* ------------------------------------------------------------------------
 * The decode step in one launch: NeoX RoPE on the query and key, the KV-cache
 * write of the new token, and paged attention. It computes what
 *   tlb_rotary_embedding_neox_with_cache(positions = seq_lens - 1, ...,
 *       block_tables addressing, rot_dim = head_dim)
 * followed by tlb_paged_attention on the rotated query computes
 * (pos_encoding_kernel.cu:24-65, attention.py:96-116 and
 * attention_kernel.cu:24-150 in that order; attention.py:151-166 is the layer
 * that runs them), for a decode batch: one new token per sequence, at
 * position seq_lens[s] - 1, so that token's row lies in the sequence's last
 * block, which one CTA alone reads: that CTA rotates the key, stores it and
 * the value into the caches, and then loads the block.
 *
 *   query  : [num_seqs, num_heads, head_dim] raw (not rotated), not modified
 *   key    : [num_seqs, key_stride] raw key, rotated in place (as
 *            tlb_rotary_embedding_neox leaves it)
 *   value  : [num_seqs, value_stride]
 *   cos_sin_cache : [cache_rows, head_dim] (cos | sin halves), query dtype
 * Positions outside the table leave the vectors unrotated and set
 * TLB_STATUS_BAD_POSITION; block ids outside the pool skip the write (and
 * the read, TLB_STATUS_BAD_BLOCK_ID), negative ones skip both silently.
 * Tensor-core shapes only (fp16/bf16, head_dim 64 or 128, group <= 16,
 * block_size 8..64, 16-byte aligned tensors); others return
 * TLB_ERR_UNSUPPORTED and are served by the two calls above. Workspace and
 * flags as tlb_paged_attention (TLB_ATTN_OVERLAP_PROLOGUE: the kernel before
 * writes neither block_tables nor seq_lens nor the cos/sin table).
 * No reference counterpart: a fusion of the three reference steps.
 * ---------------------------------------------------------------------- */
TLB_API int tlb_paged_attention_with_rope(void* out, const void* query, void* key,
                        const void* value, void* key_cache, void* value_cache,
                        const int32_t* block_tables, const int32_t* seq_lens,
                        const void* cos_sin_cache, int64_t cache_rows,
                        int64_t num_seqs, int64_t num_heads, int64_t num_kv_heads,
                        int64_t head_dim, int64_t num_blocks, int64_t block_size,
                        int64_t max_blocks_per_seq, int64_t key_stride,
                        int64_t value_stride, float scale, int dtype, void* workspace,
                        size_t workspace_bytes, unsigned flags, void* stream);

/* ------------------------------------------------------------------------
 * Prefill (multi-token, causal) paged attention over prompt chunks.
 *
 * No reference counterpart: the reference layer accepts decode batches only
 * (src/model_executor/layers/attention.py:139-143). Chunk c holds the query
 * rows query_start[c] .. query_start[c + 1] - 1 of the packed `query`; they are
 * the last n_c = query_start[c + 1] - query_start[c] of the first
 * context_lens[c] tokens of the chunk's sequence, whose keys and values are
 * already in the paged cache. Row j attends to tokens 0 .. p of the sequence,
 * p = context_lens[c] - n_c + j (causal), with the decode op's rules: query
 * head h uses kv head h / (num_heads / num_kv_heads), negative block ids are
 * skipped, an empty softmax gives zeros (tests/test_paged_attention.py:42-57
 * with a causal mask is the definition).
 *
 *   out, query   : [num_tokens, num_heads, head_dim] (rows of all chunks)
 *   block_tables : [num_chunks, max_blocks_per_seq] int32
 *   query_start  : [num_chunks + 1] int32, non-decreasing
 *   context_lens : [num_chunks] int32
 *   max_query_len: >= every chunk's n_c (sizes the grid)
 * fp16 / bf16, head_dim 64 or 128, 16-byte aligned tensors. Rows of `out`
 * outside every chunk are not written.
 * ---------------------------------------------------------------------- */
TLB_API int tlb_paged_prefill_attention(void* out, const void* query, const void* key_cache,
                        const void* value_cache, const int32_t* block_tables,
                        const int32_t* query_start, const int32_t* context_lens,
                        int64_t num_chunks, int64_t num_heads, int64_t num_kv_heads,
                        int64_t head_dim, int64_t num_blocks, int64_t block_size,
                        int64_t max_blocks_per_seq, int64_t max_query_len, float scale,
                        int dtype, void* stream);

/* ------------------------------------------------------------------------
 * NeoX rotary embedding.
 *
 * Replaces `rotary_embedding_neox(postions, query, key, head_size,
 * cos_sin_cache)` of cscr/pos_encoding.cpp:7-18 and the launch
 * cscr/pos_encoding_kernel.cu:70-134.
 *
 *   positions     : [num_tokens] of pos_dtype (TLB_INT32 or TLB_INT64)
 *   query         : [num_tokens, num_heads * head_size]; row stride query_stride
 *   key           : [num_tokens, num_kv_heads * head_size]; rotated IN PLACE
 *   out           : [num_tokens, num_heads * head_size]; rotated query
 *   cos_sin_cache : [cache_rows, rot_dim]; cos in [:rot_dim/2], sin after
 *
 * Pairs (i, i + rot_dim/2), i < rot_dim/2, of each head are rotated:
 * x' = x cos - y sin, y' = y cos + x sin, in fp32 with each product and
 * the sum rounded on its own (no multiply-add), then rounded once to dtype.
 * Query elements at and beyond rot_dim are copied to `out` unchanged.
 * ---------------------------------------------------------------------- */
TLB_API int tlb_rotary_embedding_neox(void* out, const void* positions, int pos_dtype,
                              const void* query, void* key, int64_t num_tokens,
                              int64_t num_heads, int64_t num_kv_heads,
                              int64_t head_size, const void* cos_sin_cache,
                              int64_t cache_rows, int64_t rot_dim,
                              int64_t query_stride, int64_t key_stride,
                              int64_t out_stride, int dtype, void* stream);

/* ------------------------------------------------------------------------
 * KV-cache write ("reshape_and_cache").
 *
 * The reference writes new keys/values with torch advanced indexing in
 * PagedAttentionWithRoPE._write_kv_cache (src/model_executor/layers/
 * attention.py:82-116); it has no native op. This entry point is that step
 * as one kernel, addressed by a slot mapping:
 *
 *   key, value  : [num_tokens, num_kv_heads, head_size]; row strides
 *                 key_stride / value_stride (elements between tokens)
 *   key_cache, value_cache : [num_blocks, num_kv_heads, block_size, head_size]
 *   slots       : [num_tokens] of slot_dtype (TLB_INT32 or TLB_INT64);
 *                 slot = block * block_size + offset; slot < 0 skips the token
 *
 * Bit-exact copy; tokens whose slot is outside the cache are skipped and
 * flagged (TLB_STATUS_BAD_SLOT).
 * ---------------------------------------------------------------------- */
TLB_API int tlb_reshape_and_cache(const void* key, const void* value, void* key_cache,
                          void* value_cache, const void* slots, int slot_dtype,
                          int64_t num_tokens, int64_t num_kv_heads,
                          int64_t head_size, int64_t num_blocks,
                          int64_t block_size, int64_t key_stride,
                          int64_t value_stride, int dtype, void* stream);

/* The same write addressed exactly as _write_kv_cache addresses it
 * (attention.py:96-116): token r goes to block
 * block_tables[r, positions[r] / block_size], offset positions[r] %
 * block_size, and is skipped when that block id is negative. No host sync. */
TLB_API int tlb_write_kv_cache(const void* key, const void* value, void* key_cache,
                       void* value_cache, const void* positions, int pos_dtype,
                       const int32_t* block_tables, int64_t max_blocks_per_seq,
                       int64_t num_tokens, int64_t num_kv_heads,
                       int64_t head_size, int64_t num_blocks,
                       int64_t block_size, int64_t key_stride,
                       int64_t value_stride, int dtype, void* stream);

/* ------------------------------------------------------------------------
 * Fused NeoX RoPE + KV-cache write: one launch that does
 * tlb_rotary_embedding_neox (query -> out, key rotated in place) and then
 * writes the rotated key and `value` into the caches, without reading the
 * rotated key back. Same argument meaning as the calls it replaces
 * (pos_encoding_kernel.cu:24-65 followed by attention.py:96-116).
 * The destination comes from `slots` (as tlb_reshape_and_cache) when it is
 * non-null, otherwise from block_tables/positions (as tlb_write_kv_cache,
 * block_tables [num_tokens, max_blocks_per_seq] int32).
 * `value_stride` is in elements between tokens; key rows use key_stride.
 *
 * flags: TLB_ROPE_OVERLAP_PREVIOUS lets the launch begin while the kernel
 * before it on `stream` finishes (programmatic dependent launch): until that
 * kernel completes this one reads only positions, slots, block_tables and
 * cos_sin_cache and writes nothing. Set it only when the preceding kernel
 * does not write those four arrays (a QKV projection or an attention
 * launch do not); leave it unset when the predecessor is unknown.
 * ---------------------------------------------------------------------- */
#define TLB_ROPE_OVERLAP_PREVIOUS 0x1u

TLB_API int tlb_rotary_embedding_neox_with_cache(
    void* out, const void* positions, int pos_dtype, const void* query,
    void* key, const void* value, void* key_cache, void* value_cache,
    const void* slots, int slot_dtype, const int32_t* block_tables,
    int64_t max_blocks_per_seq, int64_t num_tokens, int64_t num_heads,
    int64_t num_kv_heads, int64_t head_size, const void* cos_sin_cache,
    int64_t cache_rows, int64_t rot_dim, int64_t num_blocks,
    int64_t block_size, int64_t query_stride, int64_t key_stride,
    int64_t value_stride, int64_t out_stride, int dtype, unsigned flags,
    void* stream);

/* ------------------------------------------------------------------------
 * Block copies (cscr/cache.cpp:94-151, cscr/cache_kernel.cu:124-212).
 *
 * `pairs` is HOST memory: num_pairs (src_block, dst_block) int64 pairs.
 * A block is `block_bytes` contiguous bytes; block b of a cache starts at
 * base + b * block_bytes.
 *
 * tlb_copy_blocks copies, inside each of the `num_caches` device caches
 * listed in `caches` (host array of device pointers: every layer's key and
 * value cache), block src -> dst for every pair, in ONE launch.
 *
 * tlb_swap_blocks copies block src of `src` to block dst of `dst`;
 * src_on_device / dst_on_device say where each lives (1 = current device,
 * 0 = host memory). Device<->device uses a kernel, host<->device one
 * cudaMemcpyAsync per run of consecutive blocks, host<->host memcpy.
 * ---------------------------------------------------------------------- */
TLB_API int tlb_copy_blocks(void* const* caches, int64_t num_caches,
                    const int64_t* pairs, int64_t num_pairs,
                    int64_t block_bytes, void* stream);

TLB_API int tlb_swap_blocks(const void* src, int src_on_device, void* dst,
                    int dst_on_device, const int64_t* pairs, int64_t num_pairs,
                    int64_t block_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Decode metadata on the device (src/worker/worker.py:139-159): for each
 * decode sequence r, position = context_len - 1 and
 * slot = block_tables[r, position / block_size] * block_size
 *        + position % block_size
 * (-1 when the context is empty or the block id is negative).
 *   context_lens : [num_seqs] int32; block_tables [num_seqs, max_blocks] int32
 *   positions_out: [num_seqs] int64; slots_out: [num_seqs] int64
 * ---------------------------------------------------------------------- */
TLB_API int tlb_decode_metadata(const int32_t* context_lens,
                        const int32_t* block_tables, int64_t num_seqs,
                        int64_t max_blocks_per_seq, int64_t block_size,
                        int64_t* positions_out, int64_t* slots_out,
                        void* stream);

/* ------------------------------------------------------------------------
 * Metadata of a packed continuous-batching step on the device
 * (src/worker/worker.py:84-169): the tokens of every prompt first, position i
 * of prompt p at slot prompt_tables[p, i / block_size] * block_size +
 * i % block_size (:111-124), then one token per decode sequence r at position
 * context_lens[r] - 1 with its slot as tlb_decode_metadata (:144-159).
 *   prompt_lens   : [num_prompts] int32 (num_prompts <= 4096)
 *   prompt_tables : [num_prompts, prompt_max_blocks] int32
 *   context_lens  : [num_decode] int32; decode_tables [num_decode,
 *                   decode_max_blocks] int32
 *   num_tokens    : sum(prompt_lens) + num_decode, the step's packed tokens
 *   positions_out, slots_out : [round_up(num_tokens, alignment)] int64
 * Entries past num_tokens hold position 0 (the worker pads its positions with
 * 0 to a multiple of 8, :163-164) and slot -1 (skipped by the cache writes).
 * A negative block id, or a position beyond its table, gives slot -1 (the
 * latter also sets TLB_STATUS_BAD_SLOT). No reference counterpart as a
 * native op: the worker computes these lists in Python and discards the
 * slots.
 * ---------------------------------------------------------------------- */
TLB_API int tlb_step_metadata(const int32_t* prompt_lens, const int32_t* prompt_tables,
                        int64_t num_prompts, int64_t prompt_max_blocks,
                        const int32_t* context_lens, const int32_t* decode_tables,
                        int64_t num_decode, int64_t decode_max_blocks,
                        int64_t block_size, int64_t num_tokens, int64_t alignment,
                        int64_t* positions_out, int64_t* slots_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TINYLLAMA_B200_H_ */
