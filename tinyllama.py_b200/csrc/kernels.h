// Internal launch interface between the C ABI (abi.cu) and the kernel files.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace tlb {

// Message returned by tlb_last_error() on this thread (defined in abi.cu).
void set_last_error(const char* msg);

// The argument checks and path choice of tlb_paged_attention, without
// launching (abi.cu). On TLB_OK, `total` is the workspace the call will use
// and `zeroed` the prefix that must be zero when it starts; both are 0 when
// the kernel that serves the call needs no workspace. No CUDA call beyond
// device and occupancy queries.
int attention_workspace_plan(const void* out, const void* query, const void* key_cache,
                             const void* value_cache, const int32_t* block_tables,
                             const int32_t* seq_lens, int64_t num_seqs, int64_t num_heads,
                             int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks,
                             int64_t block_size, int64_t max_blocks_per_seq, int dtype,
                             unsigned flags, size_t* total, size_t* zeroed);

// Marks the allocation-free entry point's static scratch on `dev` as not
// known to be zero (static_scratch.cu), so its next call clears it.
void no_alloc_scratch_dirty(int dev);

// ------------------------------------------------------------ attention
namespace attn {

constexpr int kConsumerWarps = 4;   // warps that run the mma / softmax
constexpr int kTileRows = 16;       // tokens per warp tile (mma k / n extent)
constexpr int kStageRows = kConsumerWarps * kTileRows;  // tokens per pipeline stage
constexpr int kGMax = 16;           // largest query-head group on the tensor-core path
#ifndef TLB_ATTN_CTAS_PER_SM
#define TLB_ATTN_CTAS_PER_SM 2
#endif
// Persistent grid: at most this many CTAs per SM (also sizes the workspace).
constexpr int kMaxCtasPerSm = TLB_ATTN_CTAS_PER_SM;
constexpr int kWorkspaceHeader = 256;
// Fewest context tokens (per kv head) a CTA of the tensor-core path is given
// before another CTA joins: below this, a split's merge costs more than the
// parallelism saves.
#ifndef TLB_ATTN_MIN_TOKENS
#define TLB_ATTN_MIN_TOKENS 128
#endif
// Work items per CTA of the grid the partial-result slots are sized for: one
// static range per CTA plus at most two tail chunks per CTA.
constexpr int kItemsPerCta = 3;

struct TcParams {
    void* out;
    const void* query;
    const int32_t* block_tables;
    const int32_t* seq_lens;
    float* ws_o;              // [2 * grid][gpad][head_dim] unnormalised partial outputs
    float* ws_ml;             // [2 * grid][gpad][2] (running max, running sum) per partial
    unsigned int* counters;   // [num_seqs * num_kv_heads] arrival counters (self-resetting)
    unsigned int* sched;      // [2] tail-chunk counter, finished-CTA counter (self-resetting)
    long long num_blocks;
    int num_seqs;
    int num_heads;
    int num_kv_heads;
    int group;                // num_heads / num_kv_heads
    int block_size;
    int max_blocks;
    int min_tokens;           // fewest tokens (per kv head) a CTA is given before more join
    float scale_log2;         // softmax scale * log2(e)
    unsigned wait_limit;      // mbarrier probes before a pipeline wait gives up
    // Fused decode step (cos_sin != nullptr): the new token of sequence s sits
    // at position seq_lens[s] - 1. `query` is then the raw query, rotated in
    // the kernel (NeoX, rot_dim == head_dim); the CTA that reads a sequence's
    // last block first writes that kv head's rotated key and its value into
    // the caches there (and the rotated key back into `key_new`).
    const void* cos_sin;      // [cache_rows, head_dim]: cos | sin halves
    long long cache_rows;
    void* key_new;            // [num_seqs, key_stride] raw key, rotated in place
    const void* value_new;    // [num_seqs, value_stride]
    long long key_stride;     // elements between tokens
    long long value_stride;
    void* key_cache;          // the caches, for the new rows' stores
    void* value_cache;
};

struct GenericParams {
    void* out;
    const void* query;
    const void* key_cache;
    const void* value_cache;
    const int32_t* block_tables;
    const int32_t* seq_lens;
    long long num_blocks;
    int num_seqs;
    int num_heads;
    int num_kv_heads;
    int group;
    int head_dim;
    int block_size;
    int max_blocks;
    float scale_log2;
};

// Returns true when the tensor-core path serves this shape / dtype.
bool tc_supported(int dtype, int head_dim, int group, int block_size);
// Heads per partial slot in the workspace for a group size.
int tc_gpad(int group);
// Number of CTAs the tensor-core kernel launches on `device` (persistent grid).
int tc_grid(int device, int dtype, int head_dim, int group, cudaError_t* err);

// `overlap`: launch with programmatic stream serialization (the kernel reads
// metadata before griddepcontrol.wait; see TLB_ATTN_OVERLAP_PROLOGUE).
cudaError_t launch_tc(int dtype, int head_dim, int group, const TcParams& p,
                      const CUtensorMap& tm_k, const CUtensorMap& tm_v, int grid, bool overlap,
                      cudaStream_t stream);
cudaError_t launch_generic(int dtype, const GenericParams& p, cudaStream_t stream);

}  // namespace attn

// ---------------------------------------------------- rope + cache writes
struct RopeCacheParams {
    void* out;                 // rotated query (may be null when no query work)
    const void* positions;
    const void* query;
    void* key;
    const void* value;
    void* key_cache;
    void* value_cache;
    const void* slots;         // slot mapping, or null with block_tables
    const int32_t* block_tables;
    const void* cos_sin;
    long long cache_rows;
    long long num_tokens;
    long long query_stride, key_stride, value_stride, out_stride;
    long long num_blocks;
    int max_blocks;
    int num_heads;
    int num_kv_heads;
    int head_size;
    int rot_dim;
    int block_size;
    int overlap;               // launched with programmatic stream serialization
};

// Rope only (query -> out, key in place).
cudaError_t launch_rope(int dtype, int pos_dtype, int vec, const RopeCacheParams& p,
                        cudaStream_t stream);
// Rope + write rotated key and value into the cache through `slots`, or
// through block_tables[t, pos / block_size] when by_block_table is set.
cudaError_t launch_rope_cache(int dtype, int pos_dtype, int slot_dtype, bool by_block_table,
                              int vec, const RopeCacheParams& p, cudaStream_t stream);
// Cache write only: `slots` (slot_dtype) or positions + block_tables.
cudaError_t launch_cache_write(int dtype, int index_dtype, bool by_block_table, int vec,
                               const RopeCacheParams& p, cudaStream_t stream);
cudaError_t launch_decode_metadata(const int32_t* context_lens, const int32_t* block_tables,
                                   long long num_seqs, int max_blocks, int block_size,
                                   int64_t* positions, int64_t* slots, cudaStream_t stream);

// Positions and slots of a packed step: prompts' tokens, then one token per
// decode sequence, padded to `num_padded` entries (step_metadata.cu).
constexpr int kStepMaxPrompts = 4096;
cudaError_t launch_step_metadata(const int32_t* prompt_lens, const int32_t* prompt_tables,
                                 int num_prompts, int prompt_max_blocks,
                                 const int32_t* context_lens, const int32_t* decode_tables,
                                 long long num_decode, int decode_max_blocks, int block_size,
                                 long long num_padded, int64_t* positions, int64_t* slots,
                                 cudaStream_t stream);

// Causal paged attention of prompt chunks (prefill_attention.cu).
cudaError_t launch_prefill_attention(int dtype, int head_dim, void* out, const void* query,
                                     const void* key_cache, const void* value_cache,
                                     const int32_t* block_tables, const int32_t* query_start,
                                     const int32_t* context_lens, long long num_blocks,
                                     int num_chunks, int num_heads, int num_kv_heads,
                                     int block_size, int max_blocks, int max_query_len,
                                     float scale_log2, const CUtensorMap* tm_k,
                                     const CUtensorMap* tm_v, cudaStream_t stream);
// Cache rows per TMA copy of the prefill kernel for this block size (a block,
// or a 64-row part of one), 0 when the block size needs the cp.async loader.
int prefill_box_rows(int block_size);

// ------------------------------------------------------------ block copies
constexpr int kCopyMaxCaches = 128;
constexpr int kCopyMaxPairs = 1024;
struct CopyParams {
    long long block_bytes;
    int num_caches;
    int num_pairs;
    char* dst[kCopyMaxCaches];
    const char* src[kCopyMaxCaches];
    long long pairs[2 * kCopyMaxPairs];
};
cudaError_t launch_copy_blocks(const CopyParams& p, bool vec16, cudaStream_t stream);

}  // namespace tlb
