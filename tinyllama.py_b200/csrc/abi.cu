// C ABI of libtinyllama_b200.so: argument checks, path selection, tensor-map
// encoding and launches. See include/tinyllama_b200.h for the contract.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "tinyllama_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace tlb {
__device__ unsigned int g_status = 0;
}

namespace {

thread_local std::string g_last_error;
// Probes before a pipeline wait of the attention kernels gives up
// (tlb_attention_set_wait_limit).
std::atomic<uint32_t> g_wait_limit{TLB_WAIT_LIMIT_DEFAULT};

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(TLB_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

#define TLB_REQUIRE(cond, ...)                                   \
    do {                                                         \
        if (!(cond)) return fail(TLB_ERR_INVALID_ARGUMENT, __VA_ARGS__); \
    } while (0)

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

inline int elem_bytes(int dtype) {
    switch (dtype) {
        case TLB_FLOAT32: return 4;
        case TLB_FLOAT16: return 2;
        case TLB_BFLOAT16: return 2;
        case TLB_INT32: return 4;
        case TLB_INT64: return 8;
        default: return 0;
    }
}
inline bool is_float(int dtype) {
    return dtype == TLB_FLOAT32 || dtype == TLB_FLOAT16 || dtype == TLB_BFLOAT16;
}
inline bool is_index(int dtype) { return dtype == TLB_INT32 || dtype == TLB_INT64; }

// ------------------------------------------------------------ tensor maps
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
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

struct MapKey {
    uintptr_t ptr;
    uint64_t rows;
    int head_dim;
    int box_rows;
    int box_chunks;
    bool operator==(const MapKey& o) const {
        return ptr == o.ptr && rows == o.rows && head_dim == o.head_dim &&
               box_rows == o.box_rows && box_chunks == o.box_chunks;
    }
};
struct MapKeyHash {
    size_t operator()(const MapKey& k) const {
        return std::hash<uintptr_t>()(k.ptr) ^ (std::hash<uint64_t>()(k.rows) * 31u) ^
               ((size_t)k.head_dim << 20) ^ ((size_t)k.box_rows << 40) ^
               ((size_t)k.box_chunks << 56);
    }
};

// A cache [rows = blocks * kv_heads * block_size, head_dim] of 16-bit elements
// viewed as a 3-D tensor {64 columns, rows, head_dim / 64 column chunks}
// (strides: a row, 128 bytes). A box holds box_rows rows of box_chunks chunks,
// stored in shared memory chunk-major: [chunk][box_rows rows][128 bytes],
// 128-byte swizzle, so every 8-row group of a chunk is one 1024-byte swizzle
// atom. The decode kernel takes one (block, kv head) tile with every chunk per
// box; the prefill kernel one chunk of it (its tiles keep a chunk's 64 rows
// together).
int kv_tensor_map(const void* base, uint64_t rows, int head_dim, int box_rows, int box_chunks,
                  CUtensorMap* out) {
    static std::mutex mu;
    static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
    const MapKey key{reinterpret_cast<uintptr_t>(base), rows, head_dim, box_rows, box_chunks};
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = cache.find(key);
        if (it != cache.end()) {
            *out = it->second;
            return TLB_OK;
        }
    }
    auto fn = encode_fn();
    if (fn == nullptr) return fail(TLB_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
    const cuuint32_t chunks = (cuuint32_t)(head_dim / 64);
    cuuint64_t dims[3] = {64, (cuuint64_t)rows, chunks};
    cuuint64_t strides[2] = {(cuuint64_t)head_dim * 2, 128};
    cuuint32_t box[3] = {64, (cuuint32_t)box_rows, (cuuint32_t)box_chunks};
    cuuint32_t estr[3] = {1, 1, 1};
    CUtensorMap m;
    CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(base), dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(TLB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    {
        std::lock_guard<std::mutex> lk(mu);
        if (cache.size() > 4096) cache.clear();
        cache.emplace(key, m);
    }
    *out = m;
    return TLB_OK;
}

// The same cache viewed as a 4-D tensor {64 columns, 8 rows, head_dim / 64
// chunks, rows / 8 groups of 8 rows} (strides: a row, 128 bytes, 8 rows): a
// box {64, 8, chunks, box_rows / 8} holds box_rows rows with every chunk,
// stored [8-row group][chunk][8 rows][128 bytes] with 128-byte swizzle (the
// prefill kernel's K / V tiles: one stride between 8-row groups whichever
// block they come from). rows and box_rows are multiples of 8.
int kv_group_tensor_map(const void* base, uint64_t rows, int head_dim, int box_rows,
                        CUtensorMap* out) {
    static std::mutex mu;
    static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
    const MapKey key{reinterpret_cast<uintptr_t>(base), rows, head_dim, box_rows, -1};
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = cache.find(key);
        if (it != cache.end()) {
            *out = it->second;
            return TLB_OK;
        }
    }
    auto fn = encode_fn();
    if (fn == nullptr) return fail(TLB_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
    const cuuint32_t chunks = (cuuint32_t)(head_dim / 64);
    cuuint64_t dims[4] = {64, 8, chunks, (cuuint64_t)(rows / 8)};
    cuuint64_t strides[3] = {(cuuint64_t)head_dim * 2, 128, (cuuint64_t)head_dim * 2 * 8};
    cuuint32_t box[4] = {64, 8, chunks, (cuuint32_t)(box_rows / 8)};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUtensorMap m;
    CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, const_cast<void*>(base), dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(TLB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    {
        std::lock_guard<std::mutex> lk(mu);
        if (cache.size() > 4096) cache.clear();
        cache.emplace(key, m);
    }
    *out = m;
    return TLB_OK;
}

int current_device(int* dev) {
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    return TLB_OK;
}

// Workspace layout of the tensor-core attention path.
struct WsLayout {
    size_t counters, ml, o, total, zeroed;
};
WsLayout ws_layout(int64_t num_seqs, int64_t num_kv_heads, int64_t head_dim, int gpad, int grid) {
    WsLayout w;
    w.counters = tlb::attn::kWorkspaceHeader;
    w.ml = w.counters + align_up((size_t)num_seqs * num_kv_heads * 4, 256);
    w.zeroed = w.ml;
    const size_t slots = (size_t)2 * tlb::attn::kItemsPerCta * grid;
    w.o = w.ml + align_up(slots * gpad * 2 * 4, 256);
    w.total = w.o + align_up(slots * gpad * head_dim * 4, 256);
    return w;
}

}  // namespace

void tlb::set_last_error(const char* msg) { g_last_error = msg ? msg : ""; }

extern "C" {

const char* tlb_last_error(void) { return g_last_error.c_str(); }

const char* tlb_version(void) { return "tinyllama_b200 0.1.0 (sm_100a)"; }

int tlb_attention_set_wait_limit(uint32_t tries) {
    g_wait_limit.store(tries, std::memory_order_relaxed);
    return TLB_OK;
}

int tlb_get_device_status(uint32_t* status_out, int clear, void* stream) {
    TLB_REQUIRE(status_out != nullptr, "status_out must not be null");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    unsigned int v = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(&v, tlb::g_status, sizeof(v), 0,
                                              cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess && clear) {
        static const unsigned int zero = 0;
        e = cudaMemcpyToSymbolAsync(tlb::g_status, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice,
                                    st);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "reading the device status word");
    if (v & TLB_STATUS_WAIT_TIMEOUT) {
        // A kernel that gave up a wait may have left arrival counters set in
        // its scratch: the library's own static scratch is cleared again
        // before its next use (caller-owned workspaces are the caller's).
        int dev = 0;
        if (cudaGetDevice(&dev) == cudaSuccess) tlb::no_alloc_scratch_dirty(dev);
    }
    *status_out = v;
    return TLB_OK;
}

// ------------------------------------------------------------ prefill
int tlb_paged_prefill_attention(void* out, const void* query, const void* key_cache,
                                const void* value_cache, const int32_t* block_tables,
                                const int32_t* query_start, const int32_t* context_lens,
                                int64_t num_chunks, int64_t num_heads, int64_t num_kv_heads,
                                int64_t head_dim, int64_t num_blocks, int64_t block_size,
                                int64_t max_blocks_per_seq, int64_t max_query_len, float scale,
                                int dtype, void* stream) {
    TLB_REQUIRE(dtype == TLB_FLOAT16 || dtype == TLB_BFLOAT16,
                "prefill attention supports float16 and bfloat16");
    TLB_REQUIRE(head_dim == 64 || head_dim == 128, "prefill attention supports head_dim 64 or 128");
    TLB_REQUIRE(num_chunks >= 0 && max_query_len >= 0, "counts must not be negative");
    TLB_REQUIRE(num_heads > 0 && num_kv_heads > 0 && num_blocks > 0 && block_size > 0 &&
                    max_blocks_per_seq > 0,
                "sizes must be positive");
    TLB_REQUIRE(num_heads % num_kv_heads == 0, "num_heads must be divisible by num_kv_heads");
    TLB_REQUIRE(num_chunks < 65536 && num_heads < 65536 && max_query_len < (1ll << 22) &&
                    max_blocks_per_seq * block_size < (1ll << 31),
                "sizes exceed the supported range");
    if (num_chunks == 0 || max_query_len == 0) return TLB_OK;
    TLB_REQUIRE(out && query && key_cache && value_cache && block_tables && query_start &&
                    context_lens,
                "tensor pointers must not be null");
    TLB_REQUIRE(aligned(out, 16) && aligned(query, 16) && aligned(key_cache, 16) &&
                    aligned(value_cache, 16),
                "query, out and the caches must be 16-byte aligned");
    // K and V tiles by TMA where a box can tile the blocks and every cache row
    // has a 32-bit coordinate; otherwise the kernel's cp.async loader
    CUtensorMap tk, tv;
    const CUtensorMap *ptk = nullptr, *ptv = nullptr;
    const int box_rows = tlb::prefill_box_rows((int)block_size);
    const long long rows = num_blocks * num_kv_heads * block_size;
    if (box_rows > 0 && rows < (1ll << 31) && num_blocks < (1ll << 31)) {
        if (int rc = kv_group_tensor_map(key_cache, (uint64_t)rows, (int)head_dim, box_rows, &tk))
            return rc;
        if (int rc = kv_group_tensor_map(value_cache, (uint64_t)rows, (int)head_dim, box_rows, &tv))
            return rc;
        ptk = &tk;
        ptv = &tv;
    }
    cudaError_t e = tlb::launch_prefill_attention(
        dtype, (int)head_dim, out, query, key_cache, value_cache, block_tables, query_start,
        context_lens, num_blocks, (int)num_chunks, (int)num_heads, (int)num_kv_heads,
        (int)block_size, (int)max_blocks_per_seq, (int)max_query_len,
        scale * 1.4426950408889634f, ptk, ptv, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "launching prefill attention");
    return TLB_OK;
}

// ------------------------------------------------------------ attention
int tlb_paged_attention_workspace_size(int64_t num_seqs, int64_t num_heads, int64_t num_kv_heads,
                                       int64_t head_dim, int dtype, size_t* bytes_out) {
    TLB_REQUIRE(bytes_out != nullptr, "bytes_out must not be null");
    TLB_REQUIRE(num_seqs > 0 && num_heads > 0 && num_kv_heads > 0 && head_dim > 0,
                "sizes must be positive");
    TLB_REQUIRE(num_heads % num_kv_heads == 0, "num_heads must be divisible by num_kv_heads");
    const int group = (int)(num_heads / num_kv_heads);
    // Block size does not change the workspace; any supported one answers.
    if (!tlb::attn::tc_supported(dtype, (int)head_dim, group, 16)) {
        *bytes_out = 0;
        return TLB_OK;
    }
    int dev;
    if (int rc = current_device(&dev)) return rc;
    cudaError_t e;
    const int grid = tlb::attn::tc_grid(dev, dtype, (int)head_dim, group, &e);
    if (grid <= 0) return cuda_fail(e, "sizing the attention grid");
    *bytes_out = ws_layout(num_seqs, num_kv_heads, head_dim, tlb::attn::tc_gpad(group), grid).total;
    return TLB_OK;
}

int tlb_paged_attention_workspace_zeroed_bytes(int64_t num_seqs, int64_t num_kv_heads,
                                               size_t* bytes_out) {
    TLB_REQUIRE(bytes_out != nullptr, "bytes_out must not be null");
    TLB_REQUIRE(num_seqs > 0 && num_kv_heads > 0, "sizes must be positive");
    *bytes_out = ws_layout(num_seqs, num_kv_heads, 64, 8, 1).zeroed;
    return TLB_OK;
}

namespace {
// The decode step's RoPE and cache write, folded into the attention launch.
struct FusedRope {
    const void* cos_sin;
    int64_t cache_rows;
    void* key;
    const void* value;
    int64_t key_stride, value_stride;
};

// Argument checks and path choice of a paged-attention call, before any
// launch. `ws` gets the workspace layout of the tensor-core path (all zero when
// the generic kernel serves the call: it uses no workspace).
struct AttnPlan {
    bool tc = false;
    int grid = 0;
    int gpad = 0;
    int group = 0;
    uint64_t rows = 0;
    WsLayout ws{};
};

int plan_attention(const void* out, const void* query, const void* key_cache,
                   const void* value_cache, const int32_t* block_tables, const int32_t* seq_lens,
                   int64_t num_seqs, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                   int64_t num_blocks, int64_t block_size, int64_t max_blocks_per_seq, int dtype,
                   unsigned flags, AttnPlan* pl) {
    TLB_REQUIRE(is_float(dtype), "dtype must be float16, bfloat16 or float32");
    TLB_REQUIRE((flags & ~TLB_ATTN_OVERLAP_PROLOGUE) == 0, "unknown flags");
    TLB_REQUIRE(num_seqs > 0, "query must contain at least one sequence");
    TLB_REQUIRE(num_heads > 0 && num_kv_heads > 0 && head_dim > 0 && num_blocks > 0 &&
                    block_size > 0 && max_blocks_per_seq > 0,
                "sizes must be positive");
    TLB_REQUIRE(num_heads % num_kv_heads == 0, "num_heads must be divisible by num_kv_heads");
    TLB_REQUIRE(head_dim <= 1024, "head_dim too large for the reference kernel");
    TLB_REQUIRE(out && query && key_cache && value_cache && block_tables && seq_lens,
                "tensor pointers must not be null");
    TLB_REQUIRE(num_seqs < (1ll << 31) && num_heads < (1 << 16) && max_blocks_per_seq < (1ll << 31),
                "sizes exceed the supported range");
    const int esz = elem_bytes(dtype);
    TLB_REQUIRE(aligned(query, esz) && aligned(out, esz) && aligned(key_cache, esz) &&
                    aligned(value_cache, esz),
                "tensor pointers must be aligned to the element size");
    pl->group = (int)(num_heads / num_kv_heads);
    pl->rows = (uint64_t)num_blocks * num_kv_heads * block_size;
    pl->tc = tlb::attn::tc_supported(dtype, (int)head_dim, pl->group, (int)block_size) &&
             aligned(query, 16) && aligned(key_cache, 16) && aligned(value_cache, 16) &&
             pl->rows < (1ull << 31);
    pl->ws = WsLayout{};
    if (!pl->tc) return TLB_OK;
    int dev;
    if (int rc = current_device(&dev)) return rc;
    cudaError_t e;
    pl->grid = tlb::attn::tc_grid(dev, dtype, (int)head_dim, pl->group, &e);
    if (pl->grid <= 0) return cuda_fail(e, "sizing the attention grid");
    pl->gpad = tlb::attn::tc_gpad(pl->group);
    pl->ws = ws_layout(num_seqs, num_kv_heads, head_dim, pl->gpad, pl->grid);
    return TLB_OK;
}

int attention_impl(void* out, const void* query, const void* key_cache,
                   const void* value_cache, const int32_t* block_tables,
                   const int32_t* seq_lens, int64_t num_seqs, int64_t num_heads,
                   int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks,
                   int64_t block_size, int64_t max_blocks_per_seq, float scale, int dtype,
                   void* workspace, size_t workspace_bytes, unsigned flags, void* stream,
                   const FusedRope* fr) {
    AttnPlan pl;
    if (int rc = plan_attention(out, query, key_cache, value_cache, block_tables, seq_lens,
                                num_seqs, num_heads, num_kv_heads, head_dim, num_blocks,
                                block_size, max_blocks_per_seq, dtype, flags, &pl))
        return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int group = pl.group;
    const float scale_log2 = scale * 1.4426950408889634f;
    const uint64_t rows = pl.rows;
    const bool tc = pl.tc;
    if (fr != nullptr && !(tc && aligned(fr->cos_sin, 16) && aligned(fr->key, 16) &&
                           aligned(fr->value, 16) && fr->key_stride % 8 == 0 &&
                           fr->value_stride % 8 == 0))
        return fail(TLB_ERR_UNSUPPORTED,
                    "the fused decode step needs the tensor-core path (fp16/bf16, head_dim 64 "
                    "or 128, group <= 16, block_size 8..64, 16-byte aligned tensors)");
    if (tc) {
        cudaError_t e;
        const int grid = pl.grid;
        const WsLayout& w = pl.ws;
        if (workspace == nullptr || workspace_bytes < w.total || !aligned(workspace, 256))
            return fail(TLB_ERR_WORKSPACE,
                        "paged_attention needs a 256-byte aligned workspace of %zu bytes (got %zu)",
                        w.total, workspace_bytes);
        CUtensorMap tk, tv;
        const int chunks = (int)head_dim / 64;
        if (int rc = kv_tensor_map(key_cache, rows, (int)head_dim, (int)block_size, chunks, &tk))
            return rc;
        if (int rc = kv_tensor_map(value_cache, rows, (int)head_dim, (int)block_size, chunks, &tv))
            return rc;
        tlb::attn::TcParams p{};
        char* ws = static_cast<char*>(workspace);
        p.out = out;
        p.query = query;
        p.block_tables = block_tables;
        p.seq_lens = seq_lens;
        p.ws_o = reinterpret_cast<float*>(ws + w.o);
        p.ws_ml = reinterpret_cast<float*>(ws + w.ml);
        p.counters = reinterpret_cast<unsigned int*>(ws + w.counters);
        p.sched = reinterpret_cast<unsigned int*>(ws);  // header: zeroed, self-resetting
        p.num_blocks = num_blocks;
        p.num_seqs = (int)num_seqs;
        p.num_heads = (int)num_heads;
        p.num_kv_heads = (int)num_kv_heads;
        p.group = group;
        p.block_size = (int)block_size;
        p.max_blocks = (int)max_blocks_per_seq;
        p.min_tokens = TLB_ATTN_MIN_TOKENS;
        p.scale_log2 = scale_log2;
        p.wait_limit = g_wait_limit.load(std::memory_order_relaxed);
        // the caches (the fused step stores the new rows there)
        p.key_cache = const_cast<void*>(key_cache);
        p.value_cache = const_cast<void*>(value_cache);
        if (fr != nullptr) {
            p.cos_sin = fr->cos_sin;
            p.cache_rows = fr->cache_rows;
            p.key_new = fr->key;
            p.value_new = fr->value;
            p.key_stride = fr->key_stride;
            p.value_stride = fr->value_stride;
        }
        e = tlb::attn::launch_tc(dtype, (int)head_dim, group, p, tk, tv, grid,
                                 (flags & TLB_ATTN_OVERLAP_PROLOGUE) != 0, st);
        if (e != cudaSuccess) return cuda_fail(e, "launching paged attention");
        return TLB_OK;
    }
    tlb::attn::GenericParams g;
    g.out = out;
    g.query = query;
    g.key_cache = key_cache;
    g.value_cache = value_cache;
    g.block_tables = block_tables;
    g.seq_lens = seq_lens;
    g.num_blocks = num_blocks;
    g.num_seqs = (int)num_seqs;
    g.num_heads = (int)num_heads;
    g.num_kv_heads = (int)num_kv_heads;
    g.group = group;
    g.head_dim = (int)head_dim;
    g.block_size = (int)block_size;
    g.max_blocks = (int)max_blocks_per_seq;
    g.scale_log2 = scale_log2;
    cudaError_t e = tlb::attn::launch_generic(dtype, g, st);
    if (e != cudaSuccess) return cuda_fail(e, "launching paged attention");
    return TLB_OK;
}
}  // namespace

}  // extern "C"

int tlb::attention_workspace_plan(const void* out, const void* query, const void* key_cache,
                                  const void* value_cache, const int32_t* block_tables,
                                  const int32_t* seq_lens, int64_t num_seqs, int64_t num_heads,
                                  int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks,
                                  int64_t block_size, int64_t max_blocks_per_seq, int dtype,
                                  unsigned flags, size_t* total, size_t* zeroed) {
    AttnPlan pl;
    if (int rc = plan_attention(out, query, key_cache, value_cache, block_tables, seq_lens,
                                num_seqs, num_heads, num_kv_heads, head_dim, num_blocks,
                                block_size, max_blocks_per_seq, dtype, flags, &pl))
        return rc;
    *total = pl.ws.total;
    *zeroed = pl.ws.zeroed;
    return TLB_OK;
}

extern "C" {

int tlb_paged_attention(void* out, const void* query, const void* key_cache,
                        const void* value_cache, const int32_t* block_tables,
                        const int32_t* seq_lens, int64_t num_seqs, int64_t num_heads,
                        int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks,
                        int64_t block_size, int64_t max_blocks_per_seq, float scale, int dtype,
                        void* workspace, size_t workspace_bytes, unsigned flags,
                        void* stream) {
    return attention_impl(out, query, key_cache, value_cache, block_tables, seq_lens, num_seqs,
                          num_heads, num_kv_heads, head_dim, num_blocks, block_size,
                          max_blocks_per_seq, scale, dtype, workspace, workspace_bytes, flags,
                          stream, nullptr);
}

int tlb_paged_attention_with_rope(void* out, const void* query, void* key, const void* value,
                                  void* key_cache, void* value_cache,
                                  const int32_t* block_tables, const int32_t* seq_lens,
                                  const void* cos_sin_cache, int64_t cache_rows,
                                  int64_t num_seqs, int64_t num_heads, int64_t num_kv_heads,
                                  int64_t head_dim, int64_t num_blocks, int64_t block_size,
                                  int64_t max_blocks_per_seq, int64_t key_stride,
                                  int64_t value_stride, float scale, int dtype, void* workspace,
                                  size_t workspace_bytes, unsigned flags, void* stream) {
    TLB_REQUIRE(key && value && cos_sin_cache, "tensor pointers must not be null");
    TLB_REQUIRE(cache_rows > 0, "cos_sin_cache must have at least one row");
    TLB_REQUIRE(key_stride >= num_kv_heads * head_dim && value_stride >= num_kv_heads * head_dim,
                "key / value rows are shorter than num_kv_heads * head_dim");
    const int esz = is_float(dtype) ? elem_bytes(dtype) : 1;
    TLB_REQUIRE(aligned(key, esz) && aligned(value, esz) && aligned(cos_sin_cache, esz),
                "tensor pointers must be aligned to the element size");
    const FusedRope fr{cos_sin_cache, cache_rows, key, value, key_stride, value_stride};
    return attention_impl(out, query, key_cache, value_cache, block_tables, seq_lens, num_seqs,
                          num_heads, num_kv_heads, head_dim, num_blocks, block_size,
                          max_blocks_per_seq, scale, dtype, workspace, workspace_bytes, flags,
                          stream, &fr);
}

// ---------------------------------------------------------------- rope etc.
namespace {

int rope_checks(const void* positions, int pos_dtype, int64_t num_tokens, int64_t num_heads,
                int64_t num_kv_heads, int64_t head_size, const void* cos_sin_cache,
                int64_t cache_rows, int64_t rot_dim, int dtype) {
    TLB_REQUIRE(is_float(dtype), "dtype must be float16, bfloat16 or float32");
    TLB_REQUIRE(is_index(pos_dtype), "positions must be int32 or int64");
    TLB_REQUIRE(num_tokens > 0, "positions must contain at least one token");
    TLB_REQUIRE(head_size > 0, "head_size must be positive");
    TLB_REQUIRE(num_heads >= 0 && num_kv_heads >= 0, "head counts must not be negative");
    TLB_REQUIRE(rot_dim > 0 && rot_dim % 2 == 0, "rotary dimension must be even and positive");
    TLB_REQUIRE(rot_dim <= head_size, "rotary dimension must not exceed head_size");
    TLB_REQUIRE(cache_rows > 0, "cos_sin_cache must have at least one row");
    TLB_REQUIRE(positions && cos_sin_cache, "tensor pointers must not be null");
    return TLB_OK;
}

// 16-byte vectors when every pointer and every row/head offset allows them.
int pick_vec(int dtype, int64_t head_size, int64_t rot_dim, std::initializer_list<int64_t> strides,
             std::initializer_list<const void*> ptrs) {
    const int v = 16 / elem_bytes(dtype);
    if (head_size % v || (rot_dim / 2) % v) return 1;
    for (int64_t s : strides)
        if (s % v) return 1;
    for (const void* p : ptrs)
        if (p && !aligned(p, 16)) return 1;
    return v;
}

}  // namespace

int tlb_rotary_embedding_neox(void* out, const void* positions, int pos_dtype, const void* query,
                              void* key, int64_t num_tokens, int64_t num_heads,
                              int64_t num_kv_heads, int64_t head_size, const void* cos_sin_cache,
                              int64_t cache_rows, int64_t rot_dim, int64_t query_stride,
                              int64_t key_stride, int64_t out_stride, int dtype, void* stream) {
    if (int rc = rope_checks(positions, pos_dtype, num_tokens, num_heads, num_kv_heads, head_size,
                             cos_sin_cache, cache_rows, rot_dim, dtype))
        return rc;
    TLB_REQUIRE(num_heads == 0 || (out && query), "query/out pointers must not be null");
    TLB_REQUIRE(num_kv_heads == 0 || key, "key pointer must not be null");
    tlb::RopeCacheParams p{};
    p.out = out;
    p.positions = positions;
    p.query = query;
    p.key = key;
    p.cos_sin = cos_sin_cache;
    p.cache_rows = cache_rows;
    p.num_tokens = num_tokens;
    p.query_stride = query_stride;
    p.key_stride = key_stride;
    p.out_stride = out_stride;
    p.num_heads = (int)num_heads;
    p.num_kv_heads = (int)num_kv_heads;
    p.head_size = (int)head_size;
    p.rot_dim = (int)rot_dim;
    p.block_size = 1;
    const int vec = pick_vec(dtype, head_size, rot_dim, {query_stride, key_stride, out_stride},
                             {out, query, key, cos_sin_cache});
    cudaError_t e = tlb::launch_rope(dtype, pos_dtype, vec, p, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "launching rotary_embedding_neox");
    return TLB_OK;
}

namespace {
int cache_checks(const void* key_cache, const void* value_cache, int64_t num_tokens,
                 int64_t num_kv_heads, int64_t head_size, int64_t num_blocks, int64_t block_size,
                 int dtype) {
    TLB_REQUIRE(is_float(dtype), "dtype must be float16, bfloat16 or float32");
    TLB_REQUIRE(num_tokens >= 0, "num_tokens must not be negative");
    TLB_REQUIRE(num_kv_heads > 0 && head_size > 0 && num_blocks > 0 && block_size > 0,
                "cache sizes must be positive");
    TLB_REQUIRE(key_cache && value_cache, "cache pointers must not be null");
    return TLB_OK;
}
}  // namespace

int tlb_reshape_and_cache(const void* key, const void* value, void* key_cache, void* value_cache,
                          const void* slots, int slot_dtype, int64_t num_tokens,
                          int64_t num_kv_heads, int64_t head_size, int64_t num_blocks,
                          int64_t block_size, int64_t key_stride, int64_t value_stride, int dtype,
                          void* stream) {
    if (int rc = cache_checks(key_cache, value_cache, num_tokens, num_kv_heads, head_size,
                              num_blocks, block_size, dtype))
        return rc;
    TLB_REQUIRE(is_index(slot_dtype), "slot_mapping must be int32 or int64");
    if (num_tokens == 0) return TLB_OK;
    TLB_REQUIRE(key && value && slots, "tensor pointers must not be null");
    tlb::RopeCacheParams p{};
    p.key = const_cast<void*>(key);
    p.value = value;
    p.key_cache = key_cache;
    p.value_cache = value_cache;
    p.slots = slots;
    p.num_tokens = num_tokens;
    p.key_stride = key_stride;
    p.value_stride = value_stride;
    p.num_blocks = num_blocks;
    p.num_kv_heads = (int)num_kv_heads;
    p.head_size = (int)head_size;
    p.rot_dim = 0;
    p.block_size = (int)block_size;
    const int vec = pick_vec(dtype, head_size, 0, {key_stride, value_stride},
                             {key, value, key_cache, value_cache});
    cudaError_t e = tlb::launch_cache_write(dtype, slot_dtype, false, vec, p,
                                            reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "launching reshape_and_cache");
    return TLB_OK;
}

int tlb_write_kv_cache(const void* key, const void* value, void* key_cache, void* value_cache,
                       const void* positions, int pos_dtype, const int32_t* block_tables,
                       int64_t max_blocks_per_seq, int64_t num_tokens, int64_t num_kv_heads,
                       int64_t head_size, int64_t num_blocks, int64_t block_size,
                       int64_t key_stride, int64_t value_stride, int dtype, void* stream) {
    if (int rc = cache_checks(key_cache, value_cache, num_tokens, num_kv_heads, head_size,
                              num_blocks, block_size, dtype))
        return rc;
    TLB_REQUIRE(is_index(pos_dtype), "positions must be int32 or int64");
    TLB_REQUIRE(max_blocks_per_seq > 0, "block_tables must have at least one column");
    if (num_tokens == 0) return TLB_OK;
    TLB_REQUIRE(key && value && positions && block_tables, "tensor pointers must not be null");
    tlb::RopeCacheParams p{};
    p.key = const_cast<void*>(key);
    p.value = value;
    p.key_cache = key_cache;
    p.value_cache = value_cache;
    p.positions = positions;
    p.block_tables = block_tables;
    p.max_blocks = (int)max_blocks_per_seq;
    p.num_tokens = num_tokens;
    p.key_stride = key_stride;
    p.value_stride = value_stride;
    p.num_blocks = num_blocks;
    p.num_kv_heads = (int)num_kv_heads;
    p.head_size = (int)head_size;
    p.rot_dim = 0;
    p.block_size = (int)block_size;
    const int vec = pick_vec(dtype, head_size, 0, {key_stride, value_stride},
                             {key, value, key_cache, value_cache});
    cudaError_t e = tlb::launch_cache_write(dtype, pos_dtype, true, vec, p,
                                            reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "launching write_kv_cache");
    return TLB_OK;
}

int tlb_rotary_embedding_neox_with_cache(
    void* out, const void* positions, int pos_dtype, const void* query, void* key,
    const void* value, void* key_cache, void* value_cache, const void* slots, int slot_dtype,
    const int32_t* block_tables, int64_t max_blocks_per_seq, int64_t num_tokens, int64_t num_heads, int64_t num_kv_heads, int64_t head_size,
    const void* cos_sin_cache, int64_t cache_rows, int64_t rot_dim, int64_t num_blocks,
    int64_t block_size, int64_t query_stride, int64_t key_stride, int64_t value_stride,
    int64_t out_stride, int dtype, unsigned flags, void* stream) {
    if (int rc = rope_checks(positions, pos_dtype, num_tokens, num_heads, num_kv_heads, head_size,
                             cos_sin_cache, cache_rows, rot_dim, dtype))
        return rc;
    TLB_REQUIRE((flags & ~TLB_ROPE_OVERLAP_PREVIOUS) == 0, "unknown flags");
    if (int rc = cache_checks(key_cache, value_cache, num_tokens, num_kv_heads, head_size,
                              num_blocks, block_size, dtype))
        return rc;
    const bool by_table = slots == nullptr;
    if (by_table) {
        TLB_REQUIRE(block_tables != nullptr && max_blocks_per_seq > 0,
                    "either slots or block_tables must be given");
    } else {
        TLB_REQUIRE(is_index(slot_dtype), "slot_mapping must be int32 or int64");
    }
    TLB_REQUIRE(out && query && key && value, "tensor pointers must not be null");
    tlb::RopeCacheParams p{};
    p.block_tables = block_tables;
    p.max_blocks = (int)max_blocks_per_seq;
    p.out = out;
    p.positions = positions;
    p.query = query;
    p.key = key;
    p.value = value;
    p.key_cache = key_cache;
    p.value_cache = value_cache;
    p.slots = slots;
    p.cos_sin = cos_sin_cache;
    p.cache_rows = cache_rows;
    p.num_tokens = num_tokens;
    p.query_stride = query_stride;
    p.key_stride = key_stride;
    p.value_stride = value_stride;
    p.out_stride = out_stride;
    p.num_blocks = num_blocks;
    p.num_heads = (int)num_heads;
    p.num_kv_heads = (int)num_kv_heads;
    p.head_size = (int)head_size;
    p.rot_dim = (int)rot_dim;
    p.block_size = (int)block_size;
    p.overlap = (flags & TLB_ROPE_OVERLAP_PREVIOUS) ? 1 : 0;
    const int vec =
        pick_vec(dtype, head_size, rot_dim, {query_stride, key_stride, value_stride, out_stride},
                 {out, query, key, value, key_cache, value_cache, cos_sin_cache});
    cudaError_t e = tlb::launch_rope_cache(dtype, pos_dtype, by_table ? TLB_INT64 : slot_dtype,
                                           by_table, vec, p,
                                           reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "launching rotary_embedding_neox_with_cache");
    return TLB_OK;
}

int tlb_decode_metadata(const int32_t* context_lens, const int32_t* block_tables,
                        int64_t num_seqs, int64_t max_blocks_per_seq, int64_t block_size,
                        int64_t* positions_out, int64_t* slots_out, void* stream) {
    TLB_REQUIRE(num_seqs >= 0 && max_blocks_per_seq > 0 && block_size > 0,
                "sizes must be positive");
    if (num_seqs == 0) return TLB_OK;
    TLB_REQUIRE(context_lens && block_tables && positions_out && slots_out,
                "tensor pointers must not be null");
    cudaError_t e = tlb::launch_decode_metadata(context_lens, block_tables, num_seqs,
                                                (int)max_blocks_per_seq, (int)block_size,
                                                positions_out, slots_out,
                                                reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "launching decode_metadata");
    return TLB_OK;
}

int tlb_step_metadata(const int32_t* prompt_lens, const int32_t* prompt_tables,
                      int64_t num_prompts, int64_t prompt_max_blocks,
                      const int32_t* context_lens, const int32_t* decode_tables,
                      int64_t num_decode, int64_t decode_max_blocks, int64_t block_size,
                      int64_t num_tokens, int64_t alignment, int64_t* positions_out,
                      int64_t* slots_out, void* stream) {
    TLB_REQUIRE(num_prompts >= 0 && num_decode >= 0 && num_tokens >= 0,
                "counts must not be negative");
    TLB_REQUIRE(num_prompts <= tlb::kStepMaxPrompts, "at most %d prompts per step",
                tlb::kStepMaxPrompts);
    TLB_REQUIRE(block_size > 0 && alignment > 0, "block_size and alignment must be positive");
    TLB_REQUIRE(num_prompts == 0 || (prompt_lens && prompt_tables && prompt_max_blocks > 0),
                "prompt_lens and prompt_tables are required when there are prompts");
    TLB_REQUIRE(num_decode == 0 || (context_lens && decode_tables && decode_max_blocks > 0),
                "context_lens and decode_tables are required when there are decode sequences");
    TLB_REQUIRE(num_tokens >= num_decode, "num_tokens must count every decode token");
    TLB_REQUIRE(prompt_max_blocks < (1ll << 31) && decode_max_blocks < (1ll << 31) &&
                    block_size < (1ll << 31),
                "sizes exceed the supported range");
    const int64_t padded = (num_tokens + alignment - 1) / alignment * alignment;
    TLB_REQUIRE(padded == 0 || (positions_out && slots_out), "output pointers must not be null");
    cudaError_t e = tlb::launch_step_metadata(
        prompt_lens, prompt_tables, (int)num_prompts, (int)prompt_max_blocks, context_lens,
        decode_tables, num_decode, (int)decode_max_blocks, (int)block_size, padded,
        positions_out, slots_out, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "launching step_metadata");
    return TLB_OK;
}

// ------------------------------------------------------------ block copies
int tlb_copy_blocks(void* const* caches, int64_t num_caches, const int64_t* pairs,
                    int64_t num_pairs, int64_t block_bytes, void* stream) {
    TLB_REQUIRE(num_caches >= 0 && num_pairs >= 0, "counts must not be negative");
    if (num_caches == 0 || num_pairs == 0) return TLB_OK;
    TLB_REQUIRE(caches && pairs, "caches and pairs must not be null");
    TLB_REQUIRE(block_bytes > 0, "block_bytes must be positive");
    bool vec16 = block_bytes % 16 == 0;
    for (int64_t c = 0; c < num_caches; ++c) {
        TLB_REQUIRE(caches[c] != nullptr, "cache pointer %lld is null", (long long)c);
        if (!aligned(caches[c], 16)) vec16 = false;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    tlb::CopyParams p;
    p.block_bytes = block_bytes;
    for (int64_t c0 = 0; c0 < num_caches; c0 += tlb::kCopyMaxCaches) {
        p.num_caches = (int)std::min<int64_t>(tlb::kCopyMaxCaches, num_caches - c0);
        for (int c = 0; c < p.num_caches; ++c) {
            p.dst[c] = static_cast<char*>(caches[c0 + c]);
            p.src[c] = static_cast<const char*>(caches[c0 + c]);
        }
        for (int64_t k0 = 0; k0 < num_pairs; k0 += tlb::kCopyMaxPairs) {
            p.num_pairs = (int)std::min<int64_t>(tlb::kCopyMaxPairs, num_pairs - k0);
            std::memcpy(p.pairs, pairs + 2 * k0, sizeof(int64_t) * 2 * p.num_pairs);
            cudaError_t e = tlb::launch_copy_blocks(p, vec16, st);
            if (e != cudaSuccess) return cuda_fail(e, "launching copy_blocks");
        }
    }
    return TLB_OK;
}

int tlb_swap_blocks(const void* src, int src_on_device, void* dst, int dst_on_device,
                    const int64_t* pairs, int64_t num_pairs, int64_t block_bytes, void* stream) {
    TLB_REQUIRE(num_pairs >= 0, "num_pairs must not be negative");
    if (num_pairs == 0) return TLB_OK;
    TLB_REQUIRE(src && dst && pairs, "pointers must not be null");
    TLB_REQUIRE(block_bytes > 0, "block_bytes must be positive");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const char* s = static_cast<const char*>(src);
    char* d = static_cast<char*>(dst);
    if (!src_on_device && !dst_on_device) {
        for (int64_t k = 0; k < num_pairs; ++k)
            std::memcpy(d + pairs[2 * k + 1] * block_bytes, s + pairs[2 * k] * block_bytes,
                        (size_t)block_bytes);
        return TLB_OK;
    }
    if (src_on_device && dst_on_device) {
        tlb::CopyParams p;
        p.block_bytes = block_bytes;
        p.num_caches = 1;
        p.dst[0] = d;
        p.src[0] = s;
        const bool vec16 = block_bytes % 16 == 0 && aligned(src, 16) && aligned(dst, 16);
        for (int64_t k0 = 0; k0 < num_pairs; k0 += tlb::kCopyMaxPairs) {
            p.num_pairs = (int)std::min<int64_t>(tlb::kCopyMaxPairs, num_pairs - k0);
            std::memcpy(p.pairs, pairs + 2 * k0, sizeof(int64_t) * 2 * p.num_pairs);
            cudaError_t e = tlb::launch_copy_blocks(p, vec16, st);
            if (e != cudaSuccess) return cuda_fail(e, "launching swap_blocks");
        }
        return TLB_OK;
    }
    // Host <-> device: one copy per run of consecutive blocks.
    const cudaMemcpyKind kind = src_on_device ? cudaMemcpyDeviceToHost : cudaMemcpyHostToDevice;
    int64_t k = 0;
    while (k < num_pairs) {
        int64_t run = 1;
        while (k + run < num_pairs && pairs[2 * (k + run)] == pairs[2 * k] + run &&
               pairs[2 * (k + run) + 1] == pairs[2 * k + 1] + run)
            ++run;
        cudaError_t e = cudaMemcpyAsync(d + pairs[2 * k + 1] * block_bytes,
                                        s + pairs[2 * k] * block_bytes,
                                        (size_t)(run * block_bytes), kind, st);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync in swap_blocks");
        k += run;
    }
    return TLB_OK;
}

}  // extern "C"
