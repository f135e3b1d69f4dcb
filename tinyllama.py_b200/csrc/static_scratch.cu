// Paged attention for callers that cannot allocate device memory.
//
// The attention kernel needs scratch (arrival counters and fp32 partial
// results of sequences split across CTAs). tlb_paged_attention takes it from
// the caller. Some callers cannot provide it: an engine that sizes its KV
// pool to fill the GPU (as the reference's worker does, handing every free
// byte after profiling to the cache) has nothing left to allocate from per
// call; a host that binds only the C header has no CUDA allocator at all.
// tlb_paged_attention_no_alloc serves them from one fixed array in device
// memory, declared below, and never allocates.
//
// The array is a file-scope __device__ variable: every GPU that loads this
// library holds kNoAllocScratchBytes of it until the process exits. In host
// code its name is only a host-side stand-in, never a device address, so the
// device address is looked up once per device with cudaGetSymbolAddress (with
// that device current) and cached. All calls on a device share the array:
// calls whose kernels overlap on the GPU (different streams, no ordering
// between them) race on it and must not be issued.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "tinyllama_b200.h"

namespace {

constexpr size_t kNoAllocScratchBytes = TLB_NO_ALLOC_SCRATCH_BYTES;

static __device__ __align__(256) unsigned char g_no_alloc_scratch[kNoAllocScratchBytes];

struct DeviceScratch {
    void* ptr = nullptr;   // device address of g_no_alloc_scratch on this device
    size_t clean = 0;      // leading bytes known to be zero when no call is in flight
};
std::mutex g_mu;
DeviceScratch g_dev[64];

int set_error(int code, const char* msg) {
    tlb::set_last_error(msg);
    return code;
}

}  // namespace

// Forget which prefix of the array is zero on `dev`: the next call clears it.
// Called when a launch failed or a bounded wait inside a kernel gave up (a
// kernel that stopped early may leave arrival counters set).
void tlb::no_alloc_scratch_dirty(int dev) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (dev >= 0 && dev < 64) g_dev[dev].clean = 0;
}

extern "C" int tlb_paged_attention_no_alloc(
    void* out, const void* query, const void* key_cache, const void* value_cache,
    const int32_t* block_tables, const int32_t* seq_lens, int64_t num_seqs, int64_t num_heads,
    int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks, int64_t block_size,
    int64_t max_blocks_per_seq, float scale, int dtype, unsigned flags, void* stream) {
    // Every argument check of tlb_paged_attention first, and the scratch this
    // call will really use (none when the kernel serving it needs none).
    size_t need = 0, zeroed = 0;
    if (int rc = tlb::attention_workspace_plan(out, query, key_cache, value_cache, block_tables,
                                               seq_lens, num_seqs, num_heads, num_kv_heads,
                                               head_dim, num_blocks, block_size,
                                               max_blocks_per_seq, dtype, flags, &need, &zeroed))
        return rc;
    if (need > kNoAllocScratchBytes || zeroed > kNoAllocScratchBytes) {
        char buf[200];
        snprintf(buf, sizeof(buf),
                 "paged_attention_no_alloc: this batch needs %zu bytes of scratch, more than "
                 "the %zu-byte static buffer (fewer sequences per call fit)",
                 need > zeroed ? need : zeroed, kNoAllocScratchBytes);
        return set_error(TLB_ERR_WORKSPACE, buf);
    }
    if (need == 0)  // served by the kernel that uses no scratch: nothing to set up
        return tlb_paged_attention(out, query, key_cache, value_cache, block_tables, seq_lens,
                                   num_seqs, num_heads, num_kv_heads, head_dim, num_blocks,
                                   block_size, max_blocks_per_seq, scale, dtype, nullptr, 0,
                                   flags, stream);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return set_error(TLB_ERR_CUDA, "paged_attention_no_alloc: no current CUDA device");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &capturing) != cudaSuccess)
        return set_error(TLB_ERR_CUDA, "paged_attention_no_alloc: cudaStreamIsCapturing failed");
    void* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        DeviceScratch& d = g_dev[dev];
        if (d.ptr == nullptr) {
            // First call on this device: find the array's device address.
            // (Make this first call outside any stream capture.)
            void* p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_no_alloc_scratch);
            if (e != cudaSuccess || p == nullptr)
                return set_error(TLB_ERR_CUDA,
                                 "paged_attention_no_alloc: cudaGetSymbolAddress failed");
            d.ptr = p;
            d.clean = 0;
        }
        // The kernel needs its counter prefix zero and leaves it zero; a call
        // with a longer prefix than the clean one clears it first (a memset
        // on the same stream, no allocation). A call recorded into a stream
        // capture always clears it: the host cannot know what ran on the
        // device between the capture and a later replay.
        if (zeroed > d.clean || capturing != cudaStreamCaptureStatusNone) {
            if (cudaMemsetAsync(d.ptr, 0, zeroed, st) != cudaSuccess)
                return set_error(TLB_ERR_CUDA, "paged_attention_no_alloc: clearing scratch failed");
        }
        d.clean = zeroed;
        scratch = d.ptr;
    }
    const int rc = tlb_paged_attention(out, query, key_cache, value_cache, block_tables,
                                       seq_lens, num_seqs, num_heads, num_kv_heads, head_dim,
                                       num_blocks, block_size, max_blocks_per_seq, scale, dtype,
                                       scratch, kNoAllocScratchBytes, flags, stream);
    if (rc != TLB_OK) tlb::no_alloc_scratch_dirty(dev);  // state unknown: clear next time
    return rc;
}
