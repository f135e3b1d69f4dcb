// Positions and slot mapping of a packed continuous-batching step, on the GPU.
//
// The reference's worker forms them with Python loops every step
// (src/worker/worker.py:84-169): the tokens of every prompt first, position i
// of a prompt at slot block_table[i / block_size] * block_size + i %
// block_size (:111-124), then one token per decode sequence at position
// context_len - 1 (:144-159), the positions padded with 0 to a multiple of 8
// (:163-164). Here one launch derives both arrays from the prompt lengths,
// context lengths and block tables already on the device.
//
// Layout of the work: a grid-stride loop over the padded token range. Each
// CTA first turns the prompt lengths into exclusive offsets in shared memory
// (a chunked block scan), then a token finds its prompt by binary search over
// those offsets. Byte work only: one int64 position and one int64 slot
// written per token, the block-table entry read per token (L2-resident).
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace tlb {
namespace {

constexpr int kMetaThreads = 256;

__global__ void __launch_bounds__(kMetaThreads)
    step_metadata_kernel(const int32_t* __restrict__ prompt_lens,
                         const int32_t* __restrict__ prompt_tables, int num_prompts,
                         int prompt_max_blocks, const int32_t* __restrict__ context_lens,
                         const int32_t* __restrict__ decode_tables, long long num_decode,
                         int decode_max_blocks, int block_size, long long num_padded,
                         int64_t* __restrict__ positions, int64_t* __restrict__ slots) {
    __shared__ long long start[kStepMaxPrompts + 1];  // exclusive prompt offsets
    __shared__ long long warp_sum[kMetaThreads / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    long long carry = 0;
    for (int base = 0; base < num_prompts; base += kMetaThreads) {
        const int i = base + tid;
        long long v = i < num_prompts ? (long long)max(prompt_lens[i], 0) : 0ll;
        // inclusive scan within the warp, then across the warps of the chunk
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const long long n = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += n;
        }
        if (lane == 31) warp_sum[warp] = v;
        __syncthreads();
        long long before = carry;
        for (int w = 0; w < warp; ++w) before += warp_sum[w];
        if (i < num_prompts) start[i + 1] = before + v;
        long long chunk = 0;
        for (int w = 0; w < kMetaThreads / 32; ++w) chunk += warp_sum[w];
        __syncthreads();  // warp_sum is rewritten by the next chunk
        carry += chunk;
    }
    if (tid == 0) start[0] = 0;
    __syncthreads();
    const long long prompt_tokens = start[num_prompts];

    for (long long t = (long long)blockIdx.x * blockDim.x + tid; t < num_padded;
         t += (long long)gridDim.x * blockDim.x) {
        long long pos = 0, slot = -1;
        if (t < prompt_tokens) {
            // the prompt p with start[p] <= t < start[p + 1]
            int lo = 0, hi = num_prompts - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (start[mid] <= t) lo = mid; else hi = mid - 1;
            }
            pos = t - start[lo];
            const long long lb = pos / block_size;
            if (lb < prompt_max_blocks) {
                const long long blk = prompt_tables[(long long)lo * prompt_max_blocks + lb];
                if (blk >= 0) slot = blk * block_size + pos % block_size;
            } else {
                flag_status(TLB_STATUS_BAD_SLOT);
            }
        } else if (t < prompt_tokens + num_decode) {
            const long long r = t - prompt_tokens;
            pos = (long long)context_lens[r] - 1;
            if (pos >= 0 && pos / block_size < decode_max_blocks) {
                const long long blk = decode_tables[r * decode_max_blocks + pos / block_size];
                if (blk >= 0) slot = blk * block_size + pos % block_size;
            } else if (pos >= 0) {
                flag_status(TLB_STATUS_BAD_SLOT);
            }
        }
        // tokens past the step's real ones: position 0 (the worker's pad)
        // and slot -1 (a cache write skips them)
        positions[t] = pos;
        slots[t] = slot;
    }
}

}  // namespace

cudaError_t launch_step_metadata(const int32_t* prompt_lens, const int32_t* prompt_tables,
                                 int num_prompts, int prompt_max_blocks,
                                 const int32_t* context_lens, const int32_t* decode_tables,
                                 long long num_decode, int decode_max_blocks, int block_size,
                                 long long num_padded, int64_t* positions, int64_t* slots,
                                 cudaStream_t stream) {
    if (num_padded <= 0) return cudaSuccess;
    long long blocks = (num_padded + kMetaThreads - 1) / kMetaThreads;
    if (blocks > 4 * 148) blocks = 4 * 148;  // grid-stride beyond a few waves
    step_metadata_kernel<<<(unsigned)blocks, kMetaThreads, 0, stream>>>(
        prompt_lens, prompt_tables, num_prompts, prompt_max_blocks, context_lens, decode_tables,
        num_decode, decode_max_blocks, block_size, num_padded, positions, slots);
    return cudaGetLastError();
}

}  // namespace tlb
