// Block copies between KV caches (cscr/cache_kernel.cu:23-40 and the
// swap/copy drivers :124-212). One launch covers every (src, dst) block pair
// of every cache (all layers' key and value caches), with the pair list
// passed in the kernel parameters instead of a synchronous host-to-device
// upload. Each CTA copies one block of one cache with 128-bit accesses.
#include "common.cuh"
#include "kernels.h"

namespace tlb {

namespace {

template <bool VEC16>
__global__ void __launch_bounds__(256) copy_blocks_kernel(const __grid_constant__ CopyParams p) {
    const int pair = blockIdx.x;
    const int cache = blockIdx.y;
    const long long sb = p.pairs[2 * pair], db = p.pairs[2 * pair + 1];
    const char* src = p.src[cache] + sb * p.block_bytes;
    char* dst = p.dst[cache] + db * p.block_bytes;
    if (VEC16) {
        const long long n = p.block_bytes / 16;
        const uint4* s4 = reinterpret_cast<const uint4*>(src);
        uint4* d4 = reinterpret_cast<uint4*>(dst);
        for (long long i = threadIdx.x; i < n; i += blockDim.x) d4[i] = s4[i];
    } else {
        for (long long i = threadIdx.x; i < p.block_bytes; i += blockDim.x) dst[i] = src[i];
    }
}

}  // namespace

cudaError_t launch_copy_blocks(const CopyParams& p, bool vec16, cudaStream_t stream) {
    if (p.num_pairs <= 0 || p.num_caches <= 0) return cudaSuccess;
    dim3 grid(p.num_pairs, p.num_caches);
    if (vec16)
        copy_blocks_kernel<true><<<grid, 256, 0, stream>>>(p);
    else
        copy_blocks_kernel<false><<<grid, 256, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace tlb
