// Prefill (multi-token, causal) paged attention for sm_100a.
//
// The reference has no such op: its layer stops at a decode-only guard
// (src/model_executor/layers/attention.py:139-143). This kernel serves the
// prompt chunks of a continuous-batching step: chunk c holds n_c new tokens,
// the last n_c of the first context_lens[c] tokens of its sequence, already
// written into the paged cache (RoPE + cache write run first, over the whole
// packed step). Query token j of the chunk sits at position
// p = context_lens[c] - n_c + j and attends to the sequence's tokens 0..p:
//     out[t, h] = softmax(scale * q[t, h] . K[0..p]^T) V[0..p]
// with K, V of kv head h / (num_heads / num_kv_heads), token k read from block
// block_tables[c, k / block_size] at offset k % block_size. Blocks with a
// negative id are skipped and a softmax with nothing left gives zeros, the
// decode op's rules (cscr/attention_kernel.cu:70-72, :102).
//
// One CTA takes 64 query tokens of one query head (four warps x 16 rows) and
// walks the 64-token KV tiles up to its last query's position:
//   * K and V tiles come from the paged cache with 16-byte cp.async copies
//     into a two-buffer ring (the next tile loads while this one computes),
//     rows XOR-swizzled by 16-byte chunk so that ldmatrix is conflict-free;
//     rows past the causal limit or in unmapped blocks are zero-filled and
//     masked.
//   * S = Q K^T and O += P V with mma.m16n8k16 (fp32 accumulate), the query
//     fragments held in registers for the whole walk, an fp32 online softmax
//     in registers (quad shuffles), P fed from the S accumulators (for bf16
//     as a hi + lo pair, 16 significant bits, like the decode kernel).
//   * CTAs of the late (heavier) query tiles are scheduled first.
// Query heads of one kv head run as neighbouring CTAs, so a KV tile is read
// from HBM about once and from L2 by the rest of the group.
#include "common.cuh"
#include "kernels.h"

namespace tlb {
namespace prefill {
namespace {

constexpr int kBQ = 64;       // query tokens per CTA (4 warps x 16 rows)
constexpr int kBK = 64;       // KV tokens per tile
constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;

template <int D>
struct Layout {
    static constexpr int kRowBytes = D * 2;
    static constexpr int kChunks = D / 8;               // 16-byte chunks per row
    static constexpr int kTile = kBK * kRowBytes;       // one K or V tile
    static constexpr int kOffQ = 0;
    static constexpr int kOffK = kOffQ + kBQ * kRowBytes;
    static constexpr int kOffV = kOffK + 2 * kTile;
    static constexpr int kOffOk = kOffV + 2 * kTile;   // [2][kBK] row usable
    static constexpr int kBytes = kOffOk + 2 * kBK;
};

// Byte offset of 16-byte chunk `ch` of row `row` in a swizzled tile: the
// chunk index is XORed with the row's low three bits, so the eight rows an
// ldmatrix reads at one logical chunk fall in eight different bank groups.
template <int D>
__device__ __forceinline__ uint32_t swz(int row, int ch) {
    return (uint32_t)(row * (D * 2) + ((ch ^ (row & 7)) << 4));
}

__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, bool pred) {
    // src-size 0 fills the 16 bytes with zeros and reads nothing
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst),
                 "l"(reinterpret_cast<uint64_t>(src)), "r"(pred ? 16 : 0)
                 : "memory");
}

struct Params {
    void* out;
    const void* query;
    const void* key_cache;
    const void* value_cache;
    const int32_t* block_tables;
    const int32_t* query_start;   // [num_chunks + 1]
    const int32_t* context_lens;  // [num_chunks]
    long long num_blocks;
    int num_chunks;
    int num_heads;
    int num_kv_heads;
    int group;
    int block_size;
    int max_blocks;
    int q_tiles;                  // tiles of the longest chunk (gridDim.x)
    float scale_log2;
};

// Loads KV tile `kt` (tokens kt*64 .. +63) of kv head `kvh` into buffer
// `buf`: one 16-byte cp.async per (row, chunk); rows at or past `kv_end`, and
// rows whose block id is negative or outside the pool, are zero-filled and
// marked unusable in `ok`.
template <typename T, int D>
__device__ __forceinline__ void load_kv_tile(const Params& p, uint8_t* smem, uint32_t sbase,
                                             int buf, int kt, int c, int kvh, int kv_end) {
    using L = Layout<D>;
    const T* kc = reinterpret_cast<const T*>(p.key_cache);
    const T* vc = reinterpret_cast<const T*>(p.value_cache);
    const int* table = p.block_tables + (long long)c * p.max_blocks;
    const uint32_t kdst = sbase + L::kOffK + buf * L::kTile;
    const uint32_t vdst = sbase + L::kOffV + buf * L::kTile;
    for (int i = threadIdx.x; i < kBK * L::kChunks; i += kThreads) {
        const int row = i / L::kChunks, ch = i % L::kChunks;
        const int tok = kt * kBK + row;
        bool use = tok < kv_end;
        long long off = 0;
        if (use) {
            const int blk = table[tok / p.block_size];
            if (blk < 0) {
                use = false;
            } else if (blk >= p.num_blocks) {
                use = false;
                if (ch == 0) flag_status(TLB_STATUS_BAD_BLOCK_ID);
            } else {
                off = (((long long)blk * p.num_kv_heads + kvh) * p.block_size +
                       tok % p.block_size) * D + ch * 8;
            }
        }
        cp_async_16(kdst + swz<D>(row, ch), kc + off, use);
        cp_async_16(vdst + swz<D>(row, ch), vc + off, use);
        if (ch == 0) smem[L::kOffOk + buf * kBK + row] = use ? 1 : 0;
    }
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 2) prefill_attention_kernel(const Params p) {
    using L = Layout<D>;
    constexpr int KS = D / 16;   // k-steps of Q K^T over the head dim
    constexpr int NO = D / 8;    // n-tiles of the output (8 dims each)
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, q4 = lane & 3;

    const int c = blockIdx.z;
    const int h = blockIdx.y;
    const int tile = p.q_tiles - 1 - (int)blockIdx.x;  // late, heavier tiles first
    const int q_begin = p.query_start[c];
    const int n_c = p.query_start[c + 1] - q_begin;
    if (tile * kBQ >= n_c) return;  // (also a chunk with no, or negative, length)
    const int ctx = p.context_lens[c];
    const int first_pos = ctx - n_c;  // position of the chunk's first query token
    const int kvh = h / p.group;
    const int rows_here = min(kBQ, n_c - tile * kBQ);
    const int cap = p.max_blocks * p.block_size;  // tokens the block table can address
    if (ctx > cap && tile == p.q_tiles - 1 && h == 0 && threadIdx.x == 0)
        flag_status(TLB_STATUS_SEQ_TOO_LONG);
    // KV tokens this tile needs: up to its last query's position
    const int kv_end = max(0, min(min(ctx, cap), first_pos + tile * kBQ + rows_here));
    const int n_kv_tiles = (kv_end + kBK - 1) / kBK;

    const T* query = reinterpret_cast<const T*>(p.query);
    const long long tok0 = (long long)q_begin + tile * kBQ;  // packed row of query 0
    // ---- query tile -> shared memory (zero rows past the chunk)
    for (int i = tid; i < kBQ * L::kChunks; i += kThreads) {
        const int row = i / L::kChunks, ch = i % L::kChunks;
        const bool use = row < rows_here;
        const T* src = query + ((tok0 + (use ? row : 0)) * p.num_heads + h) * D + ch * 8;
        cp_async_16(sbase + L::kOffQ + swz<D>(row, ch), src, use);
    }
    cp_async_commit();
    if (n_kv_tiles > 0) load_kv_tile<T, D>(p, smem, sbase, 0, 0, c, kvh, kv_end);
    cp_async_commit();

    // this thread's two query rows (g, g + 8 of the warp's 16) and positions
    const int r0 = warp * 16 + g;
    const int pos0 = first_pos + tile * kBQ + r0, pos1 = pos0 + 8;

    cp_async_wait<1>();
    __syncthreads();
    uint32_t qa[KS][4];
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
        const int row = warp * 16 + (lane & 15);
        const int ch = ks * 2 + (lane >> 4);
        ldsm_x4(sbase + L::kOffQ + swz<D>(row, ch), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
    }

    float o[NO][4];
#pragma unroll
    for (int n = 0; n < NO; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    const float sl2 = p.scale_log2;

    for (int kt = 0; kt < n_kv_tiles; ++kt) {
        const int buf = kt & 1;
        // the next tile loads into the other buffer while this one computes
        // (everyone finished reading that buffer before the last barrier)
        if (kt + 1 < n_kv_tiles) load_kv_tile<T, D>(p, smem, sbase, buf ^ 1, kt + 1, c, kvh, kv_end);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();

        const uint32_t kb = sbase + L::kOffK + buf * L::kTile;
        const uint32_t vb = sbase + L::kOffV + buf * L::kTile;
        const uint8_t* ok = smem + L::kOffOk + buf * kBK;
        // ---- S = Q K^T: 16 query rows x 64 kv tokens per warp (8 n-tiles)
        float sacc[8][4];
#pragma unroll
        for (int n = 0; n < 8; ++n) sacc[n][0] = sacc[n][1] = sacc[n][2] = sacc[n][3] = 0.f;
#pragma unroll
        for (int np = 0; np < 4; ++np) {  // pairs of n-tiles: tokens 16 np .. 16 np + 15
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                uint32_t b0, b1, b2, b3;
                const int row = np * 16 + (lane & 7) + ((lane >> 4) << 3);
                const int ch = ks * 2 + ((lane >> 3) & 1);
                ldsm_x4(kb + swz<D>(row, ch), b0, b1, b2, b3);
                mma16816<T>(sacc[2 * np], qa[ks], b0, b1);
                mma16816<T>(sacc[2 * np + 1], qa[ks], b2, b3);
            }
        }
        // ---- causal / unmapped-block mask, online softmax (base 2)
        float mx[2] = {m_run[0], m_run[1]};
#pragma unroll
        for (int n = 0; n < 8; ++n) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int col = n * 8 + 2 * q4 + (e & 1);
                const int tok = kt * kBK + col;
                const int qpos = (e < 2) ? pos0 : pos1;
                const bool keep = ok[col] && tok <= qpos;
                const float v = keep ? sacc[n][e] * sl2 : -INFINITY;
                sacc[n][e] = v;
                mx[e >> 1] = fmaxf(mx[e >> 1], v);
            }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
        }
        float alpha[2], rs[2] = {0.f, 0.f};
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            alpha[r] = mx[r] == -INFINITY ? 1.f : exp2f(m_run[r] - mx[r]);
            m_run[r] = mx[r];
        }
#pragma unroll
        for (int n = 0; n < 8; ++n) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float mr = m_run[e >> 1];
                const float pv = mr == -INFINITY ? 0.f : exp2f(sacc[n][e] - mr);
                sacc[n][e] = pv;
                rs[e >> 1] += pv;
            }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
            rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
            l_run[r] = l_run[r] * alpha[r] + rs[r];
        }
#pragma unroll
        for (int n = 0; n < NO; ++n) {
            o[n][0] *= alpha[0];
            o[n][1] *= alpha[0];
            o[n][2] *= alpha[1];
            o[n][3] *= alpha[1];
        }
        // ---- O += P V: P (16 x 64) from the S accumulators, 4 k-steps of 16
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            uint32_t ph[4], pl[4];
            split2<T>(sacc[2 * kk][0], sacc[2 * kk][1], ph[0], pl[0]);
            split2<T>(sacc[2 * kk][2], sacc[2 * kk][3], ph[1], pl[1]);
            split2<T>(sacc[2 * kk + 1][0], sacc[2 * kk + 1][1], ph[2], pl[2]);
            split2<T>(sacc[2 * kk + 1][2], sacc[2 * kk + 1][3], ph[3], pl[3]);
#pragma unroll
            for (int dp = 0; dp < NO / 2; ++dp) {  // pairs of output n-tiles (16 dims)
                uint32_t b0, b1, b2, b3;
                const int row = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
                const int ch = dp * 2 + (lane >> 4);
                ldsm_x4_trans(vb + swz<D>(row, ch), b0, b1, b2, b3);
                mma16816<T>(o[2 * dp], ph, b0, b1);
                mma16816<T>(o[2 * dp + 1], ph, b2, b3);
                if constexpr (kSplitP<T>) {
                    mma16816<T>(o[2 * dp], pl, b0, b1);
                    mma16816<T>(o[2 * dp + 1], pl, b2, b3);
                }
            }
        }
        __syncthreads();  // every warp is done with `buf` before it is refilled
    }
    cp_async_wait<0>();

    // ---- normalise and store (rows of the chunk only; an empty softmax -> 0)
    T* out = reinterpret_cast<T*>(p.out);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int row = r0 + 8 * r;
        if (row >= rows_here) continue;
        const float inv = l_run[r] > 0.f ? 1.f / l_run[r] : 0.f;
        T* dst = out + ((tok0 + row) * p.num_heads + h) * D + 2 * q4;
#pragma unroll
        for (int n = 0; n < NO; ++n) {
            const uint32_t w = pack2<T>(o[n][2 * r] * inv, o[n][2 * r + 1] * inv);
            *reinterpret_cast<uint32_t*>(dst + n * 8) = w;
        }
    }
}

}  // namespace

bool supported(int dtype, int head_dim) {
    return (dtype == TLB_FLOAT16 || dtype == TLB_BFLOAT16) && (head_dim == 64 || head_dim == 128);
}

template <typename T, int D>
cudaError_t launch_t(const Params& p, cudaStream_t st) {
    using L = Layout<D>;
    auto kern = prefill_attention_kernel<T, D>;
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (e != cudaSuccess) return e;
    dim3 grid(p.q_tiles, p.num_heads, p.num_chunks);
    kern<<<grid, kThreads, L::kBytes, st>>>(p);
    return cudaGetLastError();
}

}  // namespace prefill

cudaError_t launch_prefill_attention(int dtype, int head_dim, void* out, const void* query,
                                     const void* key_cache, const void* value_cache,
                                     const int32_t* block_tables, const int32_t* query_start,
                                     const int32_t* context_lens, long long num_blocks,
                                     int num_chunks, int num_heads, int num_kv_heads,
                                     int block_size, int max_blocks, int max_query_len,
                                     float scale_log2, cudaStream_t stream) {
    prefill::Params p;
    p.out = out;
    p.query = query;
    p.key_cache = key_cache;
    p.value_cache = value_cache;
    p.block_tables = block_tables;
    p.query_start = query_start;
    p.context_lens = context_lens;
    p.num_blocks = num_blocks;
    p.num_chunks = num_chunks;
    p.num_heads = num_heads;
    p.num_kv_heads = num_kv_heads;
    p.group = num_heads / num_kv_heads;
    p.block_size = block_size;
    p.max_blocks = max_blocks;
    p.q_tiles = (max_query_len + prefill::kBQ - 1) / prefill::kBQ;
    p.scale_log2 = scale_log2;
    if (p.q_tiles == 0 || num_chunks == 0) return cudaSuccess;
    if (dtype == TLB_BFLOAT16)
        return head_dim == 64 ? prefill::launch_t<__nv_bfloat16, 64>(p, stream)
                              : prefill::launch_t<__nv_bfloat16, 128>(p, stream);
    return head_dim == 64 ? prefill::launch_t<__half, 64>(p, stream)
                          : prefill::launch_t<__half, 128>(p, stream);
}

}  // namespace tlb
