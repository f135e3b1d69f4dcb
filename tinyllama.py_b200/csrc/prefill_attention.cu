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
// The contractions run on the 5th-generation tensor cores (tcgen05) with
// their accumulators in tensor memory. One CTA takes 128 query rows of one
// query head (tensor-memory lane r = query row r, owned by thread r for the
// softmax) and walks 64-token KV tiles up to its last query's position:
//   * Q (once), K and V come from the paged cache with 16-byte cp.async
//     copies into 128-byte-swizzled shared memory; rows past the causal
//     limit or in unmapped blocks are zero-filled and marked unusable. K is
//     single-buffered, V double-buffered: the next tile's copies start as
//     soon as the current S = Q K^T has completed (which also means the
//     previous tile's P V has, so its V buffer and P are free).
//   * S = Q K^T: M 128 x N 64, K = head dim, Q and K K-major, S in tensor
//     memory. Each thread loads its row of S (tcgen05.ld), masks, updates the
//     fp32 online softmax (base 2) and, when its running maximum moved,
//     rescales its row of O in tensor memory (tcgen05.ld / st).
//   * P (the row's probabilities in the storage type) goes to shared memory
//     K-major; O += P V: M 128 x N = head dim, K 64 tokens, V read MN-major
//     straight from its copied tile. One thread issues every MMA; commits to
//     mbarriers order them against the threads.
//   * CTAs of the late (heavier) query tiles are scheduled first. Query heads
//     of one kv head are neighbouring CTAs, so a KV tile comes from HBM about
//     once and from L2 for the rest of the group.
#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace tlb {
namespace prefill {
namespace {

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
    int bs_shift;                 // log2(block_size) when a power of two, else -1
    int max_blocks;
    int q_tiles;                  // tiles of the longest chunk (gridDim.z)
    float scale_log2;
};

// ---------------------------------------------------------------- tcgen05
// One CTA = 128 query rows of one query head (tensor-memory lane r = row r,
// thread r its softmax), KV tiles of 64 tokens.
constexpr int kTcBQ = 128;
constexpr int kTcBK = 64;
constexpr int kTcThreads = 128;
constexpr float kRebase = 8.f;  // log2 units

// With bf16 the probabilities go to the PV product as a hi + lo pair of bf16
// values (16 significant bits, as in the decode kernel; bf16 alone keeps 8):
// the layout then holds two P tiles and one V buffer instead of one P tile
// and two V buffers (the same bytes, so two CTAs still fit an SM).
template <int D, bool SPLIT>
struct TcLayout {
    static constexpr int kCh = D / 64;                       // 64-element chunks of a row
    static constexpr int kVBufs = SPLIT ? 1 : 2;
    static constexpr int kPTiles = SPLIT ? 2 : 1;
    static constexpr int kOffQ = 0;                          // [kCh][128 rows][128 B]
    static constexpr int kOffK = kOffQ + kCh * kTcBQ * 128;  // [kCh][64 tokens][128 B]
    static constexpr int kOffV = kOffK + kCh * kTcBK * 128;  // kVBufs buffers of the same
    static constexpr int kVBuf = kCh * kTcBK * 128;
    static constexpr int kOffP = kOffV + kVBufs * kVBuf;     // [kPTiles][128 rows][128 B]
    static constexpr int kPTile = kTcBQ * 128;               // 64 tokens of every row
    static constexpr int kOffOk = kOffP + kPTiles * kPTile;  // [2][64] token usable
    static constexpr int kOffBar = kOffOk + 2 * kTcBK;       // S done, O done
    static constexpr int kOffSlot = kOffBar + 16;            // tensor-memory address
    static constexpr int kBytes = kOffSlot + 16;
    static constexpr int kAlloc = kBytes + 1024;             // slack for 1024-byte alignment
    static constexpr uint32_t kTmemCols = D == 128 ? 256 : 128;  // S: 64 columns, O: D
    static_assert(kOffK % 1024 == 0 && kOffV % 1024 == 0 && kVBuf % 1024 == 0 &&
                      kOffP % 1024 == 0 && kPTile % 1024 == 0,
                  "swizzled tiles on 1024-byte boundaries");
};

// 16-byte unit `u` (of 8 per 128-byte row) of row `row` in a [rows][128 B]
// block with 128-byte swizzle.
__device__ __forceinline__ uint32_t sw128(int row, int u) {
    return (uint32_t)(row * 128 + ((u ^ (row & 7)) << 4));
}

// Row split of a KV tile copy: a thread copies one 16-byte column unit of
// kRows rows, kRowStep rows apart.
template <int D>
struct KvSplit {
    static constexpr int kUnits = D / 8;                  // 16-byte units per row
    static constexpr int kRowStep = kTcThreads / kUnits;  // rows between a thread's rows
    static constexpr int kRows = kTcBK / kRowStep;        // rows per thread
    static_assert(kTcThreads % kUnits == 0 && kTcBK % kRowStep == 0, "tile split");
};

// The block ids of this thread's rows of KV tile `kt` (-1 past kv_end). The
// loads are issued back to back and consumed a stage later, so a tile's copies
// do not wait on one table round trip per row.
template <int D>
__device__ __forceinline__ void fetch_blocks(const Params& p, int kt, int c, int kv_end,
                                             int (&blk)[KvSplit<D>::kRows]) {
    using S = KvSplit<D>;
    const int* table = p.block_tables + (long long)c * p.max_blocks;
    const int tok0 = kt * kTcBK + threadIdx.x / S::kUnits;
#pragma unroll
    for (int j = 0; j < S::kRows; ++j) {
        const int tok = tok0 + j * S::kRowStep;
        const int lb = p.bs_shift >= 0 ? tok >> p.bs_shift : tok / p.block_size;
        blk[j] = tok < kv_end ? __ldg(table + lb) : -1;
    }
}

// KV tile `kt` (tokens kt*64 .. +63) with its block ids `blk`: K into the K
// buffer (and the usable flag of every token into ok[kt % 2]), V into V buffer
// `vbuf`. Rows at or past kv_end, or in a block whose id is negative or
// outside the pool, are zero-filled and unusable. Returns whether one of this
// thread's rows below kv_end is unusable (the tile then needs the per-token
// flags; otherwise token < kv_end says it all).
template <typename T, int D, bool SPLIT, bool DO_K, bool DO_V>
__device__ __forceinline__ bool load_kv_tc(const Params& p, uint8_t* smem, uint32_t sbase,
                                           int vbuf, int kt, int kvh, int kv_end,
                                           const int (&blk)[KvSplit<D>::kRows]) {
    using L = TcLayout<D, SPLIT>;
    using S = KvSplit<D>;
    const T* kc = reinterpret_cast<const T*>(p.key_cache);
    const T* vc = reinterpret_cast<const T*>(p.value_cache);
    const int ua = threadIdx.x % S::kUnits;
    const int row0 = threadIdx.x / S::kUnits;
    bool hole = false;
#pragma unroll
    for (int j = 0; j < S::kRows; ++j) {
        const int row = row0 + j * S::kRowStep;
        const int tok = kt * kTcBK + row;
        bool use = blk[j] >= 0;
        if (use && blk[j] >= p.num_blocks) {
            use = false;
            if (ua == 0 && DO_K) flag_status(TLB_STATUS_BAD_BLOCK_ID);
        }
        long long off = 0;
        if (use) {
            const int in_blk = p.bs_shift >= 0 ? tok & (p.block_size - 1) : tok % p.block_size;
            off = (((long long)blk[j] * p.num_kv_heads + kvh) * p.block_size + in_blk) * D +
                  ua * 8;
        }
        const uint32_t dst = (uint32_t)((ua >> 3) * kTcBK * 128) + sw128(row, ua & 7);
        if (DO_K) {
            cp_async_16(sbase + L::kOffK + dst, kc + off, use);
            if (ua == 0) smem[L::kOffOk + (kt & 1) * kTcBK + row] = use ? 1 : 0;
        }
        if (DO_V) cp_async_16(sbase + L::kOffV + vbuf * L::kVBuf + dst, vc + off, use);
        hole |= !use && tok < kv_end;
    }
    return hole;
}

template <typename T, int D>
__global__ void __launch_bounds__(kTcThreads, (D == 128 || !std::is_same<T, __half>::value) ? 2 : 3)
    prefill_attention_tc_kernel(const Params p) {
    constexpr bool kBf16 = sizeof(T) == 2 && !std::is_same<T, __half>::value;
    constexpr bool kSplit = kBf16;  // P as a hi + lo pair of bf16
    using L = TcLayout<D, kSplit>;
    constexpr uint32_t kIdescS = tc5::idesc_f16(kBf16, false, kTcBQ, kTcBK);
    constexpr uint32_t kIdescO = tc5::idesc_f16(kBf16, true, kTcBQ, D);
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar_s = sbase + L::kOffBar, bar_o = bar_s + 8;
    const int tid = threadIdx.x, warp = tid >> 5;

    // grid (heads, chunks, tiles): CTAs start in x, then y, then z order, so
    // the late (heaviest) tiles of every chunk go first and the query heads of
    // one kv head run side by side
    const int h = blockIdx.x;
    const int c = blockIdx.y;
    const int tile = p.q_tiles - 1 - (int)blockIdx.z;
    const int q_begin = p.query_start[c];
    const int n_c = p.query_start[c + 1] - q_begin;
    if (tile * kTcBQ >= n_c) return;  // (also a chunk with no, or negative, length)
    const int ctx = p.context_lens[c];
    const int first_pos = ctx - n_c;
    const int kvh = h / p.group;
    const int rows_here = min(kTcBQ, n_c - tile * kTcBQ);
    const int cap = p.max_blocks * p.block_size;
    if (ctx > cap && tile == p.q_tiles - 1 && h == 0 && tid == 0)
        flag_status(TLB_STATUS_SEQ_TOO_LONG);
    const int kv_end = max(0, min(min(ctx, cap), first_pos + tile * kTcBQ + rows_here));
    const int nkt = (kv_end + kTcBK - 1) / kTcBK;

    // ---- query tile, first KV tile
    const T* query = reinterpret_cast<const T*>(p.query);
    const long long tok0 = (long long)q_begin + tile * kTcBQ;
    constexpr int kUnits = D / 8;
    for (int i = tid; i < kTcBQ * kUnits; i += kTcThreads) {
        const int row = i / kUnits, ua = i % kUnits;
        const bool use = row < rows_here;
        const T* src = query + ((tok0 + (use ? row : 0)) * p.num_heads + h) * D + ua * 8;
        cp_async_16(sbase + L::kOffQ + (uint32_t)((ua >> 3) * kTcBQ * 128) + sw128(row, ua & 7),
                    src, use);
    }
    constexpr int kRows = KvSplit<D>::kRows;
    int blk[kRows], blk_next[kRows] = {};  // block ids of tiles kt + 1 and kt + 2
    bool hole = false;
    if (nkt > 0) {
        fetch_blocks<D>(p, 0, c, kv_end, blk);
        hole = load_kv_tc<T, D, kSplit, true, true>(p, smem, sbase, 0, 0, kvh, kv_end, blk);
        fetch_blocks<D>(p, 1, c, kv_end, blk);
    }
    cp_async_commit();
    if (tid == 0) {
        mbar_init(bar_s, 1);
        mbar_init(bar_o, 1);
        fence_mbar_init();
    }
    if (warp == 0) tc5::alloc(sbase + L::kOffSlot, L::kTmemCols);
    cp_async_wait<0>();
    fence_proxy_async_smem();
    tc5::fence_before_sync();
    int tile_holes = __syncthreads_or(hole);  // tile kt has unusable tokens below kv_end
    tc5::fence_after_sync();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + L::kOffSlot);
    const uint32_t t_s = tmem, t_o = tmem + kTcBK;          // columns of S and O
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;  // this warp's lanes

    const int row = tid;  // query row of this thread
    const int qpos = first_pos + tile * kTcBQ + row;
    const float sl2 = p.scale_log2;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;

    for (int kt = 0; kt < nkt; ++kt) {
        const int buf = kt & 1;
        // ---- S = Q K^T (M 128, N 64, K = head dim), one thread issues
        if (tid == 0) {
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks) {
                const uint32_t qo = (uint32_t)((ks >> 2) * kTcBQ * 128 + (ks & 3) * 32);
                const uint32_t ko = (uint32_t)((ks >> 2) * kTcBK * 128 + (ks & 3) * 32);
                tc5::mma(t_s, tc5::desc_sw128(sbase + L::kOffQ + qo, 16, 1024),
                         tc5::desc_sw128(sbase + L::kOffK + ko, 16, 1024), kIdescS, ks > 0);
            }
            tc5::commit(bar_s);
        }
        __syncwarp();
        // S done implies every earlier MMA is done (commit tracks all prior
        // ones): the K buffer, the other V buffer, P and O are free.
        if (!mbar_wait_bounded(bar_s, (uint32_t)(kt & 1))) ok = false;
        tc5::fence_after_sync();
        // the next K (and, with two V buffers, the next V) start now
        hole = false;
        if (kt + 1 < nkt) {
            hole = load_kv_tc<T, D, kSplit, true, !kSplit>(p, smem, sbase, buf ^ 1, kt + 1, kvh,
                                                           kv_end, blk);
            fetch_blocks<D>(p, kt + 2, c, kv_end, blk_next);  // lands during the softmax
        }
        cp_async_commit();

        // ---- online softmax of this thread's row (base 2)
        float sv[64];
        {
            float a[32], b2[32];
            tc5::ld32(t_s + lane_base, a);
            tc5::ld32(t_s + lane_base + 32, b2);
#pragma unroll
            for (int j = 0; j < 32; ++j) { sv[j] = a[j]; sv[32 + j] = b2[j]; }
        }
        float mx = -INFINITY;
        if (!tile_holes) {
            // usable = below kv_end; causal = at or before this row's position
            const int lim = min(qpos, kv_end - 1) - kt * kTcBK;
#pragma unroll
            for (int j = 0; j < 64; ++j) {
                sv[j] = j <= lim ? sv[j] * sl2 : -INFINITY;
                mx = fmaxf(mx, sv[j]);
            }
        } else {
            const uint8_t* okf = smem + L::kOffOk + (kt & 1) * kTcBK;
#pragma unroll
            for (int j = 0; j < 64; ++j) {
                const bool keep = okf[j] && kt * kTcBK + j <= qpos;
                sv[j] = keep ? sv[j] * sl2 : -INFINITY;
                mx = fmaxf(mx, sv[j]);
            }
        }
        // The exponent base moves only when the row's maximum passes it by more
        // than kRebase (a factor 2^8): probabilities then stay <= 256, exact
        // to the storage type's relative precision, and O is rescaled on few
        // tiles instead of on most of the early ones. The result is the same
        // softmax (numerator and denominator share the base).
        const bool rebase = mx > m_run + kRebase;
        const float m_new = rebase ? mx : m_run;
        const float alpha = rebase && m_run != -INFINITY ? exp2f(m_run - m_new) : 1.f;
        float rs = 0.f;
#pragma unroll
        for (int j = 0; j < 64; ++j) {
            sv[j] = m_new == -INFINITY ? 0.f : exp2f(sv[j] - m_new);
            rs += sv[j];
        }
        l_run = l_run * alpha + rs;
        m_run = m_new;
        // ---- O *= alpha in tensor memory (warp-uniform: tcgen05.ld/st are
        // warp-wide; rows that need no rescale multiply by 1)
        if (kt > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
            for (int c0 = 0; c0 < D; c0 += 32) {
                float o[32];
                tc5::ld32(t_o + lane_base + c0, o);
#pragma unroll
                for (int j = 0; j < 32; ++j) o[j] *= alpha;
                tc5::st32(t_o + lane_base + c0, o);
            }
        }
        // ---- P (this row, 64 tokens) -> shared memory, K-major, swizzled
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            uint4 hi, lo;
            split2<T>(sv[8 * u + 0], sv[8 * u + 1], hi.x, lo.x);
            split2<T>(sv[8 * u + 2], sv[8 * u + 3], hi.y, lo.y);
            split2<T>(sv[8 * u + 4], sv[8 * u + 5], hi.z, lo.z);
            split2<T>(sv[8 * u + 6], sv[8 * u + 7], hi.w, lo.w);
            *reinterpret_cast<uint4*>(smem + L::kOffP + sw128(row, u)) = hi;
            if constexpr (kSplit)
                *reinterpret_cast<uint4*>(smem + L::kOffP + L::kPTile + sw128(row, u)) = lo;
        }
        fence_proxy_async_smem();
        tc5::fence_before_sync();
        __syncthreads();
        tc5::fence_after_sync();
        // ---- O += P V (M 128, N = head dim, K 64 tokens; V MN-major)
        const int vb = kSplit ? 0 : buf;
        if (tid == 0) {
#pragma unroll
            for (int ks = 0; ks < kTcBK / 16; ++ks) {
                const uint64_t bdesc = tc5::desc_sw128(
                    sbase + L::kOffV + vb * L::kVBuf + ks * 16 * 128, kTcBK * 128, 1024);
                tc5::mma(t_o, tc5::desc_sw128(sbase + L::kOffP + ks * 32, 16, 1024), bdesc,
                         kIdescO, kt > 0 || ks > 0);
                if constexpr (kSplit)
                    tc5::mma(t_o, tc5::desc_sw128(sbase + L::kOffP + L::kPTile + ks * 32, 16, 1024),
                             bdesc, kIdescO, true);
            }
            tc5::commit(bar_o);
        }
        __syncwarp();
        if constexpr (kSplit) {
            // one V buffer: the next V starts once this P V has read it
            if (kt + 1 < nkt) {
                if (!mbar_wait_bounded(bar_o, (uint32_t)(kt & 1))) ok = false;
                tc5::fence_after_sync();
                load_kv_tc<T, D, kSplit, false, true>(p, smem, sbase, 0, kt + 1, kvh, kv_end,
                                                      blk);
            }
            cp_async_commit();
        }
#pragma unroll
        for (int j = 0; j < kRows; ++j) blk[j] = blk_next[j];
        // the next tile's K and V have landed and are visible to the tensor core
        cp_async_wait<0>();
        fence_proxy_async_smem();
        tile_holes = __syncthreads_or(hole);
    }

    // ---- normalise and store (rows of the chunk only; an empty softmax -> 0)
    T* out = reinterpret_cast<T*>(p.out);
    if (nkt > 0) {
        if (!mbar_wait_bounded(bar_o, (uint32_t)((nkt - 1) & 1))) ok = false;
        tc5::fence_after_sync();
    }
    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
    T* dst = out + ((tok0 + row) * p.num_heads + h) * D;
#pragma unroll
    for (int c0 = 0; c0 < D; c0 += 32) {
        float o[32];
        if (nkt > 0) {
            tc5::ld32(t_o + lane_base + c0, o);
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] = 0.f;
        }
        if (row < rows_here) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
                uint4 w;
                w.x = pack2<T>(o[j + 0] * inv, o[j + 1] * inv);
                w.y = pack2<T>(o[j + 2] * inv, o[j + 3] * inv);
                w.z = pack2<T>(o[j + 4] * inv, o[j + 5] * inv);
                w.w = pack2<T>(o[j + 6] * inv, o[j + 7] * inv);
                *reinterpret_cast<uint4*>(dst + c0 + j) = w;
            }
        }
    }
    if (!ok && tid == 0) flag_status(TLB_STATUS_WAIT_TIMEOUT);
    tc5::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc5::dealloc(tmem, L::kTmemCols);
}

}  // namespace

bool supported(int dtype, int head_dim) {
    return (dtype == TLB_FLOAT16 || dtype == TLB_BFLOAT16) && (head_dim == 64 || head_dim == 128);
}

template <typename T, int D>
cudaError_t launch_t(const Params& p, cudaStream_t st) {
    using L = TcLayout<D, !std::is_same<T, __half>::value>;
    auto kern = prefill_attention_tc_kernel<T, D>;
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) return e;
    dim3 grid(p.num_heads, p.num_chunks, p.q_tiles);
    kern<<<grid, kTcThreads, L::kAlloc, st>>>(p);
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
    p.bs_shift = -1;
    if (block_size > 0 && (block_size & (block_size - 1)) == 0)
        p.bs_shift = __builtin_ctz((unsigned)block_size);
    p.max_blocks = max_blocks;
    p.q_tiles = (max_query_len + prefill::kTcBQ - 1) / prefill::kTcBQ;
    p.scale_log2 = scale_log2;
    if (p.q_tiles == 0 || num_chunks == 0) return cudaSuccess;
    if (dtype == TLB_BFLOAT16)
        return head_dim == 64 ? prefill::launch_t<__nv_bfloat16, 64>(p, stream)
                              : prefill::launch_t<__nv_bfloat16, 128>(p, stream);
    return head_dim == 64 ? prefill::launch_t<__half, 64>(p, stream)
                          : prefill::launch_t<__half, 128>(p, stream);
}

}  // namespace tlb
