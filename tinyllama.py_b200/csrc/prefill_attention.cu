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
//   * Q (once) comes with 16-byte cp.async copies into 128-byte-swizzled
//     shared memory. K and V come from the paged cache by TMA: a 3-D tensor
//     map over the cache rows [blocks * kv heads * block_size, head dim]
//     with one 64-column chunk per box, so one copy moves the rows of one
//     block (or the tile's part of a block) for one chunk, already swizzled;
//     the lanes of one warp issue a tile's copies (at most 32) together and
//     an mbarrier per buffer counts their bytes. 16-byte cp.async copies
//     (one per thread and row) stalled the issuing threads for ~2,800
//     cycles per tile on the SM's miss queue. Block sizes a box cannot tile
//     (not a power of two below 64, or below 8) keep the cp.async loader.
//     Rows past the context or in unmapped blocks are marked unusable; their
//     V rows are zeroed before P V (stale cache slots never leak). K is
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
    int box_rows;                 // (TMA) cache rows per copy: min(block_size, 64)
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
    // mbarriers: S done, O done, K landed, V0 / V1 landed, K seen by every
    // softmax warp (warp-specialised kernel)
    static constexpr int kOffBar = kOffOk + 2 * kTcBK;
    static constexpr int kOffHole = kOffBar + 48;            // [2] tile has unmapped blocks
    static constexpr int kOffSlot = kOffHole + 8;            // tensor-memory address
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

// ---- TMA loads (warp-specialised kernel). The cache is viewed as a 4-D
// tensor {64 columns, 8 rows, head_dim / 64 chunks, rows / 8 groups} (strides:
// a row, 128 bytes, 8 rows), so one box of {64, 8, chunks, box_rows / 8} moves
// box_rows rows of one block (all of it, or a 64-row part) with every chunk,
// stored [8-row group][chunk][8 rows][128 bytes] with 128-byte swizzle: the
// 8-row groups of a 64-token tile are then kCh * 1024 bytes apart whichever
// block they come from, one stride for the MMA descriptors. Lane b < 64 /
// box_rows of the copy warp moves part b of the tile.
__device__ __forceinline__ void tma_load_kv4(uint32_t dst, const CUtensorMap* map, int32_t group,
                                             uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(0), "r"(0), "r"(group), "r"(bar)
        : "memory");
}

// Block id of this lane's part of KV tile `kt` (-1 past kv_end or for lanes
// beyond the tile's parts).
__device__ __forceinline__ int tma_block_of(const Params& p, int kt, int c, int kv_end) {
    const int lane = threadIdx.x & 31;
    const int tok = kt * kTcBK + lane * p.box_rows;
    if (lane >= kTcBK / p.box_rows || tok >= kv_end) return -1;
    const int lb = p.bs_shift >= 0 ? tok >> p.bs_shift : tok / p.block_size;
    return __ldg(p.block_tables + (long long)c * p.max_blocks + lb);
}

// Issues one K or V tile (this lane's part, block id `blk`) into `dst`; lane 0
// first tells the buffer's mbarrier how many bytes arrive.
template <int D>
__device__ __forceinline__ void issue_kv_ws(const Params& p, const CUtensorMap* map,
                                            uint32_t dst, uint32_t bar, int kt, int kvh,
                                            int blk) {
    const int lane = threadIdx.x & 31;
    const int R = p.box_rows;
    const bool valid = blk >= 0 && blk < p.num_blocks;
    const unsigned m = __ballot_sync(0xffffffffu, valid);
    if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)__popc(m) * (uint32_t)(R * D * 2));
    __syncwarp();
    if (valid) {
        const int tok = kt * kTcBK + lane * R;
        const int in_blk = R == p.block_size ? 0
                           : p.bs_shift >= 0 ? (tok & (p.block_size - 1))
                                             : tok % p.block_size;
        const int group = ((blk * p.num_kv_heads + kvh) * p.block_size + in_blk) >> 3;
        tma_load_kv4(dst + (uint32_t)(lane * R * D * 2), map, group, bar);
    }
}

// Usable flags of KV tile `kt` (this lane's part) and whether a token below
// kv_end sits in an unmapped block; flags a block id outside the pool.
__device__ __forceinline__ bool tile_flags_ws(const Params& p, uint8_t* okf, int kt, int kv_end,
                                              int blk) {
    const int lane = threadIdx.x & 31;
    const int R = p.box_rows;
    if (lane >= kTcBK / R) return false;
    const int tok = kt * kTcBK + lane * R;
    const bool valid = blk >= 0 && blk < p.num_blocks;
    if (blk >= p.num_blocks) flag_status(TLB_STATUS_BAD_BLOCK_ID);
    for (int r = 0; r < R; ++r) okf[lane * R + r] = (valid && tok + r < kv_end) ? 1 : 0;
    return !valid && tok < kv_end;
}

// Online softmax (base 2) of KV tile `kt` for this thread's query row: reads
// the row's S (tensor-memory columns t_s..t_s+63 of its lane), keeps the
// usable tokens at or before the row's position, updates the running
// (m_run, l_run), rescales the row of O (columns t_o..) when the exponent base
// moves, and writes the row's probabilities to P in shared memory (K-major,
// 128-byte swizzle; with SPLIT a second tile holds the low parts).
template <typename T, int D, bool SPLIT>
__device__ __forceinline__ void softmax_tile(uint8_t* smem_p, const uint8_t* okf, bool holes,
                                             uint32_t t_s, uint32_t t_o, int kt, int row,
                                             int qpos, int kv_end, float sl2, float& m_run,
                                             float& l_run) {
    float sv[64];
    {
        float a[32], b2[32];
        tc5::ld32(t_s, a);
        tc5::ld32(t_s + 32, b2);
#pragma unroll
        for (int j = 0; j < 32; ++j) { sv[j] = a[j]; sv[32 + j] = b2[j]; }
    }
    // row maximum and (below) row sum as eight interleaved partials: a
    // 64-long dependent chain of max / add would leave a warp idle on
    // each step with two warps per scheduler
    float mx8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) mx8[i] = -INFINITY;
    if (!holes) {
        // usable = below kv_end; causal = at or before this row's position
        const int lim = min(qpos, kv_end - 1) - kt * kTcBK;
#pragma unroll
        for (int j = 0; j < 64; ++j) {
            sv[j] = j <= lim ? sv[j] * sl2 : -INFINITY;
            mx8[j & 7] = fmaxf(mx8[j & 7], sv[j]);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 64; ++j) {
            const bool keep = okf[j] && kt * kTcBK + j <= qpos;
            sv[j] = keep ? sv[j] * sl2 : -INFINITY;
            mx8[j & 7] = fmaxf(mx8[j & 7], sv[j]);
        }
    }
    const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                           fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
    // The exponent base moves only when the row's maximum passes it by more
    // than kRebase (a factor 2^8): probabilities then stay <= 256, exact
    // to the storage type's relative precision, and O is rescaled on few
    // tiles instead of on most of the early ones. The result is the same
    // softmax (numerator and denominator share the base).
    const bool rebase = mx > m_run + kRebase;
    const float m_new = rebase ? mx : m_run;
    const float alpha = rebase && m_run != -INFINITY ? exp2f(m_run - m_new) : 1.f;
    float rs8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) rs8[i] = 0.f;
#pragma unroll
    for (int j = 0; j < 64; ++j) {
        sv[j] = m_new == -INFINITY ? 0.f : exp2f(sv[j] - m_new);
        rs8[j & 7] += sv[j];
    }
    const float rs = ((rs8[0] + rs8[1]) + (rs8[2] + rs8[3])) + ((rs8[4] + rs8[5]) + (rs8[6] + rs8[7]));
    l_run = l_run * alpha + rs;
    m_run = m_new;
    // ---- P (this row, 64 tokens) -> shared memory, K-major, swizzled
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        uint4 hi, lo;
        split2<T>(sv[8 * u + 0], sv[8 * u + 1], hi.x, lo.x);
        split2<T>(sv[8 * u + 2], sv[8 * u + 3], hi.y, lo.y);
        split2<T>(sv[8 * u + 4], sv[8 * u + 5], hi.z, lo.z);
        split2<T>(sv[8 * u + 6], sv[8 * u + 7], hi.w, lo.w);
        *reinterpret_cast<uint4*>(smem_p + sw128(row, u)) = hi;
        if constexpr (SPLIT)
            *reinterpret_cast<uint4*>(smem_p + kTcBQ * 128 + sw128(row, u)) = lo;
    }
    // ---- O *= alpha in tensor memory, after P is out of registers (warp-
    // uniform: tcgen05.ld/st are warp-wide; rows that need no rescale
    // multiply by 1)
    if (kt > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
            float o[32];
            tc5::ld32(t_o + c0, o);
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] *= alpha;
            tc5::st32(t_o + c0, o);
        }
    }
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

    if (tid == 0) {
        mbar_init(bar_s, 1);
        mbar_init(bar_o, 1);
        fence_mbar_init();
    }

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
    // the block ids of this thread's rows of tiles kt + 1 and kt + 2
    constexpr int kRows = KvSplit<D>::kRows;
    int blk[kRows] = {}, blk_next[kRows] = {};
    bool hole = false;
    if (nkt > 0) {
        fetch_blocks<D>(p, 0, c, kv_end, blk);
        hole = load_kv_tc<T, D, kSplit, true, true>(p, smem, sbase, 0, 0, kvh, kv_end, blk);
        fetch_blocks<D>(p, 1, c, kv_end, blk);
    }
    cp_async_commit();
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
        const int vb = kSplit ? 0 : buf;  // V buffer of this tile
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
        softmax_tile<T, D, kSplit>(smem + L::kOffP, smem + L::kOffOk + (kt & 1) * kTcBK,
                                   tile_holes, t_s + lane_base, t_o + lane_base, kt, row, qpos,
                                   kv_end, sl2, m_run, l_run);
        fence_proxy_async_smem();
        tc5::fence_before_sync();
        __syncthreads();
        tc5::fence_after_sync();
        // ---- O += P V (M 128, N = head dim, K 64 tokens; V MN-major)
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
    if (!ok) flag_status(TLB_STATUS_WAIT_TIMEOUT);
    tc5::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc5::dealloc(tmem, L::kTmemCols);
}

// Shared-memory layout of the warp-specialised kernel: Q, two K and two V
// buffers (P lives in tensor memory), usable flags and unmapped-block flags of
// four tiles in flight, mbarriers.
template <int D>
struct WsLayout {
    static constexpr int kCh = D / 64;
    static constexpr int kKV = kCh * kTcBK * 128;                // one K or V tile
    static constexpr int kOffQ = 0;                              // [kCh][128 rows][128 B]
    static constexpr int kOffK = kOffQ + kCh * kTcBQ * 128;      // 2 x [8 groups][kCh][8][128 B]
    static constexpr int kOffV = kOffK + 2 * kKV;                // 2 x the same
    static constexpr int kOffOk = kOffV + 2 * kKV;               // [4][64] token usable
    static constexpr int kOffHole = kOffOk + 4 * kTcBK;          // [4] tile has unmapped blocks
    // mbarriers: S done [2], O done [2] (per S / V buffer), K landed [2], V landed [2],
    // P ready [2] (per S buffer), flags stored [4] (per flag slot)
    static constexpr int kOffBar = kOffHole + 16;
    static constexpr int kOffSlot = kOffBar + 112;               // tensor-memory address
    static constexpr int kBytes = kOffSlot + 16;
    static constexpr int kAlloc = kBytes + 1024;                 // slack for 1024-byte alignment
    // tensor memory: S / P of tiles kt and kt + 1 (64 columns each), then O
    static constexpr uint32_t kTmemCols = 256;
    static_assert(2 * kTcBK + D <= (int)kTmemCols, "S, S and O fit the allocation");
    static_assert(kOffK % 1024 == 0 && kOffV % 1024 == 0 && kKV % 1024 == 0,
                  "swizzled tiles on 1024-byte boundaries");
};

// Online softmax (base 2) of KV tile `kt` for this thread's query row, with P
// kept in tensor memory: reads the row's S (columns t_s..t_s+63 of its lane),
// keeps the usable tokens at or before the row's position, updates the
// running (m_run, l_run) and writes the row's probabilities over its S:
// columns t_s..t_s+31 hold 64 values packed in pairs (with SPLIT the high
// parts there and the low parts in t_s+32..t_s+63). Returns the factor the
// row of O must be scaled by before this tile's P V.
template <typename T, bool SPLIT>
__device__ __forceinline__ float softmax_tile_tm(const uint8_t* okf, bool holes, uint32_t t_s,
                                                 int kt, int qpos, int kv_end, float sl2,
                                                 float& m_run, float& l_run) {
    float sv[64];
    {
        float a[32], b2[32];
        tc5::ld32(t_s, a);
        tc5::ld32(t_s + 32, b2);
#pragma unroll
        for (int j = 0; j < 32; ++j) { sv[j] = a[j]; sv[32 + j] = b2[j]; }
    }
    // row maximum and (below) row sum as eight interleaved partials
    float mx8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) mx8[i] = -INFINITY;
    if (!holes) {
        // usable = below kv_end; causal = at or before this row's position
        const int lim = min(qpos, kv_end - 1) - kt * kTcBK;
#pragma unroll
        for (int j = 0; j < 64; ++j) {
            sv[j] = j <= lim ? sv[j] * sl2 : -INFINITY;
            mx8[j & 7] = fmaxf(mx8[j & 7], sv[j]);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 64; ++j) {
            const bool keep = okf[j] && kt * kTcBK + j <= qpos;
            sv[j] = keep ? sv[j] * sl2 : -INFINITY;
            mx8[j & 7] = fmaxf(mx8[j & 7], sv[j]);
        }
    }
    const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                           fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
    // lazy exponent base (see softmax_tile)
    const bool rebase = mx > m_run + kRebase;
    const float m_new = rebase ? mx : m_run;
    const float alpha = rebase && m_run != -INFINITY ? exp2f(m_run - m_new) : 1.f;
    float rs8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) rs8[i] = 0.f;
#pragma unroll
    for (int j = 0; j < 64; ++j) {
        sv[j] = m_new == -INFINITY ? 0.f : exp2f(sv[j] - m_new);
        rs8[j & 7] += sv[j];
    }
    const float rs = ((rs8[0] + rs8[1]) + (rs8[2] + rs8[3])) + ((rs8[4] + rs8[5]) + (rs8[6] + rs8[7]));
    l_run = l_run * alpha + rs;
    m_run = m_new;
    uint32_t ph[32], pl[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) split2<T>(sv[2 * j], sv[2 * j + 1], ph[j], pl[j]);
    tc5::st32u(t_s, ph);
    if constexpr (SPLIT) tc5::st32u(t_s + 32, pl);
    return alpha;
}

// ---------------------------------------------------------------- warp-specialised
// Warps 0-3 run the softmax of the CTA's 128 query rows; warp 4 issues the
// TMA copies of K and V, warp 5 the MMAs. S is double-buffered in tensor
// memory and P is written over its own S, so the tensor core runs P V of
// tile kt - 1 and S of tile kt + 1 while the softmax warps work on tile kt:
//   MMA warp: once every softmax warp has put P (kt) in place, P V (kt) -> O,
//   then S (kt + 2) -> S buffer kt % 2 (issued in order: the P V read of that
//   buffer comes first);
//   copy warp: K (kt) into K buffer kt % 2 once S (kt - 2) is done, then the
//   tile's usable flags into flag slot kt % 4, V (kt) into V buffer kt % 2
//   once P V (kt - 2) is done.
// The softmax warps never wait for one another. Every mbarrier is per buffer
// or per slot, so none can complete a second phase before its waiters have
// seen the first.
constexpr int kWsThreads = kTcThreads + 64;
constexpr int kCopyWarp = kTcThreads / 32, kMmaWarp = kCopyWarp + 1;

template <typename T, int D>
__global__ void __launch_bounds__(kWsThreads, 2)
    prefill_attention_ws_kernel(const __grid_constant__ CUtensorMap tm_k,
                                const __grid_constant__ CUtensorMap tm_v, const Params p) {
    constexpr bool kBf16 = sizeof(T) == 2 && !std::is_same<T, __half>::value;
    constexpr bool kSplit = kBf16;  // P as a hi + lo pair of bf16
    constexpr int kCh = D / 64;
    using L = WsLayout<D>;
    constexpr uint32_t kIdescS = tc5::idesc_f16(kBf16, false, kTcBQ, kTcBK);
    constexpr uint32_t kIdescO = tc5::idesc_f16(kBf16, true, kTcBQ, D);
    constexpr uint32_t kGroupStride = kCh * 1024;  // bytes between 8-token groups of K / V
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    const uint32_t sbase = smem_u32(smem);
    // buffer b: bar_s + 8 b, bar_o + 8 b, bar_k + 8 b, bar_v + 8 b, bar_p + 8 b;
    // flag slot f: bar_f + 8 f
    const uint32_t bar_s = sbase + L::kOffBar, bar_o = bar_s + 16, bar_k = bar_s + 32,
                   bar_v = bar_s + 48, bar_p = bar_s + 64, bar_f = bar_s + 80;
    volatile int* hflag = reinterpret_cast<volatile int*>(smem + L::kOffHole);
    const int tid = threadIdx.x, warp = tid >> 5;

    // grid (heads, chunks, tiles): the late (heaviest) tiles of every chunk
    // start first, the query heads of one kv head side by side
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

    if (tid == 0) {
        for (int i = 0; i < 8; ++i) mbar_init(bar_s + 8 * i, 1);
        mbar_init(bar_p, kTcThreads / 32);
        mbar_init(bar_p + 8, kTcThreads / 32);
        for (int i = 0; i < 4; ++i) mbar_init(bar_f + 8 * i, 1);
        fence_mbar_init();
    }
    if (tid == kTcThreads) {
        prefetch_tensormap(&tm_k);
        prefetch_tensormap(&tm_v);
    }
    // ---- query tile (softmax warps)
    const T* query = reinterpret_cast<const T*>(p.query);
    const long long tok0 = (long long)q_begin + tile * kTcBQ;
    constexpr int kUnits = D / 8;
    if (tid < kTcThreads) {
        for (int i = tid; i < kTcBQ * kUnits; i += kTcThreads) {
            const int row = i / kUnits, ua = i % kUnits;
            const bool use = row < rows_here;
            const T* src = query + ((tok0 + (use ? row : 0)) * p.num_heads + h) * D + ua * 8;
            cp_async_16(sbase + L::kOffQ + (uint32_t)((ua >> 3) * kTcBQ * 128) +
                            sw128(row, ua & 7),
                        src, use);
        }
    }
    cp_async_commit();
    if (warp == 0) tc5::alloc(sbase + L::kOffSlot, L::kTmemCols);
    cp_async_wait<0>();
    fence_proxy_async_smem();
    tc5::fence_before_sync();
    __syncthreads();
    tc5::fence_after_sync();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + L::kOffSlot);
    bool ok = true;

    if (warp == kCopyWarp) {
        // ======================================================== copy warp
        int blk = tma_block_of(p, 0, c, kv_end);
        for (int kt = 0; kt < nkt; ++kt) {
            const int b = kt & 1;
            const uint32_t prev = (uint32_t)(((kt - 2) >> 1) & 1);  // phase of tile kt - 2
            const int blk_next = tma_block_of(p, kt + 1, c, kv_end);  // lands while waiting
            // K buffer b is free once S of tile kt - 2 is done
            if (kt >= 2 && !__all_sync(0xffffffffu, mbar_wait_bounded(bar_s + 8 * b, prev)))
                ok = false;
            const bool hole =
                tile_flags_ws(p, smem + L::kOffOk + (kt & 3) * kTcBK, kt, kv_end, blk);
            const bool any_hole = __any_sync(0xffffffffu, hole);
            if ((tid & 31) == 0) hflag[kt & 3] = any_hole ? 1 : 0;
            __syncwarp();  // flags stored before lane 0's arrive (release) below
            if ((tid & 31) == 0) mbar_arrive(bar_f + 8 * (kt & 3));
            issue_kv_ws<D>(p, &tm_k, sbase + L::kOffK + b * L::kKV, bar_k + 8 * b, kt, kvh, blk);
            // V buffer b is free once P V of tile kt - 2 is done
            if (kt >= 2 && !__all_sync(0xffffffffu, mbar_wait_bounded(bar_o + 8 * b, prev)))
                ok = false;
            issue_kv_ws<D>(p, &tm_v, sbase + L::kOffV + b * L::kKV, bar_v + 8 * b, kt, kvh, blk);
            blk = blk_next;
        }
    } else if (warp == kMmaWarp) {
        // ========================================================= MMA warp
        if (tid == kMmaWarp * 32) {
            // S = Q K^T of tile j (M 128, N 64, K = head dim) into S buffer
            // j % 2, once K of tile j has landed
            auto issue_s = [&](int j) {
                const int b = j & 1;
                if (!mbar_wait_bounded(bar_k + 8 * b, (uint32_t)((j >> 1) & 1))) ok = false;
                tc5::fence_after_sync();
#pragma unroll
                for (int ks = 0; ks < D / 16; ++ks) {
                    const uint32_t qo = (uint32_t)((ks >> 2) * kTcBQ * 128 + (ks & 3) * 32);
                    const uint32_t ko = (uint32_t)(b * L::kKV + (ks >> 2) * 1024 + (ks & 3) * 32);
                    tc5::mma(tmem + b * kTcBK, tc5::desc_sw128(sbase + L::kOffQ + qo, 16, 1024),
                             tc5::desc_sw128(sbase + L::kOffK + ko, 16, kGroupStride), kIdescS,
                             ks > 0);
                }
                tc5::commit(bar_s + 8 * b);
            };
            for (int j = 0; j < min(2, nkt); ++j) issue_s(j);
            for (int kt = 0; kt < nkt; ++kt) {
                const int b = kt & 1;
                const uint32_t par = (uint32_t)((kt >> 1) & 1);
                // ---- O += P V (M 128, N = head dim, K 64 tokens; P from tensor
                // memory, V MN-major from shared memory), once every softmax
                // warp has put P (kt) in place and V (kt) has landed
                if (!mbar_wait_bounded(bar_p + 8 * b, par)) ok = false;
                if (!mbar_wait_bounded(bar_v + 8 * b, par)) ok = false;
                tc5::fence_after_sync();
#pragma unroll
                for (int ks = 0; ks < kTcBK / 16; ++ks) {
                    const uint64_t bdesc = tc5::desc_sw128(
                        sbase + L::kOffV + b * L::kKV + ks * 2 * kGroupStride, 1024, kGroupStride);
                    tc5::mma_ts(tmem + 2 * kTcBK, tmem + b * kTcBK + ks * 8, bdesc, kIdescO,
                                kt > 0 || ks > 0);
                    if constexpr (kSplit)
                        tc5::mma_ts(tmem + 2 * kTcBK, tmem + b * kTcBK + 32 + ks * 8, bdesc,
                                    kIdescO, true);
                }
                tc5::commit(bar_o + 8 * b);
                if (kt + 2 < nkt) issue_s(kt + 2);
            }
        }
        __syncwarp();
    } else {
        // ===================================================== softmax warps
        const uint32_t t_o = tmem + 2 * kTcBK;                   // columns of O
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;  // this warp's lanes
        const int row = tid;  // query row of this thread
        const int qpos = first_pos + tile * kTcBQ + row;
        const float sl2 = p.scale_log2;
        float m_run = -INFINITY, l_run = 0.f;
        for (int kt = 0; kt < nkt; ++kt) {
            const int b = kt & 1;
            const uint32_t par = (uint32_t)((kt >> 1) & 1);  // phase of tile kt on buffer b
            // the tile's flags are stored, and S of it is done
            if (!mbar_wait_bounded(bar_f + 8 * (kt & 3), (uint32_t)((kt >> 2) & 1))) ok = false;
            const bool holes = hflag[kt & 3] != 0;
            const uint8_t* okf = smem + L::kOffOk + (kt & 3) * kTcBK;
            if (!mbar_wait_bounded(bar_s + 8 * b, par)) ok = false;
            tc5::fence_after_sync();
            const float alpha = softmax_tile_tm<T, kSplit>(okf, holes, tmem + b * kTcBK + lane_base,
                                                           kt, qpos, kv_end, sl2, m_run, l_run);
            // ---- O *= alpha (rare with the lazy base), once P V of tile
            // kt - 1 has accumulated into it (warp-uniform: tcgen05.ld/st are
            // warp-wide; rows that need no rescale multiply by 1)
            if (kt > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
                if (!mbar_wait_bounded(bar_o + 8 * (b ^ 1), (uint32_t)(((kt - 1) >> 1) & 1)))
                    ok = false;
                tc5::fence_after_sync();
#pragma unroll
                for (int c0 = 0; c0 < D; c0 += 32) {
                    float o[32];
                    tc5::ld32(t_o + lane_base + c0, o);
#pragma unroll
                    for (int j = 0; j < 32; ++j) o[j] *= alpha;
                    tc5::st32(t_o + lane_base + c0, o);
                }
            }
            // A box moves whole blocks: V rows past the context, or of an
            // unmapped block (never copied: stale shared memory), are zeroed
            // once the tile's V has landed, so 0 x (stale NaN) never reaches O;
            // each warp zeroes its own quarter of the rows.
            if (holes || (kt == nkt - 1 && kv_end - kt * kTcBK < kTcBK)) {
                if (!mbar_wait_bounded(bar_v + 8 * b, par)) ok = false;
                for (int i = tid; i < kTcBK * kCh * 8; i += kTcThreads) {
                    const int r = i / (kCh * 8), u = i % (kCh * 8);
                    if (!okf[r])
                        *reinterpret_cast<uint4*>(smem + L::kOffV + b * L::kKV +
                                                  (r >> 3) * kGroupStride + (u >> 3) * 1024 +
                                                  (r & 7) * 128 + (u & 7) * 16) =
                            make_uint4(0u, 0u, 0u, 0u);
                }
                fence_proxy_async_smem();
            }
            // P (and any zeroed V rows) in place: the warp's arrival releases them
            tc5::fence_before_sync();
            __syncwarp();
            if ((tid & 31) == 0) mbar_arrive(bar_p + 8 * b);
        }
        // ---- normalise and store (rows of the chunk only; an empty softmax -> 0)
        T* out = reinterpret_cast<T*>(p.out);
        if (nkt > 0) {
            const int last = nkt - 1;
            if (!mbar_wait_bounded(bar_o + 8 * (last & 1), (uint32_t)((last >> 1) & 1))) ok = false;
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
    }
    if (!ok) flag_status(TLB_STATUS_WAIT_TIMEOUT);
    tc5::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc5::dealloc(tmem, WsLayout<D>::kTmemCols);
}

}  // namespace

bool supported(int dtype, int head_dim) {
    return (dtype == TLB_FLOAT16 || dtype == TLB_BFLOAT16) && (head_dim == 64 || head_dim == 128);
}

template <typename T, int D>
cudaError_t launch_d(const Params& p, const CUtensorMap* tk, const CUtensorMap* tv,
                     cudaStream_t st) {
    using L = TcLayout<D, !std::is_same<T, __half>::value>;
    const dim3 grid(p.num_heads, p.num_chunks, p.q_tiles);
    if (tk != nullptr && tv != nullptr) {
        constexpr int kAlloc = WsLayout<D>::kAlloc;
        auto kern = prefill_attention_ws_kernel<T, D>;
        cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kAlloc);
        if (e != cudaSuccess) return e;
        kern<<<grid, kWsThreads, kAlloc, st>>>(*tk, *tv, p);
    } else {
        auto kern = prefill_attention_tc_kernel<T, D>;
        cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
        if (e != cudaSuccess) return e;
        kern<<<grid, kTcThreads, L::kAlloc, st>>>(p);
    }
    return cudaGetLastError();
}

}  // namespace prefill

int prefill_box_rows(int block_size) {
    if (block_size >= 8 && block_size <= 64 && (block_size & (block_size - 1)) == 0)
        return block_size;
    if (block_size >= 64 && block_size % 64 == 0) return 64;
    return 0;
}

cudaError_t launch_prefill_attention(int dtype, int head_dim, void* out, const void* query,
                                     const void* key_cache, const void* value_cache,
                                     const int32_t* block_tables, const int32_t* query_start,
                                     const int32_t* context_lens, long long num_blocks,
                                     int num_chunks, int num_heads, int num_kv_heads,
                                     int block_size, int max_blocks, int max_query_len,
                                     float scale_log2, const CUtensorMap* tm_k,
                                     const CUtensorMap* tm_v, cudaStream_t stream) {
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
    p.box_rows = prefill_box_rows(block_size);
    p.scale_log2 = scale_log2;
    if (p.q_tiles == 0 || num_chunks == 0) return cudaSuccess;
    if (p.box_rows == 0) tm_k = tm_v = nullptr;  // the cp.async loader
    if (dtype == TLB_BFLOAT16)
        return head_dim == 64 ? prefill::launch_d<__nv_bfloat16, 64>(p, tm_k, tm_v, stream)
                              : prefill::launch_d<__nv_bfloat16, 128>(p, tm_k, tm_v, stream);
    return head_dim == 64 ? prefill::launch_d<__half, 64>(p, tm_k, tm_v, stream)
                          : prefill::launch_d<__half, 128>(p, tm_k, tm_v, stream);
}

}  // namespace tlb
