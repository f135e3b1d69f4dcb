// Paged-attention decode for sm_100a.
//
// Reference semantics (cscr/attention_kernel.cu:24-107, launch :111-150):
// for every sequence s and query head h, softmax(scale * q[s,h] . K_s^T) V_s
// over the first seq_lens[s] tokens of the sequence, where token t lives in
// physical block block_tables[s, t / block_size] at offset t % block_size and
// uses KV head h / (num_heads / num_kv_heads). Tokens whose block id is
// negative are skipped; an empty softmax gives zeros (:102).
//
// Tensor-core path (fp16 / bf16, head_dim 64 or 128, group <= 16):
//   * Work is the flat list of (sequence, kv head) units, each a run of
//     stages of 64 tokens (the last one of a sequence may be shorter) plus a
//     fixed charge for starting a piece, cut into equal contiguous ranges of
//     that cost, one per persistent CTA ("stream-K"): every CTA gets the same
//     time's worth of stages and piece starts whatever the length mix, and a
//     range boundary never leaves a partly filled stage inside a sequence.
//   * Inside a CTA one producer warp walks its range and, per pipeline stage
//     of 64 tokens, issues 2-D TMA loads (128-byte swizzle, evict-first L2
//     policy) of each KV block straight from the paged cache, plus a bulk
//     load of the query group when a new (sequence, kv head) piece starts.
//   * Four consumer warps each take 16 tokens of a stage: S = Q K^T with
//     mma.m16n8k16 (query heads of one KV head folded into the 16 rows, so a
//     KV byte is read once for the whole group), an fp32 online softmax in
//     registers with quad shuffles, and O^T += V^T P^T with the softmax
//     probabilities fed straight from the S accumulators.
//   * A piece that covers a whole (sequence, kv head) is normalised and
//     written directly. A piece cut by a range boundary writes an fp32
//     partial (O, max, sum); the CTA that arrives last on that sequence's
//     counter merges the partials and writes the output, then the counter
//     is back at zero (atomicInc wrap), so no second kernel is launched.
//
// Generic path (fp32, other head sizes / groups / block sizes): one CTA per
// (sequence, kv head, head chunk), warps stride over tokens with the query
// group folded, fp32 CUDA-core arithmetic.
#pragma once

#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace tlb {
namespace attn {

namespace {

enum : int {
    kPieceStart = 1,
    kPieceEnd = 2,
    kPieceComplete = 4,
    kTerminate = 8,
    kRopeSkip = 16,  // fused step: the position is outside the cos/sin table, no rotation
    kNewToken = 32,  // fused step: the stage carries the new token's rows (new_r, new_row)
    kCtaLast = 64,   // the last stage of the CTA's range
};

// Written by the producer as four 16-byte stores.
struct alignas(16) StageDesc {
    unsigned rows[4];  // bit r of word r / 32: stage row r holds a token of the piece
    int flags;
    int seq;
    int kvh;
    int slot;        // partial slot of this piece (when not complete)
    int nsplits;     // pieces the (sequence, kv head) is cut into
    int jfirst;      // first CTA holding a piece of it
    int first_slot1; // that CTA stored its piece in its second slot
    int u;           // sequence * num_kv_heads + kv head
    int new_r;       // (kNewToken) stage row of the new token, -1 when not in the stage
    int new_row;     // (kNewToken) its cache row ((block * kv heads + kv head) * bs + offset),
                     // -1 when its block is not mapped
    int pad[2];
};

constexpr int kSeqCache = 1024; // context lengths kept in shared memory (first 1024 seqs)
constexpr int kCombineCap = 512; // (split, head) pairs the shared-memory combine handles
constexpr int kJobRing = 8;     // producer job ring (jobs generated ahead of issue)
// Work is measured in cost units: a stage costs kCostStage, and every
// (sequence, kv head) carries kCostPiece more for starting a piece (query
// load, hand-off and merge), so ranges that start many pieces get fewer
// stages. Stage i of a unit sits at cost kCostPiece + kCostStage * i from the
// unit's start; a range owns the stages whose cost point lies inside it.
constexpr int kCostStage = 4;
#ifndef TLB_ATTN_MAX_SPLITS
#define TLB_ATTN_MAX_SPLITS 32
#endif
constexpr int kMaxSplits = TLB_ATTN_MAX_SPLITS;  // most pieces a (sequence, kv head) is cut into
constexpr int kCostPiece = 5;
#ifndef TLB_ATTN_PREFETCH
#define TLB_ATTN_PREFETCH 3
#endif
// Stage jobs generated (block ids in flight) ahead of the one being issued;
// at most two jobs are generated per issued stage, so the lookahead never
// comes as a burst between two issues.
constexpr int kPrefetch = TLB_ATTN_PREFETCH;
static_assert(kPrefetch >= 2 && kPrefetch <= 6,
              "the job after the one issued is in the ring; cp.async waits handle <= 5 pending");
#ifndef TLB_ATTN_TAIL_DEN
#define TLB_ATTN_TAIL_DEN 0
#endif
// 1/kTailDen of the work is handed out as dynamically taken tail chunks
// (0: purely static ranges).
constexpr int kTailDen = TLB_ATTN_TAIL_DEN;

// One stage job of the producer: a run of <= blocks_per_stage KV blocks of a
// single (sequence, kv head) piece.
struct alignas(8) Job {
    int s, h, cb, nblk;
    int ns;          // stages of the sequence (clamped)
    int seqlen;
    int b_lo, b_hi;  // block range of the piece
    int st_hi;       // end of the piece in stages of the sequence
    long long pre;   // stages of all sequences before s
    // Per piece, computed once when the piece starts (a few divisions):
    int nsplits;     // pieces its (sequence, kv head) is cut into (1 = complete)
    int jfirst;      // first work range holding a piece of it
    int first_slot1; // that range stored its piece in its second slot
    int item;        // work item the piece belongs to (partial slot 2*item + !first)
    int first;       // first piece of its item
    int valid;
    int pos;         // position of the sequence's new token (its length - 1)
};

// Merge arithmetic of split pieces, shared by the epilogue warp's merge and
// the consumer warps' merge of a CTA's last piece: explicit roundings, so
// either path gives the same bits for the same pieces.
//
// Weights of one head over pieces j < cn: w[j * stride] holds piece j's max
// on entry and its weight exp2(m_j - M) on exit; returns lt + sum_j w_j l_j.
__device__ __forceinline__ float piece_weights(float* w, const float* l, int cn, int stride,
                                               float M, float lt) {
    for (int j = 0; j < cn; ++j) {
        const float wt = M == -INFINITY ? 0.f : exp2f(w[j * stride] - M);
        w[j * stride] = wt;
        lt = __fmaf_rn(wt, l[j * stride], lt);
    }
    return lt;
}
// a += w0 v0 + w1 v1, elementwise (pieces are summed in pairs, ascending)
__device__ __forceinline__ void add_pair(float4& a, float w0, const float4& v0, float w1,
                                         const float4& v1) {
    a.x = __fadd_rn(a.x, __fmaf_rn(w1, v1.x, __fmul_rn(w0, v0.x)));
    a.y = __fadd_rn(a.y, __fmaf_rn(w1, v1.y, __fmul_rn(w0, v0.y)));
    a.z = __fadd_rn(a.z, __fmaf_rn(w1, v1.z, __fmul_rn(w0, v0.z)));
    a.w = __fadd_rn(a.w, __fmaf_rn(w1, v1.w, __fmul_rn(w0, v0.w)));
}
// Most pieces the consumer warps merge themselves (the (m, l) of every piece
// sit in the hand-off buffer meanwhile, which bounds the count); a unit cut
// into more goes to the epilogue warp.
constexpr int kConsumerMergeMax = 120;
// With head dim 64 a piece's partial is half as large and the epilogue
// warp's merge correspondingly quicker: there the consumer warps take a
// CTA's last piece only when its unit is cut into at least this many pieces
// (measured on the shape sweep: fewer pieces lose more to the consumers'
// barrier phases than the wider merge wins).
constexpr int kConsumerMinPieces64 = 8;

#ifndef TLB_ATTN_TPW64
#define TLB_ATTN_TPW64 2
#endif
template <int D, int NT, int NSTAGE, int CW, bool FUSED>
struct TcLayout {
    // 16-token tiles each consumer warp takes per stage: head dim 64 takes two,
    // so a stage carries as many bytes (32 KB of K and V) as with head dim 128
    // and the per-stage costs are paid once per 32 KB either way.
    static constexpr int kTpw = D == 64 ? TLB_ATTN_TPW64 : 1;
    static constexpr int kRows = CW * kTileRows * kTpw;  // tokens per stage
    static constexpr int kChunks = D / 64;            // 128-byte column chunks per row
    static constexpr int kStageKV = kRows * D * 2;  // bytes of K (or V) per stage
    // query group of the piece, then (fused decode step) the cos/sin row of
    // the new token's position and that token's raw key and value rows
    static constexpr int kQBytes = 8 * NT * D * 2 + (FUSED ? 3 * D * 2 : 0);
    static constexpr int kGP = 8 * NT;                 // padded heads per piece
    static constexpr int kOFloats = CW * kGP * D;
    static constexpr int kOffK = 0;
    static constexpr int kOffV = kOffK + NSTAGE * kStageKV;
    static constexpr int kOffQ = kOffV + NSTAGE * kStageKV;
    static constexpr int kOffO = kOffQ + NSTAGE * kQBytes;
    static constexpr int kOffM = kOffO + kOFloats * 4;
    static constexpr int kOffL = kOffM + CW * kGP * 4;
    static constexpr int kOffDesc = (kOffL + CW * kGP * 4 + 15) / 16 * 16;
    static constexpr int kOffBar = (kOffDesc + NSTAGE * (int)sizeof(StageDesc) + 7) / 8 * 8;
    // + epilogue full/empty + consumer warps' own barrier
    static constexpr int kOffMisc = kOffBar + (2 * NSTAGE + 3) * 8;
    static constexpr int kMiscInts = 64;
    static constexpr int kOffProd = kOffMisc + kMiscInts * 4;  // producer scratch
    static constexpr int kProdBytes = kSeqCache * 8 + kJobRing * (int)sizeof(Job) + kJobRing * (kRows / 8) * 4;
    static constexpr int kOffEpi = (kOffProd + kProdBytes + 15) / 16 * 16;  // hand-off descriptor
    static constexpr int kOffW = kOffEpi + (int)sizeof(StageDesc);     // merge weights, M, L
    static constexpr int kOffCW = kOffW + (CW * kGP + 2 * kGP) * 4;
    static constexpr int kOffOwn = kOffCW + 2 * kCombineCap * 4;      // combine weights, sums
    static constexpr int kBytes = kOffOwn + kGP * D * 4;  // a merging piece's own partial
    // TMA destinations sit on 1024-byte swizzle atoms; float4 / 16-byte
    // structures on 16 bytes.
    static_assert(kOffK % 1024 == 0 && kOffV % 1024 == 0 && kStageKV % 1024 == 0, "TMA tiles");
    static_assert(kOffQ % 16 == 0 && kQBytes % 16 == 0, "bulk copy of the query");
    static_assert(kOffO % 16 == 0 && kOffDesc % 16 == 0 && kOffEpi % 16 == 0 && kOffW % 16 == 0,
                  "16-byte accesses");
    static_assert(kOffOwn % 16 == 0 && kOffBar % 8 == 0 && kOffProd % 8 == 0,
                  "aligned words");
    static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
};

// Block-wide inclusive scan of a 64-bit value over blockDim.x threads.
__device__ __forceinline__ long long block_incl_scan(long long v, long long* warp_sums,
                                                     long long* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nwarps = (blockDim.x + 31) >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        long long n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
    }
    if (lane == 31) warp_sums[warp] = v;
    __syncthreads();
    long long before = 0, all = 0;
    for (int w = 0; w < nwarps; ++w) {
        const long long ws = warp_sums[w];
        if (w < warp) before += ws;
        all += ws;
    }
    __syncthreads();
    *total = all;
    return v + before;
}

// Quotient of non-negative a and positive b: one 32-bit division when both
// fit in 32 bits (every launch below 2^32 cost units), else the 64-bit one.
__device__ __forceinline__ long long div_nn(long long a, long long b) {
    return ((unsigned long long)(a | b) >> 32) == 0ull
               ? (long long)((unsigned)a / (unsigned)b)
               : a / b;
}
// CTA whose unit range [floor(j W / P), floor((j+1) W / P)) contains unit x.
__device__ __forceinline__ int cta_of(long long x, long long W, int P) {
    return (int)div_nn((x + 1) * (long long)P - 1, W);
}
__device__ __forceinline__ long long range_start(int j, long long W, int P) {
    return div_nn((long long)j * W, P);
}
__host__ __device__ constexpr int ilog2_c(int v) { return v <= 1 ? 0 : 1 + ilog2_c(v >> 1); }



}  // namespace

// One head tile (NT == 1) keeps two CTAs per SM: at most 168 registers.
template <typename T, int D, int NT, int NSTAGE, int CW, bool FUSED, bool INJECT>
__global__ void __launch_bounds__((CW + 2) * 32, (NT == 1 && CW == 4) ? 2 : 1)
    paged_attention_tc_kernel(const __grid_constant__ CUtensorMap tm_k,
                              const __grid_constant__ CUtensorMap tm_v, const TcParams p) {
    using L = TcLayout<D, NT, NSTAGE, CW, FUSED>;
    constexpr int ROWS = L::kRows;        // tokens per stage
    constexpr int kBpsMax = ROWS / 8;     // most KV blocks in a stage (block_size >= 8)
    constexpr int kCS = kCostStage * ROWS / 64;  // cost of one stage of ROWS tokens
    constexpr int GP = L::kGP;
    constexpr int KS = D / 16;  // k-steps of QK, m-tiles of PV
    // probes before a pipeline wait gives up (copy drains keep the default);
    // a compile-time constant except in the failure-injection instances
    const uint32_t wlim = INJECT ? p.wait_limit : kWaitLimit;

    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
    const uint32_t sbase = smem_u32(smem);

    float* sO = reinterpret_cast<float*>(smem + L::kOffO);
    float* sM = reinterpret_cast<float*>(smem + L::kOffM);
    float* sL = reinterpret_cast<float*>(smem + L::kOffL);
    StageDesc* sDesc = reinterpret_cast<StageDesc*>(smem + L::kOffDesc);
    const uint32_t bar_full = sbase + L::kOffBar;           // NSTAGE x 8 bytes
    const uint32_t bar_empty = bar_full + NSTAGE * 8;       // NSTAGE x 8 bytes
    const uint32_t bar_epi_full = bar_empty + NSTAGE * 8;   // consumers -> epilogue
    const uint32_t bar_epi_empty = bar_epi_full + 8;        // epilogue -> consumers
    const uint32_t bar_cons = bar_epi_empty + 8;            // consumer warps among themselves
    StageDesc* sEpi = reinterpret_cast<StageDesc*>(smem + L::kOffEpi);
    float* sW = reinterpret_cast<float*>(smem + L::kOffW);
    float* sHM = sW + CW * GP;
    float* sHL = sHM + GP;
    float* sCW = reinterpret_cast<float*>(smem + L::kOffCW);
    float* sCL = sCW + kCombineCap;
    float* sOwn = reinterpret_cast<float*>(smem + L::kOffOwn);
    long long* sScan = reinterpret_cast<long long*>(smem + L::kOffMisc);  // 8 warp sums
    int* sMisc = reinterpret_cast<int*>(smem + L::kOffMisc + 8 * 8);

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int S = p.num_seqs;
    const int KVH = p.num_kv_heads;
    const int G = p.group;
    const int bs = p.block_size;
    const int cap_tokens = p.max_blocks * bs;
    // Block sizes are powers of two (8 to 64; the host checks), so every
    // division by the block size or by the blocks per stage is a shift.
    const int bs_sh = __ffs(bs) - 1;
    static_assert((ROWS & (ROWS - 1)) == 0, "stage rows are a power of two");

    if (tid == 0) {
        for (int i = 0; i < NSTAGE; ++i) {
            mbar_init(bar_full + 8 * i, 1);
            mbar_init(bar_empty + 8 * i, CW);
        }
        mbar_init(bar_epi_full, CW * 32);
        mbar_init(bar_epi_empty, 32);
        mbar_init(bar_cons, CW * 32);
        fence_mbar_init();
        fence_proxy_async_smem();
    }
    if (warp == CW && lane == 0) {
        prefetch_tensormap(&tm_k);
        prefetch_tensormap(&tm_v);
    }
    // The next kernel on the stream, if launched programmatically, may start
    // its own prologue once SMs free up; it waits for this grid to finish
    // before it writes or reads anything this kernel produces.
    grid_launch_dependents();

    // ---- pass 1: context lengths -> shared memory, exclusive prefix of
    // cost per sequence (per kv head), total. Thread t owns sequences [t*per, t*per+per):
    // one batch of independent loads, one block scan.
    int* sSeqLen = reinterpret_cast<int*>(smem + L::kOffProd);
    unsigned* sPre = reinterpret_cast<unsigned*>(smem + L::kOffProd + kSeqCache * 4);
    auto len_of = [&](int s) -> int { return s < kSeqCache ? sSeqLen[s] : p.seq_lens[s]; };
    auto blocks_of = [&](int len) -> int {
        len = min(len, cap_tokens);
        return len > 0 ? (len + bs - 1) >> bs_sh : 0;
    };
    const int bps = ROWS >> bs_sh;  // KV blocks per stage
    constexpr int kRowsSh = ilog2_c(ROWS);
    const int bps_sh = kRowsSh - bs_sh;
    auto stages_of = [&](int len) -> int { return (blocks_of(len) + bps - 1) >> bps_sh; };
    auto cost_of = [&](int len) -> int {  // per kv head
        const int ns = stages_of(len);
        return ns > 0 ? kCostPiece + kCS * ns : 0;
    };
    long long total_cost;
    {
        const int per = (S + (int)blockDim.x - 1) / (int)blockDim.x;
        const int s0 = min(S, tid * per), s1 = min(S, s0 + per);
        long long mine = 0;
        unsigned bad_len = 0;
        for (int s = s0; s < s1; ++s) {
            const int len = p.seq_lens[s];
            if (s < kSeqCache) sSeqLen[s] = len;
            if (len > cap_tokens) bad_len = 1;
            mine += cost_of(len);
        }
        if (bad_len) flag_status(TLB_STATUS_SEQ_TOO_LONG);
        long long run = block_incl_scan(mine, sScan, &total_cost) - mine;
        for (int s = s0; s < min(s1, kSeqCache); ++s) {
            sPre[s] = (unsigned)run;
            run += cost_of(sSeqLen[s]);
        }
        if (tid == 0 && S < kSeqCache) sPre[S] = (unsigned)total_cost;
        __syncthreads();
    }

    // Until griddepcontrol.wait this kernel only reads metadata (seq_lens,
    // block_tables) and writes nothing but its own status word: with
    // programmatic launch it may be running beside the kernel before it.
    T* out = reinterpret_cast<T*>(p.out);
    // Sequences with no context get zeros (attention_kernel.cu:102); CTA j
    // covers sequences j, j + grid, ... with the threads [first, first + n).
    auto zero_empty_outputs = [&](int first, int n) {
        for (int s = blockIdx.x; s < S; s += gridDim.x) {
            if (len_of(s) <= 0) {
                const long long base = (long long)s * p.num_heads * D;
                for (int e = first; e < p.num_heads * D; e += n)
                    out[base + e] = Elem<T>::from_f(0.f);
            }
        }
    };

    const long long W = total_cost * KVH;
    if (W == 0) {
        grid_dependency_wait();
        zero_empty_outputs(tid, blockDim.x);
        return;
    }
    // ---- work items. Items [0, P) split the first Ws units into equal
    // contiguous ranges, one per CTA (stream-K). With the prefix cached, the
    // last quarter of the units forms T tail chunks of C units, taken in order
    // from an atomic counter by whichever CTA is free first, so CTAs that
    // stream faster take more of them and all finish together.
    const bool cached = S < kSeqCache && total_cost < (1ll << 32);
    const long long Ws = (cached && kTailDen > 0) ? W - W / (kTailDen > 0 ? kTailDen : 1) : W;
    int P = (int)gridDim.x;
    {
        // Ranges of at least min_tokens, and long enough that a
        // (sequence, kv head) of average cost is cut into at most kMaxSplits
        // pieces: the last piece merges the others one pair at a time.
        const long long avg_unit = div_nn(W, (long long)S * KVH);
        // Every range is at least one stage's cost long, so a range inside a
        // unit always holds a stage point and each piece count (nsplits) is
        // exact: ranges are floor(Ws / P) or longer.
        const long long min_cost = max((long long)max(1, p.min_tokens / ROWS) * kCS,
                                       (avg_unit + kMaxSplits - 1) / kMaxSplits);
        const long long want = div_nn(Ws, min_cost);
        if (want < P) P = (int)(want > 0 ? want : 1);
    }
    const long long Wt = W - Ws;
    long long C = div_nn(Wt + 2ll * gridDim.x - 1, 2ll * gridDim.x);
    if (C < kCS) C = kCS;  // a chunk holds at least one stage point
    const int T_tail = (int)div_nn(Wt + C - 1, C);
    // Range starts and the range holding a cost point are computed where
    // they are needed, not tabulated: with operands below 2^32 each is one
    // 32-bit division, cheaper than filling a table of all range starts
    // before the producer's first lookup.
    auto static_start = [&](int i) -> long long { return range_start(i, Ws, P); };
    auto item_start = [&](int i) -> long long {
        return i < P ? static_start(i) : Ws + (long long)(i - P) * C;
    };
    auto item_end = [&](int i) -> long long {
        return i < P ? static_start(i + 1) : min(W, Ws + (long long)(i - P + 1) * C);
    };
    auto item_of = [&](long long x) -> int {
        if (x >= Ws) return P + (int)div_nn(x - Ws, C);
        return cta_of(x, Ws, P);
    };
    const int j = blockIdx.x;

    // Sequence holding cost point x and its cost prefix: binary search of the
    // cached prefix, or (uncached) a block-wide scan for the static item.
    // The largest s with sPre[s] * KVH <= x. The prefix is non-decreasing
    // from sPre[0] = 0, so the sequences that pass form a prefix: with at
    // most 64 sequences two warp ballots count them (all 32 lanes call this).
    auto locate_cached = [&](long long x, long long& pre) -> int {
        int lo;
        if (S <= 64) {
            const unsigned t0 = __ballot_sync(0xffffffffu, lane < S && (long long)sPre[lane] * KVH <= x);
            const unsigned t1 =
                __ballot_sync(0xffffffffu, lane + 32 < S && (long long)sPre[lane + 32] * KVH <= x);
            lo = __popc(t0) + __popc(t1) - 1;
        } else {
            lo = 0;
            int hi = S - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if ((long long)sPre[mid] * KVH <= x) lo = mid; else hi = mid - 1;
            }
        }
        pre = sPre[lo];
        return lo;
    };
    int s_first = 0;
    long long pre_first = 0;
    if (j < P && !cached) {
        const long long ustart = item_start(j);
        if (tid == 0) sMisc[0] = -1;
        __syncthreads();
        long long base = 0;
        for (int c0 = 0; c0 < S; c0 += blockDim.x) {
            const int s = c0 + tid;
            const long long nb = s < S ? cost_of(len_of(s)) : 0;
            long long chunk_total;
            const long long incl = block_incl_scan(nb, sScan, &chunk_total);
            const long long excl = incl - nb;
            if (nb > 0 && (base + excl) * KVH <= ustart && ustart < (base + incl) * KVH) {
                sMisc[0] = s;
                reinterpret_cast<long long*>(sMisc)[1] = base + excl;
            }
            __syncthreads();
            base += chunk_total;
            if (base * KVH > ustart) break;
        }
        __syncthreads();
        s_first = sMisc[0];
        pre_first = reinterpret_cast<long long*>(sMisc)[1];
        if (s_first < 0) {  // cannot happen for ustart < W; never walk from garbage
            grid_dependency_wait();
            zero_empty_outputs(tid, blockDim.x);
            return;
        }
    }

    if (warp == CW) {
        // ===================================================== producer warp
        const uint64_t pol = l2_policy_evict_first();
        constexpr bool fused = FUSED;  // p.cos_sin != nullptr
        const T* cos_sin = reinterpret_cast<const T*>(p.cos_sin);
        const T* key_new = reinterpret_cast<const T*>(p.key_new);
        const T* value_new = reinterpret_cast<const T*>(p.value_new);
        // Fused decode step: the new token (position job.pos) has a cos/sin row.
        auto pos_ok = [&](const Job& job) -> bool {
            return job.pos >= 0 && (long long)job.pos < p.cache_rows;
        };
        // Whether this job is the last stage of a piece that runs to its
        // (sequence, kv head)'s end: that stage alone holds the sequence's
        // last block, so it carries the new token's rows.
        auto carries_new_token = [&](const Job& job) -> bool {
            return fused && job.st_hi == job.ns && job.cb + job.nblk == job.b_hi;
        };
        // Whether the new token's block is among this stage's blocks.
        auto new_token_here = [&](const Job& job) -> bool {
            const int blk_i = job.pos >> bs_sh;  // used only when pos >= 0
            return job.pos >= 0 && job.pos < cap_tokens && blk_i >= job.cb &&
                   blk_i < job.cb + job.nblk;
        };
        const T* query = reinterpret_cast<const T*>(p.query);
        Job* sJob = reinterpret_cast<Job*>(smem + L::kOffProd + kSeqCache * 8);
        const uint32_t sBid = sbase + L::kOffProd + kSeqCache * 8 + kJobRing * (int)sizeof(Job);
        const int* sBidPtr = reinterpret_cast<const int*>(smem + L::kOffProd + kSeqCache * 8 +
                                                          kJobRing * (int)sizeof(Job));

        // First job of the first piece at or after cost point x (inside
        // sequence s, whose cost prefix is `pre`, or a later one) of work
        // item `item`; invalid when the item holds no further stage.
        auto piece_job = [&](long long x, int s, long long pre, int item, bool first) -> Job {
            Job jb;
            jb.valid = 0;
            const long long iend = item_end(item);
            while (true) {
                if (x >= iend || s >= S) return jb;
                const int len = len_of(s);
                const int ns = stages_of(len);
                if (ns == 0) {  // empty sequence: no cost, nothing to do
                    ++s;
                    continue;
                }
                const int L1 = kCostPiece + kCS * ns;  // cost of one unit
                const long long rel = x - pre * KVH;          // < KVH * L1
                int h, r;
                if (rel < 0x7fffffffll) {
                    h = (int)((unsigned)rel / (unsigned)L1);
                    r = (int)((unsigned)rel - (unsigned)h * (unsigned)L1);
                } else {
                    h = (int)(rel / L1);
                    r = (int)(rel % L1);
                }
                const long long U = pre * KVH + (long long)h * L1;  // unit start
                // first stage whose cost point is at or after x
                const int i_lo = r <= kCostPiece ? 0 : (r - kCostPiece + kCS - 1) / kCS;
                if (i_lo >= ns) {  // past this unit's last stage: next unit
                    x = U + L1;
                    if (h + 1 >= KVH) {
                        pre += L1;
                        ++s;
                    }
                    continue;
                }
                const long long end_r = iend - U;
                const int i_hi =
                    end_r <= kCostPiece
                        ? 0
                        : (int)min((long long)ns,
                                   (end_r - kCostPiece + kCS - 1) / kCS);
                if (i_hi <= i_lo) return jb;  // the range ends before the next stage
                const int nb = blocks_of(len);
                jb.s = s;
                jb.h = h;
                jb.st_hi = i_hi;
                jb.b_lo = i_lo * bps;
                jb.b_hi = min(nb, i_hi * bps);
                jb.cb = jb.b_lo;
                jb.nblk = min(bps, jb.b_hi - jb.cb);
                jb.ns = ns;
                jb.seqlen = max(0, min(len, cap_tokens));
                jb.pos = len - 1;
                jb.pre = pre;
                jb.item = item;
                jb.first = first ? 1 : 0;
                if (i_lo == 0 && i_hi == ns) {
                    jb.nsplits = 1;
                    jb.jfirst = item;
                    jb.first_slot1 = 0;
                } else {
                    // owners of the first and the last stage; the first owner
                    // holds an earlier stage (the previous unit's last, at
                    // U - kCS) when its range starts at or before it
                    const int jf = item_of(U + kCostPiece);
                    jb.nsplits = item_of(U + kCostPiece + (long long)kCS * (ns - 1)) - jf + 1;
                    jb.jfirst = jf;
                    jb.first_slot1 = (U > 0 && item_start(jf) <= U - kCS) ? 1 : 0;
                }
                jb.valid = 1;
                return jb;
            }
        };
        auto first_job_of = [&](int item) -> Job {
            long long pre;
            const long long x = item_start(item);
            const int s = locate_cached(x, pre);
            return piece_job(x, s, pre, item, true);
        };
        // Next tail chunk, or an invalid job when none is left. Every lane of
        // the producer warp runs the job generator in lockstep; lane 0 alone
        // takes the chunk and broadcasts it.
        auto grab = [&]() -> Job {
            Job none;
            none.valid = 0;
            if (T_tail == 0) return none;
            unsigned t = 0;
            if (lane == 0) t = atomicAdd(p.sched, 1u);
            t = __shfl_sync(0xffffffffu, t, 0);
            if ((int)t >= T_tail) return none;
            return first_job_of(P + (int)t);
        };
        auto next_job = [&](const Job& jb) -> Job {
            if (jb.cb + jb.nblk < jb.b_hi) {
                Job n = jb;
                n.cb = jb.cb + jb.nblk;
                n.nblk = min(bps, jb.b_hi - n.cb);
                return n;
            }
            // piece finished: the next unit of the item when the piece ran to
            // its unit's end, else (or if nothing is left) the next item
            if (jb.st_hi == jb.ns) {
                const long long x = jb.pre * KVH + (long long)(jb.h + 1) * (kCostPiece + kCS * jb.ns);
                const Job n = jb.h + 1 < KVH
                                  ? piece_job(x, jb.s, jb.pre, jb.item, false)
                                  : piece_job(x, jb.s + 1, jb.pre + kCostPiece + kCS * jb.ns,
                                              jb.item, false);
                if (n.valid) return n;
            }
            return grab();
        };

        // Jobs are generated up to kPrefetch stages ahead of the one being
        // issued: the job goes to a shared ring and its block ids are copied
        // there with cp.async, so the dependent global read of the block
        // table never sits between two TMA issues. New jobs are generated
        // right after a stage is issued, while the producer would otherwise
        // wait for a free stage, so the per-piece bookkeeping (divisions
        // and range lookups) never delays an issue. `pj` is the next job to store; it
        // is advanced lazily, so nothing is taken from the tail counter
        // before griddepcontrol.wait.
        Job pj;
        pj.valid = 0;
        bool have_pj = false;
        if (j < P) {
            if (cached) {
                pj = first_job_of(j);
            } else {
                pj = piece_job(item_start(j), s_first, pre_first, j, true);
            }
            have_pj = true;
        }
        auto prefetch = [&](int k) {
            if (!have_pj) {
                pj = grab();
                have_pj = true;
            } else if (k > 0 && pj.valid) {
                pj = next_job(pj);
            }
            const int slot = k % kJobRing;
            if (lane == 0) sJob[slot] = pj;
            // The query group of a new piece is pulled into L2 (and its page
            // into the TLB) kPrefetch stages before its bulk load. L2 is the
            // coherence point, so this is safe before griddepcontrol.wait.
            if (lane == 0 && pj.valid && pj.cb == pj.b_lo) {
                bulk_prefetch_l2(query + ((long long)pj.s * p.num_heads + (long long)pj.h * G) * D,
                                 (uint32_t)(G * D * 2));
            }
            if (lane == 0 && pj.valid && carries_new_token(pj)) {  // its raw key and value
                bulk_prefetch_l2(key_new + pj.s * p.key_stride + (long long)pj.h * D,
                                 (uint32_t)(D * 2));
                bulk_prefetch_l2(value_new + pj.s * p.value_stride + (long long)pj.h * D,
                                 (uint32_t)(D * 2));
            }
            if (pj.valid && lane < pj.nblk)
                cp_async_4(sBid + (uint32_t)(slot * kBpsMax + lane) * 4u,
                           p.block_tables + (long long)pj.s * p.max_blocks + pj.cb + lane);
            cp_async_commit();
        };
        // Waits until job k and its block ids have landed: at most
        // nf - k - 1 of the committed cp.async groups may still be pending.
        auto wait_job = [&](int nf_, int k) {
            switch (nf_ - k - 1) {
                case 0: cp_async_wait<0>(); break;
                case 1: cp_async_wait<1>(); break;
                case 2: cp_async_wait<2>(); break;
                case 3: cp_async_wait<3>(); break;
                case 4: cp_async_wait<4>(); break;
                default: cp_async_wait<5>(); break;
            }
            __syncwarp();
        };
        // Loaded blocks of stage job k (bit b: block b of the stage) and the
        // tile row of every block, in every lane.
        auto stage_blocks = [&](const Job& job, int k, int32_t (&ys)[kBpsMax]) -> unsigned {
            const int bid = lane < job.nblk ? sBidPtr[(k % kJobRing) * kBpsMax + lane] : -1;
            const bool in_range = lane < job.nblk;
            const bool valid = in_range && bid >= 0 && (long long)bid < p.num_blocks;
            if (in_range && (long long)bid >= p.num_blocks) flag_status(TLB_STATUS_BAD_BLOCK_ID);
            const int32_t my_y = (int32_t)(((long long)bid * KVH + job.h) * bs);
#pragma unroll
            for (int b = 0; b < kBpsMax; ++b) ys[b] = __shfl_sync(0xffffffffu, my_y, b);
            return __ballot_sync(0xffffffffu, valid);
        };
        // Descriptor and transaction count of a stage (elected lane).
        auto arm_stage = [&](const Job& job, int stage, unsigned vmask, bool new_tok, int new_r,
                             int new_row, bool cta_last) {
            const bool piece_start = job.cb == job.b_lo;
            const bool piece_end = job.cb + job.nblk == job.b_hi;
            // Valid rows: inside the stage, before the context end, in a
            // block that is loaded.
            const int tok0 = job.cb * bs;
            const int nv = min(job.nblk * bs, job.seqlen - tok0);
            unsigned rows[4];
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                const int lo = 32 * w;
                rows[w] = nv >= lo + 32 ? ~0u : (nv > lo ? (1u << (nv - lo)) - 1u : 0u);
            }
            for (unsigned inval = (~vmask) & ((1u << job.nblk) - 1u); inval != 0u; inval &= inval - 1u) {
                const int r0b = (__ffs(inval) - 1) * bs;  // rows [r0b, r0b + bs) of a missing block
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    const int a = max(r0b, 32 * w) - 32 * w, b = min(r0b + bs, 32 * w + 32) - 32 * w;
                    if (a < b) rows[w] &= ~((b - a >= 32 ? ~0u : ((1u << (b - a)) - 1u)) << a);
                }
            }
            const int flags = (piece_start ? kPieceStart : 0) | (piece_end ? kPieceEnd : 0) |
                              (job.nsplits == 1 ? kPieceComplete : 0) |
                              (fused && !pos_ok(job) ? kRopeSkip : 0) | (new_tok ? kNewToken : 0) |
                              (cta_last ? kCtaLast : 0);
            if (fused && piece_start && !pos_ok(job)) flag_status(TLB_STATUS_BAD_POSITION);
            int4* dw = reinterpret_cast<int4*>(&sDesc[stage]);
            dw[0] = make_int4((int)rows[0], (int)rows[1], (int)rows[2], (int)rows[3]);
            dw[1] = make_int4(flags, job.s, job.h, 2 * job.item + (job.first ? 0 : 1));
            dw[2] = make_int4(job.nsplits, job.jfirst, job.first_slot1, job.s * KVH + job.h);
            if (FUSED) dw[3] = make_int4(new_r, new_row, 0, 0);
            // KV tiles, the query group and cos/sin row of a piece start, the
            // new token's key and value rows (and cos/sin row) of its stage
            const uint32_t bytes = (uint32_t)__popc(vmask) * (uint32_t)bs * D * 2u * 2u +
                                   (piece_start ? (uint32_t)(G * D * 2 + (fused ? D * 2 : 0)) : 0u) +
                                   (new_tok ? (uint32_t)(2 * D * 2 + (piece_start ? 0 : D * 2)) : 0u);
            mbar_arrive_expect_tx(bar_full + 8 * stage, bytes);
        };
        // The copies of the blocks in `mask` (one (block, kv head) tile per
        // copy: [chunk][bs rows][128 B]) and, if asked, of the query group
        // and of the new token's rows.
        auto issue_copies = [&](const Job& job, int stage, unsigned mask,
                                const int32_t (&ys)[kBpsMax], bool with_query, bool new_tok) {
            const uint32_t fb = bar_full + 8 * stage;
            const uint32_t kdst = sbase + L::kOffK + stage * L::kStageKV;
            const uint32_t vdst = sbase + L::kOffV + stage * L::kStageKV;
#pragma unroll
            for (int b = 0; b < kBpsMax; ++b) {
                if ((mask >> b) & 1u) {
                    tma_load_3d(kdst + b * bs * D * 2, &tm_k, 0, ys[b], 0, fb, pol);
                    tma_load_3d(vdst + b * bs * D * 2, &tm_v, 0, ys[b], 0, fb, pol);
                }
            }
            if (with_query) {
                const T* qsrc = query + ((long long)job.s * p.num_heads + (long long)job.h * G) * D;
                bulk_load(sbase + L::kOffQ + stage * L::kQBytes, qsrc, (uint32_t)(G * D * 2), fb);
            }
            const uint32_t cdst = sbase + L::kOffQ + stage * L::kQBytes + GP * D * 2;
            if (fused && (with_query || new_tok))  // cos/sin row of the new token (row 0 when out of the table)
                bulk_load(cdst, cos_sin + (pos_ok(job) ? (long long)job.pos * D : 0ll),
                          (uint32_t)(D * 2), fb);
            if (new_tok) {
                bulk_load(cdst + D * 2, key_new + job.s * p.key_stride + (long long)job.h * D,
                          (uint32_t)(D * 2), fb);
                bulk_load(cdst + 2 * D * 2, value_new + job.s * p.value_stride + (long long)job.h * D,
                          (uint32_t)(D * 2), fb);
            }
        };
        int nf = 0;  // jobs generated (cp.async groups committed)
        int stage = 0;
        uint32_t phase = 0;
        if (have_pj) {
            prefetch(nf++);
            prefetch(nf++);
        }
        // Everything above reads only metadata; the query and the cache may
        // still be written by the kernel launched just before this one.
        grid_dependency_wait();
        while (nf < 2) prefetch(nf++);
        bool ok = true;
        for (int k = 0;; ++k) {
            if (k >= nf) break;  // never read a ring slot no job was written to
            wait_job(nf, k);
            const Job job = sJob[k % kJobRing];
            if (!job.valid) break;

            bool waited = true;  // the first NSTAGE slots are fresh: no wait
            if (k >= NSTAGE) {
                if (lane == 0) waited = mbar_wait_bounded(bar_empty + 8 * stage, phase ^ 1, wlim);
                waited = __shfl_sync(0xffffffffu, waited, 0);
            }
            if (!waited) {
                if (lane == 0) flag_status(TLB_STATUS_WAIT_TIMEOUT);
                ok = false;
                break;
            }
            int32_t ys[kBpsMax];
            const unsigned vmask = stage_blocks(job, k, ys);
            // Fused decode step: where the new token sits in this stage and in
            // the cache (the consumers write its rows; see below).
            const bool new_tok = carries_new_token(job);
            int new_r = -1, new_row = -1;
            if (new_tok && new_token_here(job)) {
                const int b = (job.pos >> bs_sh) - job.cb;
                new_r = job.pos - job.cb * bs;
                int32_t y = 0;
#pragma unroll
                for (int bb = 0; bb < kBpsMax; ++bb) y = bb == b ? ys[bb] : y;
                if ((vmask >> b) & 1u) new_row = y + (job.pos & (bs - 1));
            }
            if (elect_one()) {
                // jobs up to k + kPrefetch are in the ring: an invalid next job
                // means this stage ends the CTA's range
                arm_stage(job, stage, vmask, new_tok, new_r, new_row,
                          !sJob[(k + 1) % kJobRing].valid);
                issue_copies(job, stage, vmask, ys, job.cb == job.b_lo, new_tok);
            }
            __syncwarp();
            if (++stage == NSTAGE) { stage = 0; phase ^= 1; }
            for (int t = 0; t < 2 && nf < k + 1 + kPrefetch; ++t) prefetch(nf++);
        }
        cp_async_wait<0>();
        // outputs of sequences with no context (after the stream: they are
        // not on the way to the first copy)
        zero_empty_outputs(lane, 32);
        if (T_tail > 0 && lane == 0) {
            // The last CTA to finish taking tail chunks resets the counters
            // for the next launch (they live in the zeroed workspace prefix).
            if (atomicAdd(p.sched + 1, 1u) == gridDim.x - 1) {
                atomicExch(p.sched, 0u);
                atomicExch(p.sched + 1, 0u);
            }
        }
        bool drain = !ok;
        if (ok) {
            bool waited = true;
            if (lane == 0) waited = mbar_wait_bounded(bar_empty + 8 * stage, phase ^ 1, wlim);
            waited = __shfl_sync(0xffffffffu, waited, 0);
            if (lane == 0) {
                if (waited) {
                    sDesc[stage].flags = kTerminate;
                    mbar_arrive(bar_full + 8 * stage);
                } else {
                    flag_status(TLB_STATUS_WAIT_TIMEOUT);
                }
            }
            drain = !waited;
        }
        if (drain) {
            // A wait gave up: let the copies already issued land before the
            // CTA's shared memory is released (these waits keep the default
            // bound: an issued copy always lands). Stage `stage` was not
            // issued; the NSTAGE-1 before it may have been.
            if (lane == 0) {
                int st = stage;
                uint32_t ph = phase;
                for (int k = 0; k < NSTAGE - 1; ++k) {
                    if (st == 0) { st = NSTAGE - 1; ph ^= 1; } else { --st; }
                    mbar_wait_bounded(bar_full + 8 * st, ph);
                }
            }
        }
        return;
    }

    if (warp == CW + 1) {
        // ===================================================== epilogue warp
        // Merges the consumer warps' (m, l, O) of each finished piece, frees
        // the hand-off buffer, then writes the output (whole piece) or an fp32
        // partial; the last partial of a (sequence, kv head) to arrive merges
        // all of them. None of this stalls the KV stream.
        constexpr int kPer4 = GP * D / 128;  // float4 groups of the piece per lane
        uint32_t ephase = 0;
        while (true) {
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(bar_epi_full, ephase, wlim))) {
                if (lane == 0) flag_status(TLB_STATUS_WAIT_TIMEOUT);
                break;
            }
            const StageDesc e = *sEpi;
            if (e.flags & kTerminate) break;
            if (lane < G) {
                float M = -INFINITY;
#pragma unroll
                for (int w = 0; w < CW; ++w) M = fmaxf(M, sM[w * GP + lane]);
                float lt = 0.f;
#pragma unroll
                for (int w = 0; w < CW; ++w) {
                    const float wt = M == -INFINITY ? 0.f : exp2f(sM[w * GP + lane] - M);
                    sW[w * GP + lane] = wt;
                    lt += wt * sL[w * GP + lane];
                }
                sHM[lane] = M;
                sHL[lane] = lt;
            }
            __syncwarp();
            // Lane `lane` owns the float4 groups el4 = lane + 32 * i (elements
            // 4 * el4 .. + 3 of the piece, all of one head): 16-byte shared
            // and global accesses, independent across i.
            float4 acc[kPer4];
#pragma unroll
            for (int i = 0; i < kPer4; ++i) {
                const int el = 4 * (lane + 32 * i);
                const int h = el / D, dd = el % D;
                float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
                if (h < G) {
#pragma unroll
                    for (int w = 0; w < CW; ++w) {
                        const float wt = sW[w * GP + h];
                        const float4 v = *reinterpret_cast<const float4*>(sO + (w * GP + h) * D + dd);
                        a.x += wt * v.x; a.y += wt * v.y; a.z += wt * v.z; a.w += wt * v.w;
                    }
                }
                acc[i] = a;
            }
            __syncwarp();
            mbar_arrive(bar_epi_empty);  // hand-off buffer free again
            ephase ^= 1;

            const long long out_base = ((long long)e.seq * p.num_heads + (long long)e.kvh * G) * D;
            auto store_out = [&](int i, float scale) {
                const int el = 4 * (lane + 32 * i);
                Vec4Out<T>::store(out + out_base + el, acc[i], scale);
            };
            if (e.flags & kPieceComplete) {
#pragma unroll
                for (int i = 0; i < kPer4; ++i) {
                    const int h = 4 * (lane + 32 * i) / D;
                    if (h < G) {
                        const float lt = sHL[h];
                        store_out(i, lt > 0.f ? 1.f / lt : 0.f);
                    }
                }
                continue;
            }
            // A piece of a split (sequence, kv head). If every other piece
            // has already published its partial (counter at nsplits - 1),
            // this one is the last: it merges straight from registers and
            // skips its own partial and the atomic. Otherwise it publishes
            // and takes a ticket; the last ticket merges from the workspace.
            const int n = e.nsplits;
            auto slot_k = [&](int k) -> long long {
                return 2ll * (e.jfirst + k) + ((k == 0 && e.first_slot1) ? 1 : 0);
            };
            unsigned seen = 0;
            if (lane == 0) seen = ld_acquire_gpu(p.counters + e.u);
            seen = __shfl_sync(0xffffffffu, seen, 0);
            const bool own_in_regs = seen == (unsigned)(n - 1);
            if (own_in_regs) {
                if (lane == 0) st_relaxed_gpu(p.counters + e.u, 0u);  // ready for the next launch
            } else {
                float* wo = p.ws_o + (long long)e.slot * GP * D;
#pragma unroll
                for (int i = 0; i < kPer4; ++i) {
                    const int el = 4 * (lane + 32 * i);
                    if (el / D < G) *reinterpret_cast<float4*>(wo + el) = acc[i];
                }
                if (lane < G) {
                    p.ws_ml[((long long)e.slot * GP + lane) * 2 + 0] = sHM[lane];
                    p.ws_ml[((long long)e.slot * GP + lane) * 2 + 1] = sHL[lane];
                }
                // The warp barrier orders every lane's partial stores before
                // lane 0's release-acquire increment (cumulativity); its
                // acquire side orders the other pieces' stores before this
                // warp's reads below.
                __syncwarp();
                unsigned last = 0;
                if (lane == 0)
                    last = atomic_inc_acq_rel(p.counters + e.u, (unsigned)(n - 1)) ==
                           (unsigned)(n - 1);
                last = __shfl_sync(0xffffffffu, last, 0);
                if (!last) continue;
            }

            // Last piece of this (sequence, kv head) to finish: merge them
            // all. A piece that was not published keeps its partial in shared
            // memory; every piece is read the same way and summed in the same
            // order (pairs, ascending), whichever came last, so the result is
            // the same bits every run. Pieces go through shared memory in
            // chunks of kChunk; with more than one chunk the per-head maxima
            // of all pieces are found first.
            constexpr int kChunk = kCombineCap / GP;  // even: pairs never straddle chunks
            static_assert(kChunk % 2 == 0, "combine chunks hold whole pairs");
            float* sGM = sW;       // per-head max over all pieces
            float* sGL = sW + GP;  // per-head weighted sum of l (its reciprocal at the end)
            int own = -1;
            if (own_in_regs) {
                for (int k = 0; k < n; ++k)
                    if (slot_k(k) == e.slot) own = k;
#pragma unroll
                for (int i = 0; i < kPer4; ++i)
                    *reinterpret_cast<float4*>(sOwn + 4 * (lane + 32 * i)) = acc[i];
            }
            auto m_of = [&](int k, int h) -> float2 {
                if (k == own) return make_float2(sHM[h], sHL[h]);
                return __ldcg(reinterpret_cast<const float2*>(p.ws_ml + (slot_k(k) * GP + h) * 2));
            };
            const bool one_chunk = n <= kChunk;
            if (!one_chunk) {
                for (int h = 0; h < G; ++h) {
                    float mx = -INFINITY;
                    for (int k = lane; k < n; k += 32) mx = fmaxf(mx, m_of(k, h).x);
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                    if (lane == 0) sGM[h] = mx;
                }
            }
            auto load_piece = [&](int k, int i) -> float4 {
                const int el = 4 * (lane + 32 * i);
                if (el / D >= G) return make_float4(0.f, 0.f, 0.f, 0.f);
                if (k == own) return *reinterpret_cast<const float4*>(sOwn + el);
                return __ldcg(reinterpret_cast<const float4*>(p.ws_o + slot_k(k) * GP * D + el));
            };
#pragma unroll
            for (int i = 0; i < kPer4; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int c0 = 0; c0 < n; c0 += kChunk) {
                const int cn = min(kChunk, n - c0);
                __syncwarp();
                for (int idx = lane; idx < cn * G; idx += 32) {
                    const int kk = idx / G, h = idx - (idx / G) * G;
                    const float2 ml = m_of(c0 + kk, h);
                    sCW[kk * GP + h] = ml.x;
                    sCL[kk * GP + h] = ml.y;
                }
                for (int kk = 0; kk < cn; kk += 2) {
                    const bool two = kk + 1 < cn;
                    float4 v0[kPer4], v1[kPer4];
#pragma unroll
                    for (int i = 0; i < kPer4; ++i) {
                        v0[i] = load_piece(c0 + kk, i);
                        v1[i] = two ? load_piece(c0 + kk + 1, i) : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                    if (kk == 0) {  // the chunk's weights, while its first pair loads
                        __syncwarp();
                        if (lane < G) {
                            float M = one_chunk ? -INFINITY : sGM[lane];
                            if (one_chunk)
                                for (int j = 0; j < cn; ++j) M = fmaxf(M, sCW[j * GP + lane]);
                            const float lt = piece_weights(sCW + lane, sCL + lane, cn, GP, M,
                                                           c0 == 0 ? 0.f : sGL[lane]);
                            // after the last chunk: the reciprocal, for the store
                            sGL[lane] = c0 + cn < n ? lt : (lt > 0.f ? 1.f / lt : 0.f);
                        }
                        __syncwarp();
                    }
#pragma unroll
                    for (int i = 0; i < kPer4; ++i) {
                        const int h = min(4 * (lane + 32 * i) / D, GP - 1);
                        const float w0 = sCW[kk * GP + h], w1 = two ? sCW[(kk + 1) * GP + h] : 0.f;
                        add_pair(acc[i], w0, v0[i], w1, v1[i]);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < kPer4; ++i) {
                const int h = 4 * (lane + 32 * i) / D;
                if (h < G) store_out(i, sGL[h]);
            }
            __syncwarp();
        }
        return;
    }

    // ======================================================== consumer warps
    const int g = lane >> 2;  // row group of the mma fragments
    const int q4 = lane & 3;  // thread in group
    const uint32_t mi = lane >> 3;
    const int ld_row = (lane & 7) + ((mi >> 1) << 3);  // ldmatrix row within a 16-row tile
    const int ld_kk = (int)(mi & 1);
    constexpr int TPW = L::kTpw;
    // Tile t of this warp is stage rows [(t * CW + warp) * 16, +16). Stage row
    // r lives in block tile r / bs at row r % bs; chunk c of a tile starts
    // c * bs * 128 bytes in. Row offset of this lane's ldmatrix row per tile:
    uint32_t ld_off_t[TPW];
#pragma unroll
    for (int t = 0; t < TPW; ++t) {
        const int ld_r = (t * CW + warp) * kTileRows + ld_row;
        ld_off_t[t] = (uint32_t)((ld_r >> bs_sh) * (bs * D * 2) + (ld_r & (bs - 1)) * 128);
    }
    const uint32_t chunk_bytes = (uint32_t)(bs * 128);
    const int ld_swz = ld_row & 7;  // bs and tile starts are multiples of 8

    float m_run[2], l_run[2];
    float o[NT][KS][4];
    uint32_t qa[KS][4];
    m_run[0] = m_run[1] = -INFINITY;
    l_run[0] = l_run[1] = 0.f;

    int stage = 0;
    uint32_t phase = 0;
    uint32_t ephase = 0;
    constexpr bool fused_q = FUSED;
    T* key_new = reinterpret_cast<T*>(p.key_new);
    T* kc_new = reinterpret_cast<T*>(p.key_cache);
    T* vc_new = reinterpret_cast<T*>(p.value_cache);
    // Fused decode step. The stage that holds a sequence's last block (the
    // last of the piece that runs to the end of its (sequence, kv head))
    // brought the new token's raw key and value rows and its cos/sin row into
    // the stage's query slot. One warp (the one whose tile holds the token, or
    // warp 0 when the token is in no stage) rotates the key, writes it back
    // into the key tensor and, when the token's block is mapped, into both
    // caches and over the token's row of the stage, where the copy of the
    // block brought the row as it was before this step. Nothing else reads
    // that cache row during the launch, so the global stores need no ordering.
    auto write_new_token = [&](int stg, const StageDesc& dd) {
        constexpr int kU = D / 8;    // 16-byte units of a row
        constexpr int kHU = kU / 2;  // units of its first half
        const uint8_t* slot = smem + L::kOffQ + stg * L::kQBytes + GP * D * 2;
        const uint4* cs = reinterpret_cast<const uint4*>(slot);
        const uint4* kraw = reinterpret_cast<const uint4*>(slot + D * 2);
        const uint4* vraw = reinterpret_cast<const uint4*>(slot + 2 * D * 2);
        const bool store = dd.new_row >= 0;  // implies new_r >= 0
        const long long grow = (long long)dd.new_row * D;
        // the token's row in the stage: block tile new_r / bs, row rr, with
        // the 128-byte swizzle of the copies on its 16-byte units
        const int rr = store ? dd.new_r & (bs - 1) : 0;
        const int roff = store ? (dd.new_r >> bs_sh) * (bs * D * 2) + rr * 128 : 0;
        auto unit_off = [&](int u) -> int {
            return roff + (u >> 3) * (int)chunk_bytes + (((u & 7) ^ (rr & 7)) << 4);
        };
        if (lane < kHU) {
            uint4 x = kraw[lane], y = kraw[lane + kHU];
            if (!(dd.flags & kRopeSkip)) {
                const uint4 c = cs[lane], sn = cs[lane + kHU];
                rope_packed2<T>(x.x, y.x, c.x, sn.x);
                rope_packed2<T>(x.y, y.y, c.y, sn.y);
                rope_packed2<T>(x.z, y.z, c.z, sn.z);
                rope_packed2<T>(x.w, y.w, c.w, sn.w);
            }
            uint4* kn = reinterpret_cast<uint4*>(key_new + (long long)dd.seq * p.key_stride +
                                                 (long long)dd.kvh * D);
            kn[lane] = x;
            kn[lane + kHU] = y;
            if (store) {
                uint4* kc = reinterpret_cast<uint4*>(kc_new + grow);
                kc[lane] = x;
                kc[lane + kHU] = y;
                uint8_t* kst = smem + L::kOffK + stg * L::kStageKV;
                *reinterpret_cast<uint4*>(kst + unit_off(lane)) = x;
                *reinterpret_cast<uint4*>(kst + unit_off(lane + kHU)) = y;
            }
        } else if (lane >= 16 && lane < 16 + kU && store) {
            const int u = lane - 16;
            const uint4 v = vraw[u];
            reinterpret_cast<uint4*>(vc_new + grow)[u] = v;
            *reinterpret_cast<uint4*>(smem + L::kOffV + stg * L::kStageKV + unit_off(u)) = v;
        }
        // The proxy fence that orders these generic writes before the
        // stage's next copy, and the warp barrier before the tile's reads,
        // come after the call (shared with the zeroing of unused V rows).
    };
    // The CTA's last piece is finished by the consumer warps themselves once
    // their (m, l, O) are in the hand-off buffer: no other piece follows it,
    // so they are free, and the epilogue warp may still be busy with the
    // piece before it. The four warps combine their partials, and a split
    // piece that is the last of its (sequence, kv head) to finish merges
    // every piece with the partials of up to four pieces per thread in
    // flight at once (a single warp takes one round trip per pair).
    // Phases are separated by an mbarrier of the consumer threads with
    // bounded waits; a wait that gives up flags the status and abandons the
    // piece.
    uint32_t cphase = 0;
    auto csync = [&]() -> bool {
        mbar_arrive(bar_cons);
        const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar_cons, cphase, wlim));
        cphase ^= 1;
        if (!ok && lane == 0) flag_status(TLB_STATUS_WAIT_TIMEOUT);
        return ok;
    };
    auto finish_last_piece = [&](const StageDesc& e) {
        constexpr int NC = CW * 32;
        constexpr int kGroups = GP * D / 4 / NC;  // float4 groups per thread
        static_assert(GP * D / 4 % NC == 0, "groups split evenly over the consumer threads");
        const bool split = !(e.flags & kPieceComplete);
        const int n = e.nsplits;
        // the arrival counter, read while the warps combine
        unsigned seen = 0;
        if (split && tid == 0) seen = ld_acquire_gpu(p.counters + e.u);
        if (!csync()) return;  // every warp's (m, l, O) is in shared memory
        // combine the warps' partials: per head h, M = max_w m_w, weights
        // 2^(m_w - M), l = sum_w w l_w
        float4 a[kGroups];
        float scale[kGroups];
#pragma unroll
        for (int j = 0; j < kGroups; ++j) {
            const int el = 4 * (tid + NC * j), h = el / D, dd = el % D;
            a[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            scale[j] = 0.f;
            if (h < G) {
                float M = -INFINITY;
#pragma unroll
                for (int w = 0; w < CW; ++w) M = fmaxf(M, sM[w * GP + h]);
                float lt = 0.f;
#pragma unroll
                for (int w = 0; w < CW; ++w) {
                    const float wt = M == -INFINITY ? 0.f : exp2f(sM[w * GP + h] - M);
                    lt += wt * sL[w * GP + h];
                    const float4 v = *reinterpret_cast<const float4*>(sO + (w * GP + h) * D + dd);
                    a[j].x += wt * v.x; a[j].y += wt * v.y; a[j].z += wt * v.z; a[j].w += wt * v.w;
                }
                scale[j] = lt;
            }
        }
        const long long out_base = ((long long)e.seq * p.num_heads + (long long)e.kvh * G) * D;
        if (!split) {
#pragma unroll
            for (int j = 0; j < kGroups; ++j) {
                const int el = 4 * (tid + NC * j);
                if (el / D < G)
                    Vec4Out<T>::store(out + out_base + el, a[j], scale[j] > 0.f ? 1.f / scale[j] : 0.f);
            }
            return;
        }
        float hm = -INFINITY, hl = 0.f;  // (m, l) of head tid of this piece
        if (tid < G) {
#pragma unroll
            for (int w = 0; w < CW; ++w) hm = fmaxf(hm, sM[w * GP + tid]);
#pragma unroll
            for (int w = 0; w < CW; ++w) {
                const float wt = hm == -INFINITY ? 0.f : exp2f(sM[w * GP + tid] - hm);
                hl += wt * sL[w * GP + tid];
            }
        }
        auto slot_k = [&](int k) -> long long {
            return 2ll * (e.jfirst + k) + ((k == 0 && e.first_slot1) ? 1 : 0);
        };
        int* sDecide = sMisc + 16;  // the prologue's words are long since read
        // If every other piece has published (counter at n - 1), this one is
        // the last and merges with its own partial in registers; otherwise
        // it publishes and takes a ticket.
        if (tid == 0) *sDecide = seen == (unsigned)(n - 1) ? 1 : 0;
        if (!csync()) return;  // also: every read of the hand-off buffer is done
        const bool own_regs = *sDecide != 0;
        if (own_regs) {
            if (tid == 0) st_relaxed_gpu(p.counters + e.u, 0u);  // ready for the next launch
        } else {
            float* wo = p.ws_o + (long long)e.slot * GP * D;
#pragma unroll
            for (int j = 0; j < kGroups; ++j) {
                const int el = 4 * (tid + NC * j);
                if (el / D < G) *reinterpret_cast<float4*>(wo + el) = a[j];
            }
            if (tid < G) {
                p.ws_ml[((long long)e.slot * GP + tid) * 2 + 0] = hm;
                p.ws_ml[((long long)e.slot * GP + tid) * 2 + 1] = hl;
            }
            __threadfence();  // every thread's partial stores before the release below
            if (!csync()) return;
            if (tid == 0)
                *sDecide = atomic_inc_acq_rel(p.counters + e.u, (unsigned)(n - 1)) == (unsigned)(n - 1);
            if (!csync()) return;
            if (*sDecide == 0) return;
        }
        // Merge all n pieces. The other pieces' partials are staged into the
        // CTA's K and V stage buffers, free now (the producer has issued its
        // last copy and every stage has been consumed), with 16-byte cp.async
        // copies, kStageP pieces per round trip; each thread copies exactly
        // the float4 groups it sums, so it needs only its own copies to land.
        // Meanwhile the pieces' (m, l) go through the hand-off buffer into
        // per-head weights. Every thread then sums its groups over the pieces
        // in pairs, ascending (this piece's own partial from registers).
        int own = -1;
        if (own_regs)
            for (int k = 0; k < n; ++k)
                if (slot_k(k) == e.slot) own = k;
        float* sMW = sO;                // [n][GP] maxima, then weights
        float* sML = sMW + n * GP;      // [n][GP] sums
        float* sFL = sML + n * GP;      // [GP] 1 / total
        static_assert(2 * kConsumerMergeMax * GP + GP <= L::kOFloats,
                      "the weights of every piece fit the hand-off buffer");
        constexpr int kPieceF = GP * D;  // floats of one partial
        constexpr int kStageP = (2 * NSTAGE * L::kStageKV) / (kPieceF * 4) / 2 * 2;  // even
        static_assert(kStageP >= 2 && L::kOffK == 0 && L::kOffV == NSTAGE * L::kStageKV,
                      "the K and V stage buffers are one run of kStageP partials");
        const uint32_t sPart = sbase + L::kOffK;
        auto stage_chunk = [&](int c0) {
            const int cn = min(kStageP, n - c0);
            for (int kk = 0; kk < cn; ++kk) {
                const int k = c0 + kk;
                if (k == own) continue;
                const float* src = p.ws_o + slot_k(k) * kPieceF;
#pragma unroll
                for (int j = 0; j < kGroups; ++j) {
                    const int el = 4 * (tid + NC * j);
                    if (el / D < G)
                        cp_async_cg16(sPart + (uint32_t)(kk * kPieceF + el) * 4u, src + el);
                }
            }
            cp_async_commit();
        };
        stage_chunk(0);
        for (int idx = tid; idx < n * G; idx += NC) {
            const int k = idx / G, h = idx - (idx / G) * G;
            if (k == own) continue;  // written below by the thread that holds it
            const float2 ml =
                __ldcg(reinterpret_cast<const float2*>(p.ws_ml + (slot_k(k) * GP + h) * 2));
            sMW[k * GP + h] = ml.x;
            sML[k * GP + h] = ml.y;
        }
        if (own >= 0 && tid < G) {
            sMW[own * GP + tid] = hm;
            sML[own * GP + tid] = hl;
        }
        // A failed phase still waits for this thread's copies: the stage
        // buffers must not be written once the CTA has left.
        if (!csync()) { cp_async_wait<0>(); return; }
        if (tid < G) {
            float M = -INFINITY;
            for (int k = 0; k < n; ++k) M = fmaxf(M, sMW[k * GP + tid]);
            const float lt = piece_weights(sMW + tid, sML + tid, n, GP, M, 0.f);
            sFL[tid] = lt > 0.f ? 1.f / lt : 0.f;
        }
        if (!csync()) { cp_async_wait<0>(); return; }
        float4 acc[kGroups];
#pragma unroll
        for (int j = 0; j < kGroups; ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        const float* sPartF = reinterpret_cast<const float*>(smem + L::kOffK);
        for (int c0 = 0; c0 < n; c0 += kStageP) {
            cp_async_wait<0>();  // this thread's copies of the chunk
            const int cn = min(kStageP, n - c0);
#pragma unroll
            for (int j = 0; j < kGroups; ++j) {
                const int el = 4 * (tid + NC * j), h = el / D;
                if (h >= G) continue;
                auto piece = [&](int kk) -> float4 {
                    if (kk >= cn) return make_float4(0.f, 0.f, 0.f, 0.f);
                    if (c0 + kk == own) return a[j];
                    return *reinterpret_cast<const float4*>(sPartF + kk * kPieceF + el);
                };
                for (int kk = 0; kk < cn; kk += 2) {
                    const int k = c0 + kk;
                    add_pair(acc[j], sMW[k * GP + h], piece(kk),
                             k + 1 < n ? sMW[(k + 1) * GP + h] : 0.f, piece(kk + 1));
                }
            }
            // the next chunk overwrites only this thread's own groups
            if (c0 + kStageP < n) stage_chunk(c0 + kStageP);
        }
#pragma unroll
        for (int j = 0; j < kGroups; ++j) {
            const int el = 4 * (tid + NC * j), h = el / D;
            if (h < G) Vec4Out<T>::store(out + out_base + el, acc[j], sFL[h]);
        }
    };

    while (true) {
        bool got = true;
        // warp-uniform outcome: the warp's mma and shuffles below need all lanes
        got = __all_sync(0xffffffffu, mbar_wait_bounded(bar_full + 8 * stage, phase, wlim));
        if (!got) {
            if (lane == 0) flag_status(TLB_STATUS_WAIT_TIMEOUT);
            break;
        }
        const StageDesc d = sDesc[stage];
        if (d.flags & kTerminate) break;

        if (d.flags & kPieceStart) {
            const T* sq = reinterpret_cast<const T*>(smem + L::kOffQ + stage * L::kQBytes);
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                const int c0 = ks * 16 + 2 * q4;
                qa[ks][0] = g < G ? *reinterpret_cast<const uint32_t*>(sq + g * D + c0) : 0u;
                qa[ks][1] = g + 8 < G ? *reinterpret_cast<const uint32_t*>(sq + (g + 8) * D + c0) : 0u;
                qa[ks][2] = g < G ? *reinterpret_cast<const uint32_t*>(sq + g * D + c0 + 8) : 0u;
                qa[ks][3] =
                    g + 8 < G ? *reinterpret_cast<const uint32_t*>(sq + (g + 8) * D + c0 + 8) : 0u;
            }
            if (fused_q && !(d.flags & kRopeSkip)) {
                // Fused decode step: rotate the raw query group in registers
                // with the cos/sin row that came with it. Columns c and
                // c + D/2 of a fragment word sit in k-steps ks and ks + KS/2
                // of the same lane, so each lane rotates its own pairs.
                // Words 1 and 3 hold head g + 8, words 0 and 2 head g: heads
                // at or beyond the group are zero padding and stay zero.
                const T* cs = sq + GP * D;
#pragma unroll
                for (int ks = 0; ks < KS / 2; ++ks)
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        if (NT == 1 && (r & 1)) continue;  // head g + 8 >= 8 >= G
                        if ((r & 1) ? g + 8 >= G : g >= G) continue;
                        const int col = ks * 16 + 2 * q4 + (r >= 2 ? 8 : 0);
                        rope_packed2<T>(qa[ks][r], qa[ks + KS / 2][r],
                                        *reinterpret_cast<const uint32_t*>(cs + col),
                                        *reinterpret_cast<const uint32_t*>(cs + D / 2 + col));
                    }
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int mt = 0; mt < KS; ++mt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) o[nt][mt][e] = 0.f;
            m_run[0] = m_run[1] = -INFINITY;
            l_run[0] = l_run[1] = 0.f;
        }

#pragma unroll
        for (int t = 0; t < TPW; ++t) {
        const int r0 = (t * CW + warp) * kTileRows;
        const uint32_t ld_off = ld_off_t[t];
        // Valid rows of this 16-token tile.
        const unsigned vmask = (sDesc[stage].rows[r0 >> 5] >> (r0 & 31)) & 0xffffu;
        if (FUSED && (d.flags & kNewToken) &&
            (d.new_r >= 0 ? d.new_r / kTileRows == t * CW + warp : (t == 0 && warp == 0))) {
            write_new_token(stage, d);
            if (vmask == 0u || vmask == 0xffffu) {  // no zeroing below to share the fence
                fence_proxy_async_smem();  // before the stage's next copy overwrites the rows
                __syncwarp();
            }
        }

        if (vmask != 0u) {
            const uint32_t kbase = sbase + L::kOffK + stage * L::kStageKV;
            const uint32_t vbase = sbase + L::kOffV + stage * L::kStageKV;
            if (vmask != 0xffffu) {
                // Rows that hold no token of this piece may contain anything
                // (stale stage data, unwritten cache slots): zero V there so
                // that P = 0 really contributes nothing.
                uint8_t* vrow = smem + L::kOffV + stage * L::kStageKV;
                for (int idx = lane; idx < 16 * L::kChunks * 8; idx += 32) {
                    const int r = idx / (L::kChunks * 8);
                    const int c = (idx / 8) % L::kChunks;
                    const int k = idx & 7;
                    const int sr = r0 + r;
                    if (!((vmask >> r) & 1u))
                        *reinterpret_cast<uint4*>(vrow + (sr >> bs_sh) * (bs * D * 2) + c * chunk_bytes +
                                                  (sr & (bs - 1)) * 128 + k * 16) =
                            make_uint4(0u, 0u, 0u, 0u);
                }
                fence_proxy_async_smem();
                __syncwarp();
            }

            // ---- S = Q K^T for 16 tokens (two 8-token n-tiles). All K
            // fragments are loaded first; the k-steps then feed kQkChains
            // independent accumulators per n-tile (mma.sync latency is far
            // above its issue interval), summed at the end.
            constexpr int kQkChains = KS < 4 ? KS : 4;
            uint32_t kf[KS][4];
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                const int c = ks >> 2;
                const int kk = ((ks & 3) << 1) + ld_kk;
                ldsm_x4(kbase + ld_off + c * chunk_bytes + ((kk ^ ld_swz) << 4), kf[ks][0],
                        kf[ks][1], kf[ks][2], kf[ks][3]);
            }
            float s_part[kQkChains][2][4];
#pragma unroll
            for (int ch = 0; ch < kQkChains; ++ch)
#pragma unroll
                for (int n = 0; n < 2; ++n)
#pragma unroll
                    for (int e = 0; e < 4; ++e) s_part[ch][n][e] = 0.f;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                mma16816<T>(s_part[ks % kQkChains][0], qa[ks], kf[ks][0], kf[ks][1]);
                mma16816<T>(s_part[ks % kQkChains][1], qa[ks], kf[ks][2], kf[ks][3]);
            }
            float s_acc[2][4];
#pragma unroll
            for (int n = 0; n < 2; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    float v = s_part[0][n][e];
#pragma unroll
                    for (int ch = 1; ch < kQkChains; ++ch) v += s_part[ch][n][e];
                    s_acc[n][e] = v;
                }

            // ---- online softmax (log2 domain); heads g (and g + 8).
            float x[2][4];
#pragma unroll
            for (int n = 0; n < 2; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int tok = n * 8 + 2 * q4 + (e & 1);
                    x[n][e] = ((vmask >> tok) & 1u) ? s_acc[n][e] * p.scale_log2 : -INFINITY;
                }
            float alpha[2];
            float pr[2][4];
#pragma unroll
            for (int hh = 0; hh < NT; ++hh) {
                float mx = fmaxf(fmaxf(x[0][2 * hh], x[0][2 * hh + 1]),
                                 fmaxf(x[1][2 * hh], x[1][2 * hh + 1]));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                const float m_new = fmaxf(m_run[hh], mx);
                const float mu = m_new == -INFINITY ? 0.f : m_new;
                alpha[hh] = exp2f(m_run[hh] - mu);
                float rs = 0.f;
#pragma unroll
                for (int n = 0; n < 2; ++n)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const float pv = exp2f(x[n][2 * hh + e] - mu);
                        pr[n][2 * hh + e] = pv;
                        rs += pv;
                    }
                l_run[hh] = l_run[hh] * alpha[hh] + rs;
                m_run[hh] = m_new;
            }
            // Rescale O^T columns (heads nt*8 + 2*q4 + {0,1}) by their alphas.
            const bool need = __any_sync(0xffffffffu, alpha[0] != 1.f || (NT == 2 && alpha[1] != 1.f));
            if (need) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    const float a0 = __shfl_sync(0xffffffffu, alpha[nt], (2 * q4) * 4);
                    const float a1 = __shfl_sync(0xffffffffu, alpha[nt], (2 * q4 + 1) * 4);
#pragma unroll
                    for (int mt = 0; mt < KS; ++mt) {
                        o[nt][mt][0] *= a0;
                        o[nt][mt][1] *= a1;
                        o[nt][mt][2] *= a0;
                        o[nt][mt][3] *= a1;
                    }
                }
            }
            // P^T as the B operand: tokens (2q, 2q+1) and (8+2q, 8+2q+1) of head g.
            // bf16 keeps 8 mantissa bits, so P goes in as hi + lo bf16 pairs
            // (two mmas) and the weights match the fp32 row sums to ~2^-16.
            uint32_t pb[NT][2], pl[NT][2];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                split2<T>(pr[0][2 * nt], pr[0][2 * nt + 1], pb[nt][0], pl[nt][0]);
                split2<T>(pr[1][2 * nt], pr[1][2 * nt + 1], pb[nt][1], pl[nt][1]);
            }
            // ---- O^T += V^T P^T, one 16-wide slice of head_dim per m-tile:
            // all V fragments first, then the hi products of every m-tile,
            // then the lo products, so no mma waits on the one before it.
            uint32_t vf[KS][4];
#pragma unroll
            for (int mt = 0; mt < KS; ++mt) {
                const int c = mt >> 2;
                const int kk = ((mt & 3) << 1) + ld_kk;
                ldsm_x4_trans(vbase + ld_off + c * chunk_bytes + ((kk ^ ld_swz) << 4), vf[mt][0],
                              vf[mt][1], vf[mt][2], vf[mt][3]);
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int mt = 0; mt < KS; ++mt) mma16816<T>(o[nt][mt], vf[mt], pb[nt][0], pb[nt][1]);
            if constexpr (kSplitP<T>) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int mt = 0; mt < KS; ++mt)
                        mma16816<T>(o[nt][mt], vf[mt], pl[nt][0], pl[nt][1]);
            }
        }
        }  // tiles of this warp
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_empty + 8 * stage);
        if (++stage == NSTAGE) { stage = 0; phase ^= 1; }

        if (!(d.flags & kPieceEnd)) continue;

        // ======== piece end: hand (m, l, O) of this warp to the epilogue warp
        float lsum[2];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            float v = l_run[hh];
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            lsum[hh] = v;
        }
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(bar_epi_empty, ephase ^ 1, wlim))) {
            if (lane == 0) flag_status(TLB_STATUS_WAIT_TIMEOUT);
            break;
        }
        if (q4 == 0) {
            sM[warp * GP + g] = m_run[0];
            sL[warp * GP + g] = lsum[0];
            if (NT == 2) {
                sM[warp * GP + 8 + g] = m_run[1];
                sL[warp * GP + 8 + g] = lsum[1];
            }
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int mt = 0; mt < KS; ++mt) {
                const int h0 = nt * 8 + 2 * q4;
                const int d0 = mt * 16 + g;
                float* base = sO + (warp * GP + h0) * D + d0;
                base[0] = o[nt][mt][0];
                base[D] = o[nt][mt][1];
                base[8] = o[nt][mt][2];
                base[D + 8] = o[nt][mt][3];
            }
        if ((d.flags & kCtaLast) && d.nsplits <= kConsumerMergeMax &&
            (D == 128 || d.nsplits >= kConsumerMinPieces64)) {
            finish_last_piece(d);
            continue;  // the next stage is the terminate
        }
        if (tid == 0) *sEpi = d;
        mbar_arrive(bar_epi_full);
        ephase ^= 1;
    }
    // Let the epilogue warp finish once it has taken the last piece.
    if (__all_sync(0xffffffffu, mbar_wait_bounded(bar_epi_empty, ephase ^ 1, wlim))) {
        if (tid == 0) sEpi->flags = kTerminate;
        mbar_arrive(bar_epi_full);
    } else if (lane == 0) {
        flag_status(TLB_STATUS_WAIT_TIMEOUT);
    }
}

// ============================================================ host side
namespace {

template <typename T, int D, int NT, int NSTAGE, int CW, bool FUSED, bool INJECT>
cudaError_t launch_tc_t(const TcParams& p, const CUtensorMap& tk, const CUtensorMap& tv,
                        int grid, bool overlap, cudaStream_t st) {
    using L = TcLayout<D, NT, NSTAGE, CW, FUSED>;
    auto kern = paged_attention_tc_kernel<T, D, NT, NSTAGE, CW, FUSED, INJECT>;
    static std::once_flag once[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static cudaError_t attr_err[64];
    std::call_once(once[dev & 63], [&] {
        attr_err[dev & 63] =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    });
    if (attr_err[dev & 63] != cudaSuccess) return attr_err[dev & 63];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3((CW + 2) * 32);
    cfg.dynamicSmemBytes = L::kAlloc;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = overlap ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, tk, tv, p);
}

// Pipeline depth per head size: one CTA per SM keeps this many 64-token
// stages (K, V and the query group) in flight, ~160 KB per SM, enough to
// cover HBM latency under full load (bytes in flight = bandwidth x latency).
#ifndef TLB_ATTN_STAGES_64
#define TLB_ATTN_STAGES_64 (TLB_ATTN_TPW64 == 2 ? 2 : 4)
#endif
#ifndef TLB_ATTN_STAGES_128
#define TLB_ATTN_STAGES_128 2
#endif
constexpr int kStages64 = TLB_ATTN_STAGES_64;
constexpr int kStages128 = TLB_ATTN_STAGES_128;
// Consumer warps of the one-head-tile kernels (the two-tile ones, group > 8,
// need more registers per thread and keep kConsumerWarps).
#ifndef TLB_ATTN_CW1
#define TLB_ATTN_CW1 4
#endif
#ifndef TLB_ATTN_CW1_64
#define TLB_ATTN_CW1_64 4
#endif
constexpr int kCw1 = TLB_ATTN_CW1;        // head_dim 128
constexpr int kCw1_64 = TLB_ATTN_CW1_64;  // head_dim 64

// The fused decode step (cos/sin table given) and plain attention are
// separate instances, so plain attention carries none of the fused code.
template <typename T, bool FUSED, bool INJECT>
cudaError_t dispatch_tc_f(int head_dim, int group, const TcParams& p, const CUtensorMap& tk,
                          const CUtensorMap& tv, int grid, bool ov, cudaStream_t st) {
    const bool two = group > 8;
    if (head_dim == 64)
        return two ? launch_tc_t<T, 64, 2, kStages64, kConsumerWarps, FUSED, INJECT>(p, tk, tv, grid, ov, st)
                   : launch_tc_t<T, 64, 1, kStages64, kCw1_64, FUSED, INJECT>(p, tk, tv, grid, ov, st);
    return two ? launch_tc_t<T, 128, 2, kStages128, kConsumerWarps, FUSED, INJECT>(p, tk, tv, grid, ov, st)
               : launch_tc_t<T, 128, 1, kStages128, kCw1, FUSED, INJECT>(p, tk, tv, grid, ov, st);
}

template <typename T, bool INJECT>
cudaError_t dispatch_tc(int head_dim, int group, const TcParams& p, const CUtensorMap& tk,
                        const CUtensorMap& tv, int grid, bool ov, cudaStream_t st) {
    return p.cos_sin != nullptr ? dispatch_tc_f<T, true, INJECT>(head_dim, group, p, tk, tv, grid, ov, st)
                                : dispatch_tc_f<T, false, INJECT>(head_dim, group, p, tk, tv, grid, ov, st);
}

}  // namespace

// The same dispatch, every instance waiting at most TcParams::wait_limit
// probes (paged_attention_inject.cu): launched instead of the default
// instances only while tlb_attention_set_wait_limit holds another limit.
cudaError_t launch_tc_inject(int dtype, int head_dim, int group, const TcParams& p,
                             const CUtensorMap& tm_k, const CUtensorMap& tm_v, int grid,
                             bool overlap, cudaStream_t stream);

}  // namespace attn
}  // namespace tlb
