// NeoX rotary embedding and the KV-cache writes of the decode step.
//
// Rotation (cscr/pos_encoding_kernel.cu:24-65): for each token and head,
// pairs (i, i + rot/2), i < rot/2, become
//   x' = x * cos[pos, i] - y * sin[pos, i],  y' = y * cos[pos, i] + x * sin[pos, i]
// with cos/sin read from the dtype-rounded cos_sin_cache row, the math in
// fp32 and one rounding to the storage dtype. The query is written to a new
// tensor, the key is rewritten in place.
//
// Cache write (src/model_executor/layers/attention.py:96-116): key/value row
// of token t lands at cache[block, :, offset] with block/offset taken from a
// slot mapping (slot = block * block_size + offset, negative = skip) or, as
// the reference does it, from block_tables[t, pos / block_size] and
// pos % block_size.
//
// All three are one flat grid over 16-byte work items (8 half-precision or
// 4 fp32 elements): items never straddle a head, every load and store is a
// 128-bit access when the pointers and strides allow it (VEC > 1), and the
// fused variant writes the rotated key to the cache from registers.
#include "common.cuh"
#include "kernels.h"

namespace tlb {

namespace {

template <typename T, int VEC>
struct VecIO {
    static __device__ __forceinline__ void load(const T* p, float (&f)[VEC]) {
        if constexpr (VEC * sizeof(T) == 16) {
            const uint4 u = *reinterpret_cast<const uint4*>(p);
            const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
            for (int i = 0; i < VEC; ++i) f[i] = Elem<T>::to_f(e[i]);
        } else {
#pragma unroll
            for (int i = 0; i < VEC; ++i) f[i] = Elem<T>::to_f(p[i]);
        }
    }
    static __device__ __forceinline__ void store(T* p, const float (&f)[VEC]) {
        if constexpr (VEC * sizeof(T) == 16) {
            uint4 u;
            T* e = reinterpret_cast<T*>(&u);
#pragma unroll
            for (int i = 0; i < VEC; ++i) e[i] = Elem<T>::from_f(f[i]);
            *reinterpret_cast<uint4*>(p) = u;
        } else {
#pragma unroll
            for (int i = 0; i < VEC; ++i) p[i] = Elem<T>::from_f(f[i]);
        }
    }
    // Raw copy of VEC elements (bit-exact). The source is a query, key or
    // value row, so the copy first waits for the preceding kernel when the
    // launch was programmatic (a no-op otherwise).
    static __device__ __forceinline__ void copy(T* dst, const T* src) {
        grid_dependency_wait();
        if constexpr (VEC * sizeof(T) == 16) {
            *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
        } else {
#pragma unroll
            for (int i = 0; i < VEC; ++i) dst[i] = src[i];
        }
    }
};

template <typename I>
__device__ __forceinline__ long long load_index(const void* p, long long i) {
    return (long long)reinterpret_cast<const I*>(p)[i];
}

// Destination row of token t in the cache for kv head h, or -1 to skip.
// Mode 0: `slots`; mode 1: positions + block_tables (one row per token).
template <typename SI, bool BY_TABLE>
__device__ __forceinline__ long long cache_row_base(const RopeCacheParams& p, long long t,
                                                    long long pos) {
    long long blk, off;
    if constexpr (BY_TABLE) {
        if (pos < 0 || pos / p.block_size >= p.max_blocks) {
            flag_status(TLB_STATUS_BAD_SLOT);
            return -1;
        }
        blk = p.block_tables[t * p.max_blocks + pos / p.block_size];
        if (blk < 0) return -1;
        off = pos % p.block_size;
    } else {
        const long long slot = load_index<SI>(p.slots, t);
        if (slot < 0) return -1;
        blk = slot / p.block_size;
        off = slot % p.block_size;
    }
    if (blk >= p.num_blocks) {
        flag_status(TLB_STATUS_BAD_SLOT);
        return -1;
    }
    // element offset of (blk, head 0, off, 0)
    return ((blk * p.num_kv_heads) * p.block_size + off) * p.head_size;
}

// Rotation of VEC pairs starting at pair index i0 of one head.
template <typename T, int VEC>
__device__ __forceinline__ void rotate(const T* src, T* dst, const T* cs, int half, int i0,
                                       T* also = nullptr) {
    float x[VEC], y[VEC], c[VEC], s[VEC];
    VecIO<T, VEC>::load(cs + i0, c);
    VecIO<T, VEC>::load(cs + half + i0, s);
    grid_dependency_wait();
    VecIO<T, VEC>::load(src + i0, x);
    VecIO<T, VEC>::load(src + i0 + half, y);
    float xo[VEC], yo[VEC];
#pragma unroll
    for (int k = 0; k < VEC; ++k) rope_pair(x[k], y[k], c[k], s[k], xo[k], yo[k]);
    VecIO<T, VEC>::store(dst + i0, xo);
    VecIO<T, VEC>::store(dst + i0 + half, yo);
    if (also != nullptr) {
        VecIO<T, VEC>::store(also + i0, xo);
        VecIO<T, VEC>::store(also + i0 + half, yo);
    }
}

// Items per token (each VEC elements wide):
//   [0, nq_rot)            query rotation: head = i / hv, pair vector = i % hv
//   [.., + nq_pass)        query elements >= rot copied to out
//   [.., + nk_rot)         key rotation (in place; to the cache when WITH_CACHE)
//   [.., + nk_pass)        WITH_CACHE: key elements >= rot copied to the cache
//   [.., + nv)             WITH_CACHE: value row copied to the cache
// IX is the index type of the item arithmetic: 32-bit unsigned when the
// launch has fewer than 2^31 items (the usual case; its divisions are a few
// instructions), 64-bit otherwise.
template <typename T, typename PI, typename SI, int VEC, bool WITH_QUERY, bool WITH_CACHE,
          bool BY_TABLE, typename IX>
__global__ void __launch_bounds__(256) rope_cache_kernel(const RopeCacheParams p) {
    // A kernel launched after this one with programmatic serialization (the
    // attention kernel) may start its metadata prologue now; it still waits
    // for this grid to finish before reading anything written here.
    grid_launch_dependents();
    // When this kernel itself is launched programmatically (p.overlap), it
    // overlaps the tail of the kernel before it on the stream. Until
    // grid_dependency_wait() it reads only positions, slot_mapping,
    // block_tables and the cos/sin table - never query, key or value, which
    // the kernel before it (the QKV projection in a model) produces - and it
    // writes nothing. Without a programmatic launch the wait returns at once.
    const int half = p.rot_dim / 2;
    const IX hv = (IX)(half / VEC);                       // pair vectors per head
    const IX pv = (IX)((p.head_size - p.rot_dim) / VEC);  // pass-through vectors per head
    const IX dv = (IX)(p.head_size / VEC);
    const IX nq_rot = WITH_QUERY ? (IX)p.num_heads * hv : 0;
    const IX nq_pass = WITH_QUERY ? (IX)p.num_heads * pv : 0;
    const IX nk_rot = WITH_QUERY ? (IX)p.num_kv_heads * hv : 0;
    const IX nk_pass = WITH_CACHE && WITH_QUERY ? (IX)p.num_kv_heads * pv : 0;
    const IX nk_copy = WITH_CACHE && !WITH_QUERY ? (IX)p.num_kv_heads * dv : 0;
    const IX nv = WITH_CACHE ? (IX)p.num_kv_heads * dv : 0;
    const IX per_tok = nq_rot + nq_pass + nk_rot + nk_pass + nk_copy + nv;
    const IX total = per_tok * (IX)p.num_tokens;

    const T* query = reinterpret_cast<const T*>(p.query);
    T* key = reinterpret_cast<T*>(p.key);
    const T* value = reinterpret_cast<const T*>(p.value);
    T* out = reinterpret_cast<T*>(p.out);
    T* kc = reinterpret_cast<T*>(p.key_cache);
    T* vc = reinterpret_cast<T*>(p.value_cache);
    const T* cs_all = reinterpret_cast<const T*>(p.cos_sin);

    for (IX idx = (IX)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (IX)gridDim.x * blockDim.x) {
        const long long t = (long long)(idx / per_tok);
        IX r = idx - (IX)t * per_tok;

        long long pos = 0;
        const T* cs = nullptr;
        if (WITH_QUERY || BY_TABLE) {
            pos = load_index<PI>(p.positions, t);
        }
        if (WITH_QUERY) {
            if (pos >= 0 && pos < p.cache_rows) {
                cs = cs_all + pos * p.rot_dim;
            } else {
                flag_status(TLB_STATUS_BAD_POSITION);
            }
        }

        if (r < nq_rot) {
            const int h = (int)(r / hv), i0 = (int)(r % hv) * VEC;
            const T* src = query + t * p.query_stride + (long long)h * p.head_size;
            T* dst = out + t * p.out_stride + (long long)h * p.head_size;
            if (cs) {
                rotate<T, VEC>(src, dst, cs, half, i0);
            } else {  // out-of-table position: pass the pair through unchanged
                VecIO<T, VEC>::copy(dst + i0, src + i0);
                VecIO<T, VEC>::copy(dst + i0 + half, src + i0 + half);
            }
            continue;
        }
        r -= nq_rot;
        if (r < nq_pass) {
            const int h = (int)(r / pv), i0 = p.rot_dim + (int)(r % pv) * VEC;
            VecIO<T, VEC>::copy(out + t * p.out_stride + (long long)h * p.head_size + i0,
                                query + t * p.query_stride + (long long)h * p.head_size + i0);
            continue;
        }
        r -= nq_pass;
        if (r < nk_rot) {
            const int h = (int)(r / hv), i0 = (int)(r % hv) * VEC;
            T* kh = key + t * p.key_stride + (long long)h * p.head_size;
            T* also = nullptr;
            if (WITH_CACHE) {
                const long long base = cache_row_base<SI, BY_TABLE>(p, t, pos);
                if (base >= 0) also = kc + base + (long long)h * p.block_size * p.head_size;
            }
            if (cs) {
                rotate<T, VEC>(kh, kh, cs, half, i0, also);
            } else if (also) {
                VecIO<T, VEC>::copy(also + i0, kh + i0);
                VecIO<T, VEC>::copy(also + i0 + half, kh + i0 + half);
            }
            continue;
        }
        r -= nk_rot;
        if (WITH_CACHE) {
            if (r < nk_pass + nk_copy) {
                // Key elements that need no rotation (the tail beyond rot_dim
                // with the fused path, the whole row for a plain cache write).
                const int per_head = nk_pass ? pv : dv;
                const int h = (int)(r / per_head);
                const int i0 = (nk_pass ? p.rot_dim : 0) + (int)(r % per_head) * VEC;
                const long long base = cache_row_base<SI, BY_TABLE>(p, t, pos);
                if (base >= 0)
                    VecIO<T, VEC>::copy(kc + base + (long long)h * p.block_size * p.head_size + i0,
                                        key + t * p.key_stride + (long long)h * p.head_size + i0);
                continue;
            }
            r -= nk_pass + nk_copy;
            {
                const int h = (int)(r / dv), i0 = (int)(r % dv) * VEC;
                const long long base = cache_row_base<SI, BY_TABLE>(p, t, pos);
                if (base >= 0)
                    VecIO<T, VEC>::copy(vc + base + (long long)h * p.block_size * p.head_size + i0,
                                        value + t * p.value_stride + (long long)h * p.head_size + i0);
            }
        }
    }
}

__global__ void decode_metadata_kernel(const int32_t* __restrict__ context_lens,
                                       const int32_t* __restrict__ block_tables,
                                       long long num_seqs, int max_blocks, int block_size,
                                       int64_t* __restrict__ positions,
                                       int64_t* __restrict__ slots) {
    for (long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x; r < num_seqs;
         r += (long long)gridDim.x * blockDim.x) {
        const long long pos = (long long)context_lens[r] - 1;
        long long slot = -1;
        if (pos >= 0 && pos / block_size < max_blocks) {
            const long long blk = block_tables[r * max_blocks + pos / block_size];
            if (blk >= 0) slot = blk * block_size + pos % block_size;
        } else if (pos >= 0) {
            flag_status(TLB_STATUS_BAD_SLOT);
        }
        positions[r] = pos;
        slots[r] = slot;
    }
}

int grid_for(long long items) {
    static int sms = 0;
    if (sms == 0) {
        int dev = 0, n = 148;
        if (cudaGetDevice(&dev) == cudaSuccess &&
            cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
            sms = n;
        else
            sms = 148;
    }
    const long long blocks = (items + 255) / 256;
    const long long cap = (long long)sms * 8;
    return (int)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

long long items_per_token(const RopeCacheParams& p, int vec, bool q, bool cache) {
    const long long hv = p.rot_dim / 2 / vec, pv = (p.head_size - p.rot_dim) / vec,
                    dv = p.head_size / vec;
    long long n = 0;
    if (q) n += (long long)p.num_heads * (hv + pv) + (long long)p.num_kv_heads * hv;
    if (cache) n += (long long)p.num_kv_heads * ((q ? pv : dv) + dv);
    return n;
}

template <typename T, typename PI, typename SI, int VEC, bool Q, bool C, bool BT>
cudaError_t go(const RopeCacheParams& p, cudaStream_t st) {
    const long long items = items_per_token(p, VEC, Q, C) * p.num_tokens;
    if (items == 0) return cudaSuccess;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid_for(items));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = p.overlap ? 1 : 0;
    if (items < (1ll << 31))
        return cudaLaunchKernelEx(&cfg, rope_cache_kernel<T, PI, SI, VEC, Q, C, BT, unsigned>, p);
    return cudaLaunchKernelEx(&cfg, rope_cache_kernel<T, PI, SI, VEC, Q, C, BT,
                                                      unsigned long long>, p);
}

template <typename T, int VEC, bool Q, bool C, bool BT>
cudaError_t by_index(int pos_dtype, int slot_dtype, const RopeCacheParams& p, cudaStream_t st) {
    const bool p64 = pos_dtype == TLB_INT64, s64 = slot_dtype == TLB_INT64;
    if (p64)
        return s64 ? go<T, int64_t, int64_t, VEC, Q, C, BT>(p, st)
                   : go<T, int64_t, int32_t, VEC, Q, C, BT>(p, st);
    return s64 ? go<T, int32_t, int64_t, VEC, Q, C, BT>(p, st)
               : go<T, int32_t, int32_t, VEC, Q, C, BT>(p, st);
}

template <bool Q, bool C, bool BT>
cudaError_t by_type(int dtype, int pos_dtype, int slot_dtype, int vec, const RopeCacheParams& p,
                    cudaStream_t st) {
    switch (dtype) {
        case TLB_FLOAT32:
            return vec > 1 ? by_index<float, 4, Q, C, BT>(pos_dtype, slot_dtype, p, st)
                           : by_index<float, 1, Q, C, BT>(pos_dtype, slot_dtype, p, st);
        case TLB_FLOAT16:
            return vec > 1 ? by_index<__half, 8, Q, C, BT>(pos_dtype, slot_dtype, p, st)
                           : by_index<__half, 1, Q, C, BT>(pos_dtype, slot_dtype, p, st);
        default:
            return vec > 1 ? by_index<__nv_bfloat16, 8, Q, C, BT>(pos_dtype, slot_dtype, p, st)
                           : by_index<__nv_bfloat16, 1, Q, C, BT>(pos_dtype, slot_dtype, p, st);
    }
}

}  // namespace

cudaError_t launch_rope(int dtype, int pos_dtype, int vec, const RopeCacheParams& p,
                        cudaStream_t stream) {
    return by_type<true, false, false>(dtype, pos_dtype, TLB_INT64, vec, p, stream);
}

cudaError_t launch_rope_cache(int dtype, int pos_dtype, int slot_dtype, bool by_block_table,
                              int vec, const RopeCacheParams& p, cudaStream_t stream) {
    if (by_block_table) return by_type<true, true, true>(dtype, pos_dtype, slot_dtype, vec, p, stream);
    return by_type<true, true, false>(dtype, pos_dtype, slot_dtype, vec, p, stream);
}

cudaError_t launch_cache_write(int dtype, int index_dtype, bool by_block_table, int vec,
                               const RopeCacheParams& p, cudaStream_t stream) {
    if (by_block_table)
        return by_type<false, true, true>(dtype, index_dtype, TLB_INT64, vec, p, stream);
    return by_type<false, true, false>(dtype, TLB_INT64, index_dtype, vec, p, stream);
}

cudaError_t launch_decode_metadata(const int32_t* context_lens, const int32_t* block_tables,
                                   long long num_seqs, int max_blocks, int block_size,
                                   int64_t* positions, int64_t* slots, cudaStream_t stream) {
    if (num_seqs <= 0) return cudaSuccess;
    const int blocks = (int)((num_seqs + 255) / 256);
    decode_metadata_kernel<<<blocks < 1024 ? blocks : 1024, 256, 0, stream>>>(
        context_lens, block_tables, num_seqs, max_blocks, block_size, positions, slots);
    return cudaGetLastError();
}

}  // namespace tlb
