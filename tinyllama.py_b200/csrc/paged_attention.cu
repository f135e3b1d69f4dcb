// Paged-attention decode for sm_100a: host side, the generic kernel and the
// default instances of the tensor-core kernel (paged_attention_tc.cuh).
#include "paged_attention_tc.cuh"

#include <mutex>

namespace tlb {
namespace attn {

// ============================================================= generic path
template <typename T, int NPL, int HG>
__global__ void __launch_bounds__(256) paged_attention_generic_kernel(const GenericParams p) {
    constexpr int kWarps = 8;
    extern __shared__ float gsm[];
    const int D = p.head_dim;
    float* q_s = gsm;                         // [HG][32 * NPL]
    float* o_s = q_s + HG * 32 * NPL;         // [kWarps][HG][32 * NPL]
    float* m_s = o_s + kWarps * HG * 32 * NPL;  // [kWarps][HG]
    float* l_s = m_s + kWarps * HG;           // [kWarps][HG]

    const int s = blockIdx.x;
    const int kvh = blockIdx.y;
    const int h0 = blockIdx.z * HG;
    const int G = p.group;
    const int nh = min(HG, G - h0);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const T* query = reinterpret_cast<const T*>(p.query);
    const T* kc = reinterpret_cast<const T*>(p.key_cache);
    const T* vc = reinterpret_cast<const T*>(p.value_cache);
    T* out = reinterpret_cast<T*>(p.out);

    for (int e = tid; e < HG * 32 * NPL; e += blockDim.x) {
        const int hh = e / (32 * NPL), dd = e % (32 * NPL);
        float v = 0.f;
        if (hh < nh && dd < D)
            v = Elem<T>::to_f(query[((long long)s * p.num_heads + (long long)kvh * G + h0 + hh) * D + dd]);
        q_s[e] = v;
    }
    __syncthreads();

    const int cap = p.max_blocks * p.block_size;
    int len = p.seq_lens[s];
    if (len > cap) {
        if (tid == 0) flag_status(TLB_STATUS_SEQ_TOO_LONG);
        len = cap;
    }

    float m[HG], l[HG], acc[HG][NPL];
#pragma unroll
    for (int hh = 0; hh < HG; ++hh) {
        m[hh] = -INFINITY;
        l[hh] = 0.f;
#pragma unroll
        for (int i = 0; i < NPL; ++i) acc[hh][i] = 0.f;
    }

    for (int t = warp; t < len; t += kWarps) {
        const int bid = p.block_tables[(long long)s * p.max_blocks + t / p.block_size];
        if (bid < 0) continue;
        if ((long long)bid >= p.num_blocks) {
            if (lane == 0) flag_status(TLB_STATUS_BAD_BLOCK_ID);
            continue;
        }
        const long long row =
            (((long long)bid * p.num_kv_heads + kvh) * p.block_size + t % p.block_size) * D;
        float kv[NPL];
#pragma unroll
        for (int i = 0; i < NPL; ++i) {
            const int dd = lane + 32 * i;
            kv[i] = dd < D ? Elem<T>::to_f(kc[row + dd]) : 0.f;
        }
        float pw[HG], al[HG];
#pragma unroll
        for (int hh = 0; hh < HG; ++hh) {
            float part = 0.f;
#pragma unroll
            for (int i = 0; i < NPL; ++i) part += q_s[hh * 32 * NPL + lane + 32 * i] * kv[i];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
            const float sc = part * p.scale_log2;
            const float mn = fmaxf(m[hh], sc);
            al[hh] = exp2f(m[hh] - mn);
            pw[hh] = exp2f(sc - mn);
            l[hh] = l[hh] * al[hh] + pw[hh];
            m[hh] = mn;
        }
#pragma unroll
        for (int i = 0; i < NPL; ++i) {
            const int dd = lane + 32 * i;
            const float vv = dd < D ? Elem<T>::to_f(vc[row + dd]) : 0.f;
#pragma unroll
            for (int hh = 0; hh < HG; ++hh) acc[hh][i] = acc[hh][i] * al[hh] + pw[hh] * vv;
        }
    }

    if (lane == 0) {
#pragma unroll
        for (int hh = 0; hh < HG; ++hh) {
            m_s[warp * HG + hh] = m[hh];
            l_s[warp * HG + hh] = l[hh];
        }
    }
#pragma unroll
    for (int hh = 0; hh < HG; ++hh)
#pragma unroll
        for (int i = 0; i < NPL; ++i) o_s[(warp * HG + hh) * 32 * NPL + lane + 32 * i] = acc[hh][i];
    __syncthreads();

    for (int e = tid; e < nh * D; e += blockDim.x) {
        const int hh = e / D, dd = e % D;
        float M = -INFINITY;
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, m_s[w * HG + hh]);
        float a = 0.f, lt = 0.f;
        if (M != -INFINITY) {
            for (int w = 0; w < kWarps; ++w) {
                const float wt = exp2f(m_s[w * HG + hh] - M);
                a += wt * o_s[(w * HG + hh) * 32 * NPL + dd];
                lt += wt * l_s[w * HG + hh];
            }
        }
        out[((long long)s * p.num_heads + (long long)kvh * G + h0 + hh) * D + dd] =
            Elem<T>::from_f(lt > 0.f ? a / lt : 0.f);
    }
}

// ============================================================ host side
namespace {

// Occupancy of the fused instance, whose shared memory is the larger: the
// grid it sizes fits both instances.
template <typename T, int D, int NT, int NSTAGE, int CW>
int occupancy_t() {
    using L = TcLayout<D, NT, NSTAGE, CW, true>;
    auto kern = paged_attention_tc_kernel<T, D, NT, NSTAGE, CW, true, false>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc) !=
        cudaSuccess)
        return 0;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, (CW + 2) * 32,
                                                      L::kAlloc) != cudaSuccess)
        return 0;
    return n;
}

template <typename T>
int occupancy_dispatch(int head_dim, int group) {
    const bool two = group > 8;
    if (head_dim == 64)
        return two ? occupancy_t<T, 64, 2, kStages64, kConsumerWarps>()
                   : occupancy_t<T, 64, 1, kStages64, kCw1_64>();
    return two ? occupancy_t<T, 128, 2, kStages128, kConsumerWarps>()
               : occupancy_t<T, 128, 1, kStages128, kCw1>();
}

template <typename T, int NPL>
cudaError_t launch_generic_npl(const GenericParams& p, cudaStream_t st) {
    constexpr int HG = NPL >= 32 ? 1 : 32 / NPL;
    const size_t smem = (size_t)(HG * 32 * NPL + 8 * HG * 32 * NPL + 16 * HG) * sizeof(float);
    auto kern = paged_attention_generic_kernel<T, NPL, HG>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid(p.num_seqs, p.num_kv_heads, (p.group + HG - 1) / HG);
    kern<<<grid, 256, smem, st>>>(p);
    return cudaGetLastError();
}

template <typename T>
cudaError_t launch_generic_t(const GenericParams& p, cudaStream_t st) {
    const int D = p.head_dim;
    if (D <= 32) return launch_generic_npl<T, 1>(p, st);
    if (D <= 64) return launch_generic_npl<T, 2>(p, st);
    if (D <= 128) return launch_generic_npl<T, 4>(p, st);
    if (D <= 256) return launch_generic_npl<T, 8>(p, st);
    if (D <= 512) return launch_generic_npl<T, 16>(p, st);
    return launch_generic_npl<T, 32>(p, st);
}

}  // namespace

bool tc_supported(int dtype, int head_dim, int group, int block_size) {
    if (dtype != TLB_FLOAT16 && dtype != TLB_BFLOAT16) return false;
    if (head_dim != 64 && head_dim != 128) return false;
    if (group < 1 || group > kGMax) return false;
    if (block_size != 8 && block_size != 16 && block_size != 32 && block_size != 64) return false;
    return true;
}

int tc_gpad(int group) { return group > 8 ? 16 : 8; }

int tc_grid(int device, int dtype, int head_dim, int group, cudaError_t* err) {
    static std::mutex mu;
    static int cache[64][2][2][2];  // device x dtype x head_dim x two-tiles
    const int di = dtype == TLB_BFLOAT16 ? 1 : 0, hi = head_dim == 128 ? 1 : 0,
              ti = group > 8 ? 1 : 0;
    std::lock_guard<std::mutex> lk(mu);
    int& c = cache[device & 63][di][hi][ti];
    *err = cudaSuccess;
    if (c == 0) {
        int sms = 0;
        cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
        if (e != cudaSuccess) { *err = e; return 0; }
        int occ = dtype == TLB_BFLOAT16 ? occupancy_dispatch<__nv_bfloat16>(head_dim, group)
                                        : occupancy_dispatch<__half>(head_dim, group);
        if (occ <= 0) { *err = cudaErrorInvalidConfiguration; return 0; }
        if (occ > kMaxCtasPerSm) occ = kMaxCtasPerSm;
        c = sms * occ;
    }
    return c;
}

cudaError_t launch_tc(int dtype, int head_dim, int group, const TcParams& p,
                      const CUtensorMap& tm_k, const CUtensorMap& tm_v, int grid, bool overlap,
                      cudaStream_t stream) {
    if (p.wait_limit != kWaitLimit)
        return launch_tc_inject(dtype, head_dim, group, p, tm_k, tm_v, grid, overlap, stream);
    if (dtype == TLB_BFLOAT16)
        return dispatch_tc<__nv_bfloat16, false>(head_dim, group, p, tm_k, tm_v, grid, overlap,
                                                  stream);
    return dispatch_tc<__half, false>(head_dim, group, p, tm_k, tm_v, grid, overlap, stream);
}

cudaError_t launch_generic(int dtype, const GenericParams& p, cudaStream_t stream) {
    switch (dtype) {
        case TLB_FLOAT32: return launch_generic_t<float>(p, stream);
        case TLB_FLOAT16: return launch_generic_t<__half>(p, stream);
        default: return launch_generic_t<__nv_bfloat16>(p, stream);
    }
}

}  // namespace attn
}  // namespace tlb
