// Split-KV combine and output projection.
//
// For every (token b, head h) the partial records of its group row are merged with
// the log-sum-exp identity (records hold m in log2 units):
//     M = max_k m_k,  L = sum_k l_k 2^(m_k - M),  o_lat = sum_k 2^(m_k - M) o_k / L
// and projected through W_UV: out[b, h, j] = sum_i o_lat[i] * W_UV[h*dv + j, i]
// (the projection of src/fused_mla.cu:258-267 / src/fused_mla_batched.cu:97-105).
// Block = (head h, chunk of kTok tokens), so each W_UV[h] slice is read from
// HBM once per chunk and reused for every token of the chunk.
#include <cfloat>

#include "mla_internal.cuh"

namespace mla {

namespace {
constexpr int kTok = 8;
constexpr int kThreads = 256;
constexpr int kChunk = 64;  // latent columns of W_UV staged per step
constexpr float kLn2 = 0.6931471805599453f;
}  // namespace

// out[b, h, :] for the kTok tokens whose normalised o_lat rows are in o_s (kTok x dc).
template <typename T>
__device__ void project_wuv(int h, int b0, int B, int H, int dc, int dv, const float* o_s,
                            float* w_s, const T* __restrict__ W_UV, float* __restrict__ out) {
    // thread -> (token t, column j): t = idx % kTok, j = idx / kTok (several j per thread)
    const int nout = kTok * dv;
    float acc[(kTok * 256 + kThreads - 1) / kThreads];  // dv <= 256
    const int per = (nout + kThreads - 1) / kThreads;
    for (int k = 0; k < per; ++k) acc[k] = 0.f;
    const T* W = W_UV + static_cast<long long>(h) * dv * dc;
    for (int c0 = 0; c0 < dc; c0 += kChunk) {
        const int cw = (dc - c0) < kChunk ? (dc - c0) : kChunk;
        __syncthreads();
        for (int i = threadIdx.x; i < dv * kChunk; i += kThreads) {
            int j = i / kChunk, c = i % kChunk;
            w_s[j * (kChunk + 1) + c] = c < cw ? ElemTraits<T>::to_f(W[static_cast<long long>(j) * dc + c0 + c]) : 0.f;
        }
        __syncthreads();
        for (int k = 0; k < per; ++k) {
            int idx = threadIdx.x + k * kThreads;
            if (idx >= nout) break;
            int t = idx % kTok, j = idx / kTok;
            const float* o = o_s + t * dc + c0;
            const float* wr = w_s + j * (kChunk + 1);
            float a = acc[k];
            for (int c = 0; c < cw; ++c) a = fmaf(o[c], wr[c], a);
            acc[k] = a;
        }
    }
    for (int k = 0; k < per; ++k) {
        int idx = threadIdx.x + k * kThreads;
        if (idx >= nout) break;
        int t = idx % kTok, j = idx / kTok;
        int b = b0 + t;
        if (b < B) out[(static_cast<long long>(b) * H + h) * dv + j] = acc[k];
    }
}

// Merge the records of (b, h). Writes normalised o_lat to o_dst (dc floats) and,
// when part_ml/part_o are given, the unnormalised partial (natural-log m).
__device__ void merge_records(const DecodePlan& P, int b, int h, const float* __restrict__ rec_ml,
                              const float* __restrict__ rec_o, float* o_dst, float* part_ml,
                              float* part_o) {
    const int lane = threadIdx.x & 31;
    int g, r;
    if (P.shared) {
        int f = b * P.H + h;
        g = f / kGroupRows;
        r = f % kGroupRows;
    } else {
        g = b * P.head_blocks + h / kGroupRows;
        r = h % kGroupRows;
    }
    const int T = total_tiles(P);
    const int gt0 = tile_prefix(P, g), gt1 = tile_prefix(P, g + 1);
    float M = -INFINITY;
    int w0 = 0, w1 = -1;
    if (gt1 > gt0 && T > 0) {
        w0 = worker_of_tile(T, P.W, gt0);
        w1 = worker_of_tile(T, P.W, gt1 - 1);
    }
    for (int w = w0; w <= w1; ++w) {
        if (worker_begin(T, P.W, w) == worker_begin(T, P.W, w + 1)) continue;
        M = fmaxf(M, rec_ml[(static_cast<long long>(g + w) * kGroupRows + r) * 2]);
    }
    float L = 0.f;
    for (int w = w0; w <= w1; ++w) {
        if (worker_begin(T, P.W, w) == worker_begin(T, P.W, w + 1)) continue;
        const float* ml = rec_ml + (static_cast<long long>(g + w) * kGroupRows + r) * 2;
        L += ml[1] * exp2f(ml[0] - M);
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    for (int c = lane; c < P.dc; c += 32) {
        float a = 0.f;
        for (int w = w0; w <= w1; ++w) {
            if (worker_begin(T, P.W, w) == worker_begin(T, P.W, w + 1)) continue;
            long long rr = static_cast<long long>(g + w) * kGroupRows + r;
            a += exp2f(rec_ml[rr * 2] - M) * rec_o[rr * P.dc + c];
        }
        if (o_dst) o_dst[c] = a * inv;
        if (part_o) part_o[(static_cast<long long>(b) * P.H + h) * P.dc + c] = a;
    }
    if (part_ml && lane == 0) {
        float* pm = part_ml + (static_cast<long long>(b) * P.H + h) * 2;
        pm[0] = L > 0.f ? M * kLn2 : -INFINITY;
        pm[1] = L;
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
combine_kernel(DecodePlan P, const float* __restrict__ rec_ml, const float* __restrict__ rec_o,
               const T* __restrict__ W_UV, float* __restrict__ out, float* part_ml, float* part_o) {
    extern __shared__ float smem[];
    float* o_s = smem;                       // kTok * dc
    float* w_s = o_s + kTok * P.dc;          // dv * (kChunk + 1)
    const int h = blockIdx.x, b0 = blockIdx.y * kTok;
    const int warp = threadIdx.x >> 5;
    if (P.status && *reinterpret_cast<volatile int*>(P.status) != kStatusOk) {
        // the decode kernel gave up on a wait: make the failure visible in the output
        for (int i = threadIdx.x; i < kTok * P.dv; i += kThreads) {
            int b = b0 + i / P.dv;
            if (b < P.B && out) out[(static_cast<long long>(b) * P.H + h) * P.dv + i % P.dv] = __int_as_float(0x7fc00000);
        }
        if (part_ml && threadIdx.x < kTok && b0 + static_cast<int>(threadIdx.x) < P.B)
            part_ml[(static_cast<long long>(b0 + threadIdx.x) * P.H + h) * 2 + 1] = __int_as_float(0x7fc00000);
        return;
    }
    for (int t = warp; t < kTok; t += kThreads / 32) {
        int b = b0 + t;
        if (b < P.B) merge_records(P, b, h, rec_ml, rec_o, o_s + t * P.dc, part_ml, part_o);
        else for (int c = threadIdx.x & 31; c < P.dc; c += 32) o_s[t * P.dc + c] = 0.f;
    }
    if (out == nullptr) return;  // partial-only mode
    project_wuv<T>(h, b0, P.B, P.H, P.dc, P.dv, o_s, w_s, W_UV, out);
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
combine_parts_kernel(int B, int H, int dc, int dv, int parts, const float* __restrict__ part_ml,
                     const float* __restrict__ part_o, const T* __restrict__ W_UV,
                     float* __restrict__ out) {
    extern __shared__ float smem[];
    float* o_s = smem;
    float* w_s = o_s + kTok * dc;
    const int h = blockIdx.x, b0 = blockIdx.y * kTok;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long stride = static_cast<long long>(B) * H;
    for (int t = warp; t < kTok; t += kThreads / 32) {
        int b = b0 + t;
        float* dst = o_s + t * dc;
        if (b >= B) {
            for (int c = lane; c < dc; c += 32) dst[c] = 0.f;
            continue;
        }
        long long bh = static_cast<long long>(b) * H + h;
        float M = -INFINITY;
        for (int p = 0; p < parts; ++p) M = fmaxf(M, part_ml[(p * stride + bh) * 2]);
        float L = 0.f;
        for (int p = 0; p < parts; ++p) {
            const float* ml = part_ml + (p * stride + bh) * 2;
            if (ml[1] > 0.f) L += ml[1] * expf(ml[0] - M);
        }
        const float inv = L > 0.f ? 1.f / L : 0.f;
        for (int c = lane; c < dc; c += 32) {
            float a = 0.f;
            for (int p = 0; p < parts; ++p) {
                const float* ml = part_ml + (p * stride + bh) * 2;
                if (ml[1] > 0.f) a += expf(ml[0] - M) * part_o[(p * stride + bh) * dc + c];
            }
            dst[c] = a * inv;
        }
    }
    project_wuv<T>(h, b0, B, H, dc, dv, o_s, w_s, W_UV, out);
}

static size_t combine_smem(int dc, int dv) {
    return (static_cast<size_t>(kTok) * dc + static_cast<size_t>(dv) * (kChunk + 1)) * sizeof(float);
}

template <typename T>
cudaError_t launch_combine(const DecodePlan& P, const float* rec_ml, const float* rec_o, const T* W_UV,
                           float* out, float* part_ml, float* part_o, cudaStream_t s) {
    size_t smem = combine_smem(P.dc, P.dv);
    cudaError_t e = cudaFuncSetAttribute(combine_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    dim3 grid(P.H, ceil_div(P.B, kTok));
    combine_kernel<T><<<grid, kThreads, smem, s>>>(P, rec_ml, rec_o, W_UV, out, part_ml, part_o);
    return cudaGetLastError();
}

template <typename T>
cudaError_t launch_combine_parts(int B, int H, int dc, int dv, int parts, const float* part_ml,
                                 const float* part_o, const T* W_UV, float* out, cudaStream_t s) {
    size_t smem = combine_smem(dc, dv);
    cudaError_t e = cudaFuncSetAttribute(combine_parts_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    dim3 grid(H, ceil_div(B, kTok));
    combine_parts_kernel<T><<<grid, kThreads, smem, s>>>(B, H, dc, dv, parts, part_ml, part_o, W_UV, out);
    return cudaGetLastError();
}

#define MLA_INST(T)                                                                                   \
    template cudaError_t launch_combine<T>(const DecodePlan&, const float*, const float*, const T*,  \
                                           float*, float*, float*, cudaStream_t);                    \
    template cudaError_t launch_combine_parts<T>(int, int, int, int, int, const float*, const float*, \
                                                 const T*, float*, cudaStream_t);
MLA_INST(__half)
MLA_INST(__nv_bfloat16)
#undef MLA_INST

}  // namespace mla
