// Split-KV combine and output projection.
//
// For every (token b, head h) the partial records of its group row are merged with
// the log-sum-exp identity (records hold m in log2 units, l, and o_k, or o_k / l_k in fp16):
//     M = max_k m_k,  L = sum_k l_k 2^(m_k - M),  o_lat = sum_k 2^(m_k - M) o_k / L
// and projected through W_UV: out[b, h, j] = sum_i o_lat[i] * W_UV[h*dv + j, i]
// (the projection of src/fused_mla.cu:258-267 / src/fused_mla_batched.cu:97-105).
//
// Block = (head h, chunk of up to kTok tokens), 256 threads:
//   1. warp t computes token t's record list and normalised weights (shared memory);
//   2. all threads merge the records column by column (coalesced over d_c);
//   3. warp w projects rows j = w, w + 8, ...: the W_UV[h] row is read once into
//      registers and dotted with every token's o_lat, so W_UV[h] is read once per
//      chunk of tokens.
#include <cfloat>

#include "mla_internal.cuh"
#include "peer.cuh"

namespace mla {

namespace {
constexpr int kTok = 8;
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxRec = 128;  // records per (b, h): at most the worker count (planner caps W at 128)
constexpr float kLn2 = 0.6931471805599453f;

struct MergeList {
    int count[kTok];
    int row[kTok];                 // record row (r) of the token
    int rec[kTok][kMaxRec];
    float wgt[kTok][kMaxRec];
    float m[kTok], l[kTok];        // merged max (log2) and sum
};
}  // namespace

// Record list and weights of (b, h) -> slot t (executed by one warp).
__device__ void build_merge_list(const DecodePlan& P, int b, int h, const float* __restrict__ rec_ml,
                                 MergeList& ml, int t, bool normalise, bool rec_normalised) {
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
    int w0 = 0, w1 = -1;
    if (gt1 > gt0 && T > 0) {
        w0 = worker_of_tile(T, P.W, gt0);
        w1 = worker_of_tile(T, P.W, gt1 - 1);
    }
    const int n = w1 - w0 + 1;  // <= W <= kMaxRec
    // pass 1: per-record m (lane k handles records k, k + 32, ...), warp max
    float M = -INFINITY;
    for (int k = lane; k < n; k += 32) {
        const int w = w0 + k;
        const bool valid = worker_begin(T, P.W, w) != worker_begin(T, P.W, w + 1);
        const int rec = g + w;
        float m = valid ? rec_ml[(static_cast<long long>(rec) * kGroupRows + r) * 2] : -INFINITY;
        ml.rec[t][k] = valid ? rec : -1;
        ml.wgt[t][k] = m;  // stash m
        M = fmaxf(M, m);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    float L = 0.f;
    for (int k = lane; k < n; k += 32) {
        const int rec = ml.rec[t][k];
        float a = 0.f;
        if (rec >= 0) {
            const float l = rec_ml[(static_cast<long long>(rec) * kGroupRows + r) * 2 + 1];
            a = exp2f(ml.wgt[t][k] - M);
            L += a * l;
            if (rec_normalised) a *= l;   // a record holding o / l: its weight carries its row sum
        }
        ml.wgt[t][k] = a;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
    if (normalise) {
        const float inv = L > 0.f ? 1.f / L : 0.f;
        for (int k = lane; k < n; k += 32) ml.wgt[t][k] *= inv;
    }
    if (lane == 0) {
        ml.count[t] = n < 0 ? 0 : n;
        ml.row[t] = r;
        ml.m[t] = M;
        ml.l[t] = L;
    }
}

// out[b, h, :] for the tokens of the chunk whose o_lat rows are in o_s (ntok x dc).
// Warp w handles rows j = w, w + 8, ..., four rows at a time; with d_c a multiple
// of 256 each lane reads 16-byte vectors (8 elements), so a warp keeps 4 * d_c / 256
// independent W_UV loads in flight.
template <typename T>
__device__ void project_rows(int h, int b0, int ntok, int H, int dc, int dv, const float* o_s,
                             const T* __restrict__ W_UV, float* __restrict__ out) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const T* W = W_UV + static_cast<long long>(h) * dv * dc;
    constexpr int kRows = 4;
    if (dc % 256 == 0 && dc <= 1024) {
        const int nv = dc / 256;  // 16-byte vectors per lane per row
        for (int j0 = warp * kRows; j0 < dv; j0 += kWarps * kRows) {
            uint4 wv[kRows][4];
#pragma unroll
            for (int q = 0; q < kRows; ++q)
#pragma unroll
                for (int v = 0; v < 4; ++v)
                    if (v < nv && j0 + q < dv)
                        wv[q][v] = __ldg(reinterpret_cast<const uint4*>(W + static_cast<long long>(j0 + q) * dc +
                                                                         256 * v + 8 * lane));
            float acc[kRows][kTok];
#pragma unroll
            for (int q = 0; q < kRows; ++q)
#pragma unroll
                for (int t = 0; t < kTok; ++t) acc[q][t] = 0.f;
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                if (v >= nv) break;
#pragma unroll
                for (int t = 0; t < kTok; ++t) {
                    if (t >= ntok) break;
                    const float4 o0 = *reinterpret_cast<const float4*>(o_s + t * dc + 256 * v + 8 * lane);
                    const float4 o1 = *reinterpret_cast<const float4*>(o_s + t * dc + 256 * v + 8 * lane + 4);
#pragma unroll
                    for (int q = 0; q < kRows; ++q) {
                        const uint32_t* u = reinterpret_cast<const uint32_t*>(&wv[q][v]);
                        const float2 w0 = ElemTraits<T>::to_f2(*reinterpret_cast<const typename ElemTraits<T>::T2*>(&u[0]));
                        const float2 w1 = ElemTraits<T>::to_f2(*reinterpret_cast<const typename ElemTraits<T>::T2*>(&u[1]));
                        const float2 w2 = ElemTraits<T>::to_f2(*reinterpret_cast<const typename ElemTraits<T>::T2*>(&u[2]));
                        const float2 w3 = ElemTraits<T>::to_f2(*reinterpret_cast<const typename ElemTraits<T>::T2*>(&u[3]));
                        float a = acc[q][t];
                        a = fmaf(w0.x, o0.x, a); a = fmaf(w0.y, o0.y, a); a = fmaf(w1.x, o0.z, a); a = fmaf(w1.y, o0.w, a);
                        a = fmaf(w2.x, o1.x, a); a = fmaf(w2.y, o1.y, a); a = fmaf(w3.x, o1.z, a); a = fmaf(w3.y, o1.w, a);
                        acc[q][t] = a;
                    }
                }
            }
#pragma unroll
            for (int q = 0; q < kRows; ++q) {
                if (j0 + q >= dv) break;
#pragma unroll
                for (int t = 0; t < kTok; ++t) {
                    if (t >= ntok) break;
                    float a = acc[q][t];
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
                    if (lane == 0) out[(static_cast<long long>(b0 + t) * H + h) * dv + j0 + q] = a;
                }
            }
        }
        return;
    }
    for (int j = warp; j < dv; j += kWarps) {
        const T* wr = W + static_cast<long long>(j) * dc;
        float acc[kTok];
#pragma unroll
        for (int t = 0; t < kTok; ++t) acc[t] = 0.f;
        for (int c = lane; c < dc; c += 32) {
            const float wv = ElemTraits<T>::to_f(wr[c]);
#pragma unroll
            for (int t = 0; t < kTok; ++t)
                if (t < ntok) acc[t] = fmaf(wv, o_s[t * dc + c], acc[t]);
        }
#pragma unroll
        for (int t = 0; t < kTok; ++t) {
            if (t >= ntok) break;
            float a = acc[t];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
            if (lane == 0) out[(static_cast<long long>(b0 + t) * H + h) * dv + j] = a;
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
combine_kernel(DecodePlan P, const float* __restrict__ rec_ml, const T* __restrict__ rec_o,
               const T* __restrict__ W_UV, float* __restrict__ out, PartOut part, PeerSig sig) {
    extern __shared__ float o_s[];  // kTok * dc
    __shared__ MergeList ml;
    const int h = blockIdx.x, b0 = blockIdx.y * kTok;
    const int ntok = (P.B - b0) < kTok ? (P.B - b0) : kTok;
    const int warp = threadIdx.x >> 5;
    const bool partial = out == nullptr;
    if (P.status && *reinterpret_cast<volatile int*>(P.status) != kStatusOk) {
        // the decode kernel gave up on a wait: make the failure visible in the output
        const float nan = __int_as_float(0x7fc00000);
        for (int i = threadIdx.x; i < ntok * P.dv; i += kThreads)
            if (out) out[(static_cast<long long>(b0 + i / P.dv) * P.H + h) * P.dv + i % P.dv] = nan;
        if (partial && static_cast<int>(threadIdx.x) < ntok)
            part.ml_at(b0 + threadIdx.x, h, P.B, P.H, P.dc)[1] = nan;
    } else {
        if (warp < ntok) build_merge_list(P, b0 + warp, h, rec_ml, ml, warp, !partial, RecNorm<T>::value);
        __syncthreads();
        // merge: thread -> (token, column)
        for (int i = threadIdx.x; i < ntok * P.dc; i += kThreads) {
            const int t = i / P.dc, c = i % P.dc;
            const int r = ml.row[t];
            float a = 0.f;
            for (int k = 0; k < ml.count[t]; ++k) {
                const int rec = ml.rec[t][k];
                if (rec >= 0)
                    a = fmaf(ml.wgt[t][k],
                             ElemTraits<T>::to_f(rec_o[(static_cast<long long>(rec) * kGroupRows + r) * P.dc + c]), a);
            }
            if (partial) part.o_at(b0 + t, h, P.B, P.H, P.dc)[c] = a;
            else o_s[t * P.dc + c] = a;
        }
        if (partial) {
            if (static_cast<int>(threadIdx.x) < ntok) {
                const int t = threadIdx.x;
                float* pm = part.ml_at(b0 + t, h, P.B, P.H, P.dc);
                pm[0] = ml.l[t] > 0.f ? ml.m[t] * kLn2 : -INFINITY;  // natural-log units for the caller
                pm[1] = ml.l[t];
                if (part.slices) pm[2] = pm[3] = 0.f;
            }
        } else {
            __syncthreads();
            project_rows<T>(h, b0, ntok, P.H, P.dc, P.dv, o_s, W_UV, out);
        }
    }
    // every block of head slice q (hs heads x gridDim.y token blocks) stores into q's receiver
    if (part.to_peers()) {
        const int hs = P.H / part.slices;
        peer_block_done(sig, h / hs, static_cast<unsigned int>(hs) * gridDim.y);
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
combine_parts_kernel(int B, int H, int dc, int dv, int parts, const float* __restrict__ part_ml,
                     const float* __restrict__ part_o, int ml_stride, int o_stride, const T* __restrict__ W_UV,
                     float* __restrict__ out) {
    extern __shared__ float o_s[];
    __shared__ float wgt[kTok][64];
    const int h = blockIdx.x, b0 = blockIdx.y * kTok;
    const int ntok = (B - b0) < kTok ? (B - b0) : kTok;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long stride = static_cast<long long>(B) * H;
    if (warp < ntok) {
        const long long bh = static_cast<long long>(b0 + warp) * H + h;
        float M = -INFINITY;
        for (int p = lane; p < parts; p += 32) {
            const float* pm = part_ml + (p * stride + bh) * ml_stride;
            if (pm[1] > 0.f) M = fmaxf(M, pm[0]);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
        float L = 0.f;
        for (int p = lane; p < parts; p += 32) {
            const float* pm = part_ml + (p * stride + bh) * ml_stride;
            const float a = pm[1] > 0.f ? expf(pm[0] - M) : 0.f;
            wgt[warp][p] = a;
            L += a * pm[1];
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
        const float inv = L > 0.f ? 1.f / L : 0.f;
        __syncwarp();
        for (int p = lane; p < parts; p += 32) wgt[warp][p] *= inv;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < ntok * dc; i += kThreads) {
        const int t = i / dc, c = i % dc;
        const long long bh = static_cast<long long>(b0 + t) * H + h;
        float a = 0.f;
        for (int p = 0; p < parts; ++p) a = fmaf(wgt[t][p], part_o[(p * stride + bh) * o_stride + c], a);
        o_s[t * dc + c] = a;
    }
    __syncthreads();
    project_rows<T>(h, b0, ntok, H, dc, dv, o_s, W_UV, out);
}

template <typename T>
cudaError_t launch_combine(const DecodePlan& P, const float* rec_ml, const T* rec_o, const T* W_UV,
                           float* out, const PartOut& part, const PeerSig& sig, cudaStream_t s) {
    if (P.W > kMaxRec) return cudaErrorInvalidValue;
    const size_t smem = static_cast<size_t>(kTok) * P.dc * sizeof(float);
    cudaError_t e =
        ensure_dynamic_smem(reinterpret_cast<const void*>(combine_kernel<T>), static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    dim3 grid(P.H, ceil_div(P.B, kTok));
    combine_kernel<T><<<grid, kThreads, smem, s>>>(P, rec_ml, rec_o, W_UV, out, part, sig);
    count_launches(1);
    return cudaGetLastError();
}

template <typename T>
cudaError_t launch_combine_parts(int B, int H, int dc, int dv, int parts, const float* part_ml,
                                 const float* part_o, int ml_stride, int o_stride, const T* W_UV, float* out,
                                 cudaStream_t s) {
    if (parts > 64) return cudaErrorInvalidValue;
    const size_t smem = static_cast<size_t>(kTok) * dc * sizeof(float);
    cudaError_t e =
        ensure_dynamic_smem(reinterpret_cast<const void*>(combine_parts_kernel<T>), static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    dim3 grid(H, ceil_div(B, kTok));
    combine_parts_kernel<T><<<grid, kThreads, smem, s>>>(B, H, dc, dv, parts, part_ml, part_o, ml_stride, o_stride,
                                                         W_UV, out);
    count_launches(1);
    return cudaGetLastError();
}

#define MLA_INST(T)                                                                                   \
    template cudaError_t launch_combine<T>(const DecodePlan&, const float*, const T*, const T*,      \
                                           float*, const PartOut&, const PeerSig&, cudaStream_t);    \
    template cudaError_t launch_combine_parts<T>(int, int, int, int, int, const float*, const float*, \
                                                 int, int, const T*, float*, cudaStream_t);
MLA_INST(__half)
MLA_INST(__nv_bfloat16)
#undef MLA_INST

}  // namespace mla
