// Generic split-KV decode on CUDA cores: any d_c (multiple of 32, <= 1024) and
// even d_R (<= 128). It serves configurations the tensor-core kernel does not
// cover (the reference accepts any MLAConfig, src/mla_config.cuh:7-41), and is
// the independent cross-check of the tensor-core kernel in the GPU tests.
//
// Block = (worker w, row block of 8 rows); warp i owns row 8*blockIdx.y + i.
// Per tile of 32 positions the block stages the packed rows in shared memory
// (row stride padded by one 32-bit word so "lane = position" reads are
// conflict-free), rotates the tile's k_rope in fp32 with the caller's tables or
// on-the-fly cos / sin (the rotation of src/fused_mla.cu:34-54), then every warp scores its row
// against the 32 positions (lane j <-> position j), does an online-softmax
// update in log2 units, and accumulates o += 2^(s-m) * c_t with lane l owning
// latent columns l, l+32, ... .
#include <cfloat>

#include "mla_internal.cuh"

namespace mla {

namespace {
constexpr int kTile = 32;
constexpr int kWarps = 8;
constexpr int kMaxDcPerLane = 32;  // d_c <= 1024
}  // namespace

template <typename T>
__global__ void __launch_bounds__(kWarps * 32)
decode_simt_kernel(DecodePlan P, const T* __restrict__ kv, const T* __restrict__ qpack,
                   const float* __restrict__ rope_cos, const float* __restrict__ rope_sin,
                   float* __restrict__ rec_ml, T* __restrict__ rec_o) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int dc = P.dc, dR = P.dR, K = dc + dR, half = dR / 2;
    const int ldt = K / 2 + 1;                   // tile row stride in 32-bit words (padded)
    uint32_t* tile_w = reinterpret_cast<uint32_t*>(smem_raw);            // kTile * ldt words
    float* kr_s = reinterpret_cast<float*>(tile_w + kTile * ldt);        // kTile * (dR + 1)
    float* q_s = kr_s + kTile * (dR + 1);                                 // kWarps * K
    const int ldr = dR + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int w = blockIdx.x;
    const int row = blockIdx.y * kWarps + warp;

    const int ntiles = total_tiles(P);
    if (ntiles <= 0 || w >= P.W) return;
    int t = worker_begin(ntiles, P.W, w);
    const int t_end = worker_begin(ntiles, P.W, w + 1);
    if (t >= t_end) return;
    int g = group_of_tile(P, t);
    const int nper = dc / 32;

    while (t < t_end) {
        const int gt0 = tile_prefix(P, g), gt1 = tile_prefix(P, g + 1);
        const int lt0 = t - gt0;
        const int lt1 = (t_end < gt1 ? t_end : gt1) - gt0;
        const int len = group_len(P, g);
        const int64_t row0 = group_kv_row0(P, g);
        const bool active_block = blockIdx.y * kWarps < group_rows(P, g);  // block-uniform

        if (active_block) {
            // this warp's query row, fp32
            const T* qrow = qpack + (static_cast<long long>(g) * kGroupRows + row) * K;
            for (int k = lane; k < K; k += 32) q_s[warp * K + k] = ElemTraits<T>::to_f(qrow[k]);
        }
        float m = -INFINITY, l = 0.f;
        float acc[kMaxDcPerLane];
#pragma unroll
        for (int i = 0; i < kMaxDcPerLane; ++i) acc[i] = 0.f;

        for (int lt = lt0; lt < lt1 && active_block; ++lt) {
            const int p0 = lt * kTile;
            const int np = (len - p0) < kTile ? (len - p0) : kTile;
            const int64_t kvr = tile_kv_row(P, g, row0, p0);   // -1: page outside the cache, read nothing
            if (kvr < 0 && threadIdx.x == 0) atomicCAS(P.status, 0, kStatusBadPage);
            __syncthreads();
            // stage the packed rows (32-bit words; K is even)
            const int wpr = K / 2;
            for (int i = threadIdx.x; i < kTile * wpr; i += blockDim.x) {
                int j = i / wpr, c = i % wpr;
                uint32_t v = 0;
                if (j < np && kvr >= 0) {
                    const uint32_t* src = reinterpret_cast<const uint32_t*>(
                        kv + (kvr + j) * static_cast<int64_t>(P.row_stride));
                    v = src[c];
                }
                tile_w[j * ldt + c] = v;
            }
            __syncthreads();
            // rotate k_rope (fp32)
            for (int i = threadIdx.x; i < kTile * half; i += blockDim.x) {
                int j = i / half, d = i % half;
                float r0 = 0.f, r1 = 0.f;
                if (j < np) {
                    const T* kr = reinterpret_cast<const T*>(tile_w + j * ldt) + dc;
                    float k0 = ElemTraits<T>::to_f(kr[d]), k1 = ElemTraits<T>::to_f(kr[d + half]);
                    long long pos = static_cast<long long>(P.kv_pos_offset) + p0 + j;
                    float c, s;
                    rope_cs(P, rope_cos, rope_sin, pos, d, &c, &s);
                    r0 = k0 * c - k1 * s;
                    r1 = k0 * s + k1 * c;
                }
                kr_s[j * ldr + d] = r0;
                kr_s[j * ldr + d + half] = r1;
            }
            __syncthreads();
            // scores: lane j <-> position p0 + j
            float s = -INFINITY;
            if (lane < np) {
                const float* q = q_s + warp * K;
                const uint32_t* trow = tile_w + lane * ldt;
                float a0 = 0.f, a1 = 0.f;
                for (int c2 = 0; c2 < dc / 2; ++c2) {
                    uint32_t v = trow[c2];
                    float2 f = ElemTraits<T>::to_f2(*reinterpret_cast<const typename ElemTraits<T>::T2*>(&v));
                    a0 = fmaf(q[2 * c2], f.x, a0);
                    a1 = fmaf(q[2 * c2 + 1], f.y, a1);
                }
                const float* kr = kr_s + lane * ldr;
                for (int d = 0; d < dR; ++d) a0 = fmaf(q[dc + d], kr[d], a0);
                s = a0 + a1;
            }
            float tmax = s;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
            const float m_new = fmaxf(m, tmax);
            const float alpha = m == -INFINITY ? 0.f : exp2f(m - m_new);
            const float p = lane < np ? exp2f(s - m_new) : 0.f;
            float psum = p;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
            l = l * alpha + psum;
            m = m_new;
#pragma unroll
            for (int i = 0; i < kMaxDcPerLane; ++i) acc[i] *= alpha;
            const T* tile_e = reinterpret_cast<const T*>(tile_w);
            for (int j = 0; j < np; ++j) {
                float pj = __shfl_sync(0xffffffffu, p, j);
                const T* crow = tile_e + j * (2 * ldt);
#pragma unroll
                for (int i = 0; i < kMaxDcPerLane; ++i)
                    if (i < nper) acc[i] = fmaf(pj, ElemTraits<T>::to_f(crow[lane + 32 * i]), acc[i]);
            }
        }
        if (active_block && row < group_rows(P, g)) {
            const int rec = g + w;
            // the record holds o (bf16) or o / l (fp16) in T (l >= 1: the row's largest score contributes 2^0)
            T* o = rec_o + (static_cast<long long>(rec) * kGroupRows + row) * dc;
            const float inv_l = RecNorm<T>::value ? (l > 0.f ? 1.f / l : 0.f) : 1.f;
#pragma unroll
            for (int i = 0; i < kMaxDcPerLane; ++i)
                if (i < nper) o[lane + 32 * i] = ElemTraits<T>::from_f(acc[i] * inv_l);
            if (lane == 0) {
                float* ml = rec_ml + (static_cast<long long>(rec) * kGroupRows + row) * 2;
                ml[0] = m;
                ml[1] = l;
            }
        }
        t = gt0 + lt1;
        ++g;
        while (g < P.G && tile_prefix(P, g + 1) <= t) ++g;  // skip empty groups
    }
}

template <typename T>
cudaError_t launch_decode_simt(const DecodePlan& P, const T* kv, const T* qpack, const float* cos,
                               const float* sin, float* rec_ml, T* rec_o, cudaStream_t s) {
    const int K = P.dc + P.dR;
    size_t smem = static_cast<size_t>(kTile) * (K / 2 + 1) * 4 + static_cast<size_t>(kTile) * (P.dR + 1) * 4 +
                  static_cast<size_t>(kWarps) * K * 4;
    cudaError_t e =
        ensure_dynamic_smem(reinterpret_cast<const void*>(decode_simt_kernel<T>), static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    dim3 grid(P.W, kGroupRows / kWarps);
    decode_simt_kernel<T><<<grid, kWarps * 32, smem, s>>>(P, kv, qpack, cos, sin, rec_ml, rec_o);
    count_launches(1);
    return cudaGetLastError();
}

int simt_tile() { return kTile; }

template cudaError_t launch_decode_simt<__half>(const DecodePlan&, const __half*, const __half*,
                                                const float*, const float*, float*, __half*, cudaStream_t);
template cudaError_t launch_decode_simt<__nv_bfloat16>(const DecodePlan&, const __nv_bfloat16*,
                                                       const __nv_bfloat16*, const float*, const float*,
                                                       float*, __nv_bfloat16*, cudaStream_t);

}  // namespace mla
